/*
** ec_transformer.h -- host-side mirror of the reference's inference API
** (src/inference/inference.h:188-202) over libengine_cuda.so.
**
** A caller of transformer_init / transformer_forward switches to
** ec_transformer_init / ec_transformer_forward with the same meaning:
** forward(t, token, pos) runs one decode token and returns a pointer to
** vocab_size host floats (the reference's s->logits contract,
** inference.c:695), valid until the next call.  Errors return NULL / a
** negative EC_ERR_* code instead of exit(1).
*/
#ifndef EC_TRANSFORMER_H
# define EC_TRANSFORMER_H
# include "engine_cuda.h"

# ifdef __cplusplus
extern "C" {
# endif

typedef struct s_ec_transformer
{
	ec_model_config	config;
	ec_ctx			*ctx;
	float			*logits;	/* host [vocab_size] */
	int				last_token;	/* argmax of the last forward */
	int				last_error;
}	t_ec_transformer;

/* transformer_init (model.c:146) minus file I/O: allocate the device state. */
int		ec_transformer_init(t_ec_transformer *t, const ec_model_config *c,
			int device);

/* Map one named tensor the way model.c:167-265 does: "layers.N.<name>" with
** the LLaMA (attention.wq, feed_forward.w1, attention_norm, ...) or
** HuggingFace (self_attn.q_proj, mlp.gate_proj, input_layernorm, ...)
** spellings, plus tok_embeddings / norm / output (or model.embed_tokens,
** model.norm, lm_head).  A matrix passed with `scales` is already in the
** context's weight format (as ec_set_weight); with scales == NULL it is the
** reference's BF16 tensor and is quantised on the device
** (ec_set_weight_bf16). */
int		ec_transformer_set_tensor(t_ec_transformer *t, const char *name,
			const void *data, const float *scales);

/* transformer_forward (inference.c:60): one token of sequence 0. */
float	*ec_transformer_forward(t_ec_transformer *t, int token, int pos);

/* greedy token of the last forward (sample_argmax, sampler.c:145) */
int		ec_transformer_argmax(const t_ec_transformer *t);

/* start a new context (paged_kv_reset + lsh_index_reset) */
int		ec_transformer_reset(t_ec_transformer *t);

void	ec_transformer_free(t_ec_transformer *t);

# ifdef __cplusplus
}
# endif
#endif
