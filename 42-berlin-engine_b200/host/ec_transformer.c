/*
** ec_transformer.c -- the reference's transformer_init / transformer_forward
** contract (src/inference/inference.h:188-202) on top of libengine_cuda.
*/
#include "ec_transformer.h"
#include <stdlib.h>
#include <string.h>

int	ec_transformer_init(t_ec_transformer *t, const ec_model_config *c,
		int device)
{
	int	rc;

	if (!t || !c)
		return (EC_ERR_ARG);
	memset(t, 0, sizeof(*t));
	t->config = *c;
	rc = ec_create(c, device, &t->ctx);
	if (rc != EC_OK)
		return (rc);
	t->logits = calloc((size_t)c->vocab_size, sizeof(float));
	if (!t->logits)
	{
		ec_destroy(t->ctx);
		t->ctx = NULL;
		return (EC_ERR_OOM);
	}
	return (EC_OK);
}

/* name patterns of model.c:186-236, tried in order */
static const struct
{
	const char	*pat;
	int			which;
}	g_layer_names[] = {
	{"attention.wq", EC_WQ}, {"self_attn.q_proj", EC_WQ},
	{"attention.wk", EC_WK}, {"self_attn.k_proj", EC_WK},
	{"attention.wv", EC_WV}, {"self_attn.v_proj", EC_WV},
	{"attention.wo", EC_WO}, {"self_attn.o_proj", EC_WO},
	{"feed_forward.w1", EC_W1}, {"mlp.gate_proj", EC_W1},
	{"feed_forward.w2", EC_W2}, {"mlp.down_proj", EC_W2},
	{"feed_forward.w3", EC_W3}, {"mlp.up_proj", EC_W3},
	{"attention_norm", EC_ATTN_NORM}, {"input_layernorm", EC_ATTN_NORM},
	{"ffn_norm", EC_FFN_NORM}, {"post_attention_layernorm", EC_FFN_NORM},
};

/* A matrix with scales is already quantised (the context's INT8 / FP8
** format); without scales it is the reference's BF16 tensor, quantised on
** the device (ec_set_weight_bf16).  Vectors are BF16 either way. */
static int	set_one(t_ec_transformer *t, int layer, int which, const void *data,
		const float *scales)
{
	const int	matrix = (layer >= 0 && which <= EC_W3) || which == EC_LM_HEAD;

	if (matrix && !scales)
		return (ec_set_weight_bf16(t->ctx, layer, which, data, 0));
	return (ec_set_weight(t->ctx, layer, which, data, matrix ? scales : NULL, 0));
}

int	ec_transformer_set_tensor(t_ec_transformer *t, const char *name,
		const void *data, const float *scales)
{
	const char	*lm;
	int			layer;
	size_t		i;

	if (!t || !t->ctx || !name || !data)
		return (EC_ERR_ARG);
	lm = strstr(name, "layers.");
	if (lm)
	{
		layer = atoi(lm + 7);
		if (layer < 0 || layer >= t->config.n_layers)
			return (EC_ERR_ARG);
		for (i = 0; i < sizeof(g_layer_names) / sizeof(g_layer_names[0]); i++)
			if (strstr(name, g_layer_names[i].pat))
				return (set_one(t, layer, g_layer_names[i].which, data, scales));
		return (EC_ERR_ARG);
	}
	if (!strcmp(name, "tok_embeddings.weight")
		|| !strcmp(name, "model.embed_tokens.weight"))
		return (ec_set_weight(t->ctx, -1, EC_EMBEDDING, data, NULL, 0));
	if (!strcmp(name, "norm.weight") || !strcmp(name, "model.norm.weight"))
		return (ec_set_weight(t->ctx, -1, EC_FINAL_NORM, data, NULL, 0));
	if (!strcmp(name, "output.weight") || !strcmp(name, "lm_head.weight"))
		return (set_one(t, -1, EC_LM_HEAD, data, scales));
	return (EC_ERR_ARG);
}

float	*ec_transformer_forward(t_ec_transformer *t, int token, int pos)
{
	int	rc;

	if (!t || !t->ctx)
		return (NULL);
	rc = ec_decode_step(t->ctx, &token, &pos, 1, t->logits, &t->last_token);
	t->last_error = rc;
	return (rc == EC_OK ? t->logits : NULL);
}

int	ec_transformer_argmax(const t_ec_transformer *t)
{
	return (t ? t->last_token : -1);
}

int	ec_transformer_reset(t_ec_transformer *t)
{
	if (!t || !t->ctx)
		return (EC_ERR_ARG);
	return (ec_reset(t->ctx, 0));
}

void	ec_transformer_free(t_ec_transformer *t)
{
	if (!t)
		return ;
	ec_destroy(t->ctx);
	free(t->logits);
	memset(t, 0, sizeof(*t));
}
