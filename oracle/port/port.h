/*
** port.h -- TEST INFRASTRUCTURE ONLY (oracle).
**
** A plain-C restatement of the reference engine's decode hot path
** (fgroo/42-Berlin-Engine, src/inference/inference.c:60 and the ops it calls),
** written so that every floating-point operation happens in the same order,
** with the same fused multiply-adds, as the reference compiled with its own
** release flags pinned to AVX2+FMA.  Each function cites the reference
** location it restates.  It serves three purposes:
**   1. the checker the CUDA library is compared against in tests/;
**   2. the oracle for settings the reference cannot express (INT8 / FP8
**      weights with general scales, LSH with L tables x b bits and G-token
**      hash units);
**   3. the "port" CPU baseline in bench.py.
** It is pinned against the reference itself (oracle/_ref) by tests/.
** The product (libengine_cuda.so) never links or loads it.
*/
#ifndef PORT_H
# define PORT_H
# include <stdint.h>
# include <stddef.h>

/* ---- numerics primitives ---------------------------------------------- */
float	port_bf16_to_f32(uint16_t b);
uint16_t	port_f32_to_bf16(float f);
float	port_fast_expf(float x);
float	port_fast_expf_vec(float x);
float	port_fp8_e4m3_to_f32(uint8_t code);
float	port_dot_f32(const float *a, const float *b, int n);
float	port_dot_bf16_f32(const uint16_t *a, const float *b, int n);

/* ---- ops ---------------------------------------------------------------- */
void	port_gemv_bf16(float *out, const uint16_t *w, const float *x, int m,
			int k);
void	port_gemv_q8(float *out, const int8_t *w, const float *scale,
			const float *x, int m, int k);
void	port_gemv_fp8(float *out, const uint8_t *w, float scale,
			const float *x, int m, int k);
void	port_rmsnorm(float *out, const float *x, const uint16_t *w, int n,
			float eps);
void	port_rope_tables(float *cos_t, float *sin_t, int head_dim, int max_seq,
			float theta);
void	port_rope(float *data, int n_heads, int head_dim, int pos,
			const float *cos_t, const float *sin_t, int max_seq);
void	port_silu_mul(float *out, const float *g, const float *u, int n);
float	port_quant_int8(int8_t *out, const float *in, int n);
int		port_argmax(const float *x, int n);
int		port_heap_topk(const float *scores, const int *idx, int n, int k,
			int *out);

/* ---- LSH with L tables x b bits over G-token units --------------------- */
typedef struct s_port_lsh
{
	int			n_tables;
	int			n_bits;
	int			dim;
	int			unit;			/* tokens per hashed unit (64 in the reference) */
	int			max_units;
	int			radius;
	float		*hp;			/* [n_tables][n_bits][dim] */
	uint32_t	*unit_hash;		/* [n_tables][max_units] */
	int			*unit_start;	/* [max_units] */
	int			*unit_len;		/* [max_units] */
	int			*heads;			/* [n_tables][2^n_bits] */
	int			*next;			/* [n_tables][max_units] */
	int			n_units;
	float		*acc;			/* [dim] running sum of the open unit */
	int			acc_count;
	int			acc_start;
}	t_port_lsh;

t_port_lsh	*port_lsh_create(int n_tables, int n_bits, int dim, int unit,
				int max_units, int radius, unsigned int seed);
void	port_lsh_free(t_port_lsh *l);
void	port_lsh_reset(t_port_lsh *l);
uint32_t	port_lsh_hash(const t_port_lsh *l, int table, const float *v);
void	port_lsh_update(t_port_lsh *l, const float *key, int pos);
int		port_lsh_find(const t_port_lsh *l, const uint32_t *qhash,
			int *unit_ids, int max_units);
int		port_lsh_attend(const t_port_lsh *l, const uint16_t *k,
			const uint16_t *v, int kv_len, const float *q, int n_heads,
			int n_kv_heads, int head_dim, int window, int max_cand, int sparse_k,
			int *topk, float *out);

/* ---- paged INT8 KV cache, one layer ------------------------------------ */
# define PORT_KV_BLOCK 16

typedef struct s_port_paged
{
	int		n_kv_heads;
	int		head_dim;
	int		max_blocks;
	int		n_blocks;		/* logical blocks in use */
	int		n_tokens;
	int8_t	*k;				/* [max_blocks][kv][16][hd] */
	int8_t	*v;
	float	*ks;			/* [max_blocks][kv][16] */
	float	*vs;
	float	*centroid;		/* [max_blocks][hd] */
	int		*fill;			/* [max_blocks] tokens in block */
}	t_port_paged;

t_port_paged	*port_paged_create(int n_kv_heads, int head_dim, int max_tokens);
void	port_paged_free(t_port_paged *p);
void	port_paged_reset(t_port_paged *p);
void	port_paged_append(t_port_paged *p, const float *k, const float *v,
			int pos);
void	port_paged_attention(float *out, const float *q, const t_port_paged *p,
			const int *blocks, int n_sel, int n_heads);
void	port_paged_scores(const t_port_paged *p, const float *q, float *scores);
int		port_select_blocks(const float *scores, int n_blocks, int k,
			int *selected);

/* ---- linear BF16 KV attention over an index list ----------------------- */
void	port_linear_attention(float *out, const float *q, const uint16_t *k,
			const uint16_t *v, const int *idx, int n_idx, int n_heads,
			int n_kv_heads, int head_dim);

/* ---- whole decode step -------------------------------------------------- */
typedef struct s_port_config
{
	int		dim;
	int		hidden_dim;
	int		n_layers;
	int		n_heads;
	int		n_kv_heads;
	int		vocab_size;
	int		seq_len;
	int		head_dim;
	float	rope_theta;
	float	norm_eps;
	int		use_paged_kv;
	int		sparse_k;
	int		window;
	int		sparse_blocks_k;
	int		lsh_tables;
	int		lsh_bits;
	int		lsh_unit;
	int		lsh_max_units;
	int		lsh_radius;
	int		lsh_max_cand;
	int		weight_kind;	/* 0 = INT8 per-row scale, 1 = FP8 E4M3 per-tensor */
}	t_port_config;

typedef struct s_port_weights
{
	const uint16_t	*emb;			/* [V][D] bf16 */
	const uint16_t	*final_norm;	/* [D] bf16 */
	const void		*lm;			/* [V][D] int8/fp8 */
	const float		*lm_scale;		/* [V] (INT8) or [1] (FP8) */
	/* per layer, 7 matrices (wq wk wv wo w1 w2 w3) + 2 norms */
	const void		**mat;			/* [L*7] */
	const float		**mat_scale;	/* [L*7] */
	const uint16_t	**norm;			/* [L*2] attention_norm, ffn_norm */
}	t_port_weights;

void	*port_model_create(const t_port_config *c, const t_port_weights *w);
void	port_model_free(void *m);
void	port_model_reset(void *m);
const float	*port_model_forward(void *m, int token, int pos);
const float	*port_model_state(void *m, int which);
const t_port_lsh	*port_model_lsh(void *m);
const t_port_paged	*port_model_paged(void *m, int layer);
const uint16_t	*port_model_linear_k(void *m, int layer);
void	port_model_counters(void *m, unsigned long long *out);

/* ---- sampling (sample.c) ---------------------------------------------- */
void	port_repetition_penalty(float *logits, const int *hist, int hn,
			float penalty);
int		port_sample_top_p(float *logits, int n, const int *hist, int hn,
			float temperature, float top_p, float penalty, int block0, float r,
			int *cut_out, float *cum_out);
int		port_sample_temperature(const float *logits, int n, float temperature,
			float r);

#endif
