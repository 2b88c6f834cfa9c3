/*
** ref_driver.c -- TEST INFRASTRUCTURE ONLY (oracle).
**
** A thin C driver that is linked against the reference engine's own,
** unmodified sources (compiled in place by oracle/Makefile into
** oracle/_ref/libref_driver.so).  It lets the parity tests call the
** reference's decode hot path on seeded inputs:
**   - transformer_forward (src/inference/inference.c:60) on a t_transformer
**     that this driver assembles field by field instead of going through
**     transformer_init (src/inference/model.c:146).  That avoids the 10 MB
**     state arena that cannot hold the 8B shape (model.c:279) without
**     patching any reference file;
**   - the individual ops: op_matmul, op_rmsnorm, rope_apply_multihead_cached,
**     op_silu_mul, quant_f32_to_int8, paged_kv_append, score_blocks,
**     select_top_k_blocks, op_paged_attention(_sparse), op_attention_sparse,
**     lsh_init / lsh_hash / lsh_update / lsh_find_candidates, heap_push,
**     sample_argmax.
**
** Nothing in the product (the CUDA library) links or loads this file.
*/
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include "inference/inference.h"
#include "compute/ops.h"
#include "compute/ops_attention.h"
#include "compute/ops_rope.h"
#include "compute/ops_lsh.h"
#include "compute/ops_heap.h"
#include "compute/ops_quant.h"
#include "compute/sampler.h"
#include "memory/paged.h"
#include "memory/kv_cache.h"
#include "memory/arena.h"

typedef struct s_refd_config
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
}	t_refd_config;

typedef struct s_refd
{
	t_transformer	t;
	t_tensor		*tensors;	/* owned tensor headers */
	int				n_tensors;
}	t_refd;

static t_tensor	*mk2d(t_refd *r, const void *data, int rows, int cols)
{
	t_tensor	*x;

	x = &r->tensors[r->n_tensors++];
	memset(x, 0, sizeof(*x));
	x->data = (void *)data;
	x->ndim = 2;
	x->shape[0] = rows;
	x->shape[1] = cols;
	x->stride[0] = cols;
	x->stride[1] = 1;
	x->size = (size_t)rows * cols;
	x->dtype = DTYPE_BF16;
	return (x);
}

/*
** layer_w holds n_layers * 9 pointers, per layer in the order
** wq, wk, wv, wo, w1 (gate), w2 (down), w3 (up), attention_norm, ffn_norm.
** All weights are BF16, row-major [out_features, in_features].
*/
void	*refd_create(const t_refd_config *c, const uint16_t *emb,
			const uint16_t *final_norm, const uint16_t *lm_head,
			const uint16_t *const *layer_w)
{
	t_refd			*r;
	t_transformer	*t;
	int				L;
	int				i;
	int				qd;
	int				kvd;

	r = calloc(1, sizeof(*r));
	if (!r)
		return (NULL);
	t = &r->t;
	L = c->n_layers;
	r->tensors = calloc((size_t)L * 9 + 8, sizeof(t_tensor));
	t->config.dim = c->dim;
	t->config.hidden_dim = c->hidden_dim;
	t->config.n_layers = L;
	t->config.n_heads = c->n_heads;
	t->config.n_kv_heads = c->n_kv_heads;
	t->config.vocab_size = c->vocab_size;
	t->config.seq_len = c->seq_len;
	t->config.head_dim = c->head_dim;
	t->config.rope_theta = c->rope_theta;
	t->config.rope_factor = 1.0f;
	t->config.mscale = 1.0f;
	t->config.norm_eps = c->norm_eps;
	qd = c->n_heads * c->head_dim;
	kvd = c->n_kv_heads * c->head_dim;
	t->weights.token_embedding = mk2d(r, emb, c->vocab_size, c->dim);
	t->weights.norm = mk2d(r, final_norm, 1, c->dim);
	t->weights.output = mk2d(r, lm_head, c->vocab_size, c->dim);
	t->weights.layers = calloc(L, sizeof(t_layer_weights));
	for (i = 0; i < L; i++)
	{
		const uint16_t *const	*w = layer_w + (size_t)i * 9;
		t_layer_weights			*l = &t->weights.layers[i];

		l->wq = mk2d(r, w[0], qd, c->dim);
		l->wk = mk2d(r, w[1], kvd, c->dim);
		l->wv = mk2d(r, w[2], kvd, c->dim);
		l->wo = mk2d(r, w[3], c->dim, qd);
		l->w1 = mk2d(r, w[4], c->hidden_dim, c->dim);
		l->w2 = mk2d(r, w[5], c->dim, c->hidden_dim);
		l->w3 = mk2d(r, w[6], c->hidden_dim, c->dim);
		l->attention_norm = mk2d(r, w[7], 1, c->dim);
		l->ffn_norm = mk2d(r, w[8], 1, c->dim);
	}
	/* state buffers (same set transformer_init allocates, model.c:286-296) */
	t->state.x = calloc(c->dim, sizeof(float));
	t->state.xb = calloc(c->dim, sizeof(float));
	t->state.hb = calloc(c->hidden_dim > qd ? c->hidden_dim : qd, sizeof(float));
	t->state.hb2 = calloc(c->hidden_dim, sizeof(float));
	t->state.q = calloc(qd, sizeof(float));
	t->state.k = calloc(kvd, sizeof(float));
	t->state.v = calloc(kvd, sizeof(float));
	t->state.logits = calloc(c->vocab_size, sizeof(float));
	t->state.token_history = calloc(c->seq_len, sizeof(int));
	arena_init(&t->scratch, 64u << 20);
	t->sparse_k = c->sparse_k;
	t->nested_learning = 0;
	/* evict_weights.data stays NULL: eviction off (inference.c:200) */
	/* final_adapter / logit_bias / context_bias stay NULL: they are
	** zero-initialised no-ops in transformer_init (model.c:447-489). */
	t->state.kv_cache = calloc(L, sizeof(t_kv_cache));
	if (!c->use_paged_kv)
	{
		t_kv_init_params	kp;

		kp.max_seq = c->seq_len;
		kp.num_heads = c->n_kv_heads;
		kp.head_dim = c->head_dim;
		arena_init(&t->kv_arena,
			(size_t)L * 2 * c->seq_len * kvd * sizeof(uint16_t) + (1u << 20));
		for (i = 0; i < L; i++)
			kv_cache_init(&t->state.kv_cache[i], &t->kv_arena, &kp);
	}
	t->use_paged_kv = c->use_paged_kv;
	if (c->use_paged_kv)
	{
		int	mbpl;

		mbpl = (c->seq_len + KV_BLOCK_SIZE - 1) / KV_BLOCK_SIZE;
		if (block_manager_init(&t->block_manager, L, c->n_kv_heads,
				c->head_dim, mbpl) != 0)
			return (NULL);
		t->paged_kv = calloc(L, sizeof(t_paged_kv_cache));
		for (i = 0; i < L; i++)
		{
			t->paged_kv[i].bm = &t->block_manager;
			t->paged_kv[i].layer_idx = i;
		}
	}
	t->rope_cache = rope_cache_init(c->head_dim, c->seq_len, c->rope_theta);
	t->lsh_ctx = calloc(1, sizeof(t_lsh_ctx));
	t->lsh_index = calloc(1, sizeof(t_lsh_index));
	lsh_init((t_lsh_ctx *)t->lsh_ctx, c->head_dim, 42);
	lsh_index_init((t_lsh_index *)t->lsh_index);
	t->use_lsh = (c->sparse_k > 0);
	lsh_stats_reset_atomic(&t->lsh_stats);
	return (r);
}

float	*refd_forward(void *h, int token, int pos)
{
	return (transformer_forward(&((t_refd *)h)->t, token, pos));
}

#ifdef ENGINE_CUDA
/* drop-in build only: attach a libengine_cuda context (NULL: CPU path) */
void	refd_attach_gpu(void *h, void *ctx)
{
	((t_refd *)h)->t.gpu = (struct ec_ctx *)ctx;
}
#endif

/*
** The optional final hidden adapter (bf16 [dim][dim]) and logit bias (float
** [vocab]) that transformer_forward applies after the final norm
** (inference.c:583-651); NULL detaches.  The caller keeps the memory.
*/
void	refd_set_adapter(void *h, const uint16_t *adapter)
{
	t_refd	*r = (t_refd *)h;

	r->t.final_adapter = adapter ? mk2d(r, adapter, r->t.config.dim, r->t.config.dim) : NULL;
}

void	refd_set_logit_bias(void *h, const float *bias)
{
	((t_refd *)h)->t.logit_bias = (float *)bias;
}

/* the context-aware bias cache (inference.c:657-693); keys == NULL detaches */
void	refd_set_context_bias(void *h, const uint64_t *keys, const int *tokens,
		const float *biases, int size)
{
	t_transformer	*t = &((t_refd *)h)->t;

	t->context_bias.keys = (uint64_t *)keys;
	t->context_bias.tokens = (int *)tokens;
	t->context_bias.biases = (float *)biases;
	t->context_bias.size = size;
	t->context_bias.count = 0;
}

/*
** Fill positions 0..n-1 of every layer's paged KV cache with seeded
** synthetic keys and values through the reference's own paged_kv_append
** (paged.c:195) and layer 0's lsh_update (ops_lsh.c:296), the two calls
** transformer_forward makes per token (inference.c:169-192), without the
** projections.  Used by the timed CPU baseline to decode at a long context
** without paying for a CPU prompt.  Values: uniform in [-2, 2) from a 32-bit
** LCG (roughly the spread of the projections of the synthetic models).
*/
int	refd_fill_context(void *h, int n, unsigned seed)
{
	t_transformer	*t = &((t_refd *)h)->t;
	int				kvd;
	float			*k;
	float			*v;
	int				pos;
	int				i;
	int				d;

	if (!t->use_paged_kv || n > t->config.seq_len)
		return (-1);
	kvd = t->config.n_kv_heads * t->config.head_dim;
	k = malloc(kvd * sizeof(float));
	v = malloc(kvd * sizeof(float));
	if (!k || !v)
		return (free(k), free(v), -1);
	for (pos = 0; pos < n; pos++)
	{
		for (i = 0; i < t->config.n_layers; i++)
		{
			for (d = 0; d < kvd; d++)
			{
				seed = seed * 1664525u + 1013904223u;
				k[d] = ((float)(seed >> 8) / 16777216.0f) * 4.0f - 2.0f;
				seed = seed * 1664525u + 1013904223u;
				v[d] = ((float)(seed >> 8) / 16777216.0f) * 4.0f - 2.0f;
			}
			paged_kv_append(&t->paged_kv[i], k, v, pos);
			if (i == 0 && t->lsh_ctx && t->lsh_index)
				lsh_update((t_lsh_index *)t->lsh_index, (t_lsh_ctx *)t->lsh_ctx,
					k, t->config.head_dim, pos);
		}
	}
	free(k);
	free(v);
	return (0);
}

/* copies of intermediate state for layer-level parity checks */
const float	*refd_state(void *h, int which)
{
	t_inference_state	*s = &((t_refd *)h)->t.state;

	switch (which)
	{
		case 0: return (s->x);
		case 1: return (s->xb);
		case 2: return (s->q);
		case 3: return (s->k);
		case 4: return (s->v);
		case 5: return (s->hb);
		case 6: return (s->logits);
	}
	return (NULL);
}

const t_lsh_index	*refd_lsh_index(void *h)
{
	return ((const t_lsh_index *)((t_refd *)h)->t.lsh_index);
}

const t_lsh_ctx	*refd_lsh_ctx(void *h)
{
	return ((const t_lsh_ctx *)((t_refd *)h)->t.lsh_ctx);
}

/* paged KV introspection: the block holding (layer, logical block) */
int	refd_paged_block(void *h, int layer, int lblock, int8_t *k_out,
		int8_t *v_out, float *ks_out, float *vs_out, float *centroid_out)
{
	t_transformer	*t = &((t_refd *)h)->t;
	t_block_manager	*bm = &t->block_manager;
	int				phys;
	t_kv_block		*b;
	int				n;

	if (!t->use_paged_kv || lblock >= bm->logical_len[layer])
		return (-1);
	phys = bm->page_table[layer * bm->max_logical + lblock];
	if (phys < 0)
		return (-1);
	b = &bm->blocks[phys];
	n = bm->n_kv_heads * KV_BLOCK_SIZE;
	memcpy(k_out, b->k_quant, (size_t)n * bm->head_dim);
	memcpy(v_out, b->v_quant, (size_t)n * bm->head_dim);
	memcpy(ks_out, b->k_scales, n * sizeof(float));
	memcpy(vs_out, b->v_scales, n * sizeof(float));
	memcpy(centroid_out, b->centroid, bm->head_dim * sizeof(float));
	return (b->n_tokens);
}

/* linear BF16 KV cache introspection */
const uint16_t	*refd_linear_k(void *h, int layer)
{
	return ((const uint16_t *)((t_refd *)h)->t.state.kv_cache[layer].k.data);
}

const uint16_t	*refd_linear_v(void *h, int layer)
{
	return ((const uint16_t *)((t_refd *)h)->t.state.kv_cache[layer].v.data);
}

void	refd_lsh_counters(void *h, unsigned long long *out)
{
	t_transformer	*t = &((t_refd *)h)->t;

	out[0] = atomic_load(&t->lsh_stats.total_queries);
	out[1] = atomic_load(&t->lsh_stats.total_used_k);
}

/* ------------------------------------------------------------------ */
/* Individual ops on caller buffers                                    */
/* ------------------------------------------------------------------ */

static void	col(t_tensor *x, void *data, int n, t_dtype dt)
{
	memset(x, 0, sizeof(*x));
	x->data = data;
	x->ndim = 2;
	x->shape[0] = n;
	x->shape[1] = 1;
	x->stride[0] = 1;
	x->stride[1] = 1;
	x->size = n;
	x->dtype = dt;
}

int	refd_matmul(float *out, const uint16_t *w, const float *x, int m, int k)
{
	t_tensor	o;
	t_tensor	a;
	t_tensor	b;

	col(&o, out, m, DTYPE_F32);
	col(&b, (void *)x, k, DTYPE_F32);
	memset(&a, 0, sizeof(a));
	a.data = (void *)w;
	a.ndim = 2;
	a.shape[0] = m;
	a.shape[1] = k;
	a.size = (size_t)m * k;
	a.dtype = DTYPE_BF16;
	return (op_matmul(&o, &a, &b));
}

void	refd_rmsnorm(float *out, const float *x, const uint16_t *w, int n,
		float eps)
{
	t_tensor	o;
	t_tensor	xi;
	t_tensor	wt;

	col(&o, out, n, DTYPE_F32);
	col(&xi, (void *)x, n, DTYPE_F32);
	col(&wt, (void *)w, n, DTYPE_BF16);
	op_rmsnorm(&o, &xi, &wt, eps);
}

void	*refd_rope_create(int head_dim, int max_seq, float theta)
{
	return (rope_cache_init(head_dim, max_seq, theta));
}

const float	*refd_rope_table(void *c, int which)
{
	t_rope_cache	*rc = (t_rope_cache *)c;

	return (which == 0 ? rc->cos_table : rc->sin_table);
}

void	refd_rope_apply(void *c, float *data, int n_heads, int pos)
{
	rope_apply_multihead_cached(data, n_heads, pos, (t_rope_cache *)c);
}

void	refd_silu_mul(float *out, const float *gate, const float *up, int n)
{
	t_tensor	o;
	t_tensor	g;
	t_tensor	u;

	col(&o, out, n, DTYPE_F32);
	col(&g, (void *)gate, n, DTYPE_F32);
	col(&u, (void *)up, n, DTYPE_F32);
	op_silu_mul(&o, &g, &u);
}

float	refd_quant_int8(int8_t *out, const float *in, int n)
{
	return (quant_f32_to_int8(out, in, n));
}

int	refd_argmax(const float *logits, int n)
{
	t_tensor	l;

	col(&l, (void *)logits, n, DTYPE_F32);
	return (sample_argmax(&l));
}

/* the reference's own sample_top_p (sampler_topp.c:113) after srand(seed);
** refd_first_rand gives the draw it takes: the first rand() / RAND_MAX */
float	refd_first_rand(unsigned int seed)
{
	srand(seed);
	return ((float)rand() / (float)RAND_MAX);
}

int	refd_sample_top_p(const float *logits, int n, float temperature,
		float top_p, unsigned int seed)
{
	t_tensor	l;
	t_arena		a;
	int			tok;

	col(&l, (void *)logits, n, DTYPE_F32);
	arena_init(&a, (size_t)n * 8 + 4096);
	srand(seed);
	tok = sample_top_p(&l, temperature, top_p, &a);
	arena_free(&a);
	return (tok);
}

/* min-heap top-K exactly as inference.c:410-418 drives it */
int	refd_heap_topk(const float *scores, const int *idx, int n, int k,
		int *out)
{
	t_heap_item	*heap;
	int			size;
	int			i;

	heap = malloc(sizeof(t_heap_item) * (k > 0 ? k : 1));
	size = 0;
	for (i = 0; i < n; i++)
		heap_push(heap, &size, k, scores[i], idx[i]);
	heap_extract_indices(heap, size, out);
	free(heap);
	return (size);
}

/* LSH (single table, 16 bits, 64-token centroid units) */
void	*refd_lsh_ctx_create(int dim, unsigned int seed)
{
	t_lsh_ctx	*c;

	c = calloc(1, sizeof(*c));
	lsh_init(c, dim, seed);
	return (c);
}

const float	*refd_lsh_hyperplanes(void *c)
{
	return (&((t_lsh_ctx *)c)->hyperplanes[0][0]);
}

int	refd_lsh_hash(void *c, const float *v)
{
	return (lsh_hash((t_lsh_ctx *)c, v));
}

void	*refd_lsh_index_create(void)
{
	t_lsh_index	*ix;

	ix = calloc(1, sizeof(*ix));
	lsh_index_init(ix);
	return (ix);
}

void	refd_lsh_update(void *ix, void *c, const float *key, int dim, int pos)
{
	lsh_update((t_lsh_index *)ix, (t_lsh_ctx *)c, key, dim, pos);
}

int	refd_lsh_find(void *ix, int qhash, int *block_ids, int max_blocks)
{
	return (lsh_find_candidates((t_lsh_index *)ix, (uint16_t)qhash,
			block_ids, max_blocks));
}

/* export the index arrays: n_blocks, hashes, starts, lens, heads, next */
int	refd_lsh_index_dump(void *ix, uint16_t *hashes, int *starts, int *lens,
		int *heads, int *next)
{
	t_lsh_index	*x = (t_lsh_index *)ix;

	memcpy(hashes, x->block_hashes, sizeof(x->block_hashes));
	memcpy(starts, x->block_starts, sizeof(x->block_starts));
	memcpy(lens, x->block_lens, sizeof(x->block_lens));
	memcpy(heads, x->bucket_heads, sizeof(x->bucket_heads));
	memcpy(next, x->chain_next, sizeof(x->chain_next));
	return (x->n_blocks);
}

/* ------------------------------------------------------------------ */
/* Paged KV cache on its own (one layer view over a block manager)     */
/* ------------------------------------------------------------------ */
typedef struct s_refd_paged
{
	t_block_manager		bm;
	t_paged_kv_cache	pkv;
	t_block_score		*scores;
}	t_refd_paged;

void	*refd_paged_create(int n_kv_heads, int head_dim, int max_tokens)
{
	t_refd_paged	*p;
	int				mb;

	p = calloc(1, sizeof(*p));
	mb = (max_tokens + KV_BLOCK_SIZE - 1) / KV_BLOCK_SIZE;
	if (block_manager_init(&p->bm, 1, n_kv_heads, head_dim, mb) != 0)
		return (NULL);
	p->pkv.bm = &p->bm;
	p->pkv.layer_idx = 0;
	p->scores = calloc(mb, sizeof(t_block_score));
	return (p);
}

void	refd_paged_append(void *h, const float *k, const float *v, int pos)
{
	t_refd_paged	*p = (t_refd_paged *)h;

	paged_kv_append(&p->pkv, k, v, pos);
}

int	refd_paged_phys(void *h, int lblock)
{
	t_refd_paged	*p = (t_refd_paged *)h;

	return (p->bm.page_table[lblock]);
}

int	refd_paged_nblocks(void *h)
{
	return (((t_refd_paged *)h)->pkv.n_blocks);
}

void	refd_paged_attention(void *h, float *out, const float *q, int n_heads,
		int n_kv_heads, int head_dim)
{
	t_refd_paged	*p = (t_refd_paged *)h;

	op_paged_attention(out, q, &p->pkv, n_heads, n_kv_heads, head_dim,
		1.0f / sqrtf((float)head_dim));
}

/* score_blocks + select_top_k_blocks + op_paged_attention_sparse
** (inference.c:447-489) for one layer; returns n_selected */
int	refd_paged_sparse(void *h, float *out, const float *q, int n_heads,
		int n_kv_heads, int head_dim, int k, int *selected)
{
	t_refd_paged	*p = (t_refd_paged *)h;
	int				n;

	score_blocks(p->scores, q, &p->pkv, p->pkv.n_blocks);
	n = select_top_k_blocks(selected, p->scores, p->pkv.n_blocks, k);
	op_paged_attention_sparse(out, q, &p->bm, selected, n, n_heads,
		n_kv_heads, head_dim, 1.0f / sqrtf((float)head_dim));
	return (n);
}

void	refd_paged_scores(void *h, const float *q, float *out)
{
	t_refd_paged	*p = (t_refd_paged *)h;
	int				i;

	score_blocks(p->scores, q, &p->pkv, p->pkv.n_blocks);
	for (i = 0; i < p->pkv.n_blocks; i++)
		out[i] = p->scores[i].score;
}

/* sparse attention over a linear BF16 cache with an index list
** (op_attention_sparse, ops_attention.c:202) */
void	refd_linear_sparse_attention(float *out, const float *q,
		const uint16_t *k, const uint16_t *v, int kv_len, const int *idx,
		int n_idx, int n_heads, int n_kv_heads, int head_dim)
{
	t_kv_cache			kc;
	t_attention_params	p;

	memset(&kc, 0, sizeof(kc));
	kc.k.data = (void *)k;
	kc.v.data = (void *)v;
	kc.current_seq_len = kv_len;
	kc.num_heads = n_kv_heads;
	kc.head_dim = head_dim;
	memset(&p, 0, sizeof(p));
	p.q = (float *)q;
	p.kv_cache = &kc;
	p.output = out;
	p.n_heads = n_heads;
	p.n_kv_heads = n_kv_heads;
	p.head_dim = head_dim;
	p.scale = 1.0f / sqrtf((float)head_dim);
	p.topk_idx = (int *)idx;
	p.attend_k = n_idx;
	op_attention_sparse(&p);
}
