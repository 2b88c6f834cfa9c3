/*
** model.c -- TEST INFRASTRUCTURE ONLY (oracle): the decode step of
** transformer_forward (src/inference/inference.c:60-696) restated over
** INT8 (per-row scale) or FP8-E4M3 (per-tensor scale) weights, in both KV
** modes: paged INT8 (default, use_paged_kv = 1, src/inference/model.c:506)
** and linear BF16 with LSH-routed sparse attention (use_paged_kv = 0).
** The final adapter, logit bias and context bias of the reference are
** zero-initialised no-ops at inference (model.c:447-489) and are omitted.
*/
#include "port.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct s_port_model
{
	t_port_config	c;
	t_port_weights	w;
	float			*x;
	float			*xb;
	float			*q;
	float			*k;
	float			*v;
	float			*hb;
	float			*hb2;
	float			*logits;
	float			*cos_t;
	float			*sin_t;
	t_port_paged	**paged;
	uint16_t		**lin_k;
	uint16_t		**lin_v;
	int				*lin_len;
	t_port_lsh		*lsh;
	int				*cand;
	float			*cand_score;
	int				*topk;
	float			*blk_score;
	int				*sel;
	unsigned long long	queries;
	unsigned long long	used_k;
}	t_port_model;

static void	gemv(const t_port_model *m, float *out, int layer, int which,
				const float *x, int rows, int cols)
{
	const void	*mat;
	const float	*sc;

	if (layer < 0)
	{
		mat = m->w.lm;
		sc = m->w.lm_scale;
	}
	else
	{
		mat = m->w.mat[layer * 7 + which];
		sc = m->w.mat_scale[layer * 7 + which];
	}
	if (m->c.weight_kind == 0)
		port_gemv_q8(out, (const int8_t *)mat, sc, x, rows, cols);
	else
		port_gemv_fp8(out, (const uint8_t *)mat, sc[0], x, rows, cols);
}

void	*port_model_create(const t_port_config *c, const t_port_weights *w)
{
	t_port_model	*m;
	int				i;
	int				qd;
	int				kvd;
	int				half;

	m = calloc(1, sizeof(*m));
	m->c = *c;
	m->w = *w;
	qd = c->n_heads * c->head_dim;
	kvd = c->n_kv_heads * c->head_dim;
	m->x = calloc(c->dim, sizeof(float));
	m->xb = calloc(c->dim, sizeof(float));
	m->q = calloc(qd, sizeof(float));
	m->k = calloc(kvd, sizeof(float));
	m->v = calloc(kvd, sizeof(float));
	m->hb = calloc((c->hidden_dim > qd ? c->hidden_dim : qd), sizeof(float));
	m->hb2 = calloc(c->hidden_dim, sizeof(float));
	m->logits = calloc(c->vocab_size, sizeof(float));
	half = c->head_dim / 2;
	m->cos_t = malloc(sizeof(float) * (size_t)c->seq_len * half);
	m->sin_t = malloc(sizeof(float) * (size_t)c->seq_len * half);
	port_rope_tables(m->cos_t, m->sin_t, c->head_dim, c->seq_len,
		c->rope_theta);
	if (c->use_paged_kv)
	{
		m->paged = calloc(c->n_layers, sizeof(*m->paged));
		for (i = 0; i < c->n_layers; i++)
			m->paged[i] = port_paged_create(c->n_kv_heads, c->head_dim,
					c->seq_len);
		m->blk_score = calloc(c->seq_len / PORT_KV_BLOCK + 1, sizeof(float));
		m->sel = calloc(c->sparse_blocks_k + 2, sizeof(int));
	}
	else
	{
		m->lin_k = calloc(c->n_layers, sizeof(*m->lin_k));
		m->lin_v = calloc(c->n_layers, sizeof(*m->lin_v));
		m->lin_len = calloc(c->n_layers, sizeof(int));
		for (i = 0; i < c->n_layers; i++)
		{
			m->lin_k[i] = calloc((size_t)c->seq_len * kvd, sizeof(uint16_t));
			m->lin_v[i] = calloc((size_t)c->seq_len * kvd, sizeof(uint16_t));
		}
	}
	m->cand = calloc(c->seq_len, sizeof(int));
	m->cand_score = calloc(c->seq_len, sizeof(float));
	m->topk = calloc(c->seq_len, sizeof(int));
	m->lsh = port_lsh_create(c->lsh_tables, c->lsh_bits, c->head_dim,
			c->lsh_unit, c->lsh_max_units, c->lsh_radius, 42);
	return (m);
}

void	port_model_free(void *p)
{
	t_port_model	*m = p;
	int				i;

	if (!m)
		return ;
	for (i = 0; i < m->c.n_layers; i++)
	{
		if (m->paged)
			port_paged_free(m->paged[i]);
		if (m->lin_k)
		{
			free(m->lin_k[i]);
			free(m->lin_v[i]);
		}
	}
	free(m->paged);
	free(m->lin_k);
	free(m->lin_v);
	free(m->lin_len);
	free(m->x);
	free(m->xb);
	free(m->q);
	free(m->k);
	free(m->v);
	free(m->hb);
	free(m->hb2);
	free(m->logits);
	free(m->cos_t);
	free(m->sin_t);
	free(m->cand);
	free(m->cand_score);
	free(m->topk);
	free(m->blk_score);
	free(m->sel);
	port_lsh_free(m->lsh);
	free(m);
}

void	port_model_reset(void *p)
{
	t_port_model	*m = p;
	int				i;

	for (i = 0; i < m->c.n_layers; i++)
	{
		if (m->paged)
			port_paged_reset(m->paged[i]);
		if (m->lin_len)
			m->lin_len[i] = 0;
	}
	port_lsh_reset(m->lsh);
	m->queries = 0;
	m->used_k = 0;
}

static int	cmp_int(const void *a, const void *b)
{
	return (*(const int *)a - *(const int *)b);
}

/*
** Linear-mode candidate selection, inference.c:228-423: sliding window of
** the last `window` positions, plus the positions of LSH units found with
** the mean query that end before the window; sorted ascending; scored with
** sum over KV heads of bf16-key . (first query head of the group); then the
** min-heap top-K in heap order.  Returns attend_k, or -1 for dense.
*/
static int	linear_select(t_port_model *m, int layer, int kv_len)
{
	const t_port_config	*c = &m->c;
	int					nc;
	int					ws;
	int					i;
	int					h;
	int					d;
	int					u;
	int					p;
	int					kvh;
	float				s;
	float				qm[256];
	uint32_t			qh[16];
	int					units[4096];
	int					nu;
	int					kvd;

	nc = 0;
	ws = (kv_len > c->window) ? kv_len - c->window : 0;
	for (i = ws; i < kv_len; i++)
		m->cand[nc++] = i;
	if (ws > 0 && m->lsh->n_units > 0)
	{
		for (d = 0; d < c->head_dim; d++)
			qm[d] = 0.0f;
		for (h = 0; h < c->n_heads; h++)
			for (d = 0; d < c->head_dim; d++)
				qm[d] = qm[d] + m->q[h * c->head_dim + d];
		for (d = 0; d < c->head_dim; d++)
			qm[d] = qm[d] / (float)c->n_heads;
		for (i = 0; i < c->lsh_tables; i++)
			qh[i] = port_lsh_hash(m->lsh, i, qm);
		nu = port_lsh_find(m->lsh, qh, units, c->lsh_max_cand);
		for (u = 0; u < nu && nc < kv_len; u++)
		{
			int	st = m->lsh->unit_start[units[u]];
			int	ln = m->lsh->unit_len[units[u]];

			if (st + ln <= ws)
				for (p = 0; p < ln && nc < kv_len; p++)
					if (st + p < ws)
						m->cand[nc++] = st + p;
		}
	}
	if (nc > 1)
		qsort(m->cand, nc, sizeof(int), cmp_int);
	kvd = c->n_kv_heads * c->head_dim;
	for (i = 0; i < nc; i++)
	{
		s = 0.0f;
		for (kvh = 0; kvh < c->n_kv_heads; kvh++)
			s = s + port_dot_bf16_f32(m->lin_k[layer]
					+ (size_t)m->cand[i] * kvd + kvh * c->head_dim,
					m->q + (size_t)kvh * (c->n_heads / c->n_kv_heads)
					* c->head_dim, c->head_dim);
		m->cand_score[i] = s;
	}
	m->queries++;
	i = port_heap_topk(m->cand_score, m->cand, nc,
			nc < c->sparse_k ? nc : c->sparse_k, m->topk);
	m->used_k += (unsigned long long)i;
	return (i);
}

static void	attention(t_port_model *m, int layer)
{
	const t_port_config	*c = &m->c;
	int					n;
	int					i;
	int					kv_len;
	int					ak;

	if (c->use_paged_kv)
	{
		t_port_paged	*p = m->paged[layer];

		n = p->n_blocks;
		if (n > c->sparse_blocks_k)
		{
			port_paged_scores(p, m->q, m->blk_score);
			i = port_select_blocks(m->blk_score, n, c->sparse_blocks_k, m->sel);
			port_paged_attention(m->hb, m->q, p, m->sel, i, c->n_heads);
		}
		else
		{
			for (i = 0; i < n; i++)
				m->topk[i] = i;
			port_paged_attention(m->hb, m->q, p, m->topk, n, c->n_heads);
		}
		return ;
	}
	kv_len = m->lin_len[layer];
	ak = -1;
	if (c->sparse_k > 0 && kv_len > c->sparse_k)
		ak = linear_select(m, layer, kv_len);
	if (ak > 0 && ak < kv_len)
		port_linear_attention(m->hb, m->q, m->lin_k[layer], m->lin_v[layer],
			m->topk, ak, c->n_heads, c->n_kv_heads, c->head_dim);
	else
	{
		for (i = 0; i < kv_len; i++)
			m->topk[i] = i;
		port_linear_attention(m->hb, m->q, m->lin_k[layer], m->lin_v[layer],
			m->topk, kv_len, c->n_heads, c->n_kv_heads, c->head_dim);
	}
}

const float	*port_model_forward(void *p, int token, int pos)
{
	t_port_model		*m = p;
	const t_port_config	*c = &m->c;
	int					i;
	int					d;
	int					qd;
	int					kvd;

	qd = c->n_heads * c->head_dim;
	kvd = c->n_kv_heads * c->head_dim;
	for (d = 0; d < c->dim; d++)
		m->x[d] = port_bf16_to_f32(m->w.emb[(size_t)token * c->dim + d]);
	for (i = 0; i < c->n_layers; i++)
	{
		port_rmsnorm(m->xb, m->x, m->w.norm[i * 2], c->dim, c->norm_eps);
		gemv(m, m->q, i, 0, m->xb, qd, c->dim);
		gemv(m, m->k, i, 1, m->xb, kvd, c->dim);
		gemv(m, m->v, i, 2, m->xb, kvd, c->dim);
		port_rope(m->q, c->n_heads, c->head_dim, pos, m->cos_t, m->sin_t,
			c->seq_len);
		port_rope(m->k, c->n_kv_heads, c->head_dim, pos, m->cos_t, m->sin_t,
			c->seq_len);
		if (c->use_paged_kv)
			port_paged_append(m->paged[i], m->k, m->v, pos);
		else if (m->lin_len[i] < c->seq_len)
		{
			for (d = 0; d < kvd; d++)
			{
				m->lin_k[i][(size_t)m->lin_len[i] * kvd + d]
					= port_f32_to_bf16(m->k[d]);
				m->lin_v[i][(size_t)m->lin_len[i] * kvd + d]
					= port_f32_to_bf16(m->v[d]);
			}
			m->lin_len[i]++;
		}
		if (i == 0)
			port_lsh_update(m->lsh, m->k, pos);
		attention(m, i);
		gemv(m, m->xb, i, 3, m->hb, c->dim, qd);
		for (d = 0; d < c->dim; d++)
			m->x[d] = m->x[d] + m->xb[d];
		port_rmsnorm(m->xb, m->x, m->w.norm[i * 2 + 1], c->dim, c->norm_eps);
		gemv(m, m->hb, i, 4, m->xb, c->hidden_dim, c->dim);
		gemv(m, m->hb2, i, 6, m->xb, c->hidden_dim, c->dim);
		port_silu_mul(m->hb, m->hb, m->hb2, c->hidden_dim);
		gemv(m, m->xb, i, 5, m->hb, c->dim, c->hidden_dim);
		for (d = 0; d < c->dim; d++)
			m->x[d] = m->x[d] + m->xb[d];
	}
	port_rmsnorm(m->x, m->x, m->w.final_norm, c->dim, c->norm_eps);
	gemv(m, m->logits, -1, 0, m->x, c->vocab_size, c->dim);
	return (m->logits);
}

const float	*port_model_state(void *p, int which)
{
	t_port_model	*m = p;

	switch (which)
	{
		case 0: return (m->x);
		case 1: return (m->xb);
		case 2: return (m->q);
		case 3: return (m->k);
		case 4: return (m->v);
		case 5: return (m->hb);
		case 6: return (m->logits);
	}
	return (NULL);
}

const t_port_lsh	*port_model_lsh(void *p)
{
	return (((t_port_model *)p)->lsh);
}

const t_port_paged	*port_model_paged(void *p, int layer)
{
	t_port_model	*m = p;

	return (m->paged ? m->paged[layer] : NULL);
}

const uint16_t	*port_model_linear_k(void *p, int layer)
{
	t_port_model	*m = p;

	return (m->lin_k ? m->lin_k[layer] : NULL);
}

void	port_model_counters(void *p, unsigned long long *out)
{
	out[0] = ((t_port_model *)p)->queries;
	out[1] = ((t_port_model *)p)->used_k;
}
