/*
** kv.c -- TEST INFRASTRUCTURE ONLY (oracle): restated paged INT8 KV cache,
** block-centroid routing, online-softmax attention and the LSH index.
*/
#include "port.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* paged INT8 KV (src/memory/paged.c, one layer)                             */
/* ------------------------------------------------------------------------ */

t_port_paged	*port_paged_create(int n_kv_heads, int head_dim, int max_tokens)
{
	t_port_paged	*p;
	size_t			nb;

	p = calloc(1, sizeof(*p));
	p->n_kv_heads = n_kv_heads;
	p->head_dim = head_dim;
	p->max_blocks = (max_tokens + PORT_KV_BLOCK - 1) / PORT_KV_BLOCK;
	nb = (size_t)p->max_blocks;
	p->k = calloc(nb * n_kv_heads * PORT_KV_BLOCK * head_dim, 1);
	p->v = calloc(nb * n_kv_heads * PORT_KV_BLOCK * head_dim, 1);
	p->ks = calloc(nb * n_kv_heads * PORT_KV_BLOCK, sizeof(float));
	p->vs = calloc(nb * n_kv_heads * PORT_KV_BLOCK, sizeof(float));
	p->centroid = calloc(nb * head_dim, sizeof(float));
	p->fill = calloc(nb, sizeof(int));
	return (p);
}

void	port_paged_free(t_port_paged *p)
{
	if (!p)
		return ;
	free(p->k);
	free(p->v);
	free(p->ks);
	free(p->vs);
	free(p->centroid);
	free(p->fill);
	free(p);
}

void	port_paged_reset(t_port_paged *p)
{
	size_t	nb;

	nb = (size_t)p->max_blocks;
	memset(p->centroid, 0, nb * p->head_dim * sizeof(float));
	memset(p->fill, 0, nb * sizeof(int));
	p->n_blocks = 0;
	p->n_tokens = 0;
}

/* calc_block_centroid_int8, src/memory/paged.c:350-393 (KV head 0) */
static void	centroid(t_port_paged *p, int b)
{
	const int8_t	*kq;
	const float		*ks;
	float			*c;
	float			inv;
	int				t;
	int				d;
	int				hd;

	hd = p->head_dim;
	kq = p->k + (size_t)b * p->n_kv_heads * PORT_KV_BLOCK * hd;
	ks = p->ks + (size_t)b * p->n_kv_heads * PORT_KV_BLOCK;
	c = p->centroid + (size_t)b * hd;
	for (d = 0; d < hd; d++)
		c[d] = 0.0f;
	for (t = 0; t < p->fill[b]; t++)
		for (d = 0; d < hd; d++)
			c[d] = c[d] + (float)kq[t * hd + d] * ks[t];
	inv = 1.0f / (float)p->fill[b];
	for (d = 0; d < hd; d++)
		c[d] = c[d] * inv;
}

/* paged_kv_append, src/memory/paged.c:195-272 */
void	port_paged_append(t_port_paged *p, const float *k, const float *v,
			int pos)
{
	int		b;
	int		off;
	int		h;
	int		hd;
	size_t	base;

	b = pos / PORT_KV_BLOCK;
	off = pos % PORT_KV_BLOCK;
	hd = p->head_dim;
	if (b >= p->n_blocks)
		p->n_blocks = b + 1;
	for (h = 0; h < p->n_kv_heads; h++)
	{
		base = ((size_t)b * p->n_kv_heads + h) * PORT_KV_BLOCK + off;
		p->ks[base] = port_quant_int8(p->k + base * hd, k + (size_t)h * hd, hd);
		p->vs[base] = port_quant_int8(p->v + base * hd, v + (size_t)h * hd, hd);
	}
	p->fill[b] = off + 1;
	p->n_tokens = pos + 1;
	if (p->fill[b] == PORT_KV_BLOCK)
		centroid(p, b);
}

/*
** One head over one block: attention_block_int8,
** src/compute/ops_attention.c:292-348.  The running-sum update
** `sum * sf + re` is contracted to one FMA in the reference build.
*/
static void	attend_block(float *out, const float *q, const t_port_paged *p,
			int b, int kvh, float scale, float *mx, float *sum)
{
	const int8_t	*kq;
	const int8_t	*vq;
	const float		*ks;
	const float		*vs;
	float			kb[256];
	float			vb[256];
	int				t;
	int				d;
	int				hd;
	float			s;
	float			prev;
	float			sf;
	float			re;

	hd = p->head_dim;
	kq = p->k + (((size_t)b * p->n_kv_heads + kvh) * PORT_KV_BLOCK) * hd;
	vq = p->v + (((size_t)b * p->n_kv_heads + kvh) * PORT_KV_BLOCK) * hd;
	ks = p->ks + ((size_t)b * p->n_kv_heads + kvh) * PORT_KV_BLOCK;
	vs = p->vs + ((size_t)b * p->n_kv_heads + kvh) * PORT_KV_BLOCK;
	for (t = 0; t < p->fill[b]; t++)
	{
		for (d = 0; d < hd; d++)
		{
			kb[d] = (float)kq[t * hd + d] * ks[t];
			vb[d] = (float)vq[t * hd + d] * vs[t];
		}
		s = port_dot_f32(q, kb, hd) * scale;
		prev = *mx;
		if (s > prev)
			*mx = s;
		sf = port_fast_expf(prev - *mx);
		re = port_fast_expf(s - *mx);
		*sum = fmaf(*sum, sf, re);
		for (d = 0; d < hd; d++)
			out[d] = fmaf(re, vb[d], out[d] * sf);
	}
}

/*
** op_paged_attention / op_paged_attention_sparse
** (src/compute/ops_attention.c:354-461): per query head h, KV head
** h / (H / KV), blocks in the order given (logical block ids here).
*/
void	port_paged_attention(float *out, const float *q, const t_port_paged *p,
			const int *blocks, int n_sel, int n_heads)
{
	int		h;
	int		i;
	int		d;
	int		hd;
	float	mx;
	float	sum;
	float	scale;
	float	inv;

	hd = p->head_dim;
	scale = 1.0f / sqrtf((float)hd);
	for (h = 0; h < n_heads; h++)
	{
		float	*o = out + (size_t)h * hd;

		mx = -INFINITY;
		sum = 0.0f;
		for (d = 0; d < hd; d++)
			o[d] = 0.0f;
		for (i = 0; i < n_sel; i++)
			if (blocks[i] >= 0)
				attend_block(o, q + (size_t)h * hd, p, blocks[i],
					h / (n_heads / p->n_kv_heads), scale, &mx, &sum);
		if (sum > 0.0f)
		{
			inv = 1.0f / sum;
			for (d = 0; d < hd; d++)
				o[d] = o[d] * inv;
		}
	}
}

/* score_blocks, src/memory/paged.c:401-431 (query head 0 . centroid) */
void	port_paged_scores(const t_port_paged *p, const float *q, float *scores)
{
	int	b;

	for (b = 0; b < p->n_blocks; b++)
		scores[b] = port_dot_f32(q, p->centroid + (size_t)b * p->head_dim,
				p->head_dim);
}

/* select_top_k_blocks, src/memory/paged.c:439-495 */
int	port_select_blocks(const float *scores, int n_blocks, int k, int *selected)
{
	int	n;
	int	ak;
	int	*ids;
	int	m;
	int	i;

	if (n_blocks <= 0)
		return (0);
	selected[0] = 0;
	n = 1;
	if (n_blocks > 1)
		selected[n++] = n_blocks - 1;
	if (n_blocks <= 2 || k <= 2)
		return (n);
	ak = k - 2;
	if (ak > n_blocks - 2)
		ak = n_blocks - 2;
	if (ak > 62)
		ak = 62;
	ids = malloc(sizeof(int) * n_blocks);
	for (i = 1; i < n_blocks - 1; i++)
		ids[i - 1] = i;
	m = port_heap_topk(scores + 1, ids, n_blocks - 2, ak, selected + n);
	free(ids);
	return (n + m);
}

/* ------------------------------------------------------------------------ */
/* linear BF16 KV (attention_head_sparse, src/compute/ops_attention.c:131)  */
/* ------------------------------------------------------------------------ */
void	port_linear_attention(float *out, const float *q, const uint16_t *k,
			const uint16_t *v, const int *idx, int n_idx, int n_heads,
			int n_kv_heads, int head_dim)
{
	int		h;
	int		i;
	int		d;
	int		kvh;
	int		stride;
	float	mx;
	float	sum;
	float	s;
	float	prev;
	float	sf;
	float	re;
	float	scale;
	float	inv;

	stride = n_kv_heads * head_dim;
	scale = 1.0f / sqrtf((float)head_dim);
	for (h = 0; h < n_heads; h++)
	{
		float			*o = out + (size_t)h * head_dim;
		const float		*qh = q + (size_t)h * head_dim;

		kvh = h / (n_heads / n_kv_heads);
		mx = -INFINITY;
		sum = 0.0f;
		for (d = 0; d < head_dim; d++)
			o[d] = 0.0f;
		for (i = 0; i < n_idx; i++)
		{
			const uint16_t	*kr = k + (size_t)idx[i] * stride + kvh * head_dim;
			const uint16_t	*vr = v + (size_t)idx[i] * stride + kvh * head_dim;

			s = port_dot_bf16_f32(kr, qh, head_dim) * scale;
			prev = mx;
			mx = (s > prev) ? s : prev;
			sf = port_fast_expf(prev - mx);
			re = port_fast_expf(s - mx);
			sum = fmaf(sum, sf, re);
			for (d = 0; d < head_dim; d++)
				o[d] = fmaf(re, port_bf16_to_f32(vr[d]), o[d] * sf);
		}
		if (sum > 0.0f)
		{
			inv = 1.0f / sum;
			for (d = 0; d < head_dim; d++)
				o[d] = o[d] * inv;
		}
	}
}

/* ------------------------------------------------------------------------ */
/* LSH: L tables x b bits over G-token units (src/compute/ops_lsh.c)        */
/* With L = 1, b = 16, G = 64 this is the reference's index exactly.        */
/* ------------------------------------------------------------------------ */

/* rand_gaussian, src/compute/ops_lsh.c:22-34: LCG + Box-Muller */
static float	rand_gaussian(unsigned int *seed)
{
	float	u1;
	float	u2;

	*seed = *seed * 1103515245u + 12345u;
	u1 = (float)((*seed >> 16) & 0x7FFF) / 32767.0f;
	*seed = *seed * 1103515245u + 12345u;
	u2 = (float)((*seed >> 16) & 0x7FFF) / 32767.0f;
	if (u1 < 1e-6f)
		u1 = 1e-6f;
	return (sqrtf(-2.0f * logf(u1)) * cosf(2.0f * 3.14159265f * u2));
}

/*
** lsh_init, src/compute/ops_lsh.c:40-85; table t uses seed + t.
** The squared-norm accumulation is a separate multiply and add (not fused)
** in the reference build.
*/
t_port_lsh	*port_lsh_create(int n_tables, int n_bits, int dim, int unit,
				int max_units, int radius, unsigned int seed)
{
	t_port_lsh		*l;
	int				t;
	int				h;
	int				d;
	unsigned int	s;
	float			norm;
	float			*hp;

	l = calloc(1, sizeof(*l));
	l->n_tables = n_tables;
	l->n_bits = n_bits;
	l->dim = dim;
	l->unit = unit;
	l->max_units = max_units;
	l->radius = radius;
	l->hp = calloc((size_t)n_tables * n_bits * dim, sizeof(float));
	l->unit_hash = calloc((size_t)n_tables * max_units, sizeof(uint32_t));
	l->unit_start = calloc(max_units, sizeof(int));
	l->unit_len = calloc(max_units, sizeof(int));
	l->heads = malloc(sizeof(int) * ((size_t)n_tables << n_bits));
	l->next = calloc((size_t)n_tables * max_units, sizeof(int));
	l->acc = calloc(dim, sizeof(float));
	for (t = 0; t < n_tables; t++)
	{
		s = seed + (unsigned int)t;
		for (h = 0; h < n_bits; h++)
		{
			hp = l->hp + ((size_t)t * n_bits + h) * dim;
			norm = 0.0f;
			for (d = 0; d < dim; d++)
			{
				hp[d] = rand_gaussian(&s);
				norm = norm + hp[d] * hp[d];
			}
			norm = sqrtf(norm);
			if (norm > 1e-6f)
				for (d = 0; d < dim; d++)
					hp[d] = hp[d] / norm;
		}
	}
	port_lsh_reset(l);
	return (l);
}

void	port_lsh_free(t_port_lsh *l)
{
	if (!l)
		return ;
	free(l->hp);
	free(l->unit_hash);
	free(l->unit_start);
	free(l->unit_len);
	free(l->heads);
	free(l->next);
	free(l->acc);
	free(l);
}

/* lsh_index_init, src/compute/ops_lsh.c:90-104 */
void	port_lsh_reset(t_port_lsh *l)
{
	size_t	i;

	for (i = 0; i < ((size_t)l->n_tables << l->n_bits); i++)
		l->heads[i] = -1;
	memset(l->acc, 0, sizeof(float) * l->dim);
	l->n_units = 0;
	l->acc_count = 0;
	l->acc_start = 0;
}

/* lsh_hash, src/compute/ops_lsh.c:138-242: bit h = (in-order FMA chain) > 0 */
uint32_t	port_lsh_hash(const t_port_lsh *l, int table, const float *v)
{
	uint32_t	code;
	int			h;
	int			d;
	float		a;
	const float	*hp;

	code = 0;
	for (h = 0; h < l->n_bits; h++)
	{
		hp = l->hp + ((size_t)table * l->n_bits + h) * l->dim;
		a = 0.0f;
		for (d = 0; d < l->dim; d++)
			a = fmaf(v[d], hp[d], a);
		if (a > 0.0f)
			code |= 1u << h;
	}
	return (code);
}

/* lsh_update + lsh_insert_block, src/compute/ops_lsh.c:256-349 */
void	port_lsh_update(t_port_lsh *l, const float *key, int pos)
{
	int		d;
	int		t;
	int		id;
	float	sc;
	uint32_t	code;

	if (l->acc_count == 0)
		l->acc_start = pos;
	for (d = 0; d < l->dim; d++)
		l->acc[d] = l->acc[d] + key[d];
	l->acc_count++;
	if (l->acc_count < l->unit)
		return ;
	sc = 1.0f / (float)l->acc_count;
	for (d = 0; d < l->dim; d++)
		l->acc[d] = l->acc[d] * sc;
	if (l->n_units < l->max_units)
	{
		id = l->n_units;
		l->unit_start[id] = l->acc_start;
		l->unit_len[id] = l->acc_count;
		for (t = 0; t < l->n_tables; t++)
		{
			code = port_lsh_hash(l, t, l->acc);
			l->unit_hash[(size_t)t * l->max_units + id] = code;
			l->next[(size_t)t * l->max_units + id]
				= l->heads[((size_t)t << l->n_bits) + code];
			l->heads[((size_t)t << l->n_bits) + code] = id;
		}
		l->n_units++;
	}
	memset(l->acc, 0, sizeof(float) * l->dim);
	l->acc_count = 0;
}

/*
** lsh_find_candidates, src/compute/ops_lsh.c:361-418, table by table:
** probe 0 = the query code, probe p = code with bit p-1 flipped; walk each
** bucket chain newest first; keep units within the Hamming radius that were
** not seen before; stop at max_units.
*/
int	port_lsh_find(const t_port_lsh *l, const uint32_t *qhash, int *unit_ids,
		int max_units)
{
	unsigned char	*seen;
	int				n;
	int				t;
	int				p;
	int				id;
	uint32_t		probe;
	uint32_t		hh;

	seen = calloc(l->max_units, 1);
	n = 0;
	for (t = 0; t < l->n_tables && n < max_units; t++)
		for (p = 0; p <= l->n_bits && n < max_units; p++)
		{
			probe = (p == 0) ? qhash[t] : (qhash[t] ^ (1u << (p - 1)));
			id = l->heads[((size_t)t << l->n_bits) + probe];
			while (id != -1 && n < max_units)
			{
				hh = l->unit_hash[(size_t)t * l->max_units + id];
				if (__builtin_popcount(qhash[t] ^ hh) <= l->radius && !seen[id])
				{
					seen[id] = 1;
					unit_ids[n++] = id;
				}
				id = l->next[(size_t)t * l->max_units + id];
			}
		}
	free(seen);
	return (n);
}
