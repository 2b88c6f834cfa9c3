/*
** Restatement (TEST INFRASTRUCTURE ONLY) of the reference's linear-mode LSH
** sparse attention for ONE query over a linear BF16 KV cache, the isolated
** form of BASELINE configuration 3.  Selection follows inference.c:228-423
** (window of the last `window` positions plus the positions of the LSH units
** found for the mean query that end before the window; ascending; scores =
** sum over KV heads of simd_dot_bf16_f32(K[pos][kv], q[kv * H/KV]); min-heap
** top-K in heap array order, ops_heap.h:40-133), attention follows
** attention_head_sparse (ops_attention.c:131-170) over that order.  The index
** is whatever port_lsh_update built (L tables x b bits x G-token units; the
** reference is L = 1, b = 16, G = 64).  Returns the number of positions
** attended; topk receives them.
*/
#include <stdlib.h>
#include <string.h>

#include "port.h"

static int	cmp_pos(const void *a, const void *b)
{
	return (*(const int *)a - *(const int *)b);
}

int	port_lsh_attend(const t_port_lsh *l, const uint16_t *k, const uint16_t *v,
		int kv_len, const float *q, int n_heads, int n_kv_heads, int head_dim,
		int window, int max_cand, int sparse_k, int *topk, float *out)
{
	int			*cand;
	float		*score;
	int			*units;
	int			nc;
	int			ws;
	int			i;
	int			n;
	float		qm[256];
	uint32_t	qh[16];

	if (!(sparse_k > 0 && kv_len > sparse_k))
	{
		for (i = 0; i < kv_len; i++)
			topk[i] = i;
		port_linear_attention(out, q, k, v, topk, kv_len, n_heads, n_kv_heads,
			head_dim);
		return (kv_len);
	}
	cand = malloc(sizeof(int) * (size_t)kv_len);
	score = malloc(sizeof(float) * (size_t)kv_len);
	units = malloc(sizeof(int) * (size_t)(max_cand > 0 ? max_cand : 1));
	nc = 0;
	ws = (kv_len > window) ? kv_len - window : 0;
	for (i = ws; i < kv_len; i++)
		cand[nc++] = i;
	if (ws > 0 && l->n_units > 0)
	{
		int	d;
		int	h;
		int	u;

		for (d = 0; d < head_dim; d++)
			qm[d] = 0.0f;
		for (h = 0; h < n_heads; h++)
			for (d = 0; d < head_dim; d++)
				qm[d] = qm[d] + q[h * head_dim + d];
		for (d = 0; d < head_dim; d++)
			qm[d] = qm[d] / (float)n_heads;
		for (i = 0; i < l->n_tables; i++)
			qh[i] = port_lsh_hash(l, i, qm);
		n = port_lsh_find(l, qh, units, max_cand);
		for (u = 0; u < n && nc < kv_len; u++)
		{
			int	st = l->unit_start[units[u]];
			int	ln = l->unit_len[units[u]];
			int	p;

			if (st + ln <= ws)
				for (p = 0; p < ln && nc < kv_len; p++)
					if (st + p < ws)
						cand[nc++] = st + p;
		}
	}
	if (nc > 1)
		qsort(cand, nc, sizeof(int), cmp_pos);
	for (i = 0; i < nc; i++)
	{
		float	s = 0.0f;
		int		kvh;

		for (kvh = 0; kvh < n_kv_heads; kvh++)
			s = s + port_dot_bf16_f32(k + ((size_t)cand[i] * n_kv_heads + kvh)
					* head_dim, q + (size_t)kvh * (n_heads / n_kv_heads)
					* head_dim, head_dim);
		score[i] = s;
	}
	n = port_heap_topk(score, cand, nc, nc < sparse_k ? nc : sparse_k, topk);
	port_linear_attention(out, q, k, v, topk, n, n_heads, n_kv_heads, head_dim);
	free(cand);
	free(score);
	free(units);
	return (n);
}
