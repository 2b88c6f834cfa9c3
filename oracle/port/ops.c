/*
** ops.c -- TEST INFRASTRUCTURE ONLY (oracle): restated reference ops.
**
** Built with -ffp-contract=off: every fused multiply-add below is an explicit
** fmaf(), placed exactly where the reference's AVX2 intrinsics (or gcc's
** contraction of its scalar C under -O3 -mfma) fuse.  The placement of the
** compiler-contracted ones was established by input/output comparison with
** the reference build (the golden vectors that tests/golden/make_golden.py
** writes from oracle/_ref, checked by tests/test_golden.py), not by reading
** its generated code.
*/
#include "port.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

float	port_bf16_to_f32(uint16_t b)
{
	uint32_t	u;
	float		f;

	u = (uint32_t)b << 16;
	memcpy(&f, &u, 4);
	return (f);
}

/* round-to-nearest-even on the bit pattern (src/tensor/tensor.c:67-76) */
uint16_t	port_f32_to_bf16(float f)
{
	uint32_t	u;

	memcpy(&u, &f, 4);
	u += 0x7FFFu + ((u >> 16) & 1u);
	return ((uint16_t)(u >> 16));
}

/*
** Schraudolph's exponential (N. Schraudolph, "A fast, compact approximation
** of the exponential function", Neural Computation 11(4), 1999), scalar form
** of src/compute/ops_math_fast.h:48-64: inputs below -87 give 0, inputs above
** 87 are clamped, then the integer (2^23/ln2) * x + (127 << 23), truncated
** toward zero, is read as a float bit pattern.  The reference's scalar
** expression is contracted to one FMA.
*/
float	port_fast_expf(float x)
{
	int32_t	i;
	float	f;

	if (x < -87.0f)
		return (0.0f);
	if (x > 87.0f)
		x = 87.0f;
	i = (int32_t)fmaf(12102203.0f, x, 1065353216.0f);
	memcpy(&f, &i, 4);
	return (f);
}

/*
** Vector form of the same method (ops_math_fast.h:105-126): clamp with
** max/min (a NaN input takes the clamp value), one FMA, then conversion with
** round-to-nearest-even.
*/
float	port_fast_expf_vec(float x)
{
	int32_t	i;
	float	f;

	x = (x > -87.0f) ? x : -87.0f;
	x = (x < 87.0f) ? x : 87.0f;
	i = (int32_t)nearbyintf(fmaf(x, 12102203.0f, 1065353216.0f));
	memcpy(&f, &i, 4);
	return (f);
}

/*
** E4M3 decode as the reference defines it (src/compute/ops_quant.c:27-50):
** exponent field 0 -> mant/8 * 2^-6, else (1 + mant/8) * 2^(exp-7); there is
** no NaN code (0x7F decodes to 480).
*/
float	port_fp8_e4m3_to_f32(uint8_t code)
{
	int		e;
	int		m;
	float	v;

	e = (code >> 3) & 0xF;
	m = code & 7;
	if (e == 0)
		v = ldexpf((float)m / 8.0f, -6);
	else
		v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
	return ((code & 0x80) ? -v : v);
}

/* ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)): simd_hsum_ps,
** src/compute/simd_kernels.h:57-68 */
static float	hsum8(const float *v)
{
	float	a;
	float	b;

	a = (v[0] + v[4]) + (v[1] + v[5]);
	b = (v[2] + v[6]) + (v[3] + v[7]);
	return (a + b);
}

/* simd_dot_f32_f32, simd_kernels.h:162-191 */
float	port_dot_f32(const float *a, const float *b, int n)
{
	float	acc[8];
	float	s;
	int		i;
	int		l;

	for (l = 0; l < 8; l++)
		acc[l] = 0.0f;
	for (i = 0; i + 7 < n; i += 8)
		for (l = 0; l < 8; l++)
			acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
	s = hsum8(acc);
	for (; i < n; i++)
		s = fmaf(a[i], b[i], s);
	return (s);
}

/* simd_dot_bf16_f32 with AVX-512 off, simd_kernels.h:97-156 */
float	port_dot_bf16_f32(const uint16_t *a, const float *b, int n)
{
	float	acc[8];
	float	s;
	int		i;
	int		l;

	for (l = 0; l < 8; l++)
		acc[l] = 0.0f;
	for (i = 0; i + 7 < n; i += 8)
		for (l = 0; l < 8; l++)
			acc[l] = fmaf(port_bf16_to_f32(a[i + l]), b[i + l], acc[l]);
	s = 0.0f + hsum8(acc);
	for (; i < n; i++)
		s = fmaf(port_bf16_to_f32(a[i]), b[i], s);
	return (s);
}

/*
** One GEMV row in the order of matvec_bf16_f32_blocked
** (src/compute/ops_matmul.c:57-141): 32 lanes in 4 groups of 8; lane L
** accumulates elements j == L (mod 32) with one FMA each, in increasing j;
** an 8-wide cleanup loop adds into group 0; groups combine as
** (g0+g1)+(g2+g3); then the 8-lane horizontal sum; then a scalar tail.
*/
#define ROW_BODY(DECODE) \
	float	g[4][8]; \
	float	c[8]; \
	float	s; \
	int		j; \
	int		l; \
	int		q; \
	for (q = 0; q < 4; q++) \
		for (l = 0; l < 8; l++) \
			g[q][l] = 0.0f; \
	for (j = 0; j + 31 < k; j += 32) \
		for (q = 0; q < 4; q++) \
			for (l = 0; l < 8; l++) \
				g[q][l] = fmaf(DECODE(row[j + 8 * q + l]), x[j + 8 * q + l], \
					g[q][l]); \
	for (; j + 7 < k; j += 8) \
		for (l = 0; l < 8; l++) \
			g[0][l] = fmaf(DECODE(row[j + l]), x[j + l], g[0][l]); \
	for (l = 0; l < 8; l++) \
		c[l] = (g[0][l] + g[1][l]) + (g[2][l] + g[3][l]); \
	s = hsum8(c); \
	for (; j < k; j++) \
		s = fmaf(DECODE(row[j]), x[j], s);

#define DEC_BF16(v) port_bf16_to_f32(v)
#define DEC_I8(v) ((float)(v))
#define DEC_FP8(v) port_fp8_e4m3_to_f32(v)

static float	row_bf16(const uint16_t *row, const float *x, int k)
{
	ROW_BODY(DEC_BF16)
	return (s);
}

static float	row_i8(const int8_t *row, const float *x, int k)
{
	ROW_BODY(DEC_I8)
	return (s);
}

static float	row_fp8(const uint8_t *row, const float *x, int k)
{
	ROW_BODY(DEC_FP8)
	return (s);
}

void	port_gemv_bf16(float *out, const uint16_t *w, const float *x, int m,
			int k)
{
	int	i;

	#pragma omp parallel for schedule(static)
	for (i = 0; i < m; i++)
		out[i] = row_bf16(w + (size_t)i * k, x, k);
}

/*
** INT8 weight-only GEMV: y[i] = (row sum of q[i][j] * x[j] in the reference
** lane order) * scale[i].  With power-of-two scales this equals, bit for bit,
** op_matmul on the BF16 matrix q * scale (scaling by 2^e commutes with every
** rounding in the normal range).
*/
void	port_gemv_q8(float *out, const int8_t *w, const float *scale,
			const float *x, int m, int k)
{
	int	i;

	#pragma omp parallel for schedule(static)
	for (i = 0; i < m; i++)
		out[i] = row_i8(w + (size_t)i * k, x, k) * scale[i];
}

void	port_gemv_fp8(float *out, const uint8_t *w, float scale,
			const float *x, int m, int k)
{
	int	i;

	#pragma omp parallel for schedule(static)
	for (i = 0; i < m; i++)
		out[i] = row_fp8(w + (size_t)i * k, x, k) * scale;
}

/* rmsnorm_f32_avx2, src/compute/ops_norm.c:27-124 */
void	port_rmsnorm(float *out, const float *x, const uint16_t *w, int n,
			float eps)
{
	float	acc[8];
	float	ss;
	float	inv;
	int		j;
	int		l;

	for (l = 0; l < 8; l++)
		acc[l] = 0.0f;
	for (j = 0; j + 7 < n; j += 8)
		for (l = 0; l < 8; l++)
			acc[l] = fmaf(x[j + l], x[j + l], acc[l]);
	ss = hsum8(acc);
	for (; j < n; j++)
		ss = fmaf(x[j], x[j], ss);
	ss = ss / (float)n;
	inv = 1.0f / sqrtf(ss + eps);
	for (j = 0; j < n; j++)
		out[j] = (x[j] * inv) * port_bf16_to_f32(w[j]);
}

/* rope_cache_init, src/compute/ops_rope.c:30-96 (host libm) */
void	port_rope_tables(float *cos_t, float *sin_t, int head_dim, int max_seq,
			float theta)
{
	int		half;
	int		i;
	int		p;
	float	*inv;
	float	a;

	half = head_dim / 2;
	inv = malloc(sizeof(float) * half);
	for (i = 0; i < half; i++)
		inv[i] = 1.0f / powf(theta, (float)(i * 2) / (float)head_dim);
	for (p = 0; p < max_seq; p++)
		for (i = 0; i < half; i++)
		{
			a = (float)p * inv[i];
			cos_t[(size_t)p * half + i] = cosf(a);
			sin_t[(size_t)p * half + i] = sinf(a);
		}
	free(inv);
}

/*
** rope_apply_multihead_cached, src/compute/ops_rope.c:192-231: rotate-half
** pairs (i, i + hd/2).  The reference's `v0*c - v1*s` and `v0*s + v1*c`
** compile to fma(v0, c, -(v1*s)) and fma(v0, s, v1*c).
*/
void	port_rope(float *data, int n_heads, int head_dim, int pos,
			const float *cos_t, const float *sin_t, int max_seq)
{
	int			half;
	int			h;
	int			i;
	float		*hd;
	const float	*cr;
	const float	*sr;
	float		v0;
	float		v1;

	if (pos >= max_seq)
		return ;
	half = head_dim / 2;
	cr = cos_t + (size_t)pos * half;
	sr = sin_t + (size_t)pos * half;
	for (h = 0; h < n_heads; h++)
	{
		hd = data + (size_t)h * head_dim;
		for (i = 0; i < half; i++)
		{
			v0 = hd[i];
			v1 = hd[i + half];
			hd[i] = fmaf(v0, cr[i], -(v1 * sr[i]));
			hd[i + half] = fmaf(v0, sr[i], v1 * cr[i]);
		}
	}
}

/* op_silu_mul_fused_f32, src/compute/ops_activation.c:48-102 */
void	port_silu_mul(float *out, const float *g, const float *u, int n)
{
	int		i;
	int		l;
	float	gv;
	float	sig;

	for (i = 0; i + 8 <= n; i += 8)
		for (l = i; l < i + 8; l++)
		{
			gv = g[l];
			sig = 1.0f / (1.0f + port_fast_expf_vec(0.0f - gv));
			out[l] = (gv * sig) * u[l];
		}
	for (; i < n; i++)
	{
		gv = g[i];
		sig = 1.0f / (1.0f + port_fast_expf(-gv));
		out[i] = (gv * sig) * u[i];
	}
}

/* quant_f32_to_int8, src/compute/ops_quant.c:229-273 */
float	port_quant_int8(int8_t *out, const float *in, int n)
{
	float	mx;
	float	scale;
	float	inv;
	int		i;
	int		v;

	mx = 0.0f;
	for (i = 0; i < n; i++)
		if (fabsf(in[i]) > mx)
			mx = fabsf(in[i]);
	if (mx > 0.0f)
	{
		scale = mx / 127.0f;
		inv = 127.0f / mx;
	}
	else
	{
		scale = 1.0f;
		inv = 1.0f;
	}
	for (i = 0; i < n; i++)
	{
		v = (int)roundf(in[i] * inv);
		if (v > 127)
			v = 127;
		if (v < -127)
			v = -127;
		out[i] = (int8_t)v;
	}
	return (scale);
}

/* argmax_simd_f32, src/compute/sampler.c:42-120 */
int	port_argmax(const float *x, int n)
{
	float	bm[8];
	int		bi[8];
	float	best;
	int		idx;
	int		i;
	int		l;

	if (n < 8)
	{
		idx = 0;
		best = x[0];
		for (i = 1; i < n; i++)
			if (x[i] > best)
			{
				best = x[i];
				idx = i;
			}
		return (idx);
	}
	for (l = 0; l < 8; l++)
	{
		bm[l] = x[l];
		bi[l] = l;
	}
	for (i = 8; i + 7 < n; i += 8)
		for (l = 0; l < 8; l++)
			if (x[i + l] > bm[l])
			{
				bm[l] = x[i + l];
				bi[l] = i + l;
			}
	best = bm[0];
	idx = bi[0];
	for (l = 1; l < 8; l++)
		if (bm[l] > best)
		{
			best = bm[l];
			idx = bi[l];
		}
	for (; i < n; i++)
		if (x[i] > best)
		{
			best = x[i];
			idx = i;
		}
	return (idx);
}

/* heap_push / heap_extract_indices, src/compute/ops_heap.h:40-133 */
typedef struct s_item
{
	float	score;
	int		index;
}	t_item;

static void	sift_down(t_item *h, int size, int i)
{
	int		s;
	int		l;
	int		r;
	t_item	t;

	while (1)
	{
		s = i;
		l = 2 * i + 1;
		r = 2 * i + 2;
		if (l < size && h[l].score < h[s].score)
			s = l;
		if (r < size && h[r].score < h[s].score)
			s = r;
		if (s == i)
			break ;
		t = h[i];
		h[i] = h[s];
		h[s] = t;
		i = s;
	}
}

static void	sift_up(t_item *h, int i)
{
	int		p;
	t_item	t;

	while (i > 0)
	{
		p = (i - 1) / 2;
		if (h[p].score <= h[i].score)
			break ;
		t = h[i];
		h[i] = h[p];
		h[p] = t;
		i = p;
	}
}

int	port_heap_topk(const float *scores, const int *idx, int n, int k, int *out)
{
	t_item	*h;
	int		size;
	int		i;

	h = malloc(sizeof(t_item) * (k > 0 ? k : 1));
	size = 0;
	for (i = 0; i < n; i++)
	{
		if (size < k)
		{
			h[size].score = scores[i];
			h[size].index = idx[i];
			sift_up(h, size);
			size++;
		}
		else if (k > 0 && scores[i] > h[0].score)
		{
			h[0].score = scores[i];
			h[0].index = idx[i];
			sift_down(h, size, 0);
		}
	}
	for (i = 0; i < size; i++)
		out[i] = h[i].index;
	free(h);
	return (size);
}
