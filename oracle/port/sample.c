/*
** sample.c -- TEST INFRASTRUCTURE ONLY (oracle).
**
** The reference server's sampling, restated with its float sequence:
**   - repetition penalty over a token history, worker.c:436-442 / 477-490
**     (prompt tokens then generated ones, every occurrence applied);
**   - UNK blocked, worker.c:444 / 492 (logits[0] = -1e9f);
**   - compute_softmax, sampler_topp.c:82-108 (max, expf((l - m) / t)
**     summed in index order in float, then each divided by the sum);
**   - sample_top_p, sampler_topp.c:113-158 (probabilities sorted in
**     descending order, the prefix whose running float sum first exceeds
**     top_p, the draw r * cum and the first running sum above it);
**   - sample_temperature, sampler_temp.c:96-115 with sample_from_probs
**     :74-94 (running sum in index order, the first index with r < cum).
** The draw r is an argument (the reference takes rand() / RAND_MAX for
** top-p and its own LCG for temperature).  The reference sorts with qsort,
** whose order among equal probabilities is unspecified; this restatement
** takes ties in index order.
*/
#include <math.h>
#include <stdlib.h>
#include "port.h"

typedef struct s_pi
{
	float	p;
	int		i;
}	t_pi;

static int	cmp_desc(const void *a, const void *b)
{
	const t_pi	*x = a;
	const t_pi	*y = b;

	if (x->p > y->p)
		return (-1);
	if (x->p < y->p)
		return (1);
	return ((x->i > y->i) - (x->i < y->i));
}

void	port_repetition_penalty(float *logits, const int *hist, int hn,
			float penalty)
{
	for (int j = 0; j < hn; j++)
	{
		if (logits[hist[j]] > 0)
			logits[hist[j]] /= penalty;
		else
			logits[hist[j]] *= penalty;
	}
}

static float	softmax_into(t_pi *pi, const float *l, int n, float t)
{
	float	m = l[0];
	float	sum = 0.0f;

	for (int i = 1; i < n; i++)
		if (l[i] > m)
			m = l[i];
	for (int i = 0; i < n; i++)
	{
		pi[i].p = expf((l[i] - m) / t);
		pi[i].i = i;
		sum += pi[i].p;
	}
	for (int i = 0; i < n; i++)
		pi[i].p /= sum;
	return (sum);
}

/* returns the token; *cut_out / *cum_out / *r_out describe the nucleus and
** the scaled draw, so a test can tell draws that fall within rounding of a
** boundary */
int	port_sample_top_p(float *logits, int n, const int *hist, int hn,
		float temperature, float top_p, float penalty, int block0, float r,
		int *cut_out, float *cum_out)
{
	t_pi	*pi = malloc((size_t)n * sizeof(*pi));
	float	cum = 0.0f;
	float	run = 0.0f;
	int		i = 0;
	int		tok;

	if (hist)
		port_repetition_penalty(logits, hist, hn, penalty);
	if (block0)
		logits[0] = -1e9f;
	softmax_into(pi, logits, n, temperature);
	qsort(pi, (size_t)n, sizeof(*pi), cmp_desc);
	while (i < n)
	{
		cum += pi[i].p;
		i++;
		if (cum > top_p)
			break ;
	}
	r = r * cum;
	tok = pi[i - 1].i;
	for (int j = 0; j < i; j++)
	{
		run += pi[j].p;
		if (run > r)
		{
			tok = pi[j].i;
			break ;
		}
	}
	if (cut_out)
		*cut_out = i;
	if (cum_out)
		*cum_out = cum;
	free(pi);
	return (tok);
}

int	port_sample_temperature(const float *logits, int n, float temperature,
		float r)
{
	float	*p = malloc((size_t)n * sizeof(float));
	float	m = -1e9f;
	float	sum = 0.0f;
	float	cum = 0.0f;
	int		idx = 0;

	for (int i = 0; i < n; i++)
		if (logits[i] > m)
			m = logits[i];
	for (int i = 0; i < n; i++)
	{
		p[i] = expf((logits[i] - m) / temperature);
		sum += p[i];
	}
	for (int i = 0; i < n; i++)
		p[i] /= sum;
	while (idx < n)
	{
		cum += p[idx];
		if (r < cum)
			break ;
		idx++;
	}
	free(p);
	return (idx);
}
