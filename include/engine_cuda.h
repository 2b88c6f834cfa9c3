/*
** engine_cuda.h -- C ABI of libengine_cuda.so, the B200 (sm_100a) decode hot
** path for fgroo/42-Berlin-Engine.
**
** Plain C: pointers, sizes and status codes; no CUDA, C++ or torch types.
** Streams are passed as `void *` (a cudaStream_t, NULL = legacy default).
** Every function returns EC_OK (0) or a negative EC_ERR_* code; it never
** exits the process.  ec_last_error() gives a human-readable reason.
**
** Two layers:
**   1. The fused decode path (ec_create ... ec_decode_step): one context per
**      t_transformer owns the device copy of the weights (INT8 per-row or
**      FP8-E4M3 per-tensor), the KV cache, the RoPE tables and the LSH index,
**      and runs transformer_forward (src/inference/inference.c:60) for B
**      independent sequences per call.
**   2. Per-op entry points (ec_op_*) on caller-owned device buffers, one per
**      reference op on that path, for hosts that keep their own loop.
** The file:line after each declaration names the reference interface it
** replaces.
*/
#ifndef ENGINE_CUDA_H
# define ENGINE_CUDA_H
# include <stddef.h>
# include <stdint.h>

# ifdef __cplusplus
extern "C" {
# endif

# define EC_OK 0
# define EC_ERR_ARG (-1)          /* bad argument / shape */
# define EC_ERR_CUDA (-2)         /* CUDA runtime error */
# define EC_ERR_OOM (-3)          /* device allocation failed / pool full */
# define EC_ERR_STATE (-4)        /* call out of order (e.g. weights missing) */
# define EC_ERR_UNSUPPORTED (-5)  /* shape or mode this build does not run */
# define EC_ERR_TIMEOUT (-6)      /* a bounded device wait gave up */

/* weight formats */
# define EC_W_INT8 0   /* int8 [rows][cols] + fp32 scale per row */
# define EC_W_FP8 1    /* E4M3 [rows][cols] + one fp32 scale per matrix */
# define EC_W_BF16 2   /* bf16 [rows][cols], no scale (per-op GEMV only) */

/* matrix ids for ec_set_weight (layer >= 0) */
# define EC_WQ 0
# define EC_WK 1
# define EC_WV 2
# define EC_WO 3
# define EC_W1 4       /* gate */
# define EC_W2 5       /* down */
# define EC_W3 6       /* up */
# define EC_ATTN_NORM 7
# define EC_FFN_NORM 8
/* global tensors (layer = -1) */
# define EC_EMBEDDING 16
# define EC_FINAL_NORM 17
# define EC_LM_HEAD 18
/* optional global tensors (inference.c:583-651); a tensor that is all zero
** (the reference's zero-initialised state) is kept switched off */
# define EC_FINAL_ADAPTER 19	/* bf16 [dim][dim]: x += 16 * (A . x) after the
								** final RMSNorm, before the LM head */
# define EC_LOGIT_BIAS 20		/* float [vocab_size]: logits += bias */

typedef struct ec_model_config
{
	int		dim;
	int		hidden_dim;
	int		n_layers;
	int		n_heads;
	int		n_kv_heads;
	int		vocab_size;
	int		seq_len;		/* max positions per sequence (RoPE table rows) */
	int		head_dim;
	float	rope_theta;
	float	norm_eps;
	int		weight_kind;	/* EC_W_INT8 or EC_W_FP8 */
	int		use_paged_kv;	/* 1: paged INT8 KV (reference default);
							** 0: linear BF16 KV with LSH-routed top-K */
	int		sparse_k;		/* linear mode top-K (SPARSE_K, config.h:67) */
	int		window;			/* ATTN_WINDOW_SIZE (config.h:79) */
	int		sparse_blocks_k;/* SPARSE_BLOCKS_K (config.h:73) */
	int		lsh_tables;		/* 1 in the reference */
	int		lsh_bits;		/* LSH_NUM_HASHES (ops_lsh.h:33), <= 16 */
	int		lsh_unit;		/* LSH_BLOCK_SIZE (ops_lsh.h:35): tokens per hash */
	int		lsh_max_units;	/* LSH_MAX_BLOCKS (ops_lsh.h:36) */
	int		lsh_radius;		/* LSH_HAMMING_RADIUS (ops_lsh.h:37) */
	int		lsh_max_cand;	/* candidate units per query (inference.c:300) */
	int		max_batch;		/* sequences per decode step */
	int		tensor_min_batch;	/* INT8 steps of at least this many sequences run
							** their GEMMs on the tensor cores (ec_op_gemm_tc
							** arithmetic: deterministic, not bit-identical
							** to the reference); 0 = never (default) */
	int		attention_mode;	/* paged KV decode attention:
							** EC_ATTN_REFERENCE (default): the reference's
							**   heap order and sequential online softmax,
							**   bit-identical;
							** EC_ATTN_SPLIT: steps of 1-3 sequences run
							**   the reference's selection (block heap
							**   replayed exactly) in one kernel and split
							**   each KV head's visiting order over a
							**   cluster of CTAs with the reference's
							**   softmax weights (only the additions are
							**   regrouped: within the tests' tolerance);
							**   larger batches keep the grouped
							**   reference-order attention */
	int		wait_limit;		/* bounded device waits between the GEMV chain's
							** phases: 0 = the default (about a second);
							** n > 0: n polls; n < 0: -n polls for a count
							** that is never reached (tests the timeout
							** path: the step returns EC_ERR_TIMEOUT) */
}	ec_model_config;

# define EC_ATTN_REFERENCE 0
# define EC_ATTN_SPLIT 1

typedef struct ec_ctx	ec_ctx;

const char	*ec_last_error(void);

/* Fill `c` with the reference's compile-time defaults (config.h, ops_lsh.h)
** and the Llama-3-8B shape; callers then override the shape. */
int		ec_config_default(ec_model_config *c);

/* transformer_init (src/inference/model.c:146): bind a device, allocate the
** KV pool, upload RoPE tables and LSH hyperplanes computed on the host by
** the reference's formulas (ops_rope.c:30-96, ops_lsh.c:22-85). */
int		ec_create(const ec_model_config *c, int device, ec_ctx **out);
void	ec_destroy(ec_ctx *ctx);

/* Tensor parallelism over `world` GPUs (one process or thread per GPU, one
** context each): rank r holds query heads, KV heads, hidden (FFN) rows and
** vocabulary rows [r * n, (r + 1) * n) of the model `c` describes (each
** count must divide by world).  QKV, gate/up and the LM head are split by
** rows, o and down by columns; ec_set_weight still takes the WHOLE tensor
** and keeps this rank's shard.  Row-split projections are all-gathered and
** added in rank order, the reference's cross-head quantities (the LSH
** query mean over all heads, candidate scores summed over KV heads,
** inference.c:290-353; the paged block selection from query head 0 and KV
** head 0, paged.c:401-495; the layer-0 LSH key) are exchanged so that every
** rank holds the same activations, selections and whole logits.  Not
** bit-identical to one GPU (the row-split sums are regrouped by rank):
** within 2e-2 of the logit range, equal greedy tokens in the tests.
** Collectives are NCCL (libnccl.so.2, loaded on first use) on the context
** stream.  `id` holds 128 bytes from ec_tp_unique_id on one rank, shared
** with the others by the caller; every rank calls ec_create_tp with the
** same id (it blocks until all have).  Reference-order attention and the
** exact GEMV chain only (attention_mode EC_ATTN_REFERENCE,
** tensor_min_batch 0); no prefill, adapter or logit bias. */
int		ec_tp_unique_id(void *out, size_t n);
int		ec_create_tp(const ec_model_config *c, int device, int rank, int world,
			const void *id, ec_ctx **out);

/* Register one tensor (model.c:167-265 weight mapping).  `data` is a host
** pointer unless `on_device` is nonzero.  Matrices are row-major
** [out_features][in_features] in the context's weight_kind; `scales` holds
** one float per row (INT8) or one float (FP8).  Norm weights and the
** embedding are BF16 and take scales = NULL.  Data is copied.  With
** on_device = 1 the call first waits for the whole device
** (cudaDeviceSynchronize: data a caller's stream still writes is complete),
** so it must not run while another stream on the device is capturing a
** graph. */
int		ec_set_weight(ec_ctx *ctx, int layer, int which, const void *data,
			const float *scales, int on_device);

/* The context-aware bias cache (t_transformer.context_bias,
** src/inference/inference.h:180-185, applied at inference.c:657-693): after
** the LM head (and logit bias) of every row, key = the previous input token
** of the sequence (1 at position 0) as uint64, slot = MurmurHash3's 64-bit
** finaliser of the key modulo `size`, linear probing over at most 16 slots;
** a slot holding the key adds biases[slot] to the logit of tokens[slot], a
** slot holding 0 ends the search.  The engine records every sequence's input
** tokens as the reference's token_history does.  Host arrays of `size`
** entries, copied; a table without a nonzero key (or size 0) switches the
** lookup off.  Not with tensor parallelism (EC_ERR_UNSUPPORTED). */
int		ec_set_context_bias(ec_ctx *ctx, const uint64_t *keys, const int *tokens,
			const float *biases, int size);

/* Quantise-at-load: the reference loads BF16 tensors only
** (loader_parse.c:35-49, t_dtype tensor.h:20-24).  `data` is a BF16 matrix
** [out_features][in_features] (host, or device when on_device); it is
** quantised on the device to the context's weight_kind and registered as
** ec_set_weight would: INT8 per row with scale = max|w| / 127 (1 / 127 for
** a zero row), q = clamp(rint(w / scale), +-127); FP8 E4M3 per tensor with
** scale = 2^ceil(log2(max|w| / 448)) (1 for an all-zero tensor) and the
** nearest E4M3 value of w / scale, ties to even, saturating.  Ids other
** than the seven matrices and EC_LM_HEAD are passed to ec_set_weight
** (they are BF16 already).  Like ec_set_weight(on_device = 1), device data
** makes the call synchronise the device first. */
int		ec_set_weight_bf16(ec_ctx *ctx, int layer, int which, const uint16_t *data,
			int on_device);

/* Start sequence `seq` fresh (paged_kv_reset, paged.c:297; lsh_index_reset,
** ops_lsh.c:111). */
int		ec_reset(ec_ctx *ctx, int seq);

/* transformer_forward (src/inference/inference.c:60) for B sequences:
** sequence b takes token tokens[b] at position pos[b] (host arrays).
** logits_host (B * vocab floats) and argmax_host (B ints, the reference's
** sample_argmax, sampler.c:145) may each be NULL.  Synchronous. */
int		ec_decode_step(ec_ctx *ctx, const int *tokens, const int *pos, int B,
			float *logits_host, int *argmax_host);

/* Same step with tokens/positions already in device memory and results left
** in device memory (ec_logits_device / ec_argmax_device); asynchronous on
** the context's stream.  `greedy_feedback` != 0 writes each sequence's argmax
** back into tokens_dev and increments pos_dev, so repeated calls decode
** greedily without host round trips. */
int		ec_decode_step_device(ec_ctx *ctx, int *tokens_dev, int *pos_dev, int B,
			int greedy_feedback);
float	*ec_logits_device(ec_ctx *ctx);
int		*ec_argmax_device(ec_ctx *ctx);
void	*ec_stream(ec_ctx *ctx);
int		ec_synchronize(ec_ctx *ctx);

/* Tracing: with profiling on, decode steps run without the CUDA graph and
** every kernel launch is bracketed by CUDA events on the context's stream.
** ec_profile_read returns, for one kernel kind (EC_K_*), the summed device
** time in ms, the number of launches and the summed algorithmic bytes. */
# define EC_K_GEMV_QKV 0
# define EC_K_GEMV_O 1
# define EC_K_GEMV_GATEUP 2
# define EC_K_GEMV_DOWN 3
# define EC_K_GEMV_LM 4
# define EC_K_KV_APPEND 5
# define EC_K_SELECT 6
# define EC_K_ATTENTION 7
# define EC_K_EMBED 8
# define EC_K_ARGMAX 9
# define EC_K_GEMV_CHAIN 10	/* one layer's o, gate/up, down (+ next QKV / LM head) */
# define EC_K_TC_GEMM 11	/* tensor-core GEMM (batched steps) */
# define EC_K_TC_QUANT 12	/* its input rows -> digit planes (RMSNorm fused) */
# define EC_K_TC_COMBINE 13	/* its tiles split between CTAs -> outputs */
# define EC_K_COUNT 14
int		ec_profile_enable(ec_ctx *ctx, int on);
int		ec_profile_read(ec_ctx *ctx, int kind, double *ms, int *launches,
			double *bytes);

/* Introspection for parity checks (device -> host copies).  ec_read_state
** `which`: 0 x, 2 rotated q, 3 rotated k, 4 v, 5 attention output, 6 logits,
** 7 FFN hidden, 8 the last selection ([count, ids...] as floats), 9 paged
** block centroids of the last layer in logical order ([max_blocks][hd]). */
int		ec_read_state(ec_ctx *ctx, int which, int seq, float *out, size_t n);
int		ec_read_lsh(ec_ctx *ctx, int seq, int *n_units, uint32_t *unit_hash,
			int *unit_start, int *unit_len, int *heads, int *next);
int		ec_read_counters(ec_ctx *ctx, int seq, unsigned long long *out2);
int		ec_launches_per_step(ec_ctx *ctx, int B);

/* ------------------------------------------------------------------------ */
/* Per-op entry points on caller-owned device buffers                        */
/* ------------------------------------------------------------------------ */

/* op_matmul for batch-1 activations (src/compute/ops.h:33,
** ops_matmul.c:366-392): y[m] = W[m][k] . x[k] in the reference's 32-lane
** accumulation order, times scale[row] (INT8) / scale[0] (FP8).
** k must be a multiple of 32. */
int		ec_op_gemv(int wkind, const void *w, const float *scale, const float *x,
			float *y, int m, int k, void *stream);

/* The same op_matmul over weights held in the layout the decode step streams
** (rows in groups of 4, interleaved by 32-byte pieces within chunks of 512
** or 32 columns; see gemv_packed.cu).  ec_gemv_packed_bytes gives the size of
** a packed m x k matrix, ec_gemv_pack fills it from row-major device weights
** (INT8 or FP8 bytes), and ec_op_gemv_packed computes y = W . x, bit-identical
** to ec_op_gemv on the row-major matrix.  k must be a multiple of 32. */
size_t	ec_gemv_packed_bytes(int m, int k);
/* op_matmul for nb activation vectors at once, each bit-identical to
** ec_op_gemv_packed on that vector alone: x [nb][k], y [nb][m] (device).
** INT8: the weights are read once per 8 vectors (FP8: once per vector).  k
** must be a multiple of 512 when nb > 1.  Uses a small counter buffer from the
** stream-ordered allocator. */
int		ec_op_gemv_packed_batch(int wkind, const void *w_packed, const float *scale,
			const float *x, float *y, int m, int k, int nb, void *stream);
int		ec_gemv_pack(const void *w_rowmajor, void *w_packed, int m, int k,
			void *stream);
int		ec_op_gemv_packed(int wkind, const void *w_packed, const float *scale,
			const float *x, float *y, int m, int k, void *stream);

/* Prompt prefill for sequence `seq` (forward_prefill_batch,
** src/inference/inference.c:718-1112): tokens[0..n) at positions
** pos0..pos0+n-1 go through the model max_batch at a time as rows of one
** batched step (each weight pass serves every row of a chunk), with every row
** addressing `seq`'s KV cache; each row's KV append, selection (paged
** blocks, or in linear mode LSH candidates from the units that end by the
** row's own position) and attention keep the decode step's arithmetic, so
** the cache, the LSH index and the logits are bit-identical to decoding the
** tokens one at a time.  With
** tensor_min_batch = m > 0 (INT8), chunks of at least m rows run their
** projections on the tensor cores instead (the tcgen05 GEMM of batched
** steps: within about 1e-6 relative, not bit-identical).  The last
** token's logits and greedy token go to logits_host / argmax_host (either
** may be NULL).  Both KV modes; one rank (not under tensor parallelism). */
int		ec_prefill(ec_ctx *ctx, int seq, const int *tokens, int n, int pos0,
			float *logits_host, int *argmax_host);

/* Speculative decoding's verification (mtp_generate, speculate.c:187-258):
** the target model runs draft tokens tokens[0..n) of sequence `seq` at
** positions pos0.. as the rows of batched steps (the ec_prefill path) and
** writes the greedy token after every row to greedy_out[0..n) -- the
** prediction the reference's token-by-token verification loop compares
** with draft token i + 1, bit-identical to n decode steps.  The caller keeps
** the accepted prefix and continues from the first mismatch; positions past
** it need no rewind (kv_cache_rewind, speculate.c:66, is a no-op: the next
** steps overwrite them).  Paged KV, one rank. */
int		ec_verify(ec_ctx *ctx, int seq, const int *tokens, int n, int pos0,
			int *greedy_out);

/* op_matmul (src/compute/ops.h:33) for nb activation rows at once on the
** tensor cores, INT8 weights only (the large-batch decode and prefill path;
** the reference runs op_matmul once per row).  ec_gemm_tc_bytes gives the
** size of an m x k matrix in the tensor-core layout (128-row tiles; k a
** multiple of 128), ec_gemm_tc_pack fills it from row-major INT8 device
** weights, and ec_op_gemm_tc computes y [nb][m] = scale . (W x) for x [nb][k]
** (device).  Each x row is rounded to 21-bit fixed point against its own
** max |x| (relative error <= 2^-22 of that max), multiplied exactly in int32
** and scaled once: not bit-identical to ec_op_gemv, but deterministic and
** independent of the launch.  Scratch comes from the stream-ordered
** allocator; k <= 51200. */
size_t	ec_gemm_tc_bytes(int m, int k);
int		ec_gemm_tc_pack(const void *w_rowmajor, void *w_tc, int m, int k, void *stream);
int		ec_op_gemm_tc(const void *w_tc, const float *scale, const float *x, float *y,
			int m, int k, int nb, void *stream);

/* op_rmsnorm (src/compute/ops.h:34, ops_norm.c:126); out may alias x. */
int		ec_op_rmsnorm(float *out, const float *x, const uint16_t *w, int n,
			float eps, void *stream);

/* rope_apply_multihead_cached (src/compute/ops_rope.h:80) with device copies
** of the cos/sin tables [max_seq][head_dim/2]. */
int		ec_op_rope(float *data, int n_heads, int head_dim, int pos,
			const float *cos_t, const float *sin_t, int max_seq, void *stream);

/* op_silu_mul (src/compute/ops.h:41); out may alias gate. */
int		ec_op_silu_mul(float *out, const float *gate, const float *up, int n,
			void *stream);

/* quant_f32_to_int8 (src/compute/ops_quant.c:229) on `rows` vectors of n. */
int		ec_op_quant_int8(int8_t *out, float *scales, const float *in, int rows,
			int n, void *stream);

/* sample_argmax (src/compute/sampler.h:19) of B rows of n logits. */
int		ec_op_argmax(const float *logits, int n, int B, int *out, void *stream);

/* The server's sampling step on the device, `rows` rows of n logits each
** (device pointers; the logits are modified in place, as the reference does):
**   repetition penalty (src/server/worker.c:436-442, 477-490): for each of
**     history_len[row] ids at history + row * history_stride (prompt then
**     generated, every occurrence), l > 0 ? l / penalty : l * penalty;
**     history may be NULL (no penalty);
**   block_token0 != 0: logits[0] = -1e9 (worker.c:444, 492);
**   sample_top_p (src/compute/sampler_topp.c:113): softmax at temperature,
**     the nucleus of the descending order whose running sum first exceeds
**     top_p, and the first token of it whose running sum exceeds r[row] times
**     the nucleus' mass.  r[row] in [0, 1] is the caller's draw (the
**     reference takes rand() / RAND_MAX).
** Equal probabilities are ordered by index (the reference's qsort leaves it
** unspecified).  Running sums are exact 2^-50 fixed point rather than the
** reference's float sequence, so a draw within float rounding of a boundary
** can pick the token next to the reference's in the sorted order.  One
** cluster of 8 CTAs per row, the row held in their shared memory
** (n <= 327680, else EC_ERR_UNSUPPORTED); no allocation. */
int		ec_op_sample_top_p(float *logits, int n, int rows, const int *history,
			const int *history_len, int history_stride, float temperature,
			float top_p, float penalty, int block_token0, const float *r,
			int *out, void *stream);

/* sample_temperature (src/compute/sampler_temp.c:96): softmax at
** temperature, then the first index, in index order, whose running sum
** exceeds r[row].  A draw above the whole mass gives n - 1 (the reference
** returns n). */
int		ec_op_sample_temperature(const float *logits, int n, int rows,
			float temperature, const float *r, int *out, void *stream);

/* One layer's paged INT8 KV cache in device memory
** (t_kv_block / t_block_manager, src/memory/paged.h:53-88).  Blocks hold 16
** tokens; within a block K rows are stored rotated by 16-byte pieces (piece p
** of token t at piece (p + t) mod (head_dim / 16)), so fill the view only
** with ec_op_paged_append.  head_dim is 32, 64 or 128. */
typedef struct ec_paged_view
{
	int8_t		*k;			/* [blocks][n_kv_heads][16][head_dim] */
	int8_t		*v;
	float		*k_scale;	/* [blocks][n_kv_heads][16] */
	float		*v_scale;
	float		*centroid;	/* [blocks][head_dim], KV head 0 mean */
	const int	*page_table;/* [max_blocks] logical -> physical block */
	int			n_kv_heads;
	int			head_dim;
	int			max_blocks;	/* logical blocks the page table maps */
}	ec_paged_view;

/* paged_kv_append (src/memory/paged.h:143) of one token at `pos`: quantise
** k, v (F32 [n_kv_heads*head_dim], device, already rotated) and store;
** computes the block centroid when the block fills
** (calc_block_centroid_int8, paged.c:350). */
int		ec_op_paged_append(const ec_paged_view *pv, const float *k,
			const float *v, int pos, void *stream);

/* Decode attention of one token over the first n_tokens cached tokens, q =
** rotated queries [n_heads * head_dim] (device), out likewise.
** sparse_blocks_k == 0: op_paged_attention (ops_attention.h:75), every block
** in order (n_tokens * head_dim <= 131072).  sparse_blocks_k in 1..64: as
** inference.c:436-496 drives it -- dense while the blocks number at most
** sparse_blocks_k, else score_blocks + select_top_k_blocks (paged.h:200-212,
** query head 0) and op_paged_attention_sparse (ops_attention.h:82) over
** first, last and the heap-ordered rest.  selected_out (device, optional,
** sparse_blocks_k ints; with sparse_blocks_k == 0, n_tokens/16 + 1) receives
** the logical blocks in the order attended, n_selected_out (device,
** optional) their number.  Uses a small scratch buffer that it allocates
** and frees on `stream` (stream-ordered allocator). */
int		ec_op_paged_attention(const ec_paged_view *pv, const float *q,
			float *out, int n_heads, int n_tokens, int sparse_blocks_k,
			int *selected_out, int *n_selected_out, void *stream);

/* ec_op_paged_attention without any allocation, for callers that cannot
** allocate device memory (code running under another runtime's allocator or
** memory pool, or required not to call cudaMalloc once started).  It has no
** counterpart in the reference, whose CPU engine allocates nothing on a GPU.
** Same arguments, checks and results as ec_op_paged_attention, with
** n_tokens <= 32768 (2048 blocks); larger contexts are rejected with
** EC_ERR_UNSUPPORTED.  Its scratch is a fixed 8 KB array in the library's
** device memory, one per device, held until the process exits.  The first
** call on a device looks up that array's address (with that device
** current), so make it before any stream capture.  All calls on a device
** share the array: calls that may overlap on the GPU (other streams, other
** threads) race and must be serialised by the caller. */
int		ec_op_paged_attention_static(const ec_paged_view *pv, const float *q,
			float *out, int n_heads, int n_tokens, int sparse_blocks_k,
			int *selected_out, int *n_selected_out, void *stream);

/* ------------------------------------------------------------------------ */
/* Isolated LSH sparse attention over a linear BF16 cache (BASELINE          */
/* configuration 3): the reference's linear-mode selection, inference.c:     */
/* 228-423, with lsh_init / lsh_update / lsh_hash / lsh_find_candidates      */
/* (ops_lsh.c:40-418) generalised to `tables` x `bits` codes over `unit`-    */
/* token units of KV head 0, then attention_head_sparse (ops_attention.c:    */
/* 131-170) over the selection in heap order.  The reference's own setting   */
/* is tables 1, bits 16, unit 64, radius 4, max_cand 64, window 128.         */
/* ------------------------------------------------------------------------ */
typedef struct ec_lsh_attn_config
{
	int		n_heads;
	int		n_kv_heads;
	int		head_dim;		/* 32, 64 or 128 */
	int		max_tokens;		/* cache capacity */
	int		tables;			/* 1..16 hash tables */
	int		bits;			/* 1..16 bits per code */
	int		unit;			/* tokens per hashed unit (mean key of KV head 0) */
	int		radius;			/* Hamming radius of a probe */
	int		max_cand;		/* candidate units per query */
	int		window;			/* always-attended recent positions */
	int		top_k;			/* 1..511 positions attended */
	int		max_queries;	/* queries per ec_lsh_attn_query call */
}	ec_lsh_attn_config;

typedef struct ec_lsh_attn	ec_lsh_attn;

int		ec_lsh_attn_create(const ec_lsh_attn_config *c, int device,
			ec_lsh_attn **out);
void	ec_lsh_attn_destroy(ec_lsh_attn *h);
/* Index the first n_tokens positions of k, v ([max_tokens][n_kv_heads]
** [head_dim] BF16, device; the handle keeps the pointers): one code per
** table per full unit, buckets newest first (lsh_update's chain order). */
int		ec_lsh_attn_build(ec_lsh_attn *h, const uint16_t *k, const uint16_t *v,
			int n_tokens, void *stream);
/* The same over a paged cache (BASELINE configuration 3's layout): k_blocks,
** v_blocks [physical block][16][n_kv_heads][head_dim] BF16 and page_table
** [logical block] -> physical block (device; the handle keeps the
** pointers).  Position p lives in row p % 16 of block page_table[p / 16];
** selection and attention are identical to the linear cache holding the
** same values.  max_tokens bounds the physical rows (blocks x 16). */
int		ec_lsh_attn_build_paged(ec_lsh_attn *h, const uint16_t *k_blocks,
			const uint16_t *v_blocks, const int *page_table, int n_tokens,
			void *stream);
/* n_queries queries q [n][n_heads][head_dim] (device, rotated) at position
** n_tokens - 1: selection then attention into out [n][n_heads][head_dim].
** selected_out [n][top_k] and n_selected_out [n] (device, optional)
** receive the attended positions in heap order (-1: all positions). */
int		ec_lsh_attn_query(ec_lsh_attn *h, const float *q, int n_queries,
			float *out, int *selected_out, int *n_selected_out, void *stream);
/* Test hook: 0 codes [tables][units] (uint32), 1 bucket offsets
** [tables][2^bits + 1], 2 per query (units found, candidates). */
int		ec_lsh_attn_read(ec_lsh_attn *h, int which, void *out, size_t n);

# ifdef __cplusplus
}
# endif
#endif
