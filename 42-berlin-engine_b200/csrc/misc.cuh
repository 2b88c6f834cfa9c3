// misc.cuh -- embedding, argmax and per-op kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace ec {
// Where the embedding launch records each row's input token (pos[b] of
// sequence seq(b)), as the reference's token_history; hist == nullptr: not.
struct TokenHistory {
  const int* pos = nullptr;
  int* hist = nullptr;     // [S][seq_len]
  int seq_len = 0;
  int seq0 = 0;            // row b is sequence seq0 + b ...
  int seq_plus1 = 0;       // ... or, when set, every row is seq_plus1 - 1
  __host__ __device__ int seq(int b) const { return seq_plus1 ? seq_plus1 - 1 : seq0 + b; }
};
// The reference's context-aware bias cache (t_transformer.context_bias).
struct ContextBias {
  const uint64_t* keys = nullptr;
  const int* tokens = nullptr;
  const float* biases = nullptr;
  int size = 0;
};
cudaError_t launch_embed(const uint16_t* emb, const int* tokens, float* x, int dim, int vocab, int B,
                         cudaStream_t s, bool pdl, const TokenHistory* th = nullptr);
cudaError_t launch_context_bias(float* logits, int V, int B, const TokenHistory& th,
                                const ContextBias& cb, cudaStream_t s);
// The decode step's argmax over kArgParts CTAs per row; scratch holds
// argmax_scratch_bytes(B), its counters zero (they return to zero).
size_t argmax_scratch_bytes(int B);
cudaError_t launch_argmax_split(const float* logits, int n, int B, int* out, int* tokens,
                                int* pos, void* scratch, cudaStream_t s, bool pdl);
cudaError_t launch_argmax(const float* logits, int n, int B, int* out, int* tokens, int* pos,
                          cudaStream_t s, bool pdl);
cudaError_t launch_rmsnorm(float* out, const float* x, const uint16_t* w, int n, float eps,
                           cudaStream_t s);
cudaError_t launch_rmsnorm_rows(float* out, const float* x, const uint16_t* w, int n, float eps,
                                int rows, long stride, cudaStream_t s);
// final hidden adapter: xa = x + 16 * (A . x) per row (B rows of D)
cudaError_t launch_adapter(const uint16_t* A, const float* x, float* xa, int D, int B,
                           cudaStream_t s);
cudaError_t launch_logit_bias(float* logits, const float* bias, int V, int B, cudaStream_t s);
// *out |= 1 when any element (16- or 32-bit) is not a signed zero
cudaError_t launch_nonzero(const void* p, long n, int bits, int* out, cudaStream_t s);
// quantise-at-load of BF16 weights: INT8 per row / FP8 E4M3 per tensor
cudaError_t launch_quant_rows_int8(const uint16_t* w, int8_t* q, float* scale, int rows, int cols,
                                   cudaStream_t s);
cudaError_t launch_absmax_bf16(const uint16_t* w, long n, unsigned* out, cudaStream_t s);
cudaError_t launch_quant_fp8(const uint16_t* w, uint8_t* q, long n, float scale, cudaStream_t s);
// tensor parallelism: x += sum over ranks (in rank order) of parts [world][n]
cudaError_t launch_tp_resid(float* x, const float* parts, int world, int n, cudaStream_t s);
cudaError_t launch_rope(float* data, int n_heads, int hd, int pos, const float* c, const float* sn,
                        int max_seq, cudaStream_t s);
cudaError_t launch_silu(float* out, const float* g, const float* u, int n, cudaStream_t s);
cudaError_t launch_quant(int8_t* out, float* scales, const float* in, int rows, int n,
                         cudaStream_t s);
}  // namespace ec
