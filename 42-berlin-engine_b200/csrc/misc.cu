// misc.cu -- embedding lookup, argmax, and the stand-alone per-op kernels
// (RMSNorm, RoPE, SwiGLU, INT8 quantisation) behind the ec_op_* entry points.
#include <cuda_fp8.h>

#include "ec_internal.cuh"
#include "misc.cuh"

namespace ec {

// simd_bf16_to_f32 of the token's embedding row (inference.c:83-88)
__global__ void embed_kernel(const uint16_t* __restrict__ emb, const int* __restrict__ tokens,
                             float* __restrict__ x, int dim, int vocab, TokenHistory th) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  int tok = tokens[b];
  // token_history[pos] = token (inference.c:69-70), for the context bias
  if (th.hist && threadIdx.x == 0) {
    const int p = th.pos[b];
    if (p >= 0 && p < th.seq_len) th.hist[(long)th.seq(b) * th.seq_len + p] = tok;
  }
  if (tok < 0 || tok >= vocab) tok = 0;
  const uint16_t* row = emb + (long)tok * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(long)b * dim + i] = bf16_to_f32(row[i]);
}

// argmax_simd_f32 (sampler.c:42-120): per lane l (of 8) the first index of the
// lane's maximum over i == l (mod 8), i < 8*floor(n/8); lanes compared in
// order with strict >; then the scalar tail with strict >.  One CTA per row.
// With `feedback`, also writes the token back and advances the position.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int n,
                                                      int* __restrict__ out, int* tokens,
                                                      int* pos) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* x = logits + (long)b * n;
  __shared__ float s_v[32][8];
  __shared__ int s_i[32][8];
  if (n < 8) {
    if (tid == 0) {
      int idx = 0;
      float best = x[0];
      for (int i = 1; i < n; i++)
        if (x[i] > best) {
          best = x[i];
          idx = i;
        }
      out[b] = idx;
      if (tokens) tokens[b] = idx;
      if (pos) pos[b] += 1;
    }
    return;
  }
  const int n8 = n & ~7;
  // blockDim.x is a multiple of 8: thread t only sees lane t % 8
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  bool have = false;
  for (int i = tid; i < n8; i += blockDim.x) {
    const float v = x[i];
    if (!have || v > bv) {
      bv = v;
      bi = i;
      have = true;
    }
  }
  // combine same-lane entries: larger value, then smaller index
#pragma unroll
  for (int o = 8; o < 32; o <<= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    const bool oh = __shfl_xor_sync(0xffffffffu, have, o);
    if (oh && (!have || ov > bv || (ov == bv && oi < bi))) {
      bv = ov;
      bi = oi;
      have = true;
    }
  }
  const int warp = tid >> 5, lane = tid & 31;
  if (lane < 8) {
    s_v[warp][lane] = have ? bv : -INFINITY;
    s_i[warp][lane] = have ? bi : 0x7fffffff;
  }
  __syncthreads();
  if (tid < 8) {
    float v = s_v[0][tid];
    int i = s_i[0][tid];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) {
      const float ov = s_v[w][tid];
      const int oi = s_i[w][tid];
      if (oi != 0x7fffffff && (i == 0x7fffffff || ov > v || (ov == v && oi < i))) {
        v = ov;
        i = oi;
      }
    }
    s_v[0][tid] = v;
    s_i[0][tid] = i;
  }
  __syncthreads();
  if (tid == 0) {
    float best = s_v[0][0];
    int idx = s_i[0][0];
    for (int l = 1; l < 8; l++)
      if (s_v[0][l] > best) {
        best = s_v[0][l];
        idx = s_i[0][l];
      }
    for (int i = n8; i < n; i++)
      if (x[i] > best) {
        best = x[i];
        idx = i;
      }
    out[b] = idx;
    if (tokens) tokens[b] = idx;
    if (pos) pos[b] += 1;
  }
}

// op_rmsnorm (ops_norm.c:105-124) of one vector per CTA (row blockIdx.x,
// `stride` floats apart).
__global__ void __launch_bounds__(256) rmsnorm_kernel(float* out, const float* x,
                                                      const uint16_t* w, int n, float eps,
                                                      long stride) {
  __shared__ float red[9];
  const int tid = threadIdx.x;
  x += blockIdx.x * stride;
  out += blockIdx.x * stride;
  if (tid < 8) {
    float acc = 0.0f;
    for (int j = tid; j < (n & ~7); j += 8) acc = __fmaf_rn(x[j], x[j], acc);
    red[tid] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    float ss = hsum8(red);
    for (int j = n & ~7; j < n; j++) ss = __fmaf_rn(x[j], x[j], ss);
    ss = __fdiv_rn(ss, (float)n);
    red[8] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, eps)));
  }
  __syncthreads();
  const float inv = red[8];
  for (int j = tid; j < n; j += blockDim.x) out[j] = __fmul_rn(__fmul_rn(x[j], inv), bf16_to_f32(w[j]));
}

__global__ void rope_kernel(float* data, int n_heads, int hd, int pos, const float* cos_t,
                            const float* sin_t, int max_seq) {
  if (pos >= max_seq) return;
  const int half = hd >> 1;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_heads * half) return;
  const int head = i / half, j = i - head * half;
  float* p = data + head * hd;
  const float c = cos_t[(long)pos * half + j], s = sin_t[(long)pos * half + j];
  const float v0 = p[j], v1 = p[j + half];
  p[j] = __fmaf_rn(v0, c, -__fmul_rn(v1, s));
  p[j + half] = __fmaf_rn(v0, s, __fmul_rn(v1, c));
}

// op_silu_mul_fused_f32 (ops_activation.c:48-102): vector form for the first
// 8*floor(n/8) elements, scalar form for the tail.
__global__ void silu_kernel(float* out, const float* g, const float* u, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = g[i];
  float sig;
  if (i < (n & ~7))
    sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf_vec(__fsub_rn(0.0f, gv))));
  else
    sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf(-gv)));
  out[i] = __fmul_rn(__fmul_rn(gv, sig), u[i]);
}

// quant_f32_to_int8 (ops_quant.c:229-273): one warp per vector.
__global__ void quant_kernel(int8_t* out, float* scales, const float* in, int rows, int n) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* x = in + (long)r * n;
  float mx = 0.0f;
  for (int i = lane; i < n; i += 32) mx = fmaxf(mx, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sc = 1.0f, inv = 1.0f;
  if (mx > 0.0f) {
    sc = __fdiv_rn(mx, 127.0f);
    inv = __fdiv_rn(127.0f, mx);
  }
  for (int i = lane; i < n; i += 32) {
    int v = (int)roundf(__fmul_rn(x[i], inv));
    v = v > 127 ? 127 : (v < -127 ? -127 : v);
    out[(long)r * n + i] = (int8_t)v;
  }
  if (lane == 0) scales[r] = sc;
}

cudaError_t launch_embed(const uint16_t* emb, const int* tokens, float* x, int dim, int vocab, int B,
                         cudaStream_t s, bool pdl, const TokenHistory* th) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_kernel, emb, tokens, x, dim, vocab,
                            th ? *th : TokenHistory{});
}

// argmax_simd_f32 split over kArgParts CTAs per row: CTA p reduces an
// 8-aligned range to its 8 lane partials (first index of the lane maximum);
// the last CTA to finish combines the ranges in order (strict >: on a tie the
// earlier range, i.e. the smaller index of that lane, stays), then the lanes
// in order (strict >), then the scalar tail -- the reference's result.
constexpr int kArgParts = 32;

__global__ void __launch_bounds__(256) argmax_split_kernel(const float* __restrict__ logits,
                                                           int n, int* __restrict__ out,
                                                           int* tokens, int* pos,
                                                           uint8_t* scratch) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y, p = blockIdx.x, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const float* x = logits + (long)b * n;
  // sequence b's slice of the scratch: partial values, indices, counter
  float* pv = reinterpret_cast<float*>(scratch + (size_t)b * (kArgParts * 8 * 8 + 4));
  int* pi = reinterpret_cast<int*>(pv + kArgParts * 8);
  int* ctr = pi + kArgParts * 8;
  const int n8 = n & ~7;
  const int per = ((n8 / kArgParts) + 7) & ~7;
  const int lo = min(n8, p * per), hi = min(n8, lo + per);
  __shared__ float s_v[8][8];
  __shared__ int s_i[8][8];
  __shared__ bool s_last;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = lo + tid; i < hi; i += blockDim.x) {  // blockDim % 8 == 0: lane tid % 8
    const float v = x[i];
    if (bi == 0x7fffffff || v > bv) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 8; o < 32; o <<= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane < 8) {
    s_v[warp][lane] = bv;
    s_i[warp][lane] = bi;
  }
  __syncthreads();
  float* gv = pv + p * 8;
  int* gi = pi + p * 8;
  if (tid < 8) {
    float v = s_v[0][tid];
    int i = s_i[0][tid];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) {
      const float ov = s_v[w][tid];
      const int oi = s_i[w][tid];
      if (oi != 0x7fffffff && (i == 0x7fffffff || ov > v || (ov == v && oi < i))) {
        v = ov;
        i = oi;
      }
    }
    gv[tid] = v;
    gi[tid] = i;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(ctr, 1) == kArgParts - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid < 8) {
    const float* av = pv;
    const int* ai = pi;
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int q = 0; q < kArgParts; q++) {
      const float ov = av[q * 8 + tid];
      const int oi = ai[q * 8 + tid];
      if (oi != 0x7fffffff && (i == 0x7fffffff || ov > v)) {
        v = ov;
        i = oi;
      }
    }
    s_v[0][tid] = v;
    s_i[0][tid] = i;
  }
  __syncthreads();
  if (tid == 0) {
    ctr[0] = 0;
    float best = s_v[0][0];
    int idx = s_i[0][0];
    for (int l = 1; l < 8; l++)
      if (s_v[0][l] > best) {
        best = s_v[0][l];
        idx = s_i[0][l];
      }
    for (int i = n8; i < n; i++)
      if (x[i] > best) {
        best = x[i];
        idx = i;
      }
    out[b] = idx;
    if (tokens) tokens[b] = idx;
    if (pos) pos[b] += 1;
  }
}

// per sequence: kArgParts x 8 partial values and indices, one counter
size_t argmax_scratch_bytes(int B) { return (size_t)B * (kArgParts * 8 * 8 + 4); }

cudaError_t launch_argmax_split(const float* logits, int n, int B, int* out, int* tokens,
                                int* pos, void* scratch, cudaStream_t s, bool pdl) {
  if (n < 8 * kArgParts) return launch_argmax(logits, n, B, out, tokens, pos, s, pdl);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kArgParts, B);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, argmax_split_kernel, logits, n, out, tokens, pos,
                            static_cast<uint8_t*>(scratch));
}

cudaError_t launch_argmax(const float* logits, int n, int B, int* out, int* tokens, int* pos,
                          cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B);
  cfg.blockDim = dim3(1024);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, argmax_kernel, logits, n, out, tokens, pos);
}

cudaError_t launch_rmsnorm(float* out, const float* x, const uint16_t* w, int n, float eps,
                           cudaStream_t s) {
  rmsnorm_kernel<<<1, 256, 0, s>>>(out, x, w, n, eps, 0L);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(float* out, const float* x, const uint16_t* w, int n, float eps,
                                int rows, long stride, cudaStream_t s) {
  rmsnorm_kernel<<<rows, 256, 0, s>>>(out, x, w, n, eps, stride);
  return cudaGetLastError();
}

// The final hidden adapter (inference.c:583-638): out[r] = simd_dot_bf16_f32
// (A[r], x) in its 8-lane order (lane l takes columns l, l + 8, ...; then
// ((l0+l4)+(l1+l5))+((l2+l6)+(l3+l7))), and xa[r] = x[r] + 16 * out[r]
// (ADAPTER_SCALE, config.h:54; a power of two, so the product is exact).
// 8 threads per row, 32 rows per CTA, grid (rows / 32, sequences).
__global__ void __launch_bounds__(256) adapter_kernel(const uint16_t* __restrict__ A,
                                                      const float* __restrict__ x,
                                                      float* __restrict__ xa, int D) {
  const int b = blockIdx.y, l = threadIdx.x & 7;
  const int r = blockIdx.x * 32 + (threadIdx.x >> 3);
  const float* xb = x + (long)b * D;
  const uint16_t* a = A + (long)min(r, D - 1) * D;
  float acc = 0.0f;
  for (int j = l; j < (D & ~7); j += 8) acc = __fmaf_rn(bf16_to_f32(a[j]), xb[j], acc);
  const float h4 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
  const float t2 = __fadd_rn(h4, __shfl_xor_sync(0xffffffffu, h4, 1));
  float sum = __fadd_rn(t2, __shfl_xor_sync(0xffffffffu, t2, 2));
  if (l == 0 && r < D) {
    for (int j = D & ~7; j < D; j++) sum = __fmaf_rn(bf16_to_f32(a[j]), xb[j], sum);
    xa[(long)b * D + r] = __fadd_rn(xb[r], __fmul_rn(16.0f, sum));
  }
}

cudaError_t launch_adapter(const uint16_t* A, const float* x, float* xa, int D, int B,
                           cudaStream_t s) {
  adapter_kernel<<<dim3((D + 31) / 32, B), 256, 0, s>>>(A, x, xa, D);
  return cudaGetLastError();
}

// logits[b][i] += bias[i] (inference.c:645-651)
__global__ void logit_bias_kernel(float* logits, const float* __restrict__ bias, int V) {
  float* row = logits + (long)blockIdx.y * V;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x)
    row[i] = __fadd_rn(row[i], bias[i]);
}

cudaError_t launch_logit_bias(float* logits, const float* bias, int V, int B, cudaStream_t s) {
  logit_bias_kernel<<<dim3(64, B), 256, 0, s>>>(logits, bias, V);
  return cudaGetLastError();
}

// The context-aware bias cache (inference.c:657-693): key = the previous
// token (token_history[pos - 1], or 1 at position 0) as uint64; slot =
// fmix64(key) % size (MurmurHash3's 64-bit finaliser); linear probing over
// at most 16 slots: a slot holding the key adds its bias to its target
// token's logit and ends the search, an empty slot (key 0) ends it.  A key
// of 0 matches an empty slot, whose bias is 0.  One thread per row.
__global__ void context_bias_kernel(float* __restrict__ logits, int V, int B, TokenHistory th,
                                    ContextBias cb) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int p = th.pos[b];
  if (p > th.seq_len) return;  // the reference reads past its history there
  const int prev = p > 0 ? th.hist[(long)th.seq(b) * th.seq_len + p - 1] : 1;
  const uint64_t key = (uint64_t)(long long)prev;
  uint64_t h = key;
  h ^= h >> 33;
  h *= 0xff51afd7ed558ccdULL;
  h ^= h >> 33;
  h *= 0xc4ceb9fe1a85ec53ULL;
  h ^= h >> 33;
  const uint32_t idx = (uint32_t)(h % (uint64_t)cb.size);
  for (int i = 0; i < 16; i++) {
    const uint32_t cur = (uint32_t)(((uint64_t)idx + i) % (uint64_t)cb.size);
    const uint64_t k = cb.keys[cur];
    if (k == key) {
      const int t = cb.tokens[cur];
      if (t >= 0 && t < V) {
        float* l = logits + (long)b * V + t;
        *l = __fadd_rn(*l, cb.biases[cur]);
      }
      break;
    }
    if (k == 0) break;
  }
}

cudaError_t launch_context_bias(float* logits, int V, int B, const TokenHistory& th,
                                const ContextBias& cb, cudaStream_t s) {
  context_bias_kernel<<<(B + 127) / 128, 128, 0, s>>>(logits, V, B, th, cb);
  return cudaGetLastError();
}

// Quantise-at-load (the reference ships BF16 weights only,
// loader_parse.c:35-49): INT8 per output row, scale = max|w| / 127 (1 / 127
// for an all-zero row), q = clamp(rint(w / scale), -127, 127) with IEEE
// division and round-half-even.  One CTA per row.
__global__ void __launch_bounds__(256) quant_rows_int8_kernel(const uint16_t* __restrict__ w,
                                                              int8_t* __restrict__ q,
                                                              float* __restrict__ scale, int cols) {
  __shared__ float s_red[8];
  const long r = blockIdx.x;
  const uint16_t* row = w + r * cols;
  float m = 0.0f;
  for (int j = threadIdx.x; j < cols; j += blockDim.x) m = fmaxf(m, fabsf(bf16_to_f32(row[j])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) amax = fmaxf(amax, s_red[i]);
  const float sc = __fdiv_rn(amax > 0.0f ? amax : 1.0f, 127.0f);
  for (int j = threadIdx.x; j < cols; j += blockDim.x) {
    float v = rintf(__fdiv_rn(bf16_to_f32(row[j]), sc));
    v = fminf(fmaxf(v, -127.0f), 127.0f);
    q[r * cols + j] = (int8_t)(int)v;
  }
  if (threadIdx.x == 0) scale[r] = sc;
}

cudaError_t launch_quant_rows_int8(const uint16_t* w, int8_t* q, float* scale, int rows, int cols,
                                   cudaStream_t s) {
  quant_rows_int8_kernel<<<rows, 256, 0, s>>>(w, q, scale, cols);
  return cudaGetLastError();
}

// max |w| over a BF16 tensor into *out (float bits; out zeroed by the caller)
__global__ void absmax_bf16_kernel(const uint16_t* __restrict__ w, long n, unsigned* out) {
  float m = 0.0f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(bf16_to_f32(w[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

cudaError_t launch_absmax_bf16(const uint16_t* w, long n, unsigned* out, cudaStream_t s) {
  absmax_bf16_kernel<<<296, 256, 0, s>>>(w, n, out);
  return cudaGetLastError();
}

// FP8 E4M3 per tensor: code = nearest E4M3 value of w / scale (ties to even,
// saturating at 448; negative zero stored as +0)
__global__ void quant_fp8_kernel(const uint16_t* __restrict__ w, uint8_t* __restrict__ q, long n,
                                 float scale) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float x = __fdiv_rn(bf16_to_f32(w[i]), scale);
    uint8_t c = (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
    q[i] = c == 0x80 ? 0 : c;
  }
}

cudaError_t launch_quant_fp8(const uint16_t* w, uint8_t* q, long n, float scale, cudaStream_t s) {
  quant_fp8_kernel<<<592, 256, 0, s>>>(w, q, n, scale);
  return cudaGetLastError();
}

// Tensor parallelism: x[i] += sum of the ranks' partials of a row-split
// projection, added in rank order (parts [world][n]); every rank computes the
// same sum, so x stays identical on all ranks.
__global__ void tp_resid_kernel(float* __restrict__ x, const float* __restrict__ parts, int world,
                                int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float sum = parts[i];
    for (int r = 1; r < world; r++) sum = __fadd_rn(sum, parts[(long)r * n + i]);
    x[i] = __fadd_rn(x[i], sum);
  }
}

cudaError_t launch_tp_resid(float* x, const float* parts, int world, int n, cudaStream_t s) {
  tp_resid_kernel<<<(n + 255) / 256 < 64 ? (n + 255) / 256 : 64, 256, 0, s>>>(x, parts, world, n);
  return cudaGetLastError();
}

// out[0] |= 1 when any of n elements of `bits`-bit width is not +0 / -0.
__global__ void nonzero_kernel(const void* p, long n, int bits, int* out) {
  int any = 0;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    if (bits == 16)
      any |= (static_cast<const uint16_t*>(p)[i] & 0x7FFFu) != 0;
    else
      any |= (static_cast<const uint32_t*>(p)[i] & 0x7FFFFFFFu) != 0;
  }
  if (__syncthreads_or(any) && threadIdx.x == 0) atomicOr(out, 1);
}

cudaError_t launch_nonzero(const void* p, long n, int bits, int* out, cudaStream_t s) {
  nonzero_kernel<<<148, 256, 0, s>>>(p, n, bits, out);
  return cudaGetLastError();
}

cudaError_t launch_rope(float* data, int n_heads, int hd, int pos, const float* c, const float* sn,
                        int max_seq, cudaStream_t s) {
  const int n = n_heads * (hd / 2);
  rope_kernel<<<(n + 255) / 256, 256, 0, s>>>(data, n_heads, hd, pos, c, sn, max_seq);
  return cudaGetLastError();
}

cudaError_t launch_silu(float* out, const float* g, const float* u, int n, cudaStream_t s) {
  silu_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, g, u, n);
  return cudaGetLastError();
}

cudaError_t launch_quant(int8_t* out, float* scales, const float* in, int rows, int n,
                         cudaStream_t s) {
  quant_kernel<<<(rows + 7) / 8, 256, 0, s>>>(out, scales, in, rows, n);
  return cudaGetLastError();
}

}  // namespace ec
