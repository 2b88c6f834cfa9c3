// misc.cu -- embedding lookup, argmax, and the stand-alone per-op kernels
// (RMSNorm, RoPE, SwiGLU, INT8 quantisation) behind the ec_op_* entry points.
#include "ec_internal.cuh"
#include "misc.cuh"

namespace ec {

// simd_bf16_to_f32 of the token's embedding row (inference.c:83-88)
__global__ void embed_kernel(const uint16_t* __restrict__ emb, const int* __restrict__ tokens,
                             float* __restrict__ x, int dim, int vocab) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  int tok = tokens[b];
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

// op_rmsnorm (ops_norm.c:105-124) of one vector; one CTA.
__global__ void __launch_bounds__(256) rmsnorm_kernel(float* out, const float* x,
                                                      const uint16_t* w, int n, float eps) {
  __shared__ float red[9];
  const int tid = threadIdx.x;
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
                         cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_kernel, emb, tokens, x, dim, vocab);
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
  rmsnorm_kernel<<<1, 256, 0, s>>>(out, x, w, n, eps);
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
