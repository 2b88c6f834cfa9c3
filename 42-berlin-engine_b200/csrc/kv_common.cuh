// kv_common.cuh -- device helpers shared by the decode attention paths
// (attn.cu: the reference-order path; attn_fast.cu: the split path): the
// paged K row layout, per-token INT8 quantisation, block centroids and the
// layer-0 LSH index update, each in the reference's arithmetic.
#pragma once
#include <cstdint>

#include "attn.cuh"
#include "ec_internal.cuh"

namespace ec {

constexpr int kBlk = 16;  // tokens per KV block (KV_BLOCK_SIZE, paged.h:35)

// Paged K rows are stored rotated: 16-byte piece p of token t (within its
// block) sits at piece (p + t) mod (hd/16), so threads scoring consecutive
// tokens read different banks.  Byte offset of element d:
__device__ __forceinline__ int kswz(int t, int d, int hd) {
  return ((((d >> 4) + t) & ((hd >> 4) - 1)) << 4) | (d & 15);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// quant_f32_to_int8 (ops_quant.c:229-273) of one vector of n <= 256 floats by
// one warp.  Returns the scale.
__device__ __forceinline__ float warp_quant_int8(const float* in, int8_t* out, int n, int lane, int rot = -1) {
  float mx = 0.0f;
  for (int i = lane; i < n; i += 32) mx = fmaxf(mx, fabsf(in[i]));
  mx = warp_max(mx);
  float scale, inv;
  if (mx > 0.0f) {
    scale = __fdiv_rn(mx, 127.0f);
    inv = __fdiv_rn(127.0f, mx);
  } else {
    scale = 1.0f;
    inv = 1.0f;
  }
  for (int i = lane; i < n; i += 32) {
    int v = (int)roundf(__fmul_rn(in[i], inv));
    v = v > 127 ? 127 : (v < -127 ? -127 : v);
    out[rot >= 0 ? kswz(rot, i, n) : i] = (int8_t)v;
  }
  return scale;
}

// calc_block_centroid_int8 (paged.c:350-393): KV head 0 mean of a full block
__device__ __forceinline__ void block_centroid(const KvLayout& kv, long blk, int tid, int nt) {
  const int KV = kv.n_kv_heads, hd = kv.head_dim;
  for (int d = tid; d < hd; d += nt) {
    float c = 0.0f;
    for (int t = 0; t < kBlk; t++)
      c = __fadd_rn(c, __fmul_rn((float)kv.kq[((blk * KV) * kBlk + t) * hd + kswz(t, d, hd)],
                                 kv.ks[(blk * KV) * kBlk + t]));
    kv.centroid[blk * hd + d] = __fmul_rn(c, __fdiv_rn(1.0f, (float)kBlk));
  }
}

// lsh_update (ops_lsh.c:296-349) of sequence `seq` with one post-RoPE key
// (layer 0, KV head 0) at position pos, by the whole CTA.
static __device__ __noinline__ void lsh_update_token(const LshLayout& lsh, int seq, const float* k, int pos, int hd) {
  const int tid = threadIdx.x;
  float* acc = lsh.acc + (long)seq * hd;
  int* meta = lsh.meta + seq * 4;
  __shared__ int s_count;
  __shared__ uint32_t s_code[16];
  if (tid == 0) {
    if (meta[0] == 0) meta[1] = pos;
    s_count = meta[0] + 1;
  }
  for (int d = tid; d < hd; d += blockDim.x) acc[d] = __fadd_rn(acc[d], k[d]);
  __syncthreads();
  const int count = s_count;
  if (count >= lsh.unit) {
    const float sc = __fdiv_rn(1.0f, (float)count);
    for (int d = tid; d < hd; d += blockDim.x) acc[d] = __fmul_rn(acc[d], sc);
    if (tid < 16) s_code[tid] = 0;
    __syncthreads();
    for (int tb = tid; tb < lsh.tables * lsh.bits; tb += blockDim.x) {
      const int t = tb / lsh.bits, hbit = tb - t * lsh.bits;
      const float* hp = lsh.hp + ((long)t * lsh.bits + hbit) * hd;
      float a = 0.0f;
      for (int d = 0; d < hd; d++) a = __fmaf_rn(acc[d], hp[d], a);
      if (a > 0.0f) atomicOr(&s_code[t], 1u << hbit);
    }
    __syncthreads();
    if (tid == 0) {
      const int nu = meta[2];
      if (nu < lsh.max_units) {
        lsh.unit_start[(long)seq * lsh.max_units + nu] = meta[1];
        lsh.unit_len[(long)seq * lsh.max_units + nu] = count;
        for (int t = 0; t < lsh.tables; t++) {
          const long tb = (long)seq * lsh.tables + t;
          const uint32_t code = s_code[t];
          lsh.unit_hash[tb * lsh.max_units + nu] = code;
          int* head = lsh.heads + (tb << lsh.bits) + code;
          lsh.next[tb * lsh.max_units + nu] = *head;
          *head = nu;
        }
        meta[2] = nu + 1;
      }
      meta[0] = 0;
    }
    __syncthreads();
    for (int d = tid; d < hd; d += blockDim.x) acc[d] = 0.0f;
  } else if (tid == 0) {
    meta[0] = count;
  }
  __syncthreads();
}

}  // namespace ec
