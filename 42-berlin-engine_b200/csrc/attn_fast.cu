// attn_fast.cu -- the split decode attention over the paged INT8 KV cache.
//
// Same operation as kv_append_kernel + paged_select_cta + attention_kernel
// (op_paged_attention(_sparse), ops_attention.c:292-461, with score_blocks /
// select_top_k_blocks, paged.c:401-495), with two differences that remove
// their serial chains from the critical path:
//
//   * append, block scores and the exact heap replay run in one CTA per
//     sequence with every dependent load issued at once;
//   * attention splits each KV head's visiting order over a cluster of CTAs,
//     every CTA computing all query heads of the group: the softmax weights
//     are the reference's bit for bit (each split learns the running max
//     entering it from the earlier splits), only the additions of the
//     output recurrence are regrouped (partials merged in visiting order).
//
// Kernels per layer: fast_select_kernel (one CTA per sequence: RoPE q and k,
// INT8 append, block centroid at block full, LSH update on layer 0, block
// scores, heap) then fast_attention_kernel (grid KV heads x splits x
// sequences, one cluster per KV head and sequence).
#include <cfloat>
#include <cooperative_groups.h>

#include "attn.cuh"
#include "ec_internal.cuh"
#include "kv_common.cuh"
#include "select.cuh"

namespace ec {

// Phase timestamps for performance work (build with -DEC_PHASE_TIMING):
// slot s of g_fast_ts gets %globaltimer when one thread passes mark s.
#ifdef EC_PHASE_TIMING
__device__ long long g_fast_ts[64];
#define FAST_MARK(cond, s)                                     \
  do {                                                         \
    if (cond) {                                                \
      long long t_;                                            \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));  \
      g_fast_ts[s] = t_;                                       \
    }                                                          \
  } while (0)
extern "C" int ec_debug_fast_times(long long* out) {
  return cudaMemcpyFromSymbol(out, g_fast_ts, sizeof(g_fast_ts)) == cudaSuccess ? 0 : -2;
}
#else
#define FAST_MARK(cond, s) \
  do {                     \
  } while (0)
#endif

constexpr int kFastThreads = 256;
constexpr int kFastMaxSel = 64;  // selected blocks (SPARSE_BLOCKS_K <= 64)
constexpr int kFastMaxSplits = 8;  // CTAs per cluster (portable cluster size)

// ------------------------------------------------------------------------
// fast_select_kernel: one CTA per sequence (batch row b).  Everything that
// was written in earlier steps (RoPE row, page table, the earlier tokens of
// the current block, the centroids) is loaded or prefetched before the wait
// for the previous kernel; after it, every dependent load is issued at once.
// ------------------------------------------------------------------------
constexpr int kSelChunk = 128;  // centroids staged in shared memory per round

// Dynamic shared memory of fast_select_kernel: the step's q/k/v rows and one
// chunk of centroids.
__host__ __device__ inline size_t fast_select_smem(int H, int KV, int hd) {
  return (size_t)(H + 2 * KV) * hd * 4 + (size_t)kSelChunk * hd * 4;
}

__global__ void __launch_bounds__(kFastThreads) fast_select_kernel(KvLayout kv, LshLayout lsh,
                                                                   StepBuffers sb, int layer) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ __align__(16) float s_q0[128];
  __shared__ __align__(16) float s_k[8][128];  // rotated keys (LSH: head 0)
  __shared__ __align__(16) float s_cos[64], s_sin[64];
  __shared__ __align__(16) float s_bsc[2048];
  __shared__ __align__(16) int s_pt[2048];
  __shared__ __align__(16) uint2 s_hp[128];
  __shared__ __align__(16) int8_t s_cb[kBlk * 128];  // head 0 K rows of a block being completed
  __shared__ float s_cs[kBlk];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim, half = hd >> 1;
  float* s_qkv = reinterpret_cast<float*>(dsm);                        // [H + 2KV][hd]
  float* s_cen = s_qkv + (size_t)(H + 2 * KV) * hd;                    // [kSelChunk][hd]
  const int pos = step_pos(sb, b);
  const int n_tok = min(pos + 1, kv.max_blocks * kBlk);
  const int nb = (n_tok + kBlk - 1) / kBlk;
  const long base = ((long)kv_seq(kv, b) * kv.n_layers + layer) * kv.max_blocks;
  const int* pt = kv.page_table + base;
  const bool sparse = nb > sb.sparse_blocks_k;
  const int nmid = nb - 2;
  const bool rope = pos < kv.seq_len;
  const int lb = pos / kBlk, off = pos - lb * kBlk;
  const bool append = lb < kv.max_blocks;
  const long blk = append ? base + pt[lb] : 0;
  const bool full = append && off == kBlk - 1;
  const bool mk = tid == 0 && b == 0 && layer == 1;
  (void)mk;
  FAST_MARK(mk, 0);
  // ---- before the wait: nothing here is written by the previous kernel
  if (rope)
    for (int j = tid; j < half; j += kFastThreads) {
      s_cos[j] = sb.rope_cos[(long)pos * half + j];
      s_sin[j] = sb.rope_sin[(long)pos * half + j];
    }
  if (full && tid >= 128) {
    // tokens 0..14 of the block this step completes (KV head 0), by the
    // warps that compute its centroid (they wait for their own copies)
    const int8_t* src = kv.kq + (blk * KV) * kBlk * hd;
    for (int i = tid - 128; i < (kBlk - 1) * hd / 16; i += 128)
      cp_async16(s_cb + 16 * i, src + 16 * i);
    if (tid - 128 < kBlk - 1) s_cs[tid - 128] = __ldcg(kv.ks + (blk * KV) * kBlk + tid - 128);
  }
  if (sparse) {
    for (int i = tid; i < nmid; i += kFastThreads) s_pt[i] = pt[1 + i];
    // the first chunk of middle-block centroids: blocks before this step's
    // block, written by earlier steps, so they load while the projection
    // that precedes this kernel finishes
    if (tid < 128) {
      const int nc = min(kSelChunk, nmid), per = hd >> 2;
      for (int i = tid; i < nc * per; i += 128) {
        const int bk = i / per, pc = i - bk * per;
        cp_async16(s_cen + (size_t)bk * hd + 4 * pc, kv.centroid + (base + pt[1 + bk]) * hd + 4 * pc);
      }
    }
  }
  pdl_launch_dependents();
  pdl_wait();
  FAST_MARK(mk, 1);
  float* qkv = sb.qkv + (long)b * (H + 2 * KV) * hd;
  float* qo = sb.qrot + (long)b * H * hd;
  int* out = sb.sel + (long)b * sb.max_sel;
  int* outp = sb.selp + (long)b * sb.max_sel;
  __syncthreads();
  if (warp < 4) {
    // ======== warps 0-3: query head 0, block scores, heap ========
    const int ta = tid;  // 0..127
    for (int j = ta; j < half; j += 128) {
      const float v0 = qkv[j], v1 = qkv[j + half];
      float r0 = v0, r1 = v1;
      if (rope) {
        r0 = __fmaf_rn(v0, s_cos[j], -__fmul_rn(v1, s_sin[j]));
        r1 = __fmaf_rn(v0, s_sin[j], __fmul_rn(v1, s_cos[j]));
      }
      s_q0[j] = r0;
      s_q0[j + half] = r1;
      qo[j] = r0;
      qo[j + half] = r1;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!sparse) {
      for (int i = ta; i < nb; i += 128) {
        out[i] = i;
        outp[i] = (int)(base + pt[i]);
      }
      if (ta == 0) sb.nsel[b] = nb;
    } else {
      // score_blocks (paged.c:401-431): q head 0 . centroid in
      // simd_dot_f32_f32's order (8 lanes, then ((c0+c4)+(c1+c5))+((c2+c6)+(c3+c7)));
      // centroids pulled into shared memory kSelChunk blocks at a time
      const int grp = ta >> 3, l = ta & 7;
      for (int c0 = 0; c0 < nmid; c0 += kSelChunk) {
        const int nc = min(kSelChunk, nmid - c0), per = hd >> 2;
        if (c0 > 0)  // (the first chunk was issued before the wait)
          for (int i = ta; i < nc * per; i += 128) {
            const int bk = i / per, pc = i - bk * per;
            cp_async16(s_cen + (size_t)bk * hd + 4 * pc,
                       kv.centroid + (base + s_pt[c0 + bk]) * hd + 4 * pc);
          }
        asm volatile("cp.async.wait_all;" ::: "memory");
        asm volatile("bar.sync 1, 128;" ::: "memory");
        // the same trip count on every lane (the shuffles name the whole warp)
        for (int b0 = 0; b0 < nc; b0 += 16) {
          const int bk = b0 + grp;
          const float* cp = s_cen + (size_t)min(bk, nc - 1) * hd;
          float acc = 0.0f;
          for (int j = l; j < hd; j += 8) acc = __fmaf_rn(s_q0[j], cp[j], acc);
          const float h4 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
          const float t2 = __fadd_rn(h4, __shfl_xor_sync(0xffffffffu, h4, 1));
          const float sum = __fadd_rn(t2, __shfl_xor_sync(0xffffffffu, t2, 2));
          if (l == 0 && bk < nc) s_bsc[c0 + bk] = sum;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      FAST_MARK(mk, 5);
      // select_top_k_blocks (paged.c:439-495): block 0, the last block, then
      // the min-heap of the middle blocks in its array order (exact replay)
      if (warp == 0) {
        int m = sb.sparse_blocks_k - 2;
        if (m > nmid) m = nmid;
        if (m > 62) m = 62;
        const int size = warp_heap_select<6>(s_bsc, nullptr, 1, nmid, m, s_hp, lane,
                                             [](int) { return true; });
        for (int i = lane; i < size; i += 32) {
          const int lbk = (int)s_hp[1 + i].y;
          out[2 + i] = lbk;
          outp[2 + i] = (int)(base + s_pt[lbk - 1]);
        }
        if (lane == 0) {
          out[0] = 0;
          out[1] = nb - 1;
          outp[0] = (int)(base + pt[0]);
          outp[1] = (int)(base + pt[nb - 1]);
          sb.nsel[b] = 2 + size;
        }
        FAST_MARK(mk, 6);
      }
    }
  } else {
    // ======== warps 4-7: RoPE of the other heads, INT8 append, centroid ========
    const int tb = tid - 128;
    const int n4 = (H + 2 * KV) * hd / 4;
    for (int i = tb; i < n4; i += 128) cp_async16(s_qkv + 4 * i, qkv + 4 * i);
    asm volatile("cp.async.wait_all;" ::: "memory");
    asm volatile("bar.sync 2, 128;" ::: "memory");
    FAST_MARK(tb == 0 && b == 0 && layer == 1, 2);
    // RoPE (rope_apply_multihead_cached, ops_rope.c:192-231): query heads
    // 1..H-1 to qrot, key heads in place (the reference rotates k in place)
    for (int i = tb + half; i < (H + KV) * half; i += 128) {
      const int head = i / half, j = i - head * half;
      const float v0 = s_qkv[head * hd + j], v1 = s_qkv[head * hd + j + half];
      float r0 = v0, r1 = v1;
      if (rope) {
        r0 = __fmaf_rn(v0, s_cos[j], -__fmul_rn(v1, s_sin[j]));
        r1 = __fmaf_rn(v0, s_sin[j], __fmul_rn(v1, s_cos[j]));
      }
      float* dst = head < H ? qo + head * hd : qkv + head * hd;
      dst[j] = r0;
      dst[j + half] = r1;
      if (head >= H) {
        s_k[head - H][j] = r0;
        s_k[head - H][j + half] = r1;
      }
    }
    asm volatile("bar.sync 2, 128;" ::: "memory");
    // paged_kv_append (paged.c:195-272): INT8 K (rows rotated) and V
    if (append) {
      for (int h = warp - 4; h < 2 * KV; h += 4) {
        const bool isv = h >= KV;
        const int kh = isv ? h - KV : h;
        int8_t* dst = (isv ? kv.vq : kv.kq) + ((blk * KV + kh) * kBlk + off) * hd;
        const float* src = isv ? s_qkv + (size_t)(H + KV + kh) * hd : s_k[kh];
        const float sc = warp_quant_int8(src, dst, hd, lane, isv ? -1 : off);
        if (lane == 0) (isv ? kv.vs : kv.ks)[(blk * KV + kh) * kBlk + off] = sc;
        if (full && h == 0) {
          // the new row of head 0 beside the block's earlier rows (the same
          // quantisation again, into shared memory)
          warp_quant_int8(s_k[0], s_cb + off * hd, hd, lane, off);
          if (lane == 0) s_cs[off] = sc;
        }
      }
      if (full) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        asm volatile("bar.sync 2, 128;" ::: "memory");
        // calc_block_centroid_int8 (paged.c:350-393), as block_centroid
        for (int d = tb; d < hd; d += 128) {
          float c = 0.0f;
          for (int t = 0; t < kBlk; t++)
            c = __fadd_rn(c, __fmul_rn((float)s_cb[t * hd + kswz(t, d, hd)], s_cs[t]));
          kv.centroid[blk * hd + d] = __fmul_rn(c, __fdiv_rn(1.0f, (float)kBlk));
        }
      }
    }
    FAST_MARK(tb == 0 && b == 0 && layer == 1, 3);
  }
  if (layer == 0 && lsh.tables > 0) {
    __syncthreads();
    lsh_update_token(lsh, kv_seq(kv, b), s_k[0], pos, hd);
  }
}

// ------------------------------------------------------------------------
// fast_attention_kernel: a cluster of `splits` CTAs per (KV head g,
// sequence b); CTA s takes a contiguous share of the visiting order (the
// selection list) and every query head of the group.
//
// The reference's online softmax over tokens t = 0..T-1 in visiting order,
//   m_t = max(m_{t-1}, s_t), e_t = fast_expf(s_t - m_t),
//   f_t = fast_expf(m_{t-1} - m_t), o_t = o_{t-1} f_t + e_t v_t,
// unrolls to o_T = sum_t e_t v_t prod_{u>t} f_u, the same for the sum.  Each
// split needs only the running max at its start (the max over earlier
// splits, exchanged through distributed shared memory) to compute its own
// e_t and f_t exactly as the reference does; it then forms its partial
// o_s = sum_{t in s} e_t v_t prod_{u in s, u>t} f_u and F_s = prod_{u in s} f_u,
// and the partials merge in order as o = (o * F_s) + o_s.  The weights are
// the reference's bit for bit; only the order of the additions differs.
// ------------------------------------------------------------------------
template <int G>
__global__ void __launch_bounds__(kFastThreads) fast_attention_kernel(KvLayout kv, StepBuffers sb,
                                                                      int layer, int splits) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  extern __shared__ __align__(16) uint8_t smem[];
  const int hd = kv.head_dim, tpc = sb.fast_tpc;
  int8_t* s_kq = reinterpret_cast<int8_t*>(smem);                           // [tpc][hd]
  int8_t* s_vq = s_kq + (size_t)tpc * hd;                                   // [tpc][hd]
  float* s_ks = reinterpret_cast<float*>(s_vq + (size_t)tpc * hd);          // [tpc]
  float* s_vs = s_ks + tpc;                                                 // [tpc]
  float* s_e = s_vs + tpc;                                                  // [G][tpc]
  float* s_f = s_e + (size_t)G * tpc;                                       // [G][tpc]
  float* s_q = s_f + (size_t)G * tpc;                                       // [G][hd]
  float* s_o = s_q + (size_t)G * hd;                                        // [G][hd]
  __shared__ float s_R[G], s_F[G], s_L[G];
  __shared__ int s_valid[256];
  const int KV = kv.n_kv_heads, H = kv.n_heads;
  const int s = (int)cl.block_rank(), g = blockIdx.x / splits, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool mk = tid == 0 && b == 0 && layer == 1 && blockIdx.x == 0;
  (void)mk;
  FAST_MARK(mk, 10);
  pdl_launch_dependents();
  pdl_wait();
  FAST_MARK(mk, 11);
  const int pos = step_pos(sb, b);
  const int n_tok = min(pos + 1, kv.max_blocks * kBlk);
  const int nb = (n_tok + kBlk - 1) / kBlk;
  __shared__ int s_blk[kFastMaxSel];  // physical blocks of the visiting order
  __shared__ int s_lb[kFastMaxSel];   // and their logical indices
  __shared__ int s_nsel;
  if (warp == 0) {
    // the count and the whole list at once (one round trip)
    const int* selp = sb.selp + (long)b * sb.max_sel;
    const int* sel = sb.sel + (long)b * sb.max_sel;
    const int n = __ldcg(sb.nsel + b);
    for (int i = lane; i < min(kFastMaxSel, sb.max_sel); i += 32) {
      s_blk[i] = __ldcg(selp + i);
      s_lb[i] = __ldcg(sel + i);
    }
    if (lane == 0) s_nsel = n;
  }
  __syncthreads();
  FAST_MARK(mk, 12);
  const int nsel = s_nsel;
  const int bps = (nsel + splits - 1) / splits;  // blocks per split
  const int k0 = s * bps, k1 = min(nsel, k0 + bps);
  const int T = k1 > k0 ? (k1 - k0) * kBlk : 0;
  const int pieces = hd >> 4;
  // this split's K and V rows (K rows keep their rotation), scales, and the
  // group's queries: asynchronous 16-byte copies, all in flight at once
  for (int e = tid; e < T * pieces; e += kFastThreads) {
    const int tt = e / pieces, pc = e - tt * pieces;
    const long row = ((long)s_blk[k0 + (tt >> 4)] * KV + g) * kBlk + (tt & 15);
    cp_async16(s_kq + (size_t)tt * hd + pc * 16, kv.kq + row * hd + pc * 16);
    cp_async16(s_vq + (size_t)tt * hd + pc * 16, kv.vq + row * hd + pc * 16);
  }
  for (int e = tid; e < (k1 - k0) * 8; e += kFastThreads) {
    const int kb = e >> 3, part = e & 7;  // 4 x 16 B of K scales, then of V scales
    const long row = ((long)s_blk[k0 + kb] * KV + g) * kBlk + (part & 3) * 4;
    if (part < 4)
      cp_async16(s_ks + kb * kBlk + (part & 3) * 4, kv.ks + row);
    else
      cp_async16(s_vs + kb * kBlk + (part & 3) * 4, kv.vs + row);
  }
  const float* qg = sb.qrot + (long)b * H * hd + (long)g * G * hd;
  for (int i = tid; i < G * hd / 4; i += kFastThreads) cp_async16(s_q + 4 * i, qg + 4 * i);
  for (int tt = tid; tt < T; tt += kFastThreads) {
    const int lbk = s_lb[k0 + (tt >> 4)];
    s_valid[tt] = lbk < nb - 1 || lbk * kBlk + (tt & 15) < n_tok;  // the last block may be partial
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  FAST_MARK(mk, 13);
  for (int tt = tid; tt < T; tt += kFastThreads)
    if (!s_valid[tt]) s_vs[tt] = 0.0f;  // past the last token: weight 0 times a finite value
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  // scores: simd_dot_f32_f32(q, k * scale_t) in its 8-lane order (lane l
  // takes elements l, l + 8, ...), then hsum, then * 1/sqrt(hd)
  for (int i = tid; i < G * T; i += kFastThreads) {
    const int h = i / T, tt = i - h * T, t = tt & 15;
    if (!s_valid[tt]) {
      s_e[h * tpc + tt] = -INFINITY;
      continue;
    }
    const uint8_t* kr = reinterpret_cast<const uint8_t*>(s_kq + (size_t)tt * hd);
    const float* q = s_q + h * hd;
    const float ksc = s_ks[tt];
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = 0.0f;
    for (int c = 0; c < pieces; c++) {
      const uint4 u = *reinterpret_cast<const uint4*>(kr + (((c + t) & (pieces - 1)) << 4));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      const float* qc = q + 16 * c;
#pragma unroll
      for (int e = 0; e < 16; e++) {
        const float kd = __fmul_rn((float)(int8_t)((w[e >> 2] >> (8 * (e & 3))) & 0xff), ksc);
        acc[e & 7] = __fmaf_rn(qc[e], kd, acc[e & 7]);
      }
    }
    s_e[h * tpc + tt] = __fmul_rn(hsum8(acc), scale);
  }
  __syncthreads();
  // the max of this split's scores, per head
  for (int h = warp; h < G; h += kFastThreads / 32) {
    float mx = -INFINITY;
    for (int tt = lane; tt < T; tt += 32) mx = fmaxf(mx, s_e[h * tpc + tt]);
    mx = warp_max(mx);
    if (lane == 0) s_R[h] = mx;
  }
  FAST_MARK(mk, 14);
  cl.sync();
  FAST_MARK(mk, 15);
  // per head (one warp): the running max entering this split, then e_t and
  // f_t in visiting order (lane j takes a contiguous chunk), the suffix
  // products W_t = e_t * prod_{u > t} f_u, F_s and the sum of W_t
  for (int h = warp; h < G; h += kFastThreads / 32) {
    float P = -INFINITY;
    for (int r = 0; r < s; r++) {
      const float* Rr = cl.map_shared_rank(s_R, r);
      const float v = Rr[h];
      P = v > P ? v : P;
    }
    const int cs = (T + 31) >> 5;
    const int t0 = min(T, lane * cs), t1 = min(T, t0 + cs);
    float* es = s_e + h * tpc;
    float* fs = s_f + h * tpc;
    float cm = -INFINITY;
    for (int tt = t0; tt < t1; tt++) cm = es[tt] > cm ? es[tt] : cm;
    // exclusive prefix max over the lanes, seeded with P
    float incl = cm;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = v > incl ? v : incl;
    }
    float prev = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) prev = -INFINITY;
    prev = prev > P ? prev : P;
    if (s == 0 && lane == 0) prev = -INFINITY;
    float cp = 1.0f;  // product of this chunk's f
    for (int tt = t0; tt < t1; tt++) {
      if (!s_valid[tt]) {
        es[tt] = 0.0f;
        fs[tt] = 1.0f;
        continue;
      }
      const float sc = es[tt];
      const float m = sc > prev ? sc : prev;
      const float f = fast_expf(__fsub_rn(prev, m));
      es[tt] = fast_expf(__fsub_rn(sc, m));
      fs[tt] = f;
      cp = __fmul_rn(cp, f);
      prev = m;
    }
    // exclusive suffix product of the chunk products over the lanes
    float sx = cp;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float v = __shfl_down_sync(0xffffffffu, sx, o);
      if (lane + o < 32) sx = __fmul_rn(sx, v);
    }
    float run = __shfl_down_sync(0xffffffffu, sx, 1);
    if (lane == 31) run = 1.0f;
    float lsum = 0.0f;
    for (int tt = t1 - 1; tt >= t0; tt--) {
      const float w = __fmul_rn(es[tt], run);
      es[tt] = w;
      lsum = __fadd_rn(lsum, w);
      run = __fmul_rn(run, fs[tt]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum = __fadd_rn(lsum, __shfl_xor_sync(0xffffffffu, lsum, o));
    const float Fs = __shfl_sync(0xffffffffu, sx, 0);
    if (lane == 0) {
      s_F[h] = Fs;
      s_L[h] = lsum;
    }
  }
  __syncthreads();
  // partial outputs o_s[h][d] = sum_t W_t * (v_t[d] * scale_t)
  for (int i = tid; i < G * hd; i += kFastThreads) {
    const int h = i / hd, d = i - h * hd;
    const float* w = s_e + h * tpc;
    float o = 0.0f;
    for (int tt = 0; tt < T; tt++)
      o = __fmaf_rn(__fmul_rn((float)s_vq[(size_t)tt * hd + d], s_vs[tt]), w[tt], o);
    s_o[i] = o;
  }
  FAST_MARK(mk, 16);
  cl.sync();
  FAST_MARK(mk, 17);
  // merge in visiting order: o = o * F_s + o_s; CTA s writes its slice of
  // the head dimensions
  const int dq = hd / splits;
  for (int i = tid; i < G * dq; i += kFastThreads) {
    const int h = i / dq, d = s * dq + (i - h * dq);
    // every peer's values first (independent remote loads), then the merge
    float Fv[kFastMaxSplits], Lv[kFastMaxSplits], Ov[kFastMaxSplits];
#pragma unroll
    for (int r = 0; r < kFastMaxSplits; r++)
      if (r < splits) {
        Fv[r] = cl.map_shared_rank(s_F, r)[h];
        Lv[r] = cl.map_shared_rank(s_L, r)[h];
        Ov[r] = cl.map_shared_rank(s_o, r)[h * hd + d];
      }
    float o = 0.0f, l = 0.0f;
#pragma unroll
    for (int r = 0; r < kFastMaxSplits; r++)
      if (r < splits) {
        o = __fadd_rn(__fmul_rn(o, Fv[r]), Ov[r]);
        l = __fadd_rn(__fmul_rn(l, Fv[r]), Lv[r]);
      }
    if (l > 0.0f) o = __fmul_rn(o, __fdiv_rn(1.0f, l));
    sb.att[(long)b * H * hd + (long)(g * G + h) * hd + d] = o;
  }
  FAST_MARK(mk, 18);
  cl.sync();  // peers' shared memory stays alive until every read is done
}

template <typename K, typename... Args>
static cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              bool pdl, int cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    n++;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

size_t fast_attention_smem(int tpc, int hd, int G) {
  return (size_t)tpc * hd * 2 + (size_t)tpc * 8 + (size_t)G * tpc * 8 + (size_t)G * hd * 8;
}

int fast_splits(int B) { return B < 4 ? 8 : 4; }

bool fast_attention_supported(const KvLayout& kv, int sparse_blocks_k) {
  const int G = kv.n_heads / kv.n_kv_heads;
  return kv.paged && kv.head_dim <= 128 && kv.head_dim >= 32 && kv.n_kv_heads <= 8 &&
         kv.n_heads * kv.head_dim <= 8192 &&
         (G == 1 || G == 2 || G == 4 || G == 8) && sparse_blocks_k <= kFastMaxSel &&
         kv.max_blocks <= 2048;
}

cudaError_t launch_fast_select(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                               int layer, int B, cudaStream_t s, bool pdl) {
  return launch_pdl(fast_select_kernel, dim3(B), dim3(kFastThreads),
                    fast_select_smem(kv.n_heads, kv.n_kv_heads, kv.head_dim), s, pdl, 1, kv, lsh,
                    sb, layer);
}

cudaError_t launch_fast_attend(const KvLayout& kv, StepBuffers sb, int layer, int B,
                               cudaStream_t s, bool pdl) {
  const int splits = fast_splits(B);
  const int G = kv.n_heads / kv.n_kv_heads;
  sb.fast_tpc = (kFastMaxSel + splits - 1) / splits * kBlk;
  const size_t smem = fast_attention_smem(sb.fast_tpc, kv.head_dim, G);
  const dim3 grid(kv.n_kv_heads * splits, B), block(kFastThreads);
  switch (G) {
    case 1: return launch_pdl(fast_attention_kernel<1>, grid, block, smem, s, pdl, splits, kv, sb, layer, splits);
    case 2: return launch_pdl(fast_attention_kernel<2>, grid, block, smem, s, pdl, splits, kv, sb, layer, splits);
    case 4: return launch_pdl(fast_attention_kernel<4>, grid, block, smem, s, pdl, splits, kv, sb, layer, splits);
    case 8: return launch_pdl(fast_attention_kernel<8>, grid, block, smem, s, pdl, splits, kv, sb, layer, splits);
  }
  return cudaErrorInvalidValue;
}

cudaError_t fast_attention_prepare(const KvLayout& kv) {
  const int G = kv.n_heads / kv.n_kv_heads;
  const int smem = (int)fast_attention_smem(16 * kBlk, kv.head_dim, G);
  cudaError_t e = cudaFuncSetAttribute(
      fast_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
      (int)fast_select_smem(kv.n_heads, kv.n_kv_heads, kv.head_dim));
  if (!e) e = cudaFuncSetAttribute(fast_attention_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (!e) e = cudaFuncSetAttribute(fast_attention_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (!e) e = cudaFuncSetAttribute(fast_attention_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (!e) e = cudaFuncSetAttribute(fast_attention_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return e;
}

}  // namespace ec
