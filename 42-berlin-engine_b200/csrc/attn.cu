// attn.cu -- per-layer KV append (RoPE, INT8 quantisation, block centroid, LSH
// index update), LSH-routed top-K selection, and online-softmax decode
// attention, each reproducing the reference's arithmetic order.
//
// Reference path (src/inference/inference.c:141-513):
//   RoPE q,k  -> paged_kv_append (quant per token & KV head, centroid at block
//   full) or BF16 linear append -> lsh_update (layer 0, KV head 0) ->
//   [linear: window + LSH candidates -> scores -> min-heap top-K] ->
//   [paged: > SPARSE_BLOCKS_K blocks -> centroid scores -> first+last+top-K]
//   -> flash-v1 online softmax per head over the selected tokens.
//
// The online softmax is a recurrence; to stay bit-exact it is kept sequential
// per (head, output dim), but everything around it runs in parallel: scores,
// the running max (a max-scan), both exponentials per token, and the
// denominator chain in its own warp.
#include <cfloat>
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

// Phase timestamps for performance work (build with -DEC_PHASE_TIMING):
// slot s of g_phase_ts gets %globaltimer when one thread passes mark s.
#ifdef EC_PHASE_TIMING
__device__ long long g_phase_ts[64];
#define PHASE_MARK(cond, s)                                                 \
  do {                                                                      \
    if (cond) {                                                             \
      long long t_;                                                         \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));               \
      g_phase_ts[s] = t_;                                                   \
    }                                                                       \
  } while (0)
#else
#define PHASE_MARK(cond, s) \
  do {                      \
  } while (0)
#endif

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// quant_f32_to_int8 (ops_quant.c:229-273) of one vector of n <= 256 floats by
// one warp.  Returns the scale.
__device__ float warp_quant_int8(const float* in, int8_t* out, int n, int lane, int rot = -1) {
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

// ------------------------------------------------------------------------
// KV append: one CTA per sequence.
// ------------------------------------------------------------------------
__device__ void paged_select_cta(const KvLayout& kv, const StepBuffers& sb, int layer, int b);

__global__ void __launch_bounds__(256) kv_append_kernel(KvLayout kv, LshLayout lsh, StepBuffers sb,
                                                        int layer) {
  const int b = blockIdx.y;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim, half = hd >> 1;
  pdl_launch_dependents();
  pdl_wait();
  if (blockIdx.x == 1) {
    paged_select_cta(kv, sb, layer, b);
    return;
  }
  const int pos = step_pos(sb, b);
  const float* q = sb.qkv + (long)b * (H + 2 * KV) * hd;
  float* qo = sb.qrot + (long)b * H * hd;
  float* k = sb.qkv + (long)b * (H + 2 * KV) * hd + H * hd;
  float* v = k + KV * hd;

  // RoPE (rope_apply_multihead_cached, ops_rope.c:192-231); no-op past the table
  if (pos < kv.seq_len) {
    const float* cr = sb.rope_cos + (long)pos * half;
    const float* sr = sb.rope_sin + (long)pos * half;
    for (int i = tid; i < (H + KV) * half; i += blockDim.x) {
      const int head = i / half, j = i - head * half;
      const float* src = (head < H) ? q + head * hd : k + (head - H) * hd;
      float* dst = (head < H) ? qo + head * hd : k + (head - H) * hd;
      const float c = cr[j], s = sr[j], v0 = src[j], v1 = src[j + half];
      dst[j] = __fmaf_rn(v0, c, -__fmul_rn(v1, s));
      dst[j + half] = __fmaf_rn(v0, s, __fmul_rn(v1, c));
    }
  } else {
    for (int i = tid; i < H * hd; i += blockDim.x) qo[i] = q[i];
  }
  __syncthreads();

  if (kv.paged) {
    const int lb = pos / kBlk, off = pos - lb * kBlk;
    if (lb < kv.max_blocks) {
      const long base = ((long)b * kv.n_layers + layer) * kv.max_blocks;
      const long blk = base + kv.page_table[base + lb];
      for (int h = warp; h < 2 * KV; h += nwarps) {
        const bool isv = h >= KV;
        const int kh = isv ? h - KV : h;
        int8_t* dst = (isv ? kv.vq : kv.kq) + ((blk * KV + kh) * kBlk + off) * hd;
        const float sc = warp_quant_int8((isv ? v : k) + kh * hd, dst, hd, lane, isv ? -1 : off);
        if (lane == 0) (isv ? kv.vs : kv.ks)[(blk * KV + kh) * kBlk + off] = sc;
      }
      __syncthreads();
      if (off == kBlk - 1) {
        // calc_block_centroid_int8 (paged.c:350-393): KV head 0 mean
        for (int d = tid; d < hd; d += blockDim.x) {
          float c = 0.0f;
          for (int t = 0; t < kBlk; t++)
            c = __fadd_rn(c, __fmul_rn((float)kv.kq[((blk * KV) * kBlk + t) * hd + kswz(t, d, hd)],
                                       kv.ks[(blk * KV) * kBlk + t]));
          kv.centroid[blk * hd + d] = __fmul_rn(c, __fdiv_rn(1.0f, (float)kBlk));
        }
      }
    }
  } else if (pos < kv.seq_len) {
    // kv_cache_append with F32 -> BF16 (kv_cache.c:55-75)
    const long row = (((long)b * kv.n_layers + layer) * kv.seq_len + pos) * KV * hd;
    for (int i = tid; i < KV * hd; i += blockDim.x) {
      kv.lk[row + i] = f32_to_bf16(k[i]);
      kv.lv[row + i] = f32_to_bf16(v[i]);
    }
  }

  // lsh_update (ops_lsh.c:296-349), layer 0, KV head 0 key
  if (layer == 0 && lsh.tables > 0) {
    float* acc = lsh.acc + (long)b * hd;
    int* meta = lsh.meta + b * 4;
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
          lsh.unit_start[(long)b * lsh.max_units + nu] = meta[1];
          lsh.unit_len[(long)b * lsh.max_units + nu] = count;
          for (int t = 0; t < lsh.tables; t++) {
            const long tb = (long)b * lsh.tables + t;
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
  }
}

// ------------------------------------------------------------------------
// Linear-mode selection (inference.c:228-423): one CTA per sequence.
// sel[b] receives the top-K positions in the reference's heap order.
// ------------------------------------------------------------------------
__device__ __forceinline__ float dot_bf16_ref(const uint16_t* a, const float* b, int n) {
  float acc[8];
#pragma unroll
  for (int l = 0; l < 8; l++) acc[l] = 0.0f;
  int i = 0;
  for (; i + 7 < n; i += 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(a + i);
    float w[8];
    dec_bf16x2(u.x, w);
    dec_bf16x2(u.y, w + 2);
    dec_bf16x2(u.z, w + 4);
    dec_bf16x2(u.w, w + 6);
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = __fmaf_rn(w[l], b[i + l], acc[l]);
  }
  float s = __fadd_rn(0.0f, hsum8(acc));
  for (; i < n; i++) s = __fmaf_rn(bf16_to_f32(a[i]), b[i], s);
  return s;
}

// Min-heap replay of heap_push (ops_heap.h:40-100) on shared arrays.
// Stored 1-based (node n at [n], children 2n, 2n+1 adjacent) so a level of
// sift-down reads both children with one 8-byte load; the element being
// placed is carried in registers ("hole" sifting).  Comparisons are the
// reference's: sift-up stops when parent <= value; sift-down picks the left
// child unless the right one is strictly smaller, and moves on only while the
// chosen child is strictly smaller than the value.
__device__ __forceinline__ void heap_up(float* hs, int* hi, int n, float v, int vi) {
  while (n > 1) {
    const int p = n >> 1;
    const float ps = hs[p];
    if (ps <= v) break;
    hs[n] = ps;
    hi[n] = hi[p];
    n = p;
  }
  hs[n] = v;
  hi[n] = vi;
}

__device__ __forceinline__ void heap_down(float* hs, int* hi, int size, float v, int vi) {
  int n = 1;
  for (;;) {
    const int l = 2 * n;
    if (l > size) break;
    int c = l;
    float cs;
    if (l + 1 <= size) {
      const float2 pr = *reinterpret_cast<const float2*>(hs + l);
      cs = pr.x;
      if (pr.y < pr.x) {
        c = l + 1;
        cs = pr.y;
      }
    } else {
      cs = hs[l];
    }
    if (!(cs < v)) break;
    hs[n] = cs;
    hi[n] = hi[c];
    n = c;
  }
  hs[n] = v;
  hi[n] = vi;
}

// Replays heap_push over (score[i], idx[i]) i < n with capacity cap, by one
// warp: a ballot drops candidates that cannot beat the current root (the
// root only grows), lane 0 performs the pushes that can.  hs/hi hold cap + 2
// entries (1-based, hs 8-byte aligned).  The result, in the reference's heap
// array order, is hi[1 .. size].  idx == nullptr means candidate i carries
// index i + idx_base.
__device__ int warp_heap_topk(const float* score, const int* idx, int n, int cap, float* hs,
                              int* hi, int lane, int idx_base = 0) {
  int size = 0;
  float root = -FLT_MAX;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const float sv = (i < n) ? score[i] : 0.0f;
    const int iv = (i < n) ? (idx ? idx[i] : i + idx_base) : 0;
    unsigned pend = __ballot_sync(0xffffffffu, i < n);
    if (size >= cap) pend &= __ballot_sync(0xffffffffu, sv > root);
    while (pend) {
      const int L = __ffs(pend) - 1;
      const float sL = __shfl_sync(0xffffffffu, sv, L);
      const int iL = __shfl_sync(0xffffffffu, iv, L);
      if (lane == 0) {
        if (size < cap)
          heap_up(hs, hi, size + 1, sL, iL);
        else if (sL > hs[1])
          heap_down(hs, hi, size, sL, iL);
      }
      __syncwarp();
      if (size < cap) size++;
      root = hs[1];
      pend &= ~(1u << L);
      if (size >= cap) pend &= __ballot_sync(0xffffffffu, sv > root);
    }
  }
  return size;
}

__global__ void __launch_bounds__(256) linear_select_kernel(KvLayout kv, LshLayout lsh,
                                                            StepBuffers sb, int layer) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim;
  const int cap_c = sb.window + lsh.max_cand * lsh.unit;  // candidate capacity
  int* cand = reinterpret_cast<int*>(smem);               // [cap_c]
  float* cscore = reinterpret_cast<float*>(cand + cap_c);  // [cap_c]
  float* hs = cscore + cap_c;                             // [sparse_k + 2], 1-based
  int* hi = reinterpret_cast<int*>(hs + sb.sparse_k + 2);  // [sparse_k + 2]
  float* qm = reinterpret_cast<float*>(hi + sb.sparse_k + 2);  // [hd]
  __shared__ uint32_t s_code[16];
  __shared__ int s_units[64];
  __shared__ int s_nu, s_nc, s_wcount;
  __shared__ unsigned s_seen[4096 / 32];
  pdl_launch_dependents();
  pdl_wait();
  const int pos = step_pos(sb, b);
  const int kv_len = min(pos + 1, kv.seq_len);
  const float* q = sb.qrot + (long)b * H * hd;
  if (!(sb.sparse_k > 0 && kv_len > sb.sparse_k)) {
    if (tid == 0) sb.nsel[b] = -1;  // dense attention over [0, kv_len)
    return;
  }
  const int ws = kv_len > sb.window ? kv_len - sb.window : 0;
  const int* meta = lsh.meta + b * 4;
  const int n_units = meta[2];
  if (tid == 0) s_nu = 0;
  __syncthreads();
  if (ws > 0 && n_units > 0 && lsh.tables > 0) {
    // q_mean over all heads (inference.c:290-295)
    for (int d = tid; d < hd; d += blockDim.x) {
      float a = 0.0f;
      for (int h = 0; h < H; h++) a = __fadd_rn(a, q[h * hd + d]);
      qm[d] = __fdiv_rn(a, (float)H);
    }
    if (tid < 16) s_code[tid] = 0;
    for (int i = tid; i < lsh.max_units / 32 + 1 && i < 4096 / 32; i += blockDim.x) s_seen[i] = 0;
    __syncthreads();
    for (int tb = tid; tb < lsh.tables * lsh.bits; tb += blockDim.x) {
      const int t = tb / lsh.bits, hbit = tb - t * lsh.bits;
      const float* hp = lsh.hp + ((long)t * lsh.bits + hbit) * hd;
      float a = 0.0f;
      for (int d = 0; d < hd; d++) a = __fmaf_rn(qm[d], hp[d], a);
      if (a > 0.0f) atomicOr(&s_code[t], 1u << hbit);
    }
    __syncthreads();
    if (tid == 0) {
      // lsh_find_candidates (ops_lsh.c:361-418), table after table
      int n = 0;
      const int maxc = lsh.max_cand < 64 ? lsh.max_cand : 64;
      for (int t = 0; t < lsh.tables && n < maxc; t++) {
        const long tb = (long)b * lsh.tables + t;
        const uint32_t qh = s_code[t];
        for (int p = 0; p <= lsh.bits && n < maxc; p++) {
          const uint32_t probe = (p == 0) ? qh : (qh ^ (1u << (p - 1)));
          int id = lsh.heads[(tb << lsh.bits) + probe];
          while (id != -1 && n < maxc) {
            const uint32_t hh = lsh.unit_hash[tb * lsh.max_units + id];
            if (__popc(qh ^ hh) <= lsh.radius && !(s_seen[id >> 5] & (1u << (id & 31)))) {
              s_seen[id >> 5] |= 1u << (id & 31);
              s_units[n++] = id;
            }
            id = lsh.next[tb * lsh.max_units + id];
          }
        }
      }
      // keep units that end before the window, ordered by start position
      int m = 0;
      for (int i = 0; i < n; i++) {
        const int u = s_units[i];
        const int st = lsh.unit_start[(long)b * lsh.max_units + u];
        const int ln = lsh.unit_len[(long)b * lsh.max_units + u];
        if (st + ln <= ws) {
          int j = m++;
          while (j > 0 && lsh.unit_start[(long)b * lsh.max_units + s_units[j - 1]] > st) {
            s_units[j] = s_units[j - 1];
            j--;
          }
          s_units[j] = u;
        }
      }
      s_nu = m;
    }
    __syncthreads();
  }
  if (tid == 0) {
    int n = 0;
    for (int i = 0; i < s_nu; i++) {
      const int u = s_units[i];
      const int st = lsh.unit_start[(long)b * lsh.max_units + u];
      const int ln = lsh.unit_len[(long)b * lsh.max_units + u];
      for (int p = 0; p < ln && n < cap_c; p++)
        if (st + p < ws) cand[n++] = st + p;
    }
    s_wcount = n;
  }
  __syncthreads();
  {
    const int n0 = s_wcount;
    for (int i = tid; i < kv_len - ws && n0 + i < cap_c; i += blockDim.x) cand[n0 + i] = ws + i;
    if (tid == 0) s_nc = min(n0 + (kv_len - ws), cap_c);
  }
  __syncthreads();
  const int nc = s_nc;
  // candidate scores (inference.c:341-353)
  const int grp = H / KV;
  const long lrow = ((long)b * kv.n_layers + layer) * kv.seq_len;
  for (int i = tid; i < nc; i += blockDim.x) {
    const uint16_t* kr = kv.lk + (lrow + cand[i]) * KV * hd;
    float s = 0.0f;
    for (int kh = 0; kh < KV; kh++) s = __fadd_rn(s, dot_bf16_ref(kr + kh * hd, q + kh * grp * hd, hd));
    cscore[i] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const int cap = nc < sb.sparse_k ? nc : sb.sparse_k;
    const int size = warp_heap_topk(cscore, cand, nc, cap, hs, hi, lane);
    int* out = sb.sel + (long)b * sb.max_sel;
    for (int i = lane; i < size; i += 32) out[i] = hi[i + 1];
    if (lane == 0) {
      sb.nsel[b] = size;
      lsh.counters[b * 2] += 1ull;
      lsh.counters[b * 2 + 1] += (unsigned long long)size;
    }
  }
}

// heap_push over score[0..n) (indices i + idx_base) with capacity cap, by
// one thread; result hi[1..size] in the reference's heap array order.
__device__ int heap_topk_seq(const float* score, int n, int cap, float* hs, int* hi,
                             int idx_base) {
  int size = 0;
  int i = 0;
  for (; i < n && size < cap; i++) heap_up(hs, hi, ++size, score[i], i + idx_base);
  float root = size ? hs[1] : 0.0f;
#pragma unroll 4
  for (; i < n; i++) {
    const float s = score[i];
    if (s > root) {
      heap_down(hs, hi, size, s, i + idx_base);
      root = hs[1];
    }
  }
  return size;
}

// ------------------------------------------------------------------------
// Paged block selection (inference.c:447-469): with more than
// SPARSE_BLOCKS_K blocks, score_blocks (paged.c:401-431, query head 0 .
// centroid) and select_top_k_blocks (paged.c:439-495: first, last, then
// heap_push of blocks 1..nb-2, heap array order).  Only full middle blocks
// are scored, so this runs concurrently with this step's append.  Writes
// sel[b] / nsel[b] (nsel = -1: attend to every block).
// ------------------------------------------------------------------------
__device__ void paged_select_cta(const KvLayout& kv, const StepBuffers& sb, int layer, int b) {
  constexpr int kChunkBlocks = 32;  // centroids staged per round (16 KB at hd 128)
  __shared__ __align__(16) float s_q[256];
  __shared__ __align__(16) float s_c[2 * kChunkBlocks * 128];
  __shared__ int s_nsel;
  __shared__ __align__(16) float s_bsc[2048];
  __shared__ __align__(16) float s_hs[68];
  __shared__ int s_hi[68];
  __shared__ __align__(8) uint64_t s_bar[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim, half = hd >> 1;
  if (!kv.paged) return;
  const int pos = step_pos(sb, b);
  const int n_tok = min(pos + 1, kv.max_blocks * kBlk);
  const int nb = (n_tok + kBlk - 1) / kBlk;
  if (nb <= sb.sparse_blocks_k || nb > 2048 || hd > 128) {
    // every block in order (listed explicitly when asked to, same result)
    const bool list = sb.list_dense && nb <= sb.max_sel;
    if (list) {
      int* out = sb.sel + (long)b * sb.max_sel;
      for (int i = tid; i < nb; i += blockDim.x) out[i] = i;
    }
    if (tid == 0) sb.nsel[b] = list ? nb : -1;
    return;
  }
  PHASE_MARK(tid == 0 && layer == 1, 0);
  if (tid == 0) {
    mbar_init(&s_bar[0], 1);
    mbar_init(&s_bar[1], 1);
    fence_mbar_init();
  }
  // query head 0, rotated here (the append CTA rotates its own copy)
  const float* q = sb.q_rotated ? sb.qrot + (long)b * H * hd : sb.qkv + (long)b * (H + 2 * KV) * hd;
  for (int j = tid; j < half; j += blockDim.x) {
    const float v0 = q[j], v1 = q[j + half];
    if (pos < kv.seq_len && !sb.q_rotated) {
      const float c = sb.rope_cos[(long)pos * half + j], s = sb.rope_sin[(long)pos * half + j];
      s_q[j] = __fmaf_rn(v0, c, -__fmul_rn(v1, s));
      s_q[j + half] = __fmaf_rn(v0, s, __fmul_rn(v1, c));
    } else {
      s_q[j] = v0;
      s_q[j + half] = v1;
    }
  }
  __syncthreads();
  const long base = ((long)b * kv.n_layers + layer) * kv.max_blocks;
  const int* pt = kv.page_table + base;
  // score_blocks over the middle blocks 1 .. nb-2: centroids staged in rounds
  // of kChunkBlocks (double-buffered); 8 threads per block run the 8 lanes of
  // simd_dot_f32_f32 and combine them in its horizontal-sum order
  const int nmid = nb - 2;
  const int nround = (nmid + kChunkBlocks - 1) / kChunkBlocks;
  auto issue = [&](int r) {
    const int c0 = 1 + r * kChunkBlocks;
    const int cn = min(kChunkBlocks, nb - 1 - c0);
    float* dst = s_c + (r & 1) * kChunkBlocks * 128;
    if (lane == 0) mbar_expect_tx(&s_bar[r & 1], (uint32_t)(cn * hd * 4));
    __syncwarp();
    for (int i = lane; i < cn; i += 32)
      bulk_g2s(dst + i * hd, kv.centroid + (base + pt[c0 + i]) * hd, hd * 4, &s_bar[r & 1]);
  };
  if (warp == 0) issue(0);
  bool ok = true;
  for (int r = 0; r < nround; r++) {
    if (warp == 0 && r + 1 < nround) issue(r + 1);
    if (ok) ok = mbar_wait(&s_bar[r & 1], (r >> 1) & 1, sb.err);
    const int c0 = 1 + r * kChunkBlocks;
    const int cn = min(kChunkBlocks, nb - 1 - c0);
    const float* cb = s_c + (r & 1) * kChunkBlocks * 128;
    const int blk = tid >> 3, l = tid & 7;
    float acc = 0.0f;
    if (blk < cn && ok)
      for (int d = l; d < hd; d += 8) acc = __fmaf_rn(s_q[d], cb[blk * hd + d], acc);
    // ((c0+c4)+(c1+c5)) + ((c2+c6)+(c3+c7))
    const float h4 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
    const float t2 = __fadd_rn(h4, __shfl_xor_sync(0xffffffffu, h4, 1));
    const float sum = __fadd_rn(t2, __shfl_xor_sync(0xffffffffu, t2, 2));
    if (blk < cn && l == 0) s_bsc[c0 + blk] = sum;
    __syncthreads();
  }
  int m = sb.sparse_blocks_k - 2;
  if (m > nb - 2) m = nb - 2;
  if (m > 62) m = 62;
  PHASE_MARK(tid == 0 && layer == 1, 1);
  if (tid == 0) {
    const int size = heap_topk_seq(s_bsc + 1, nmid, m, s_hs, s_hi, 1);
    PHASE_MARK(true && layer == 1, 2);
    s_nsel = size;
  }
  __syncthreads();
  if (warp == 0) {
    const int size = s_nsel;
    int* out = sb.sel + (long)b * sb.max_sel;
    if (lane == 0) {
      out[0] = 0;
      out[1] = nb - 1;
      sb.nsel[b] = 2 + size;
    }
    for (int i = lane; i < size; i += 32) out[2 + i] = s_hi[1 + i];
  }
}

// ------------------------------------------------------------------------
// Attention: one CTA per (query head, sequence).
//   1. the selected K rows (paged blocks in selection order, or linear-mode
//      positions) land in shared memory by bulk copies issued by one warp;
//      scores in the reference's dot order;
//   2. running max by a max-scan, both exponentials per token in parallel;
//   3. V rows land in the same buffer; threads 0..hd-1 run the output
//      recurrence for one dimension each, the next warp the denominator.
// ------------------------------------------------------------------------
constexpr int kAttnThreads = 512;

struct AttnSmemLayout {
  size_t kv, sc, sf, tks, tvs, lpos, boff, bphys, bfill, ksb, vsb, total;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline AttnSmemLayout attn_layout(int max_tok, int hd, int esize) {
  AttnSmemLayout L;
  const int nblk = max_tok / 16 + 4;  // selected blocks (partial last block included)
  size_t o = 256 * 4;  // q head
  L.kv = o;
  o = align_up(o + (size_t)max_tok * hd * esize, 16);
  L.sc = o;
  o += (size_t)max_tok * 4;
  L.sf = o;
  o += (size_t)max_tok * 4;
  L.tks = o;
  o += (size_t)max_tok * 4;
  L.tvs = o;
  o += (size_t)max_tok * 4;
  L.lpos = o;
  o += (size_t)max_tok * 4;
  L.boff = o;
  o += nblk * 4;
  L.bphys = o;
  o += nblk * 4;
  L.bfill = o;
  o += nblk * 4;
  o = align_up(o, 16);
  L.ksb = o;
  o += nblk * 16 * 4;
  L.vsb = o;
  o += nblk * 16 * 4;
  L.total = o;
  return L;
}

// stored int8 byte -> exact float of its signed value
__device__ __forceinline__ float s8_to_f32(uint32_t byte) {
  return __fsub_rn(__uint_as_float(byte ^ 0x4B000080u), 8388736.0f);
}

template <bool PAGED>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(KvLayout kv, StepBuffers sb,
                                                                 int layer, int max_tok) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int ES = PAGED ? 1 : 2;
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim;
  const int kvh = h / (H / KV);
  const AttnSmemLayout Ly = attn_layout(max_tok, hd, ES);
  float* qs = reinterpret_cast<float*>(smem);
  uint8_t* kvb = smem + Ly.kv;
  float* sc = reinterpret_cast<float*>(smem + Ly.sc);
  float* sf = reinterpret_cast<float*>(smem + Ly.sf);
  float* tks = reinterpret_cast<float*>(smem + Ly.tks);
  float* tvs = reinterpret_cast<float*>(smem + Ly.tvs);
  int* lpos = reinterpret_cast<int*>(smem + Ly.lpos);
  uint8_t* ttok = reinterpret_cast<uint8_t*>(lpos);  // paged: token index within its block
  int* boff = reinterpret_cast<int*>(smem + Ly.boff);
  int* bphys = reinterpret_cast<int*>(smem + Ly.bphys);
  int* bfill = reinterpret_cast<int*>(smem + Ly.bfill);
  float* ksb = reinterpret_cast<float*>(smem + Ly.ksb);
  float* vsb = reinterpret_cast<float*>(smem + Ly.vsb);
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ int s_ntok, s_nsel;
  __shared__ float s_wmax[kAttnThreads / 32];
  __shared__ float s_sum;
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  pdl_launch_dependents();
  pdl_wait();
  const bool mk = (h == 0 && b == 0 && layer == 1);
  (void)mk;
  PHASE_MARK(mk && tid == 0, 8);
  const int pos = step_pos(sb, b);
  const float* qg = sb.qrot + (long)b * H * hd;
  for (int d = tid; d < hd; d += blockDim.x) qs[d] = qg[h * hd + d];
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  bool ok = true;

  // ------------------------------------------ selected blocks / positions
  if constexpr (PAGED) {
    const int n_tok = min(pos + 1, kv.max_blocks * kBlk);
    const int nb = (n_tok + kBlk - 1) / kBlk;
    const long base = ((long)b * kv.n_layers + layer) * kv.max_blocks;
    const int* pt = kv.page_table + base;
    const int ns = sb.nsel[b];
    const int* sel = sb.sel + (long)b * sb.max_sel;
    const int nsel = ns > 0 ? ns : nb;  // selection order, or every block in order
    for (int k = tid; k < nsel; k += blockDim.x) {
      const int lb = ns > 0 ? sel[k] : k;
      bphys[k] = (int)(base + pt[lb]);
      bfill[k] = (lb == nb - 1) ? n_tok - lb * kBlk : kBlk;
    }
    __syncthreads();
    if (tid == 0) {
      int n = 0;
      for (int k = 0; k < nsel; k++) {
        boff[k] = n;
        n += bfill[k];
      }
      s_ntok = n;
      s_nsel = nsel;
    }
    __syncthreads();
    const int T = s_ntok;
    // K rows and both scale vectors of every selected block
    if (warp == 0) {
      if (lane == 0) mbar_expect_tx(&bar[0], (uint32_t)(T * hd + nsel * 2 * 64));
      __syncwarp();
      for (int k = lane; k < nsel; k += 32) {
        const long blk = bphys[k];
        bulk_g2s(kvb + (size_t)boff[k] * hd, kv.kq + ((blk * KV + kvh) * kBlk) * hd,
                 bfill[k] * hd, &bar[0]);
        bulk_g2s(ksb + k * 16, kv.ks + (blk * KV + kvh) * kBlk, 64, &bar[0]);
        bulk_g2s(vsb + k * 16, kv.vs + (blk * KV + kvh) * kBlk, 64, &bar[0]);
      }
    }
    ok = mbar_wait(&bar[0], 0, sb.err);
    for (int j = tid; j < nsel * kBlk; j += blockDim.x) {
      const int k = j >> 4, t = j & 15;
      if (t < bfill[k]) {
        tks[boff[k] + t] = ksb[j];
        tvs[boff[k] + t] = vsb[j];
        ttok[boff[k] + t] = (uint8_t)t;
      }
    }
  } else {
    const int kv_len = min(pos + 1, kv.seq_len);
    const int ns = sb.nsel[b];
    const int* sel = sb.sel + (long)b * sb.max_sel;
    const bool sparse = ns > 0 && ns < kv_len;
    const int T = sparse ? ns : kv_len;
    for (int i = tid; i < T; i += blockDim.x) lpos[i] = sparse ? sel[i] : i;
    if (tid == 0) s_ntok = T;
    __syncthreads();
    const long lrow = ((long)b * kv.n_layers + layer) * kv.seq_len;
    if (warp == 0) {
      if (lane == 0) mbar_expect_tx(&bar[0], (uint32_t)(T * hd * 2));
      __syncwarp();
      for (int i = lane; i < T; i += 32)
        bulk_g2s(kvb + (size_t)i * hd * 2, kv.lk + ((lrow + lpos[i]) * KV + kvh) * hd, hd * 2,
                 &bar[0]);
    }
    ok = mbar_wait(&bar[0], 0, sb.err);
  }
  __syncthreads();
  const int T = s_ntok;
  PHASE_MARK(mk && tid == 0, 9);

  // ------------------------------------------------------------- scores
  for (int i = tid; i < T && ok; i += blockDim.x) {
    float s;
    if constexpr (PAGED) {
      // piece c of this token's row sits at (c + t) mod np (stored rotated)
      const uint8_t* kr = kvb + (size_t)i * hd;
      const int t = ttok[i];
      const float ksc = tks[i];
      const int np = hd >> 4;
      float acc[8];
#pragma unroll
      for (int l = 0; l < 8; l++) acc[l] = 0.0f;
#pragma unroll
      for (int c = 0; c < 8; c++) {
        if (c >= np) break;
        const uint4 u = *reinterpret_cast<const uint4*>(kr + (((c + t) & (np - 1)) << 4));
        float w[16];
        dec_i8x4(u.x, w);
        dec_i8x4(u.y, w + 4);
        dec_i8x4(u.z, w + 8);
        dec_i8x4(u.w, w + 12);
#pragma unroll
        for (int l = 0; l < 16; l++)
          acc[l & 7] = __fmaf_rn(qs[16 * c + l], __fmul_rn(w[l], ksc), acc[l & 7]);
      }
      s = hsum8(acc);
    } else {
      s = dot_bf16_ref(reinterpret_cast<const uint16_t*>(kvb) + (size_t)i * hd, qs, hd);
    }
    sc[i] = __fmul_rn(s, scale);
  }
  __syncthreads();
  PHASE_MARK(mk && tid == 0, 10);
  // V rows into the same buffer (K is no longer needed)
  if (warp == 0 && ok) {
    if constexpr (PAGED) {
      const int nsel = s_nsel;
      if (lane == 0) mbar_expect_tx(&bar[1], (uint32_t)(T * hd));
      __syncwarp();
      for (int k = lane; k < nsel; k += 32)
        bulk_g2s(kvb + (size_t)boff[k] * hd, kv.vq + (((long)bphys[k] * KV + kvh) * kBlk) * hd,
                 bfill[k] * hd, &bar[1]);
    } else {
      const long lrow = ((long)b * kv.n_layers + layer) * kv.seq_len;
      if (lane == 0) mbar_expect_tx(&bar[1], (uint32_t)(T * hd * 2));
      __syncwarp();
      for (int i = lane; i < T; i += 32)
        bulk_g2s(kvb + (size_t)i * hd * 2, kv.lv + ((lrow + lpos[i]) * KV + kvh) * hd, hd * 2,
                 &bar[1]);
    }
  }
  // running max m_t = max(m_{t-1}, s_t) (exact), then the two exponentials
  {
    const int per = (T + blockDim.x - 1) / blockDim.x;
    const int lo = tid * per, hi = min(lo + per, T);
    float m = -INFINITY;
    for (int i = lo; i < hi; i++) m = (sc[i] > m) ? sc[i] : m;
    float incl = m;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = (t > incl) ? t : incl;
    }
    if (lane == 31) s_wmax[warp] = incl;
    __syncthreads();
    float pre = -INFINITY;
    for (int w = 0; w < warp; w++) pre = (s_wmax[w] > pre) ? s_wmax[w] : pre;
    float excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = -INFINITY;
    float run = (excl > pre) ? excl : pre;
    for (int i = lo; i < hi; i++) {
      const float s = sc[i];
      const float prev = run;
      run = (s > prev) ? s : prev;
      sf[i] = fast_expf(__fsub_rn(prev, run));
      sc[i] = fast_expf(__fsub_rn(s, run));  // raw_exp
    }
  }
  __syncthreads();
  // flag per 8 tokens: every scale factor is 1 (the running max did not move)
  int* ones = reinterpret_cast<int*>(tks);  // K scales are no longer needed
  for (int g = tid; g < (T >> 3); g += blockDim.x) {
    bool a1 = true;
#pragma unroll
    for (int u = 0; u < 8; u++) a1 = a1 && (sf[8 * g + u] == 1.0f);
    ones[g] = a1;
  }
  __syncthreads();
  PHASE_MARK(mk && tid == 0, 11);
  if (ok) ok = mbar_wait(&bar[1], 0, sb.err);
  PHASE_MARK(mk && tid == 0, 12);

  // -------------------------------------------------------- recurrences
  // out_t = fma(re_t, v_t, out_{t-1} * sf_t); with sf_t == 1 the multiply is
  // the identity and runs of eight such steps skip it.
  const int cw = (hd + 31) >> 5;  // chain warps
  if (warp == cw) {
    if (lane == 0) {
      float sum = 0.0f;
      int i = 0;
      for (; i + 8 <= T; i += 8) {
        const float4 f0 = *reinterpret_cast<const float4*>(sf + i);
        const float4 f1 = *reinterpret_cast<const float4*>(sf + i + 4);
        const float4 r0 = *reinterpret_cast<const float4*>(sc + i);
        const float4 r1 = *reinterpret_cast<const float4*>(sc + i + 4);
        sum = __fmaf_rn(sum, f0.x, r0.x);
        sum = __fmaf_rn(sum, f0.y, r0.y);
        sum = __fmaf_rn(sum, f0.z, r0.z);
        sum = __fmaf_rn(sum, f0.w, r0.w);
        sum = __fmaf_rn(sum, f1.x, r1.x);
        sum = __fmaf_rn(sum, f1.y, r1.y);
        sum = __fmaf_rn(sum, f1.z, r1.z);
        sum = __fmaf_rn(sum, f1.w, r1.w);
      }
      for (; i < T; i++) sum = __fmaf_rn(sum, sf[i], sc[i]);
      s_sum = sum;
    }
  } else if (tid < hd && ok) {
    const int d = tid;
    float o = 0.0f;
    // one group of 8 tokens: raw exps, dequantised values, all-ones flag;
    // the next group is loaded before the current one's FMA chain runs
    auto load = [&](int i, float* r, float* vv, int& fl) {
      const float4 r0 = *reinterpret_cast<const float4*>(sc + i);
      const float4 r1 = *reinterpret_cast<const float4*>(sc + i + 4);
      r[0] = r0.x; r[1] = r0.y; r[2] = r0.z; r[3] = r0.w;
      r[4] = r1.x; r[5] = r1.y; r[6] = r1.z; r[7] = r1.w;
      if constexpr (PAGED) {
        const float4 s0 = *reinterpret_cast<const float4*>(tvs + i);
        const float4 s1 = *reinterpret_cast<const float4*>(tvs + i + 4);
        const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int u = 0; u < 8; u++) vv[u] = __fmul_rn(s8_to_f32(kvb[(size_t)(i + u) * hd + d]), sv[u]);
      } else {
#pragma unroll
        for (int u = 0; u < 8; u++)
          vv[u] = bf16_to_f32(reinterpret_cast<const uint16_t*>(kvb)[(size_t)(i + u) * hd + d]);
      }
      fl = ones[i >> 3];
    };
    int i = 0;
    if (T >= 8) {
      float rn[8], vn[8];
      int fn;
      load(0, rn, vn, fn);
      for (; i + 8 <= T; i += 8) {
        float r[8], vv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
          r[u] = rn[u];
          vv[u] = vn[u];
        }
        const int fl = fn;
        if (i + 16 <= T) load(i + 8, rn, vn, fn);
        if (fl) {
#pragma unroll
          for (int u = 0; u < 8; u++) o = __fmaf_rn(r[u], vv[u], o);
        } else {
          const float4 f0 = *reinterpret_cast<const float4*>(sf + i);
          const float4 f1 = *reinterpret_cast<const float4*>(sf + i + 4);
          const float f[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
          for (int u = 0; u < 8; u++) o = __fmaf_rn(r[u], vv[u], __fmul_rn(o, f[u]));
        }
      }
    }
    for (; i < T; i++) {
      float vv;
      if constexpr (PAGED)
        vv = __fmul_rn(s8_to_f32(kvb[(size_t)i * hd + d]), tvs[i]);
      else
        vv = bf16_to_f32(reinterpret_cast<const uint16_t*>(kvb)[(size_t)i * hd + d]);
      o = __fmaf_rn(sc[i], vv, __fmul_rn(o, sf[i]));
    }
    qs[d] = o;  // q no longer needed
    PHASE_MARK(mk && d == 0, 13);
  }
  PHASE_MARK(mk && warp == cw && lane == 0, 14);
  __syncthreads();
  if (tid < hd) {
    float o = qs[tid];
    const float sum = s_sum;
    if (sum > 0.0f) o = __fmul_rn(o, __fdiv_rn(1.0f, sum));
    sb.att[(long)b * H * hd + h * hd + tid] = o;
  }
}

static int attn_max_tok(const KvLayout& kv, const StepBuffers& sb) {
  if (kv.paged) return kBlk * sb.sparse_blocks_k;
  return sb.sparse_k > 0 ? sb.sparse_k : kv.seq_len;
}

static size_t attn_smem(const KvLayout& kv, const StepBuffers& sb, int max_tok) {
  (void)sb;
  return attn_layout(max_tok, kv.head_dim, kv.paged ? 1 : 2).total;
}

template <typename K, typename... Args>
static cudaError_t launch_ex(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// paged_kv_append of one token into a one-layer view (k, v already rotated).
__global__ void __launch_bounds__(256) paged_append_view_kernel(KvLayout kv, const float* k,
                                                                const float* v, int pos) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int KV = kv.n_kv_heads, hd = kv.head_dim;
  const int lb = pos / kBlk, off = pos - lb * kBlk;
  if (lb >= kv.max_blocks) return;
  const long blk = kv.page_table[lb];
  for (int h = warp; h < 2 * KV; h += nwarps) {
    const bool isv = h >= KV;
    const int kh = isv ? h - KV : h;
    int8_t* dst = (isv ? kv.vq : kv.kq) + ((blk * KV + kh) * kBlk + off) * hd;
    const float sc = warp_quant_int8((isv ? v : k) + kh * hd, dst, hd, lane, isv ? -1 : off);
    if (lane == 0) (isv ? kv.vs : kv.ks)[(blk * KV + kh) * kBlk + off] = sc;
  }
  __syncthreads();
  if (off == kBlk - 1) {
    for (int d = tid; d < hd; d += blockDim.x) {
      float c = 0.0f;
      for (int t = 0; t < kBlk; t++)
        c = __fadd_rn(c, __fmul_rn((float)kv.kq[((blk * KV) * kBlk + t) * hd + kswz(t, d, hd)],
                                   kv.ks[(blk * KV) * kBlk + t]));
      kv.centroid[blk * hd + d] = __fmul_rn(c, __fdiv_rn(1.0f, (float)kBlk));
    }
  }
}

__global__ void __launch_bounds__(256) paged_select_kernel(KvLayout kv, StepBuffers sb) {
  paged_select_cta(kv, sb, 0, blockIdx.y);
}

#ifdef EC_PHASE_TIMING
extern "C" int ec_debug_phase_times(long long* out) {
  return cudaMemcpyFromSymbol(out, g_phase_ts, sizeof(g_phase_ts)) == cudaSuccess ? 0 : -2;
}
#endif

// Opt a kernel into the largest dynamic shared memory it can take: the
// per-block limit less its own static shared memory.
template <typename K>
cudaError_t opt_in_max_smem(K kernel) {
  cudaFuncAttributes a;
  cudaError_t e = cudaFuncGetAttributes(&a, kernel);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              227 * 1024 - (int)a.sharedSizeBytes);
}

cudaError_t attn_prepare(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb) {
  const int max_tok = attn_max_tok(kv, sb);
  const int smem = (int)attn_smem(kv, sb, max_tok);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  // the largest opt-in: per-op calls share these kernels with other sizes
  cudaError_t e = opt_in_max_smem(attention_kernel<true>);
  if (!e) e = opt_in_max_smem(attention_kernel<false>);
  const int cap_c = sb.window + lsh.max_cand * lsh.unit;
  const int ssel = cap_c * 8 + (sb.sparse_k + 2) * 8 + 256 * 4;
  if (!e && ssel <= 227 * 1024)
    e = cudaFuncSetAttribute(linear_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ssel);
  return e;
}

cudaError_t launch_paged_append_view(const KvLayout& kv, const float* k, const float* v, int pos,
                                     int* err, cudaStream_t s) {
  (void)err;
  paged_append_view_kernel<<<1, 256, 0, s>>>(kv, k, v, pos);
  return cudaGetLastError();
}

cudaError_t launch_paged_select(const KvLayout& kv, const StepBuffers& sb, cudaStream_t s) {
  paged_select_kernel<<<dim3(1, 1), 256, 0, s>>>(kv, sb);
  return cudaGetLastError();
}

size_t attention_smem_bytes(int max_tok, int hd, bool paged) {
  return attn_layout(max_tok, hd, paged ? 1 : 2).total;
}

cudaError_t launch_attention_n(const KvLayout& kv, const StepBuffers& sb, int max_tok,
                               cudaStream_t s) {
  const size_t smem = attention_smem_bytes(max_tok, kv.head_dim, kv.paged != 0);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = opt_in_max_smem(attention_kernel<true>);
  if (e != cudaSuccess) return e;
  return launch_ex(attention_kernel<true>, dim3(kv.n_heads, 1), dim3(kAttnThreads), smem, s, false,
                   kv, sb, 0, max_tok);
}

cudaError_t launch_kv_append(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                             int layer, int B, cudaStream_t s, bool pdl) {
  return launch_ex(kv_append_kernel, dim3(kv.paged ? 2 : 1, B), dim3(256), 0, s, pdl, kv, lsh, sb,
                   layer);
}

cudaError_t launch_linear_select(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                                 int layer, int B, cudaStream_t s, bool pdl) {
  const int cap_c = sb.window + lsh.max_cand * lsh.unit;
  const size_t smem = (size_t)cap_c * 8 + (size_t)(sb.sparse_k + 2) * 8 + 256 * 4;
  return launch_ex(linear_select_kernel, dim3(B), dim3(256), smem, s, pdl, kv, lsh, sb, layer);
}

cudaError_t launch_attention(const KvLayout& kv, const StepBuffers& sb, int layer, int B,
                             cudaStream_t s, bool pdl) {
  const int max_tok = attn_max_tok(kv, sb);
  const size_t smem = attn_smem(kv, sb, max_tok);
  if (kv.paged) {
    return launch_ex(attention_kernel<true>, dim3(kv.n_heads, B), dim3(kAttnThreads), smem, s, pdl,
                     kv, sb, layer, max_tok);
  }
  return launch_ex(attention_kernel<false>, dim3(kv.n_heads, B), dim3(kAttnThreads), smem, s, pdl,
                   kv, sb, layer, max_tok);
}

}  // namespace ec
