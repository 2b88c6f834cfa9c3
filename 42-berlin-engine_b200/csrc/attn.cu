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
#include <cooperative_groups.h>

#include "attn.cuh"
#include "select.cuh"
#include "ec_internal.cuh"
#include "kv_common.cuh"

namespace ec {

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

// ------------------------------------------------------------------------
// KV append: one CTA per sequence.
// ------------------------------------------------------------------------
__device__ void paged_select_cta(const KvLayout& kv, const StepBuffers& sb, int layer, int b);

__global__ void __launch_bounds__(256, 4) kv_append_kernel(KvLayout kv, LshLayout lsh, StepBuffers sb,
                                                        int layer) {
  const int b = blockIdx.y;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim, half = hd >> 1;
  pdl_launch_dependents();
  if (blockIdx.x == 1) {
    // waits for the previous kernel itself, after loads that do not depend on it
    paged_select_cta(kv, sb, layer, b);
    PHASE_MARK(tid == 0 && layer == 1 && b == 0, 3);
    return;
  }
  pdl_wait();
  PHASE_MARK(tid == 0 && layer == 1 && b == 0, 4);
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
      const long base = ((long)kv_seq(kv, b) * kv.n_layers + layer) * kv.max_blocks;
      const long blk = base + kv.page_table[base + lb];
      for (int h = warp; h < 2 * KV; h += nwarps) {
        const bool isv = h >= KV;
        const int kh = isv ? h - KV : h;
        int8_t* dst = (isv ? kv.vq : kv.kq) + ((blk * KV + kh) * kBlk + off) * hd;
        const float sc = warp_quant_int8((isv ? v : k) + kh * hd, dst, hd, lane, isv ? -1 : off);
        if (lane == 0) (isv ? kv.vs : kv.ks)[(blk * KV + kh) * kBlk + off] = sc;
      }
      __syncthreads();
      if (off == kBlk - 1 && !sb.defer_centroid) block_centroid(kv, blk, tid, blockDim.x);
    }
  } else if (pos < kv.seq_len) {
    // kv_cache_append with F32 -> BF16 (kv_cache.c:55-75)
    const long row = (((long)kv_seq(kv, b) * kv.n_layers + layer) * kv.seq_len + pos) * KV * hd;
    for (int i = tid; i < KV * hd; i += blockDim.x) {
      kv.lk[row + i] = f32_to_bf16(k[i]);
      kv.lv[row + i] = f32_to_bf16(v[i]);
    }
  }

  // lsh_update (ops_lsh.c:296-349), layer 0, KV head 0 key.  Prefill rows
  // are tokens of one sequence: lsh_update_rows_kernel applies them in order.
  if (layer == 0 && lsh.tables > 0 && !kv.seq_plus1) lsh_update_token(lsh, b, k, pos, hd);
  PHASE_MARK(tid == 0 && layer == 1 && b == 0, 6);
}

// ------------------------------------------------------------------------
// Linear-mode selection (inference.c:228-423) in three launches: candidates
// (one CTA per sequence: LSH query hash, lsh_find_candidates, window),
// scores (CTAs over candidates x KV heads), heap (one warp per sequence).
// sel[b] receives the top-K positions in the reference's heap order.
// ------------------------------------------------------------------------
__global__ void __launch_bounds__(256) linear_cand_kernel(KvLayout kv, LshLayout lsh,
                                                          StepBuffers sb, int layer) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int H = kv.n_heads, hd = kv.head_dim;
  const int cap_c = linear_cand_cap(sb, lsh);             // candidate capacity
  int* cand = sb.lcand + (long)b * cap_c;                  // [cap_c], global
  float* qm = reinterpret_cast<float*>(smem);              // [hd]
  __shared__ uint32_t s_code[16];
  __shared__ int s_units[64];
  __shared__ int s_nu, s_nc, s_wcount;
  __shared__ int s_uoff[64], s_ust[64], s_ulen[64];
  __shared__ unsigned s_seen[4096 / 32];
  pdl_launch_dependents();
  pdl_wait();
  const int pos = step_pos(sb, b);
  const int kv_len = min(pos + 1, kv.seq_len);
  // every query head (tensor parallelism: all ranks' heads, gathered)
  const int Hq = sb.q_all ? sb.h_all : H;
  const float* q = sb.q_all ? sb.q_all + (long)b * Hq * hd : sb.qrot + (long)b * H * hd;
  if (!(sb.sparse_k > 0 && kv_len > sb.sparse_k)) {
    if (tid == 0) {
      sb.nsel[b] = -1;  // dense attention over [0, kv_len)
      sb.lnc[b] = 0;
    }
    return;
  }
  const int ws = kv_len > sb.window ? kv_len - sb.window : 0;
  // the sequence whose index this row queries (prefill: every row's)
  const int sq = kv_seq(kv, b);
  const int* meta = lsh.meta + sq * 4;
  const int* ustart = lsh.unit_start + (long)sq * lsh.max_units;
  const int* ulen = lsh.unit_len + (long)sq * lsh.max_units;
  // A unit enters the index with its last token (lsh_update); a prefill row
  // at `pos` sees the index as decode would: units that end by `pos`
  // (units are added in position order, so unit 0 is the first to exist).
  const int n_units = meta[2] > 0 && ustart[0] + ulen[0] - 1 <= pos ? meta[2] : 0;
  if (tid == 0) s_nu = 0;
  __syncthreads();
  if (ws > 0 && n_units > 0 && lsh.tables > 0) {
    // q_mean over all heads (inference.c:290-295)
    for (int d = tid; d < hd; d += blockDim.x) {
      float a = 0.0f;
      for (int h = 0; h < Hq; h++) a = __fadd_rn(a, q[h * hd + d]);
      qm[d] = __fdiv_rn(a, (float)Hq);
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
        const long tb = (long)sq * lsh.tables + t;
        const uint32_t qh = s_code[t];
        for (int p = 0; p <= lsh.bits && n < maxc; p++) {
          const uint32_t probe = (p == 0) ? qh : (qh ^ (1u << (p - 1)));
          int id = lsh.heads[(tb << lsh.bits) + probe];
          while (id != -1 && n < maxc) {
            const uint32_t hh = lsh.unit_hash[tb * lsh.max_units + id];
            // units added after this row's token did not exist yet: skipped
            // without counting, the chain below them is as it was
            if (ustart[id] + ulen[id] - 1 <= pos && __popc(qh ^ hh) <= lsh.radius &&
                !(s_seen[id >> 5] & (1u << (id & 31)))) {
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
        const int st = ustart[u];
        const int ln = ulen[u];
        if (st + ln <= ws) {
          int j = m++;
          while (j > 0 && ustart[s_units[j - 1]] > st) {
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
  // the units' tokens before the window, in unit order (offsets by thread 0,
  // the copies by one warp per unit)
  if (tid == 0) {
    int n = 0;
    for (int i = 0; i < s_nu; i++) {
      const int u = s_units[i];
      const int st = ustart[u];
      const int ln = ulen[u];
      int take = ws - st < ln ? ws - st : ln;
      if (take < 0) take = 0;
      if (take > cap_c - n) take = cap_c - n;
      s_uoff[i] = n;
      s_ust[i] = st;
      s_ulen[i] = take;
      n += take;
    }
    s_wcount = n;
  }
  __syncthreads();
  for (int i = tid >> 5; i < s_nu; i += blockDim.x >> 5)
    for (int p = tid & 31; p < s_ulen[i]; p += 32) cand[s_uoff[i] + p] = s_ust[i] + p;
  {
    const int n0 = s_wcount;
    for (int i = tid; i < kv_len - ws && n0 + i < cap_c; i += blockDim.x) cand[n0 + i] = ws + i;
    if (tid == 0) s_nc = min(n0 + (kv_len - ws), cap_c);
  }
  __syncthreads();
  if (tid == 0) sb.lnc[b] = s_nc;
}

// Candidate scores (inference.c:341-353): thread (candidate, KV head) runs
// simd_dot_bf16_f32 of the candidate's key row with the group's first query
// head; the candidate's score adds the heads' dots in head order.
__global__ void __launch_bounds__(256) linear_score_kernel(KvLayout kv, StepBuffers sb, int layer,
                                                           int cap_c) {
  __shared__ float part[256];
  const int b = blockIdx.y, tid = threadIdx.x;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim, grp = H / KV;
  pdl_launch_dependents();
  pdl_wait();
  const int nc = sb.lnc[b];
  const int cpb = 256 / KV;  // candidates per CTA
  const int c = blockIdx.x * cpb + tid / KV, kh = tid % KV;
  if (blockIdx.x * cpb >= nc) return;
  const bool live = tid < cpb * KV && c < nc;
  const float* q = sb.qrot + (long)b * H * hd;
  const long lrow = ((long)(kv.shared_cache ? 0 : kv_seq(kv, b)) * kv.n_layers + layer) * kv.seq_len;
  if (live) {
    const int pos = sb.lcand[(long)b * cap_c + c];
    part[tid] = dot_bf16_ref(kv.lk + ((lrow + pos) * KV + kh) * hd, q + kh * grp * hd, hd);
  }
  __syncthreads();
  if (sb.score_parts) {
    // tensor parallelism: this rank's heads' dots, summed after the gather
    if (live) sb.score_parts[((long)b * cap_c + c) * KV + kh] = part[tid];
    return;
  }
  if (live && kh == 0) {
    float sc = 0.0f;
    for (int h = 0; h < KV; h++) sc = __fadd_rn(sc, part[tid + h]);
    sb.lscore[(long)b * cap_c + c] = sc;
  }
}

// Tensor parallelism: the candidate scores from every rank's per-head dots
// (parts_all [world][B][cap][kv_local], ranks holding consecutive KV heads),
// added in global head order from 0 as linear_score_kernel does.
__global__ void tp_sum_scores_kernel(StepBuffers sb, const float* __restrict__ parts_all,
                                     int world, int kv_local, int cap_c, int B) {
  const int b = blockIdx.y;
  const int nc = sb.lnc[b];
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < nc; c += gridDim.x * blockDim.x) {
    float sc = 0.0f;
    for (int r = 0; r < world; r++)
      for (int h = 0; h < kv_local; h++)
        sc = __fadd_rn(sc, parts_all[(((long)r * B + b) * cap_c + c) * kv_local + h]);
    sb.lscore[(long)b * cap_c + c] = sc;
  }
}

__global__ void lsh_update_key_kernel(LshLayout lsh, StepBuffers sb, const float* k, int hd) {
  lsh_update_token(lsh, 0, k, step_pos(sb, 0), hd);
}

// The top-K of the scored candidates (heap_push, inference.c:356-423): one
// warp per sequence replays the heap; sel[b] receives the positions in the
// reference's heap array order.
__global__ void __launch_bounds__(32) linear_heap_kernel(LshLayout lsh, StepBuffers sb,
                                                         int cap_c, int seq_plus1) {
  __shared__ __align__(16) uint2 hp[1024];  // heap nodes, 1-based
  const int b = blockIdx.x, lane = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const int nc = sb.lnc[b];
  if (nc <= 0) return;  // dense attention (nsel = -1 already)
  const int cap = nc < sb.sparse_k ? nc : sb.sparse_k;
  auto all = [](int) { return true; };
  const float* cscore = sb.lscore + (long)b * cap_c;
  const int* cand = sb.lcand + (long)b * cap_c;
  const int size = cap < 64 ? warp_heap_select<6>(cscore, cand, 0, nc, cap, hp, lane, all)
                            : warp_heap_select<9>(cscore, cand, 0, nc, cap, hp, lane, all);
  int* out = sb.sel + (long)b * sb.max_sel;
  for (int i = lane; i < size; i += 32) out[i] = (int)hp[i + 1].y;
  if (lane == 0) {
    // prefill rows of one sequence share its counters
    const int sq = seq_plus1 ? seq_plus1 - 1 : b;
    sb.nsel[b] = size;
    atomicAdd(&lsh.counters[sq * 2], 1ull);
    atomicAdd(&lsh.counters[sq * 2 + 1], (unsigned long long)size);
  }
}

// ------------------------------------------------------------------------
// Paged block selection (inference.c:447-469): with more than
// SPARSE_BLOCKS_K blocks, score_blocks (paged.c:401-431, query head 0 .
// centroid) and select_top_k_blocks (paged.c:439-495: first, last, then
// heap_push of blocks 1..nb-2, heap array order).  Only full middle blocks
// are scored, so this runs concurrently with this step's append.  Writes
// sel[b] / nsel[b] (nsel = -1: attend to every block).
//
// Warps 1..7 score the centroids in rounds, publishing how many are done;
// warp 0 replays the heap over the scores as they arrive.  256 threads.
// ------------------------------------------------------------------------
__device__ void paged_select_cta(const KvLayout& kv, const StepBuffers& sb, int layer, int b) {
  constexpr int kScorers = 224;
  __shared__ __align__(16) float s_q[128];
  __shared__ __align__(16) float s_bsc[2048];
  __shared__ __align__(16) uint2 s_hp[128];
  __shared__ int s_ready;  // middle-block scores [0, s_ready) are written
  __shared__ int s_nsel;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim, half = hd >> 1;
  if (!kv.paged) return;
  const int pos = step_pos(sb, b);
  const int n_tok = min(pos + 1, kv.max_blocks * kBlk);
  const int nb = (n_tok + kBlk - 1) / kBlk;
  if (nb <= sb.sparse_blocks_k || nb > 2048 || hd > 128) {
    // every block in order (listed explicitly when asked to, same result)
    pdl_wait();
    const bool list = sb.list_dense && nb <= sb.max_sel;
    if (list) {
      int* out = sb.sel + (long)b * sb.max_sel;
      for (int i = tid; i < nb; i += blockDim.x) out[i] = i;
    }
    if (tid == 0) sb.nsel[b] = list ? nb : -1;
    return;
  }
  // Page table and centroids of the full middle blocks were written in
  // earlier steps, not by the kernel this one follows: pull the centroids
  // into L2 before waiting for it (griddepcontrol.wait), while the previous
  // layer still runs.
  constexpr int kGroups = kScorers / 8, kU = 3, kD = 16;  // kD: hd / 8 at most
  const long base = ((long)kv_seq(kv, b) * kv.n_layers + layer) * kv.max_blocks;
  const int* pt = kv.page_table + base;
  const int nmid = nb - 2;
  for (int i = tid; i < nmid * (hd >> 5); i += blockDim.x) {
    const int blk = i / (hd >> 5), line = i - blk * (hd >> 5);
    const float* cp = kv.centroid + (base + pt[1 + blk]) * hd + line * 32;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(cp));
  }
  pdl_wait();
  PHASE_MARK(tid == 0 && layer == 1 && b == 0, 5);
  PHASE_MARK(tid == 0 && layer == 1, 0);
  if (tid == 0) s_ready = 0;
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
  int m = sb.sparse_blocks_k - 2;
  if (m > nmid) m = nmid;
  if (m > 62) m = 62;

  if (warp == 0) {
    // ------------------------------------------------------------ heap
    auto ready = [&](int j) -> bool {
      for (uint32_t it = 0; it < kWaitLimit; it++) {
        if (*reinterpret_cast<volatile int*>(&s_ready) > j) {
          __threadfence_block();
          PHASE_MARK(lane == 0 && layer == 1 && b == 0 && (j >> 5) < 16, 16 + (j >> 5));
          return true;
        }
        __nanosleep(32);
      }
      if (lane == 0) atomicCAS(sb.err, 0, EC_ERR_TIMEOUT);
      return false;
    };
    const int size = warp_heap_select<6>(s_bsc, nullptr, 1, nmid, m, s_hp, lane, ready);
    PHASE_MARK(lane == 0 && layer == 1, 2);
    if (lane == 0) s_nsel = size;
  } else {
    // -------------------------------------------- score_blocks
    // 8 threads per block run the 8 lanes of simd_dot_f32_f32 and combine
    // them in its horizontal-sum order.  Each group of 8 scores kU blocks per
    // round straight from global memory (page-table entries first, then every
    // centroid load of the round at once: one memory round trip per round),
    // and the round's scores are published for the heap.
    const int ct = tid - 32, grp = ct >> 3, l = ct & 7, nd = hd >> 3;
    for (int r0 = 0; r0 < nmid; r0 += kGroups * kU) {
      const float* cp[kU];
#pragma unroll
      for (int u = 0; u < kU; u++) {
        const int blk = r0 + grp + u * kGroups;
        cp[u] = blk < nmid ? kv.centroid + (base + pt[1 + blk]) * hd : nullptr;
      }
      float cv[kU][kD];
#pragma unroll
      for (int u = 0; u < kU; u++)
#pragma unroll
        for (int j = 0; j < kD; j++) cv[u][j] = (cp[u] && j < nd) ? __ldcg(cp[u] + l + 8 * j) : 0.0f;
#pragma unroll
      for (int u = 0; u < kU; u++) {
        const int blk = r0 + grp + u * kGroups;
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < kD; j++)
          if (j < nd) acc = __fmaf_rn(s_q[l + 8 * j], cv[u][j], acc);
        // ((c0+c4)+(c1+c5)) + ((c2+c6)+(c3+c7))
        const float h4 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
        const float t2 = __fadd_rn(h4, __shfl_xor_sync(0xffffffffu, h4, 1));
        const float sum = __fadd_rn(t2, __shfl_xor_sync(0xffffffffu, t2, 2));
        if (blk < nmid && l == 0) s_bsc[blk] = sum;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kScorers));  // this round's scores written
      if (ct == 0) {
        __threadfence_block();
        *reinterpret_cast<volatile int*>(&s_ready) = min(nmid, r0 + kGroups * kU);
        PHASE_MARK(layer == 1 && b == 0 && r0 / (kGroups * kU) < 8, 40 + r0 / (kGroups * kU));
      }
    }
    PHASE_MARK(ct == 0 && layer == 1, 1);
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
    for (int i = lane; i < size; i += 32) out[2 + i] = (int)s_hp[1 + i].y;
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
constexpr int kAttnThreads = 256;
constexpr int kSplit = 4;  // CTAs per (query head, sequence): one thread-block cluster

struct AttnSmemLayout {
  size_t sc, sf, tks, tvs, trow, boff, bphys, bfill, vraw, vf, total;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// One CTA of the cluster: all tokens' scores and factors, this CTA's quarter
// of the head dimensions of V (raw and dequantised).
__host__ __device__ inline AttnSmemLayout attn_layout(int max_tok, int hd, int esize,
                                                      bool vf = true) {
  AttnSmemLayout L;
  const int nblk = max_tok / 16 + 4;  // selected blocks (partial last block included)
  const size_t arr = (size_t)(max_tok + 8) * 4;
  const int dq = hd / kSplit;
  size_t o = 128 * 4;  // q head
  L.sc = o;
  o += arr;
  L.sf = o;
  o += arr;
  L.tks = o;
  o += arr;
  L.tvs = o;
  o += arr;
  L.trow = o;
  o += arr;
  L.boff = o;
  o += nblk * 4;
  L.bphys = o;
  o += nblk * 4;
  L.bfill = o;
  o += nblk * 4;
  o = align_up(o, 16);
  L.vraw = o;
  o = align_up(o + (size_t)max_tok * dq * esize, 16);
  L.vf = o;  // transposed: [dq][max_tok + 4] floats (absent without vf)
  if (vf) o += (size_t)(max_tok + 4) * dq * 4;
  L.total = o;
  return L;
}

// stored int8 byte -> exact float of its signed value
__device__ __forceinline__ float s8_to_f32(uint32_t byte) {
  return __fsub_rn(__uint_as_float(byte ^ 0x4B000080u), 8388736.0f);
}

__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}

// Attention for one (query head, sequence) by a cluster of kSplit CTAs:
// op_paged_attention(_sparse) (ops_attention.c:292-461) over the selected
// paged blocks in selection order, or attention_head_sparse
// (ops_attention.c:131-170) over linear-mode positions.
//   1. every CTA builds the token table (block offsets by a warp prefix sum)
//      and starts 16-byte asynchronous copies of ITS quarter of every V row;
//   2. CTA r scores tokens [r*T/4, (r+1)*T/4): K rows straight from global
//      memory, dot in the reference's 8-lane order (paired f32x2, same
//      roundings), times 1/sqrt(hd); each score is stored into all four
//      CTAs' shared memory (distributed shared memory), then a cluster
//      barrier;
//   3. every CTA: running max m_t = max(m_{t-1}, s_t) by a block max-scan,
//      both exponentials per token (fast_expf), its V quarter dequantised;
//   4. one warp runs the output recurrence o_t = fma(e_t, v_t, o_{t-1} * f_t)
//      for the CTA's hd/4 dimensions (the multiply skipped over runs where
//      every f_t is 1), one thread the denominator; out = o * (1/sum).
// Spreading a head over four SMs quarters the bytes each SM must pull.
// VF: dequantise this CTA's V quarter once into a float buffer read by a
// register-pipelined chain (lowest latency, one CTA per SM); without it the
// chain dequantises as it goes, the CTA needs a quarter of the shared memory
// and several CTAs share an SM (batched steps: throughput over latency).
template <bool PAGED, bool VF>
__global__ void __launch_bounds__(kAttnThreads, VF ? 1 : 3)
    attention_kernel(KvLayout kv, StepBuffers sb, int layer, int max_tok) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int ES = PAGED ? 1 : 2;
  const int r = (int)cl.block_rank();
  const int h = blockIdx.x / kSplit, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim;
  const int kvh = h / (H / KV);
  const int dq = hd / kSplit;  // this CTA's dimensions: [r*dq, (r+1)*dq)
  const AttnSmemLayout Ly = attn_layout(max_tok, hd, ES, VF);
  float* qs = reinterpret_cast<float*>(smem);
  float* sc = reinterpret_cast<float*>(smem + Ly.sc);
  float* sf = reinterpret_cast<float*>(smem + Ly.sf);
  float* tks = reinterpret_cast<float*>(smem + Ly.tks);
  float* tvs = reinterpret_cast<float*>(smem + Ly.tvs);
  int* trow = reinterpret_cast<int*>(smem + Ly.trow);  // paged: K/V row; linear: position
  int* boff = reinterpret_cast<int*>(smem + Ly.boff);
  int* bphys = reinterpret_cast<int*>(smem + Ly.bphys);
  int* bfill = reinterpret_cast<int*>(smem + Ly.bfill);
  uint8_t* vraw = smem + Ly.vraw;
  float* vf = reinterpret_cast<float*>(smem + Ly.vf);
  __shared__ __align__(8) uint64_t vbar;
  __shared__ int s_ntok, s_nsel;
  __shared__ float s_wmax[kAttnThreads / 32];
  __shared__ float s_sum;
  if (tid == 0) {
    mbar_init(&vbar, kAttnThreads);  // one cp.async arrival per thread
    fence_mbar_init();
  }
  pdl_launch_dependents();
  pdl_wait();
  const bool mk = (h == 0 && r == 0 && b == 0 && layer == 1);
  (void)mk;
  PHASE_MARK(mk && tid == 0, 8);
  const int pos = step_pos(sb, b);
  const float* qg = sb.qrot + (long)b * H * hd;
  for (int d = tid; d < hd; d += blockDim.x) qs[d] = qg[h * hd + d];
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const long lrow =
      ((long)(kv.shared_cache ? 0 : kv_seq(kv, b)) * kv.n_layers + layer) * kv.seq_len;  // linear

  // ------------------------------------------ selected blocks / positions
  if constexpr (PAGED) {
    const int n_tok = min(pos + 1, kv.max_blocks * kBlk);
    const int nb = (n_tok + kBlk - 1) / kBlk;
    const long base = ((long)kv_seq(kv, b) * kv.n_layers + layer) * kv.max_blocks;
    const int* pt = kv.page_table + base;
    const int ns = sb.nsel[b];
    const int* sel = sb.sel + (long)b * sb.max_sel;
    const int nsel = ns > 0 ? ns : nb;  // selection order, or every block in order
    if (warp == 0) {
      // block table and offsets (exclusive prefix sum of the fills)
      int carry = 0;
      for (int k0 = 0; k0 < nsel; k0 += 32) {
        const int k = k0 + lane;
        int fill = 0;
        if (k < nsel) {
          const int lb = ns > 0 ? sel[k] : k;
          bphys[k] = (int)(base + pt[lb]);
          fill = (lb == nb - 1) ? n_tok - lb * kBlk : kBlk;
          bfill[k] = fill;
        }
        int incl = fill;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        if (k < nsel) boff[k] = carry + incl - fill;
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) {
        s_ntok = carry;
        s_nsel = nsel;
      }
    }
    __syncthreads();
    const int nsl = s_nsel;
    for (int j = tid; j < nsl * kBlk; j += blockDim.x) {
      const int k = j >> 4, t = j & 15;
      if (t < bfill[k]) {
        const int i = boff[k] + t;
        const int row = (bphys[k] * KV + kvh) * kBlk + t;
        trow[i] = row;
        tks[i] = kv.ks[row];
        tvs[i] = kv.vs[row];
      }
    }
  } else {
    const int kv_len = min(pos + 1, kv.seq_len);
    const int ns = sb.nsel[b];
    const int* sel = sb.sel + (long)b * sb.max_sel;
    // list_dense: the list is explicit even when it covers every position
    // (rows of a paged cache, isolated LSH attention)
    const bool sparse = ns > 0 && (ns < kv_len || sb.list_dense);
    const int T = sparse ? ns : kv_len;
    for (int i = tid; i < T; i += blockDim.x) trow[i] = sparse ? sel[i] : i;
    if (tid == 0) s_ntok = T;
  }
  __syncthreads();
  const int T = s_ntok;
  // this CTA's quarter of every V row -> shared memory, completing on vbar
  {
    const int slice = dq * ES;  // bytes: 8, 16, 32 or 64
    const int np = slice >= 16 ? slice >> 4 : 1;
    for (int e = tid; e < T * np; e += blockDim.x) {
      const int i = e / np, pc = e - i * np;
      const uint8_t* row;
      if constexpr (PAGED)
        row = reinterpret_cast<const uint8_t*>(kv.vq) + (size_t)trow[i] * hd;
      else
        row = reinterpret_cast<const uint8_t*>(kv.lv + ((lrow + trow[i]) * KV + kvh) * hd);
      const uint8_t* src = row + r * slice + pc * 16;
      uint8_t* dst = vraw + (size_t)i * slice + pc * 16;
      if (slice >= 16)
        cp_async16(dst, src);
      else
        cp_async8(dst, src);
    }
    cp_async_arrive(&vbar);
  }
  PHASE_MARK(mk && tid == 0, 9);

  // ------------------------------------------- scores of this CTA's quarter
  {
    const int tq = (T + kSplit - 1) / kSplit;
    const int i0 = r * tq, i1 = min(T, i0 + tq);
    float* peer[kSplit];
#pragma unroll
    for (int k = 0; k < kSplit; k++) peer[k] = cl.map_shared_rank(sc, k);
    for (int i = i0 + tid; i < i1; i += blockDim.x) {
      float s;
      if constexpr (PAGED) {
        // piece c of this token's row sits at (c + t) mod np (stored rotated);
        // acc[l & 7] += q[16c + l] * (k[16c + l] * scale_t), l = 0..15
        const int row = trow[i];
        const uint8_t* kr = reinterpret_cast<const uint8_t*>(kv.kq) + (size_t)row * hd;
        const int t = row & (kBlk - 1);
        const float ksc = tks[i];
        const uint64_t ks2 = pack2(__float_as_uint(ksc), __float_as_uint(ksc));
        const int npc = hd >> 4;
        uint4 u[8];
#pragma unroll
        for (int c = 0; c < 8; c++)
          if (c < npc) u[c] = ldg_nc16(kr + (((c + t) & (npc - 1)) << 4));
        uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int c = 0; c < 8; c++) {
          if (c >= npc) break;
          const ulonglong2* q2 = reinterpret_cast<const ulonglong2*>(qs + 16 * c);
          const uint32_t wv[4] = {u[c].x, u[c].y, u[c].z, u[c].w};
#pragma unroll
          for (int g = 0; g < 4; g++) {
            uint64_t w01, w23;
            decode_pairs<EC_W_INT8>(wv[g], w01, w23);
            const ulonglong2 qq = q2[g];
            // elements 4g..4g+3 -> accumulator pairs (2g)&3 and (2g+1)&3
            fma2(acc[(2 * g) & 3], mul2(w01, ks2), qq.x);
            fma2(acc[(2 * g + 1) & 3], mul2(w23, ks2), qq.y);
          }
        }
        float a8[8];
#pragma unroll
        for (int l = 0; l < 4; l++) {
          a8[2 * l] = lo_f(acc[l]);
          a8[2 * l + 1] = hi_f(acc[l]);
        }
        s = hsum8(a8);
      } else {
        s = dot_bf16_ref(kv.lk + ((lrow + trow[i]) * KV + kvh) * hd, qs, hd);
      }
      s = __fmul_rn(s, scale);
#pragma unroll
      for (int k = 0; k < kSplit; k++) peer[k][i] = s;
    }
  }
  cl.sync();  // every CTA holds all T scores
  PHASE_MARK(mk && tid == 0, 10);

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
    if (warp == 0) {
      // exclusive max-prefix over the warps
      const int nw = blockDim.x >> 5;
      float w = lane < nw ? s_wmax[lane] : -INFINITY;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w = (t > w) ? t : w;
      }
      const float ex = __shfl_up_sync(0xffffffffu, w, 1);
      __syncwarp();
      if (lane < nw) s_wmax[lane] = lane == 0 ? -INFINITY : ex;
    }
    __syncthreads();
    const float pre = s_wmax[warp];
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
  // V quarter: v * scale_t, exact, four elements at a time
  bool ok = mbar_wait(&vbar, 0, sb.err);
  // thread -> (token i, dimensions 4g..4g+3) with i fastest, so a warp's
  // transposed stores fall in 32 consecutive words
  const int ng = VF ? dq >> 2 : 0;
  for (int w = tid; w < T * ng && ok; w += blockDim.x) {
    const int g = w / T, i = w - g * T, d = 4 * g;
    uint4 out;
    if constexpr (PAGED) {
      const uint32_t wv = *reinterpret_cast<const uint32_t*>(vraw + (size_t)i * dq + d);
      const float ts = tvs[i];
      const uint64_t s2 = pack2(__float_as_uint(ts), __float_as_uint(ts));
      uint64_t p01, p23;
      decode_pairs<EC_W_INT8>(wv, p01, p23);
      p01 = mul2(p01, s2);
      p23 = mul2(p23, s2);
      out = make_uint4((uint32_t)p01, (uint32_t)(p01 >> 32), (uint32_t)p23, (uint32_t)(p23 >> 32));
    } else {
      const uint2 wv = *reinterpret_cast<const uint2*>(vraw + ((size_t)i * dq + d) * 2);
      out = make_uint4(wv.x << 16, wv.x & 0xFFFF0000u, wv.y << 16, wv.y & 0xFFFF0000u);
    }
    const int ld = max_tok + 4;
    vf[(size_t)d * ld + i] = __uint_as_float(out.x);
    vf[(size_t)(d + 1) * ld + i] = __uint_as_float(out.y);
    vf[(size_t)(d + 2) * ld + i] = __uint_as_float(out.z);
    vf[(size_t)(d + 3) * ld + i] = __uint_as_float(out.w);
  }
  __syncthreads();
  // flag per 32 tokens: every scale factor is 1 (the running max did not move)
  int* ones = reinterpret_cast<int*>(tks);  // K scales are no longer needed
  for (int g = tid; g < (T + 31) >> 5; g += blockDim.x) {
    bool a1 = true;
    for (int u = 0; u < 32 && 32 * g + u < T; u++) a1 = a1 && (sf[32 * g + u] == 1.0f);
    ones[g] = a1;
  }
  __syncthreads();
  PHASE_MARK(mk && tid == 0, 11);

  // -------------------------------------------------------- recurrences
  float o = 0.0f;
  if (warp == 0) {
    // out_t = fma(e_t, v_t, out_{t-1} * f_t) for dimension `lane` (lanes
    // past dq shadow lane % dq and are discarded).  Chunks of 32 tokens live
    // in registers: this lane's v of each token, and e, f of token base+lane
    // (read back by shuffles); the next chunk loads while this one's chain
    // runs.  With f_t == 1 the multiply is the identity: runs of eight such
    // tokens skip it.
    // out_t = fma(e_t, v_t, out_{t-1} * f_t) for dimension `lane` (lanes
    // past dq shadow lane % dq and are discarded).  V is stored transposed,
    // so a lane reads four tokens with one 16-byte load; e and f are
    // broadcast loads.  A chunk of 32 tokens is loaded while the previous
    // one's chain runs; with f_t == 1 the multiply is the identity and runs
    // of four such tokens skip it.
    ok = __all_sync(0xffffffffu, ok);
    if constexpr (!VF) {
      // v_t dequantised in the loop (v * scale_t, exact); o * 1 == o, so the
      // multiply needs no skipping for exactness
      const int dd = lane % dq;
      for (int i = 0; i < T && ok; i++) {
        float v;
        if constexpr (PAGED)
          v = __fmul_rn(s8_to_f32(vraw[(size_t)i * dq + dd]), tvs[i]);
        else
          v = bf16_to_f32(reinterpret_cast<const uint16_t*>(vraw)[(size_t)i * dq + dd]);
        o = __fmaf_rn(sc[i], v, __fmul_rn(o, sf[i]));
      }
    }
    const float* row = vf + (size_t)(lane % dq) * (max_tok + 4);
    float4 va[8], ea[8], vb[8], eb[8];
    auto load = [&](float4* v, float4* e, int base) {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        v[j] = *reinterpret_cast<const float4*>(row + base + 4 * j);
        e[j] = *reinterpret_cast<const float4*>(sc + base + 4 * j);
      }
    };
    auto run = [&](const float4* v, const float4* e, int base) {
      if (ones[base >> 5]) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
          o = __fmaf_rn(e[j].x, v[j].x, o);
          o = __fmaf_rn(e[j].y, v[j].y, o);
          o = __fmaf_rn(e[j].z, v[j].z, o);
          o = __fmaf_rn(e[j].w, v[j].w, o);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float4 f = *reinterpret_cast<const float4*>(sf + base + 4 * j);
          o = __fmaf_rn(e[j].x, v[j].x, __fmul_rn(o, f.x));
          o = __fmaf_rn(e[j].y, v[j].y, __fmul_rn(o, f.y));
          o = __fmaf_rn(e[j].z, v[j].z, __fmul_rn(o, f.z));
          o = __fmaf_rn(e[j].w, v[j].w, __fmul_rn(o, f.w));
        }
      }
    };
    // two register buffers, one loading while the other runs
    const int T32 = (ok && VF) ? (T & ~31) : 0;
    if (T32) load(va, ea, 0);
    for (int base = 0; base < T32; base += 64) {
      if (base + 32 < T32) load(vb, eb, base + 32);
      run(va, ea, base);
      if (base + 32 >= T32) break;
      if (base + 64 < T32) load(va, ea, base + 64);
      run(vb, eb, base + 32);
    }
    for (int i = T32; i < T && ok && VF; i++) o = __fmaf_rn(sc[i], row[i], __fmul_rn(o, sf[i]));
    PHASE_MARK(mk && lane == 0, 13);
  } else if (warp == 1 && lane == 0) {
    // denominator: sum_t = fma(sum_{t-1}, f_t, e_t)
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
    PHASE_MARK(mk, 14);
  }
  __syncthreads();
  if (warp == 0 && lane < dq) {
    const float sum = s_sum;
    if (sum > 0.0f) o = __fmul_rn(o, __fdiv_rn(1.0f, sum));
    sb.att[(long)b * H * hd + h * hd + r * dq + lane] = o;
  }
}

// ------------------------------------------------------------------------
// Batched steps, paged KV: one CTA per (KV head, sequence) computes the
// attention of every query head of the group (op_paged_attention(_sparse),
// ops_attention.c:292-461, per head, bit for bit as attention_kernel):
//   1. token table, K / V scales, and the group's V rows (all head
//      dimensions) copied to shared memory with cp.async;
//   2. each K row is read once and decoded once for all query heads of the
//      group; the dots keep the reference's 8-lane order per head;
//   3. running max per head by a 128-thread max-scan, both exponentials;
//   4. thread d runs dimension d of every query head's output recurrence
//      o_t = fma(e_t, v_t, o_{t-1} * f_t), dequantising each V element once
//      for all of them; thread 0 also runs the denominators.
// 128 threads per query head of the group; hd of them run recurrences.
struct GroupSmemLayout {
  size_t qs, sc, sf, tks, tvs, trow, boff, bphys, bfill, ones, vraw, total;
  int ld;
};

__host__ __device__ inline GroupSmemLayout group_layout(int max_tok, int hd, int hpg) {
  GroupSmemLayout L;
  L.ld = (max_tok + 31) / 32 * 32 + 32;
  const int nblk = max_tok / 16 + 4;
  size_t o = 0;
  L.qs = o;
  o += (size_t)hpg * hd * 4;
  L.sc = o;
  o += (size_t)hpg * L.ld * 4;
  L.sf = o;
  o += (size_t)hpg * L.ld * 4;
  L.tks = o;
  o += (size_t)L.ld * 4;
  L.tvs = o;
  o += (size_t)L.ld * 4;
  L.trow = o;
  o += (size_t)L.ld * 4;
  L.boff = o;
  o += nblk * 4;
  L.bphys = o;
  o += nblk * 4;
  L.bfill = o;
  o += nblk * 4;
  L.ones = o;
  o += (size_t)hpg * (L.ld / 32) * 4;
  o = align_up(o, 16);
  L.vraw = o;
  o += (size_t)L.ld * hd;
  L.total = o;
  return L;
}

constexpr int kGrpMaxHeads = 8;

template <int HPG>
__global__ void __launch_bounds__(128 * HPG, 1)
    attention_group_kernel(KvLayout kv, StepBuffers sb, int layer, int max_tok) {
  constexpr int JB = HPG < 4 ? HPG : 4;  // heads per pass over a K row
  extern __shared__ __align__(128) uint8_t smem[];
  const int g = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim;
  constexpr int hpg = HPG;
  const int h0 = g * hpg;
  const GroupSmemLayout Ly = group_layout(max_tok, hd, hpg);
  const int ld = Ly.ld;
  float* qs = reinterpret_cast<float*>(smem + Ly.qs);
  float* sc = reinterpret_cast<float*>(smem + Ly.sc);
  float* sf = reinterpret_cast<float*>(smem + Ly.sf);
  float* tks = reinterpret_cast<float*>(smem + Ly.tks);
  float* tvs = reinterpret_cast<float*>(smem + Ly.tvs);
  int* trow = reinterpret_cast<int*>(smem + Ly.trow);
  int* boff = reinterpret_cast<int*>(smem + Ly.boff);
  int* bphys = reinterpret_cast<int*>(smem + Ly.bphys);
  int* bfill = reinterpret_cast<int*>(smem + Ly.bfill);
  int* ones = reinterpret_cast<int*>(smem + Ly.ones);
  uint8_t* vraw = smem + Ly.vraw;
  __shared__ __align__(8) uint64_t vbar;
  __shared__ int s_ntok, s_nsel;
  __shared__ float s_wmax[4 * kGrpMaxHeads];
  __shared__ float s_sum[kGrpMaxHeads];
  if (tid == 0) {
    mbar_init(&vbar, blockDim.x);  // one cp.async arrival per thread
    fence_mbar_init();
  }
  pdl_launch_dependents();
  pdl_wait();
  const bool mk = g == 0 && b == 0 && layer == 0;
  (void)mk;
  PHASE_MARK(mk && tid == 0, 48);
  const int pos = step_pos(sb, b);
  const float* qg = sb.qrot + (long)b * H * hd + (long)h0 * hd;
  for (int d = tid; d < hpg * hd; d += blockDim.x) qs[d] = qg[d];
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));

  // ------------------------------------------------------ token table
  const int n_tok = min(pos + 1, kv.max_blocks * kBlk);
  const int nb = (n_tok + kBlk - 1) / kBlk;
  const long base = ((long)kv_seq(kv, b) * kv.n_layers + layer) * kv.max_blocks;
  const int* pt = kv.page_table + base;
  const int ns = sb.nsel[b];
  const int* sel = sb.sel + (long)b * sb.max_sel;
  const int nsel = ns > 0 ? ns : nb;
  if (warp == 0) {
    int carry = 0;
    for (int k0 = 0; k0 < nsel; k0 += 32) {
      const int k = k0 + lane;
      int fill = 0;
      if (k < nsel) {
        const int lb = ns > 0 ? sel[k] : k;
        bphys[k] = (int)(base + pt[lb]);
        fill = (lb == nb - 1) ? n_tok - lb * kBlk : kBlk;
        bfill[k] = fill;
      }
      int incl = fill;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (k < nsel) boff[k] = carry + incl - fill;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_ntok = carry;
      s_nsel = nsel;
    }
  }
  __syncthreads();
  const int T = s_ntok, nsl = s_nsel;
  const int Tp = (T + 31) & ~31;
  for (int j = tid; j < nsl * kBlk; j += blockDim.x) {
    const int k = j >> 4, t = j & 15;
    if (t < bfill[k]) {
      const int i = boff[k] + t;
      const int row = (bphys[k] * KV + g) * kBlk + t;
      trow[i] = row;
      tks[i] = kv.ks[row];
      tvs[i] = kv.vs[row];
      // the K row (hd bytes) on its way to L2 while V copies and the table finish
      for (int off = 0; off < hd; off += 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(
            reinterpret_cast<const uint8_t*>(kv.kq) + (size_t)row * hd + off));
    }
  }
  // padding tokens [T, Tp): e = 0, f = 1 leave every recurrence unchanged
  for (int i = T + tid; i < Tp; i += blockDim.x) tvs[i] = 0.0f;
  __syncthreads();
  // the group's V rows -> shared memory (hd bytes each), completing on vbar
  {
    const int np = hd >> 4;
    for (int e = tid; e < T * np; e += blockDim.x) {
      const int i = e / np, pc = e - i * np;
      cp_async16(vraw + (size_t)i * hd + pc * 16,
                 reinterpret_cast<const uint8_t*>(kv.vq) + (size_t)trow[i] * hd + pc * 16);
    }
    cp_async_arrive(&vbar);
  }

  PHASE_MARK(mk && tid == 0, 49);
  // ------------------------------------- scores: one K row, every head
  {
    const int npc = hd >> 4;
    for (int i = tid; i < T; i += blockDim.x) {
      const int row = trow[i];
      const uint8_t* kr = reinterpret_cast<const uint8_t*>(kv.kq) + (size_t)row * hd;
      const int t = row & (kBlk - 1);
      const float ksc = tks[i];
      const uint64_t ks2 = pack2(__float_as_uint(ksc), __float_as_uint(ksc));
#pragma unroll 1
      for (int j0 = 0; j0 < HPG; j0 += JB) {
        uint64_t acc[JB][4];
#pragma unroll
        for (int j = 0; j < JB; j++)
#pragma unroll
          for (int l = 0; l < 4; l++) acc[j][l] = 0;
        // the whole K row first (piece c sits at (c + t) mod npc: stored
        // rotated), so its loads overlap
        uint4 ur[8];
#pragma unroll
        for (int c = 0; c < 8; c++)
          if (c < npc) ur[c] = ldg_nc16(kr + (((c + t) & (npc - 1)) << 4));
#pragma unroll
        for (int c = 0; c < 8; c++) {
          if (c >= npc) break;
          const uint4 u = ur[c];
          const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int gq = 0; gq < 4; gq++) {
            uint64_t w01, w23;
            decode_pairs<EC_W_INT8>(wv[gq], w01, w23);
            w01 = mul2(w01, ks2);
            w23 = mul2(w23, ks2);
#pragma unroll
            for (int j = 0; j < JB; j++) {
              const ulonglong2 qq =
                  reinterpret_cast<const ulonglong2*>(qs + (j0 + j) * hd + 16 * c)[gq];
              fma2(acc[j][(2 * gq) & 3], w01, qq.x);
              fma2(acc[j][(2 * gq + 1) & 3], w23, qq.y);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < JB; j++) {
          float a8[8];
#pragma unroll
          for (int l = 0; l < 4; l++) {
            a8[2 * l] = lo_f(acc[j][l]);
            a8[2 * l + 1] = hi_f(acc[j][l]);
          }
          sc[(j0 + j) * ld + i] = __fmul_rn(hsum8(a8), scale);
        }
      }
    }
  }
  __syncthreads();

  PHASE_MARK(mk && tid == 0, 50);
  // ------------- running max per head (threads 128j .. 128j + 127), exps
  {
    const int j = tid >> 7, ht = tid & 127;
    float* scj = sc + j * ld;
    float* sfj = sf + j * ld;
    const int per = (T + 127) / 128;
    const int lo = ht * per, hi = min(lo + per, T);
    float m = -INFINITY;
    for (int i = lo; i < hi; i++) m = (scj[i] > m) ? scj[i] : m;
    float incl = m;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = (t > incl) ? t : incl;
    }
    if (lane == 31) s_wmax[warp] = incl;
    __syncthreads();
    float pre = -INFINITY;
    for (int w = j * 4; w < warp; w++) pre = (s_wmax[w] > pre) ? s_wmax[w] : pre;
    float excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = -INFINITY;
    float run = (excl > pre) ? excl : pre;
    for (int i = lo; i < hi; i++) {
      const float s = scj[i];
      const float prev = run;
      run = (s > prev) ? s : prev;
      sfj[i] = fast_expf(__fsub_rn(prev, run));
      scj[i] = fast_expf(__fsub_rn(s, run));
    }
    for (int i = T + ht; i < Tp; i += 128) {
      scj[i] = 0.0f;
      sfj[i] = 1.0f;
    }
  }
  __syncthreads();
  PHASE_MARK(mk && tid == 0, 51);
  // flag per head per 32 tokens: every scale factor is 1
  for (int w = tid; w < hpg * (Tp >> 5); w += blockDim.x) {
    const int j = w / (Tp >> 5), gq = w - j * (Tp >> 5);
    bool a1 = true;
    for (int u = 0; u < 32; u++) a1 = a1 && (sf[j * ld + 32 * gq + u] == 1.0f);
    ones[j * (ld / 32) + gq] = a1;
  }
  const bool ok = __syncthreads_and(mbar_wait(&vbar, 0, sb.err));

  PHASE_MARK(mk && tid == 0, 52);
  // --------------------------------------------------------- recurrences
  // thread d (< hd) runs dimension d of every query head of the group: the
  // V element is dequantised once per token (v * scale_t, exact) and feeds
  // hpg independent chains o_t = fma(e_t, v_t, o_{t-1} * f_t); thread 0 also
  // runs the denominators
  const bool chainer = tid < hd && ok;
  const int d = tid;
  const bool lead = d == 0;
  float o[HPG], sum[HPG];
#pragma unroll
  for (int jj = 0; jj < HPG; jj++) o[jj] = sum[jj] = 0.0f;
  if (chainer) {
    for (int i0 = 0; i0 < Tp; i0 += 32) {
      bool one[HPG];
#pragma unroll
      for (int jj = 0; jj < HPG; jj++) one[jj] = ones[jj * (ld / 32) + (i0 >> 5)] != 0;
      // this chunk's V bytes first, so no load sits on the chains
      uint32_t wc[32];
#pragma unroll
      for (int k = 0; k < 32; k++) wc[k] = vraw[(size_t)(i0 + k) * hd + d];
#pragma unroll
      for (int i = i0; i < i0 + 32; i += 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(tvs + i);
        const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
        float ev[HPG][4], fv[HPG][4];
#pragma unroll
        for (int jj = 0; jj < HPG; jj++) {
          const float4 e4 = *reinterpret_cast<const float4*>(sc + jj * ld + i);
          const float4 f4 = *reinterpret_cast<const float4*>(sf + jj * ld + i);
          ev[jj][0] = e4.x; ev[jj][1] = e4.y; ev[jj][2] = e4.z; ev[jj][3] = e4.w;
          fv[jj][0] = f4.x; fv[jj][1] = f4.y; fv[jj][2] = f4.z; fv[jj][3] = f4.w;
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float v = __fmul_rn(s8_to_f32(wc[i - i0 + k]), tv[k]);
#pragma unroll
          for (int jj = 0; jj < HPG; jj++) {
            const float prev = one[jj] ? o[jj] : __fmul_rn(o[jj], fv[jj][k]);
            o[jj] = __fmaf_rn(ev[jj][k], v, prev);
            if (lead) sum[jj] = __fmaf_rn(sum[jj], fv[jj][k], ev[jj][k]);
          }
        }
      }
    }
    if (lead)
#pragma unroll
      for (int jj = 0; jj < HPG; jj++) s_sum[jj] = sum[jj];
  }
  PHASE_MARK(mk && tid == 0, 53);
  __syncthreads();
  PHASE_MARK(mk && tid == 0, 54);
  if (chainer) {
#pragma unroll
    for (int jj = 0; jj < HPG; jj++) {
      const float sm = s_sum[jj];
      float r = o[jj];
      if (sm > 0.0f) r = __fmul_rn(r, __fdiv_rn(1.0f, sm));
      sb.att[(long)b * H * hd + (long)(h0 + jj) * hd + d] = r;
    }
  }
}

// Token capacity of one attention launch, a multiple of 4: the per-token
// arrays and the transposed V rows it sizes are read as float4.
static int attn_max_tok(const KvLayout& kv, const StepBuffers& sb) {
  const int t = kv.paged ? kBlk * sb.sparse_blocks_k : (sb.sparse_k > 0 ? sb.sparse_k : kv.seq_len);
  return (t + 3) & ~3;
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

// The attention kernel: grid (kSplit * heads, B) in clusters of kSplit CTAs.
template <bool PAGED, bool VF>
static cudaError_t launch_attn(const KvLayout& kv, const StepBuffers& sb, int layer, int B,
                               int max_tok, size_t smem, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kSplit * kv.n_heads, B);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, attention_kernel<PAGED, VF>, kv, sb, layer, max_tok);
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
  cudaError_t e = opt_in_max_smem(attention_kernel<true, true>);
  if (!e) e = opt_in_max_smem(attention_group_kernel<1>);
  if (!e) e = opt_in_max_smem(attention_group_kernel<2>);
  if (!e) e = opt_in_max_smem(attention_group_kernel<4>);
  if (!e) e = opt_in_max_smem(attention_group_kernel<8>);
  if (!e) e = opt_in_max_smem(attention_kernel<false, true>);
  if (!e) e = opt_in_max_smem(attention_kernel<true, false>);
  if (!e) e = opt_in_max_smem(attention_kernel<false, false>);
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
  cudaError_t e = opt_in_max_smem(attention_kernel<true, true>);
  if (e != cudaSuccess) return e;
  return launch_attn<true, true>(kv, sb, 0, 1, max_tok, smem, s, false);
}

cudaError_t launch_kv_append(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                             int layer, int B, cudaStream_t s, bool pdl) {
  // CTA 1 of each row selects blocks; a prefill launch selects after the
  // centroids instead (launch_paged_select_rows)
  return launch_ex(kv_append_kernel, dim3(kv.paged && !sb.defer_centroid ? 2 : 1, B), dim3(256), 0,
                   s, pdl, kv, lsh, sb,
                   layer);
}

// One CTA per full block of the range.
__global__ void __launch_bounds__(128) paged_centroid_kernel(KvLayout kv, int layer, int seq,
                                                             int lb0) {
  const int lb = lb0 + blockIdx.x;
  const long base = ((long)seq * kv.n_layers + layer) * kv.max_blocks;
  block_centroid(kv, base + kv.page_table[base + lb], threadIdx.x, blockDim.x);
}

// Block selection of batch row blockIdx.y at `layer`.
__global__ void __launch_bounds__(256) paged_select_layer_kernel(KvLayout kv, StepBuffers sb,
                                                                 int layer) {
  paged_select_cta(kv, sb, layer, blockIdx.y);
}

cudaError_t launch_paged_centroids(const KvLayout& kv, int layer, int seq, int first_pos, int n,
                                   cudaStream_t s) {
  // blocks lb with first_pos <= 16 lb + 15 < first_pos + n
  const int lb0 = first_pos / kBlk;                   // ceil((first_pos - 15) / 16)
  const int lb1 = (first_pos + n) / kBlk;             // exclusive: 16 lb + 15 <= first_pos + n - 1
  const int nblk = min(lb1, kv.max_blocks) - lb0;
  if (nblk <= 0) return cudaSuccess;
  paged_centroid_kernel<<<nblk, 128, 0, s>>>(kv, layer, seq, lb0);
  return cudaGetLastError();
}

// Prefill: the LSH update of every row (consecutive tokens of sequence
// seq_plus1 - 1) in row order, by one CTA, after the append rotated the keys.
__global__ void __launch_bounds__(256) lsh_update_rows_kernel(KvLayout kv, LshLayout lsh,
                                                              StepBuffers sb, int B) {
  const int H = kv.n_heads, KV = kv.n_kv_heads, hd = kv.head_dim;
  for (int r = 0; r < B; r++)
    lsh_update_token(lsh, kv_seq(kv, r), sb.qkv + (long)r * (H + 2 * KV) * hd + H * hd,
                     step_pos(sb, r), hd);
}

cudaError_t launch_lsh_update_rows(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                                   int B, cudaStream_t s) {
  if (lsh.tables <= 0) return cudaSuccess;
  lsh_update_rows_kernel<<<1, 256, 0, s>>>(kv, lsh, sb, B);
  return cudaGetLastError();
}

cudaError_t launch_paged_select_rows(const KvLayout& kv, const StepBuffers& sb, int layer, int B,
                                     cudaStream_t s) {
  paged_select_layer_kernel<<<dim3(1, B), 256, 0, s>>>(kv, sb, layer);
  return cudaGetLastError();
}

cudaError_t launch_linear_select(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                                 int layer, int B, cudaStream_t s, bool pdl) {
  const int cap_c = linear_cand_cap(sb, lsh);
  cudaError_t e = launch_ex(linear_cand_kernel, dim3(B), dim3(256), (size_t)kv.head_dim * 4, s, pdl,
                            kv, lsh, sb, layer);
  const int cpb = 256 / kv.n_kv_heads;
  if (!e)
    e = launch_ex(linear_score_kernel, dim3((cap_c + cpb - 1) / cpb, B), dim3(256), 0, s, pdl, kv,
                  sb, layer, cap_c);
  if (!e)
    e = launch_ex(linear_heap_kernel, dim3(B), dim3(32), 0, s, pdl, lsh, sb, cap_c, kv.seq_plus1);
  return e;
}

cudaError_t launch_linear_candidates(const KvLayout& kv, const LshLayout& lsh,
                                     const StepBuffers& sb, int layer, int B, cudaStream_t s) {
  return launch_ex(linear_cand_kernel, dim3(B), dim3(256), (size_t)kv.head_dim * 4, s, false, kv,
                   lsh, sb, layer);
}

cudaError_t launch_linear_score_parts(const KvLayout& kv, const LshLayout& lsh,
                                      const StepBuffers& sb, int layer, int B, cudaStream_t s) {
  const int cap_c = linear_cand_cap(sb, lsh);
  const int cpb = 256 / kv.n_kv_heads;
  return launch_ex(linear_score_kernel, dim3((cap_c + cpb - 1) / cpb, B), dim3(256), 0, s, false,
                   kv, sb, layer, cap_c);
}

cudaError_t launch_linear_sum_heap(const LshLayout& lsh, const StepBuffers& sb,
                                   const float* parts_all, int world, int kv_local, int B,
                                   cudaStream_t s) {
  const int cap_c = linear_cand_cap(sb, lsh);
  tp_sum_scores_kernel<<<dim3(32, B), 256, 0, s>>>(sb, parts_all, world, kv_local, cap_c, B);
  cudaError_t e = cudaGetLastError();
  if (!e) e = launch_ex(linear_heap_kernel, dim3(B), dim3(32), 0, s, false, lsh, sb, cap_c, 0);
  return e;
}

cudaError_t launch_lsh_update_key(const LshLayout& lsh, const StepBuffers& sb, const float* k,
                                  int hd, cudaStream_t s) {
  if (lsh.tables <= 0) return cudaSuccess;
  lsh_update_key_kernel<<<1, 256, 0, s>>>(lsh, sb, k, hd);
  return cudaGetLastError();
}

bool use_group_attention(const KvLayout& kv, const StepBuffers& sb, int B) {
  const int hpg = kv.n_heads / kv.n_kv_heads;
  return kv.paged && B >= 4 && (hpg == 1 || hpg == 2 || hpg == 4 || hpg == 8) &&
         group_layout(attn_max_tok(kv, sb), kv.head_dim, hpg).total <= 227 * 1024 - 256;
}

cudaError_t launch_attention(const KvLayout& kv, const StepBuffers& sb, int layer, int B,
                             cudaStream_t s, bool pdl) {
  const int max_tok = attn_max_tok(kv, sb);
  if (use_group_attention(kv, sb, B)) {
    const int hpg = kv.n_heads / kv.n_kv_heads;
    const size_t smem = group_layout(max_tok, kv.head_dim, hpg).total;
    const dim3 grid(kv.n_kv_heads, B), block(128 * hpg);
    switch (hpg) {
      case 1: return launch_ex(attention_group_kernel<1>, grid, block, smem, s, pdl, kv, sb, layer, max_tok);
      case 2: return launch_ex(attention_group_kernel<2>, grid, block, smem, s, pdl, kv, sb, layer, max_tok);
      case 4: return launch_ex(attention_group_kernel<4>, grid, block, smem, s, pdl, kv, sb, layer, max_tok);
      default: return launch_ex(attention_group_kernel<8>, grid, block, smem, s, pdl, kv, sb, layer, max_tok);
    }
  }
  // from 4 sequences on, throughput over latency: the smaller variant
  const bool vf = B < 4;
  const size_t smem = attn_layout(max_tok, kv.head_dim, kv.paged ? 1 : 2, vf).total;
  if (kv.paged)
    return vf ? launch_attn<true, true>(kv, sb, layer, B, max_tok, smem, s, pdl)
              : launch_attn<true, false>(kv, sb, layer, B, max_tok, smem, s, pdl);
  return vf ? launch_attn<false, true>(kv, sb, layer, B, max_tok, smem, s, pdl)
            : launch_attn<false, false>(kv, sb, layer, B, max_tok, smem, s, pdl);
}

}  // namespace ec
