// lsh_attn.cu -- isolated LSH sparse attention over a linear BF16 KV cache
// the reference's linear-mode selection
// (inference.c:228-423) generalised to L tables x b bits x G-token units,
// followed by its sparse attention (attention_head_sparse,
// ops_attention.c:131-170), for queries against a cache built in bulk.
//
// Index.  Unit u covers tokens [u*G, u*G+G) of KV head 0; its key is their
// mean (summed in token order, times 1/G: lsh_update, ops_lsh.c:296-349) and
// its code in table l has bit h set when the in-order FMA chain
// sum_d key[d] * hp[l][h][d] is > 0 (lsh_hash, ops_lsh.c:138-242).  A bucket
// lists its units newest first -- the order the reference's insertion into
// the head of the bucket's chain produces -- stored as one contiguous run
// per bucket (built on the host from the codes), so a probe reads a run.
//
// Query (one CTA per query).  Candidates: the window [kv_len-window, kv_len)
// and every token of the units found through the mean query's codes (probe 0
// = the code, probe p = bit p-1 flipped; units within the Hamming radius)
// that end before the window.  When the distinct units found number at most
// max_cand, the reference's walk order cannot matter (candidates are sorted
// by position before scoring), so units are marked in parallel; otherwise the
// walk runs in the reference's order (table, probe, newest first) until
// max_cand units, exactly like lsh_find_candidates.  Then scores (sum over KV
// heads of the BF16 dot with the group's first query head), the min-heap
// top-K in heap array order, and the attention kernel over that order.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>

#include "attn.cuh"
#include "ec_internal.cuh"
#include "engine_cuda.h"
#include "lsh_host.h"
#include "select.cuh"

struct ec_lsh_attn {
  int H, KV, hd, max_tokens, L, bits, unit, radius, max_cand, window, top_k, max_queries;
  int device = 0;
  float* hp = nullptr;         // [L][bits][hd]
  uint32_t* codes = nullptr;   // [L][max_units]
  int* boff = nullptr;         // [L][2^bits + 1]
  int* bunits = nullptr;       // [L][max_units]
  int n_tokens = 0, n_units = 0;
  const uint16_t* k = nullptr;
  const uint16_t* v = nullptr;
  const int* page_table = nullptr;  // paged cache: logical 16-token block -> physical (else null)
  int* rows = nullptr;         // [Q][max_sel] paged: the selection as physical rows
  int* rows_n = nullptr;       // [Q] their count
  int* cand = nullptr;         // [Q][max_tokens]
  float* cscore = nullptr;     // [Q][max_tokens]
  unsigned* seen = nullptr;    // [Q][max_units / 32 + 1]
  int* sel = nullptr;          // [Q][max_sel]
  int* nsel = nullptr;         // [Q]
  int* stats = nullptr;        // [Q][2]: units found, candidates
  int max_sel = 0;
  int* err = nullptr;
  std::vector<void*> allocs;
};

namespace ec {
namespace {

// Row of position p in the cache: the position itself (linear), or the
// physical row of a paged cache of 16-token blocks ([block][16][KV][hd]).
__device__ __forceinline__ long cache_row(const int* pt, int p) {
  return pt ? (long)pt[p >> 4] * 16 + (p & 15) : (long)p;
}

// code of unit u in table l
__global__ void __launch_bounds__(128) lsh_unit_codes_kernel(const uint16_t* __restrict__ k,
                                                             const int* __restrict__ pt,
                                                             int KV, int hd, int unit,
                                                             int n_units, int L, int bits,
                                                             const float* __restrict__ hp,
                                                             uint32_t* codes, int max_units) {
  const int u = blockIdx.x;
  if (u >= n_units) return;
  __shared__ float key[256];
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float a = 0.0f;
    for (int t = 0; t < unit; t++)
      a = __fadd_rn(a, bf16_to_f32(k[(cache_row(pt, u * unit + t) * KV) * hd + d]));
    key[d] = unit > 1 ? __fmul_rn(a, __fdiv_rn(1.0f, (float)unit)) : a;
  }
  __syncthreads();
  __shared__ uint32_t code[16];
  if (threadIdx.x < 16) code[threadIdx.x] = 0;
  __syncthreads();
  for (int tb = threadIdx.x; tb < L * bits; tb += blockDim.x) {
    const int l = tb / bits, h = tb - l * bits;
    const float* w = hp + ((size_t)l * bits + h) * hd;
    float a = 0.0f;
    for (int d = 0; d < hd; d++) a = __fmaf_rn(key[d], w[d], a);
    if (a > 0.0f) atomicOr(&code[l], 1u << h);
  }
  __syncthreads();
  if (threadIdx.x < L) codes[(size_t)threadIdx.x * max_units + u] = code[threadIdx.x];
}

struct QueryArgs {
  const int* pt;  // paged cache page table (nullptr: linear)
  const float* q;  // [Q][H][hd]
  const uint16_t* k;
  const float* hp;
  const uint32_t* codes;
  const int* boff;
  const int* bunits;
  int H, KV, hd, L, bits, unit, radius, max_cand, window, top_k;
  int n_tokens, n_units, max_units, max_tokens, max_sel;
  int* cand;
  float* cscore;
  unsigned* seen;
  int* sel;
  int* nsel;
  int* stats;
  int* err;
};

__global__ void __launch_bounds__(512) lsh_query_kernel(QueryArgs a) {
  const int qi = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kv_len = a.n_tokens;
  const float* q = a.q + (size_t)qi * a.H * a.hd;
  int* cand = a.cand + (size_t)qi * a.max_tokens;
  float* cscore = a.cscore + (size_t)qi * a.max_tokens;
  unsigned* seen = a.seen + (size_t)qi * (a.max_units / 32 + 1);
  int* out = a.sel + (size_t)qi * a.max_sel;
  __shared__ float qm[256];
  __shared__ uint32_t qh[16];
  __shared__ int s_found, s_nc;
  __shared__ __align__(16) uint2 hp_nodes[1024];
  if (!(a.top_k > 0 && kv_len > a.top_k)) {
    if (tid == 0) a.nsel[qi] = -1;  // dense over [0, kv_len)
    return;
  }
  const int ws = kv_len > a.window ? kv_len - a.window : 0;
  const int nwords = a.max_units / 32 + 1;
  for (int i = tid; i < nwords; i += blockDim.x) seen[i] = 0u;
  if (tid == 0) {
    s_found = 0;
  }
  // mean query (inference.c:290-295) and its codes
  for (int d = tid; d < a.hd; d += blockDim.x) {
    float s = 0.0f;
    for (int h = 0; h < a.H; h++) s = __fadd_rn(s, q[h * a.hd + d]);
    qm[d] = __fdiv_rn(s, (float)a.H);
  }
  if (tid < 16) qh[tid] = 0;
  __syncthreads();
  const bool lsh = ws > 0 && a.n_units > 0;
  if (lsh) {
    for (int tb = tid; tb < a.L * a.bits; tb += blockDim.x) {
      const int l = tb / a.bits, h = tb - l * a.bits;
      const float* w = a.hp + ((size_t)l * a.bits + h) * a.hd;
      float acc = 0.0f;
      for (int d = 0; d < a.hd; d++) acc = __fmaf_rn(qm[d], w[d], acc);
      if (acc > 0.0f) atomicOr(&qh[l], 1u << h);
    }
  }
  __syncthreads();
  if (lsh) {
    // every (table, probe) bucket's units, marked in parallel; count distinct
    const int nb = 1 << a.bits;
    for (int tp = warp; tp < a.L * (a.bits + 1); tp += blockDim.x >> 5) {
      const int l = tp / (a.bits + 1), p = tp - l * (a.bits + 1);
      const uint32_t probe = p == 0 ? qh[l] : (qh[l] ^ (1u << (p - 1)));
      if (__popc(qh[l] ^ probe) > a.radius) continue;
      const int* run = a.bunits + (size_t)l * a.max_units;
      const int b0 = a.boff[(size_t)l * (nb + 1) + probe], b1 = a.boff[(size_t)l * (nb + 1) + probe + 1];
      for (int i = b0 + lane; i < b1; i += 32) {
        const int u = run[i];
        const unsigned bit = 1u << (u & 31);
        if (!(atomicOr(&seen[u >> 5], bit) & bit)) atomicAdd(&s_found, 1);
      }
    }
    __syncthreads();
    if (s_found > a.max_cand) {
      // the cut-off decides which units stay: the reference's walk order
      for (int i = tid; i < nwords; i += blockDim.x) seen[i] = 0u;
      __syncthreads();
      if (tid == 0) {
        int n = 0;
        for (int l = 0; l < a.L && n < a.max_cand; l++)
          for (int p = 0; p <= a.bits && n < a.max_cand; p++) {
            const uint32_t probe = p == 0 ? qh[l] : (qh[l] ^ (1u << (p - 1)));
            if (__popc(qh[l] ^ probe) > a.radius) continue;
            const int* run = a.bunits + (size_t)l * a.max_units;
            const int b0 = a.boff[(size_t)l * (nb + 1) + probe];
            const int b1 = a.boff[(size_t)l * (nb + 1) + probe + 1];
            for (int i = b0; i < b1 && n < a.max_cand; i++) {
              const int u = run[i];
              if (!(seen[u >> 5] & (1u << (u & 31)))) {
                seen[u >> 5] |= 1u << (u & 31);
                n++;
              }
            }
          }
        s_found = n;
      }
      __syncthreads();
    }
  }
  // candidates in position order: marked units ending before the window, then
  // the window (prefix sums over the marked units, one warp)
  if (warp == 0) {
    int base = 0;
    const int unit_end_lim = ws;  // unit u usable when (u + 1) * G <= ws
    const int nwu = lsh ? (min(a.n_units, unit_end_lim / a.unit) + 31) / 32 : 0;
    for (int w0 = 0; w0 < nwu; w0 += 32) {
      const int w = w0 + lane;
      unsigned m = 0;
      if (w < nwu) {
        m = seen[w];
        const int ulim = min(a.n_units, unit_end_lim / a.unit);  // units [0, ulim)
        const int hi = ulim - w * 32;
        if (hi < 32) m &= hi <= 0 ? 0u : ((1u << hi) - 1u);
      }
      const int cnt = __popc(m) * a.unit;
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      int pos = base + incl - cnt;
      while (m) {
        const int bit = __ffs(m) - 1;
        m &= m - 1;
        const int u = w * 32 + bit;
        for (int t = 0; t < a.unit; t++) cand[pos++] = u * a.unit + t;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_nc = base;
  }
  __syncthreads();
  const int n0 = s_nc;
  for (int i = tid; i < kv_len - ws; i += blockDim.x) cand[n0 + i] = ws + i;
  const int nc = n0 + (kv_len - ws);
  __syncthreads();
  // scores (inference.c:341-353)
  const int grp = a.H / a.KV;
  for (int i = tid; i < nc; i += blockDim.x) {
    const uint16_t* kr = a.k + cache_row(a.pt, cand[i]) * a.KV * a.hd;
    float s = 0.0f;
    for (int kh = 0; kh < a.KV; kh++)
      s = __fadd_rn(s, dot_bf16_ref(kr + kh * a.hd, q + kh * grp * a.hd, a.hd));
    cscore[i] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const int cap = nc < a.top_k ? nc : a.top_k;
    auto all = [](int) { return true; };
    const int size = warp_heap_select<9>(cscore, cand, 0, nc, cap, hp_nodes, lane, all);
    for (int i = lane; i < size; i += 32) out[i] = (int)hp_nodes[i + 1].y;
    if (lane == 0) {
      a.nsel[qi] = size;
      a.stats[qi * 2] = s_found;
      a.stats[qi * 2 + 1] = nc;
    }
  }
}

// Paged cache: the selection (positions, heap order) as physical rows for the
// attention kernel's linear addressing; every position in order when the
// query attends densely.
__global__ void lsh_rows_kernel(const int* __restrict__ pt, const int* __restrict__ sel,
                                const int* __restrict__ nsel, int* rows, int* rows_n, int max_sel,
                                int n_tokens) {
  const int qi = blockIdx.x;
  const int ns = nsel[qi];
  const int n = ns > 0 ? ns : n_tokens;
  if (threadIdx.x == 0) rows_n[qi] = n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int p = ns > 0 ? sel[(long)qi * max_sel + i] : i;
    rows[(long)qi * max_sel + i] = (int)cache_row(pt, p);
  }
}

}  // namespace
}  // namespace ec

// ---------------------------------------------------------------- host side
namespace {

int fail_la(int code, const char* msg) {
  ec_set_last_error(msg);
  return code;
}

template <typename T>
cudaError_t la_alloc(ec_lsh_attn* h, T** p, size_t n) {
  void* v = nullptr;
  cudaError_t e = cudaMalloc(&v, n * sizeof(T) + 16);
  if (e != cudaSuccess) return e;
  h->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return cudaSuccess;
}

}  // namespace

extern "C" void ec_lsh_attn_destroy(ec_lsh_attn* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  for (void* p : h->allocs) cudaFree(p);
  delete h;
}

extern "C" int ec_lsh_attn_create(const ec_lsh_attn_config* c, int device, ec_lsh_attn** out) {
  if (!c || !out) return fail_la(EC_ERR_ARG, "null argument");
  *out = nullptr;
  if (c->n_heads <= 0 || c->n_kv_heads <= 0 || c->n_heads % c->n_kv_heads ||
      (c->head_dim != 32 && c->head_dim != 64 && c->head_dim != 128) || c->max_tokens <= 0 ||
      c->tables < 1 || c->tables > 16 || c->bits < 1 || c->bits > 16 || c->unit < 1 ||
      c->top_k < 1 || c->top_k > 511 || c->window < 0 || c->max_cand < 1 || c->radius < 0 ||
      c->max_queries < 1)
    return fail_la(EC_ERR_UNSUPPORTED, "LSH attention settings out of range");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail_la(EC_ERR_CUDA, cudaGetErrorString(e));
  ec_lsh_attn* h = new ec_lsh_attn();
  h->H = c->n_heads;
  h->KV = c->n_kv_heads;
  h->hd = c->head_dim;
  h->max_tokens = c->max_tokens;
  h->L = c->tables;
  h->bits = c->bits;
  h->unit = c->unit;
  h->radius = c->radius;
  h->max_cand = c->max_cand;
  h->window = c->window;
  h->top_k = c->top_k;
  h->max_queries = c->max_queries;
  h->device = device;
  h->max_sel = c->top_k + 2;
  const int max_units = c->max_tokens / c->unit + 1;
  const int Q = c->max_queries;
#define TRY(x)                                                \
  do {                                                        \
    if ((e = (x)) != cudaSuccess) {                           \
      ec_lsh_attn_destroy(h);                                 \
      return fail_la(EC_ERR_CUDA, cudaGetErrorString(e));     \
    }                                                         \
  } while (0)
  const std::vector<float> hp = ec::lsh_hyperplanes(h->L, h->bits, h->hd);
  TRY(la_alloc(h, &h->hp, hp.size()));
  TRY(cudaMemcpy(h->hp, hp.data(), hp.size() * 4, cudaMemcpyHostToDevice));
  TRY(la_alloc(h, &h->codes, (size_t)h->L * max_units));
  TRY(la_alloc(h, &h->boff, (size_t)h->L * ((1 << h->bits) + 1)));
  TRY(la_alloc(h, &h->bunits, (size_t)h->L * max_units));
  TRY(la_alloc(h, &h->cand, (size_t)Q * h->max_tokens));
  TRY(la_alloc(h, &h->cscore, (size_t)Q * h->max_tokens));
  TRY(la_alloc(h, &h->seen, (size_t)Q * (max_units / 32 + 1)));
  TRY(la_alloc(h, &h->sel, (size_t)Q * h->max_sel));
  TRY(la_alloc(h, &h->rows, (size_t)Q * h->max_sel));
  TRY(la_alloc(h, &h->rows_n, (size_t)Q));
  TRY(la_alloc(h, &h->nsel, (size_t)Q));
  TRY(la_alloc(h, &h->stats, (size_t)Q * 2));
  TRY(la_alloc(h, &h->err, 1));
  TRY(cudaMemset(h->err, 0, 4));
  {
    ec::KvLayout kv{};
    kv.paged = 0;
    kv.head_dim = h->hd;
    ec::LshLayout lsh{};
    ec::StepBuffers sb{};
    sb.sparse_k = h->top_k;
    sb.window = h->window;
    TRY(ec::attn_prepare(kv, lsh, sb));
  }
#undef TRY
  *out = h;
  return EC_OK;
}

namespace {
int lsh_build(ec_lsh_attn* h, const uint16_t* k, const uint16_t* v, const int* page_table,
              int n_tokens, void* stream);
}  // namespace

extern "C" int ec_lsh_attn_build(ec_lsh_attn* h, const uint16_t* k, const uint16_t* v,
                                 int n_tokens, void* stream) {
  return lsh_build(h, k, v, nullptr, n_tokens, stream);
}

extern "C" int ec_lsh_attn_build_paged(ec_lsh_attn* h, const uint16_t* k_blocks,
                                       const uint16_t* v_blocks, const int* page_table,
                                       int n_tokens, void* stream) {
  if (!page_table) return fail_la(EC_ERR_ARG, "null page table");
  return lsh_build(h, k_blocks, v_blocks, page_table, n_tokens, stream);
}

namespace {
int lsh_build(ec_lsh_attn* h, const uint16_t* k, const uint16_t* v, const int* page_table,
              int n_tokens, void* stream) {
  if (!h || !k || !v || n_tokens <= 0 || n_tokens > h->max_tokens)
    return fail_la(EC_ERR_ARG, "bad argument");
  h->page_table = page_table;
  cudaSetDevice(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int max_units = h->max_tokens / h->unit + 1;
  const int nu = n_tokens / h->unit;  // full units only (lsh_update)
  h->k = k;
  h->v = v;
  h->n_tokens = n_tokens;
  h->n_units = nu;
  std::vector<uint32_t> codes((size_t)h->L * nu);
  if (nu > 0) {
    ec::lsh_unit_codes_kernel<<<nu, 128, 0, s>>>(k, page_table, h->KV, h->hd, h->unit, nu, h->L,
                                                 h->bits,
                                                 h->hp, h->codes, max_units);
    EC_CUDA_TRY(cudaGetLastError());
    for (int l = 0; l < h->L; l++)
      EC_CUDA_TRY(cudaMemcpyAsync(codes.data() + (size_t)l * nu, h->codes + (size_t)l * max_units,
                                  (size_t)nu * 4, cudaMemcpyDeviceToHost, s));
    EC_CUDA_TRY(cudaStreamSynchronize(s));
  }
  // buckets: units newest first (the reference inserts at the chain head)
  const int nb = 1 << h->bits;
  std::vector<int> off((size_t)h->L * (nb + 1), 0), units((size_t)h->L * (nu > 0 ? nu : 1));
  for (int l = 0; l < h->L; l++) {
    int* o = &off[(size_t)l * (nb + 1)];
    for (int u = 0; u < nu; u++) o[codes[(size_t)l * nu + u] + 1]++;
    for (int c = 0; c < nb; c++) o[c + 1] += o[c];
    std::vector<int> fill(o, o + nb);
    for (int u = nu - 1; u >= 0; u--) units[(size_t)l * nu + fill[codes[(size_t)l * nu + u]]++] = u;
  }
  EC_CUDA_TRY(cudaMemcpyAsync(h->boff, off.data(), off.size() * 4, cudaMemcpyHostToDevice, s));
  for (int l = 0; l < h->L && nu > 0; l++)
    EC_CUDA_TRY(cudaMemcpyAsync(h->bunits + (size_t)l * max_units, units.data() + (size_t)l * nu,
                                (size_t)nu * 4, cudaMemcpyHostToDevice, s));
  EC_CUDA_TRY(cudaStreamSynchronize(s));
  return EC_OK;
}
}  // namespace

extern "C" int ec_lsh_attn_query(ec_lsh_attn* h, const float* q, int n_queries, float* out,
                                 int* selected_out, int* n_selected_out, void* stream) {
  if (!h || !q || !out || n_queries <= 0 || n_queries > h->max_queries || h->n_tokens <= 0)
    return fail_la(EC_ERR_ARG, "bad argument");
  cudaSetDevice(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ec::QueryArgs a{};
  a.q = q;
  a.k = h->k;
  a.pt = h->page_table;
  a.hp = h->hp;
  a.codes = h->codes;
  a.boff = h->boff;
  a.bunits = h->bunits;
  a.H = h->H;
  a.KV = h->KV;
  a.hd = h->hd;
  a.L = h->L;
  a.bits = h->bits;
  a.unit = h->unit;
  a.radius = h->radius;
  a.max_cand = h->max_cand;
  a.window = h->window;
  a.top_k = h->top_k;
  a.n_tokens = h->n_tokens;
  a.n_units = h->n_units;
  a.max_units = h->max_tokens / h->unit + 1;
  a.max_tokens = h->max_tokens;
  a.max_sel = h->max_sel;
  a.cand = h->cand;
  a.cscore = h->cscore;
  a.seen = h->seen;
  a.sel = h->sel;
  a.nsel = h->nsel;
  a.stats = h->stats;
  a.err = h->err;
  ec::lsh_query_kernel<<<n_queries, 512, 0, s>>>(a);
  EC_CUDA_TRY(cudaGetLastError());
  // attention over the selection (or densely over [0, n_tokens))
  ec::KvLayout kv{};
  kv.n_layers = 1;
  kv.n_heads = h->H;
  kv.n_kv_heads = h->KV;
  kv.head_dim = h->hd;
  kv.seq_len = h->max_tokens;
  kv.paged = 0;
  kv.lk = const_cast<uint16_t*>(h->k);
  kv.lv = const_cast<uint16_t*>(h->v);
  kv.shared_cache = 1;
  ec::StepBuffers sb{};
  sb.pos = nullptr;
  sb.pos_fixed = h->n_tokens - 1;
  sb.qrot = const_cast<float*>(q);
  sb.att = out;
  sb.sel = h->sel;
  sb.nsel = h->nsel;
  if (h->page_table) {
    // the attention reads physical rows of the blocks in the selection's order
    ec::lsh_rows_kernel<<<n_queries, 256, 0, s>>>(h->page_table, h->sel, h->nsel, h->rows,
                                                  h->rows_n, h->max_sel, h->n_tokens);
    EC_CUDA_TRY(cudaGetLastError());
    sb.sel = h->rows;
    sb.nsel = h->rows_n;
    sb.list_dense = 1;
  }
  sb.max_sel = h->max_sel;
  sb.sparse_k = h->top_k;
  sb.window = h->window;
  sb.err = h->err;
  EC_CUDA_TRY(ec::launch_attention(kv, sb, 0, n_queries, s, false));
  for (int i = 0; i < n_queries; i++) {
    if (selected_out)
      EC_CUDA_TRY(cudaMemcpyAsync(selected_out + (size_t)i * h->top_k, h->sel + (size_t)i * h->max_sel,
                                  (size_t)h->top_k * 4, cudaMemcpyDeviceToDevice, s));
  }
  if (n_selected_out)
    EC_CUDA_TRY(cudaMemcpyAsync(n_selected_out, h->nsel, (size_t)n_queries * 4,
                                cudaMemcpyDeviceToDevice, s));
  return EC_OK;
}

extern "C" int ec_lsh_attn_read(ec_lsh_attn* h, int which, void* out, size_t n) {
  if (!h || !out) return fail_la(EC_ERR_ARG, "bad argument");
  cudaSetDevice(h->device);
  const int max_units = h->max_tokens / h->unit + 1;
  const int nb = 1 << h->bits;
  cudaError_t e = cudaSuccess;
  switch (which) {
    case 0:  // codes [L][n_units]
      for (int l = 0; l < h->L && e == cudaSuccess; l++)
        e = cudaMemcpy(static_cast<uint32_t*>(out) + (size_t)l * h->n_units,
                       h->codes + (size_t)l * max_units,
                       std::min<size_t>(h->n_units, n) * 4, cudaMemcpyDeviceToHost);
      break;
    case 1:  // bucket offsets [L][2^bits + 1]
      e = cudaMemcpy(out, h->boff, std::min<size_t>((size_t)h->L * (nb + 1), n) * 4,
                     cudaMemcpyDeviceToHost);
      break;
    case 2:  // per query: units found, candidates [Q][2]
      e = cudaMemcpy(out, h->stats, std::min<size_t>((size_t)h->max_queries * 2, n) * 4,
                     cudaMemcpyDeviceToHost);
      break;
    default:
      return fail_la(EC_ERR_ARG, "unknown item");
  }
  if (e != cudaSuccess) return fail_la(EC_ERR_CUDA, cudaGetErrorString(e));
  return EC_OK;
}
