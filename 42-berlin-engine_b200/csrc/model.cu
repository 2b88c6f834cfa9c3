// model.cu -- the decode context behind include/engine_cuda.h: device copies of
// the weights in fused layouts, the KV / LSH state, host-computed constant
// tables, and the decode step (one CUDA graph per batch shape, kernels chained
// with programmatic dependent launch).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "attn.cuh"
#include "lsh_host.h"
#include "chain.cuh"
#include "ec_internal.cuh"
#include "gemv.cuh"
#include "misc.cuh"
#include "tc_gemm.cuh"
#include "tp.cuh"

static thread_local char g_err[512];

extern "C" void ec_set_last_error(const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg ? msg : "");
}

extern "C" const char* ec_last_error(void) { return g_err; }

namespace {

// sequences per batched-chain pass
constexpr int kPack = 8;

struct Mat {
  uint8_t* w = nullptr;  // packed layout (gemv_packed.cu), rows padded to a multiple of 4
  float* scale = nullptr;  // per row (INT8 and FP8 alike, FP8 expanded)
  uint8_t* tc = nullptr;   // tensor-core layout (tc_gemm.cu) when batched steps use it
  int rows = 0, cols = 0;
};

}  // namespace

struct ec_ctx {
  ec_model_config c;   // shapes of this context (of one shard under tensor parallelism)
  ec_model_config cg;  // shapes of the whole model (== c without tensor parallelism)
  // tensor parallelism (ec_create_tp): rank, ranks, the NCCL communicator and
  // the exchange buffers of one sequence step
  int tp_rank = 0, tp_world = 1;
  void* nccl = nullptr;
  float* tp_q = nullptr;      // [H_all * hd] rotated queries of every rank
  float* tp_k = nullptr;      // [KV_all * hd] rotated keys of every rank
  float* tp_part = nullptr;   // [dim] partial of a row-split projection on this rank
  float* tp_parts = nullptr;  // [world][dim] the partials of every rank
  float* tp_sp = nullptr;     // [cap][KV] per-head candidate dots of this rank
  float* tp_sps = nullptr;    // [world][cap][KV]
  float* tp_lg = nullptr;     // [vocab / world] logits of this rank
  int device = 0;
  int n_sm = 148;
  cudaStream_t stream = nullptr;
  int esize = 1;
  // weights
  std::vector<Mat> qkv, wo, w13, w2;
  Mat lm;
  std::vector<uint16_t*> attn_norm, ffn_norm;
  uint16_t* emb = nullptr;
  uint16_t* final_norm = nullptr;
  // optional (inference.c:583-651): final hidden adapter [D][D] BF16 and
  // logit bias [V]; applied only when registered and not all zero
  uint16_t* adapter = nullptr;
  float* logit_bias = nullptr;
  bool adapter_on = false, bias_on = false;
  // the reference's token_history [S][seq_len] and context bias cache
  int* tok_hist = nullptr;
  ec::ContextBias cbias;
  uint64_t* cb_keys = nullptr;
  int* cb_tokens = nullptr;
  float* cb_biases = nullptr;
  int cb_cap = 0;
  bool cbias_on = false;
  float* xa = nullptr;  // [max_batch][D] adapted final hidden state
  std::vector<unsigned> have;  // bit per tensor per layer
  unsigned have_global = 0;
  // state
  ec::KvLayout kv{};
  ec::LshLayout lsh{};
  float *x = nullptr, *qkvb = nullptr, *qrot = nullptr, *att = nullptr, *hbuf = nullptr,
        *logits = nullptr;
  int *argmax = nullptr, *tokens = nullptr, *pos = nullptr, *sel = nullptr, *nsel = nullptr;
  int* selp = nullptr;  // split attention: physical blocks of the selection
  int *lcand = nullptr, *lnc = nullptr;  // linear mode: selection candidates per sequence
  float* lscore = nullptr;
  int cap_c = 0;
  int* err = nullptr;
  int* chain_ctr = nullptr;  // [layers][packs][kMaxChainPhases + 1]
  float* xn = nullptr;       // batched chain: RMSNorm'd rows [max_batch][dim]
  int npacks = 1;            // batched-chain passes per step (max_batch / 8, rounded up)
  void* amax = nullptr;      // split-argmax partials and counters
  bool chain = false;        // one persistent GEMV kernel per layer
  int chain_kce = 0;         // its packed chunk width
  bool tc = false;           // steps of >= tensor_min_batch sequences: tensor-core GEMMs
  int8_t* tc_digits = nullptr;
  double* tc_sx = nullptr;
  int* tc_ws = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr, *hp = nullptr;
  int max_sel = 0;
  int fast = 0;  // paged decode steps use the split attention (attention_mode)
  ec::PackedPlan p_qkv{}, p_o{}, p_w13{}, p_w2{}, p_lm{};
  // graph cache
  cudaGraphExec_t gexec = nullptr;
  int g_B = -1, g_fb = -1;
  const int *g_tok = nullptr, *g_pos = nullptr;
  int launches = 0;
  std::vector<void*> allocs;
  // profiling
  bool prof = false;
  struct Rec { int kind; cudaEvent_t a, b; double bytes; };
  std::vector<Rec> recs;
  std::vector<cudaEvent_t> ev_pool;
  double prof_ms[EC_K_COUNT] = {0};
  int prof_n[EC_K_COUNT] = {0};
  double prof_bytes[EC_K_COUNT] = {0};
};

namespace {

template <typename T>
cudaError_t dalloc(ec_ctx* c, T** p, size_t n) {
  void* v = nullptr;
  cudaError_t e = cudaMalloc(&v, n * sizeof(T) + 16);
  if (e != cudaSuccess) return e;
  c->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return cudaSuccess;
}

// EC_GEMV_ROWS_PER_THREAD=1|2 overrides the GEMV plans' choice (tuning).
int gemv_force_r() {
  const char* v = getenv("EC_GEMV_ROWS_PER_THREAD");
  return v ? atoi(v) : 0;
}

int fail(int code, const char* msg) {
  ec_set_last_error(msg);
  return code;
}

cudaEvent_t take_event(ec_ctx* c) {
  if (!c->ev_pool.empty()) {
    cudaEvent_t e = c->ev_pool.back();
    c->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Brackets one launch with events when profiling (never inside a capture).
struct ProfScope {
  ec_ctx* c;
  int kind;
  double bytes;
  cudaEvent_t a = nullptr;
  ProfScope(ec_ctx* ctx, int k, double by) : c(ctx), kind(k), bytes(by) {
    if (c->prof) {
      a = take_event(c);
      cudaEventRecord(a, c->stream);
    }
  }
  ~ProfScope() {
    if (c->prof) {
      cudaEvent_t b = take_event(c);
      cudaEventRecord(b, c->stream);
      c->recs.push_back({kind, a, b, bytes});
    }
  }
};

void prof_collect(ec_ctx* c) {
  for (auto& r : c->recs) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      c->prof_ms[r.kind] += ms;
      c->prof_n[r.kind] += 1;
      c->prof_bytes[r.kind] += r.bytes;
    }
    c->ev_pool.push_back(r.a);
    c->ev_pool.push_back(r.b);
  }
  c->recs.clear();
}

}  // namespace

extern "C" int ec_config_default(ec_model_config* c) {
  if (!c) return EC_ERR_ARG;
  memset(c, 0, sizeof(*c));
  c->dim = 4096;
  c->hidden_dim = 14336;
  c->n_layers = 32;
  c->n_heads = 32;
  c->n_kv_heads = 8;
  c->vocab_size = 128256;
  c->seq_len = 8192;
  c->head_dim = 128;
  c->rope_theta = 500000.0f;
  c->norm_eps = 1e-5f;
  c->weight_kind = EC_W_INT8;
  c->use_paged_kv = 1;
  c->sparse_k = 64;
  c->window = 128;
  c->sparse_blocks_k = 64;
  c->lsh_tables = 1;
  c->lsh_bits = 16;
  c->lsh_unit = 64;
  c->lsh_max_units = 4096;
  c->lsh_radius = 4;
  c->lsh_max_cand = 64;
  c->max_batch = 1;
  return EC_OK;
}

extern "C" void ec_destroy(ec_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  // the captured step holds NCCL work: release it before the communicator
  if (ctx->gexec) cudaGraphExecDestroy(ctx->gexec);
  ctx->gexec = nullptr;
  if (ctx->nccl) {
    cudaDeviceSynchronize();
    if (const ec::NcclApi* api = ec::nccl_api(nullptr))
      api->comm_destroy(static_cast<ncclComm_t>(ctx->nccl));
    ctx->nccl = nullptr;
  }
  cudaStreamSynchronize(ctx->stream);
  for (auto& r : ctx->recs) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (auto e : ctx->ev_pool) cudaEventDestroy(e);
  for (void* p : ctx->allocs) cudaFree(p);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

namespace {

// Context for shapes c on `device`; `global` (tensor parallelism) holds the
// shapes of the whole model, of which c is the shard of rank `rank`.
int create_ctx(const ec_model_config& c, int device, const ec_model_config* global, int rank,
               int world, ec_ctx** out) {
  if (c.dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
      c.n_heads % c.n_kv_heads || (c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128) || c.dim % 32 ||
      c.hidden_dim % 32 || c.vocab_size <= 0 || c.seq_len <= 0 || c.max_batch <= 0)
    return fail(EC_ERR_UNSUPPORTED, "unsupported model shape (head_dim 32, 64 or 128; dims % 32)");
  if (c.weight_kind != EC_W_INT8 && c.weight_kind != EC_W_FP8)
    return fail(EC_ERR_ARG, "weight_kind must be EC_W_INT8 or EC_W_FP8");
  if (c.lsh_tables < 0 || c.lsh_tables > 16 || c.lsh_bits < 1 || c.lsh_bits > 16 ||
      c.lsh_max_units > 4096 || c.lsh_unit <= 0 || c.lsh_max_cand > 64)
    return fail(EC_ERR_UNSUPPORTED, "LSH settings out of range");
  if (c.sparse_blocks_k < 1 || c.sparse_blocks_k > 64)
    return fail(EC_ERR_UNSUPPORTED, "sparse_blocks_k must be in 1..64 (select_top_k_blocks)");
  if (c.use_paged_kv && c.seq_len > 32768)
    return fail(EC_ERR_UNSUPPORTED, "paged KV supports seq_len <= 32768 (2048 blocks)");
  if (c.attention_mode != EC_ATTN_REFERENCE && c.attention_mode != EC_ATTN_SPLIT)
    return fail(EC_ERR_ARG, "attention_mode must be EC_ATTN_REFERENCE or EC_ATTN_SPLIT");
  if (!c.use_paged_kv && (c.sparse_k <= 0 || c.sparse_k > 511))
    return fail(EC_ERR_UNSUPPORTED, "linear KV mode needs sparse_k in 1..511");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
  ec_ctx* ctx = new ec_ctx();
  ctx->c = c;
  ctx->cg = global ? *global : c;
  ctx->tp_rank = rank;
  ctx->tp_world = world;
  ctx->device = device;
  cudaDeviceGetAttribute(&ctx->n_sm, cudaDevAttrMultiProcessorCount, device);
  ctx->esize = 1;
#define TRY(x)                                  \
  do {                                          \
    cudaError_t e_ = (x);                       \
    if (e_ != cudaSuccess) {                    \
      ec_set_last_error(cudaGetErrorString(e_)); \
      ec_destroy(ctx);                          \
      return e_ == cudaErrorMemoryAllocation ? EC_ERR_OOM : EC_ERR_CUDA; \
    }                                           \
  } while (0)
  TRY(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
  const int L = c.n_layers, H = c.n_heads, KV = c.n_kv_heads, hd = c.head_dim, D = c.dim;
  const int F = c.hidden_dim, V = c.vocab_size, S = c.max_batch;
  const int Vg = ctx->cg.vocab_size;  // embedding rows, logits per sequence
  ctx->qkv.resize(L);
  ctx->wo.resize(L);
  ctx->w13.resize(L);
  ctx->w2.resize(L);
  ctx->attn_norm.assign(L, nullptr);
  ctx->ffn_norm.assign(L, nullptr);
  ctx->have.assign(L, 0);
  for (int l = 0; l < L; l++) {
    Mat* ms[4] = {&ctx->qkv[l], &ctx->wo[l], &ctx->w13[l], &ctx->w2[l]};
    const int rows[4] = {(H + 2 * KV) * hd, D, 2 * F, D};
    const int cols[4] = {D, H * hd, D, F};
    for (int i = 0; i < 4; i++) {
      ms[i]->rows = rows[i];
      ms[i]->cols = cols[i];
      TRY(dalloc(ctx, &ms[i]->w, ec::packed_bytes(rows[i], cols[i])));
      TRY(cudaMemset(ms[i]->w, 0, ec::packed_bytes(rows[i], cols[i])));
      TRY(dalloc(ctx, &ms[i]->scale, (size_t)rows[i]));
    }
    TRY(dalloc(ctx, &ctx->attn_norm[l], (size_t)D));
    TRY(dalloc(ctx, &ctx->ffn_norm[l], (size_t)D));
  }
  ctx->lm.rows = V;
  ctx->lm.cols = D;
  TRY(dalloc(ctx, &ctx->lm.w, ec::packed_bytes(V, D)));
  TRY(cudaMemset(ctx->lm.w, 0, ec::packed_bytes(V, D)));
  TRY(dalloc(ctx, &ctx->lm.scale, (size_t)V));
  TRY(dalloc(ctx, &ctx->emb, (size_t)Vg * D));
  TRY(dalloc(ctx, &ctx->final_norm, (size_t)D));
  // activations
  TRY(dalloc(ctx, &ctx->x, (size_t)S * D));
  TRY(dalloc(ctx, &ctx->qkvb, (size_t)S * (H + 2 * KV) * hd));
  TRY(dalloc(ctx, &ctx->att, (size_t)S * H * hd));
  TRY(dalloc(ctx, &ctx->qrot, (size_t)S * H * hd));
  TRY(dalloc(ctx, &ctx->hbuf, (size_t)S * F));
  TRY(dalloc(ctx, &ctx->logits, (size_t)S * Vg));
  TRY(dalloc(ctx, &ctx->argmax, (size_t)S));
  TRY(dalloc(ctx, &ctx->tokens, (size_t)S));
  TRY(dalloc(ctx, &ctx->pos, (size_t)S));
  ctx->max_sel = c.sparse_k > c.sparse_blocks_k + 2 ? c.sparse_k : c.sparse_blocks_k + 2;
  TRY(dalloc(ctx, &ctx->sel, (size_t)S * ctx->max_sel));
  TRY(dalloc(ctx, &ctx->selp, (size_t)S * ctx->max_sel));
  TRY(dalloc(ctx, &ctx->nsel, (size_t)S));
  TRY(dalloc(ctx, &ctx->err, 1));
  TRY(cudaMemset(ctx->err, 0, sizeof(int)));
  {
    uint8_t* am = nullptr;
    TRY(dalloc(ctx, &am, ec::argmax_scratch_bytes(S)));
    TRY(cudaMemset(am, 0, ec::argmax_scratch_bytes(S)));
    ctx->amax = am;
  }
  {
    // one counter block per (layer, pack of up to 8 sequences), plus layer 0's QKV
    ctx->npacks = (S + kPack - 1) / kPack;
    const size_t nctr = (size_t)(L + 1) * ctx->npacks * (ec::kMaxChainPhases + 1);
    TRY(dalloc(ctx, &ctx->chain_ctr, nctr));
    TRY(cudaMemset(ctx->chain_ctr, 0, nctr * sizeof(int)));
  }
  TRY(dalloc(ctx, &ctx->xn, (size_t)S * D));
  // KV
  ec::KvLayout& kv = ctx->kv;
  kv.n_layers = L;
  kv.n_heads = H;
  kv.n_kv_heads = KV;
  kv.head_dim = hd;
  kv.seq_len = c.seq_len;
  kv.max_blocks = (c.seq_len + 15) / 16;
  kv.paged = c.use_paged_kv ? 1 : 0;
  const size_t nblk = (size_t)S * L * kv.max_blocks;
  if (kv.paged) {
    TRY(dalloc(ctx, &kv.kq, nblk * KV * 16 * hd));
    TRY(dalloc(ctx, &kv.vq, nblk * KV * 16 * hd));
    TRY(dalloc(ctx, &kv.ks, nblk * KV * 16));
    TRY(dalloc(ctx, &kv.vs, nblk * KV * 16));
    TRY(dalloc(ctx, &kv.centroid, nblk * hd));
    TRY(dalloc(ctx, &kv.page_table, nblk));
    std::vector<int> pt(nblk);
    for (size_t i = 0; i < nblk; i++) pt[i] = (int)(i % kv.max_blocks);
    TRY(cudaMemcpy(kv.page_table, pt.data(), nblk * sizeof(int), cudaMemcpyHostToDevice));
  } else {
    TRY(dalloc(ctx, &kv.lk, (size_t)S * L * c.seq_len * KV * hd));
    TRY(dalloc(ctx, &kv.lv, (size_t)S * L * c.seq_len * KV * hd));
    ctx->cap_c = c.window + c.lsh_max_cand * c.lsh_unit;
    TRY(dalloc(ctx, &ctx->lcand, (size_t)S * ctx->cap_c));
    TRY(dalloc(ctx, &ctx->lscore, (size_t)S * ctx->cap_c));
    TRY(dalloc(ctx, &ctx->lnc, (size_t)S));
  }
  // RoPE tables (rope_cache_init, ops_rope.c:30-96) on the host
  {
    const int half = hd / 2;
    std::vector<float> inv(half), ct((size_t)c.seq_len * half), st((size_t)c.seq_len * half);
    for (int i = 0; i < half; i++)
      inv[i] = 1.0f / powf(c.rope_theta, (float)(i * 2) / (float)hd);
    for (int p = 0; p < c.seq_len; p++)
      for (int i = 0; i < half; i++) {
        const float th = (float)p * inv[i];
        ct[(size_t)p * half + i] = cosf(th);
        st[(size_t)p * half + i] = sinf(th);
      }
    TRY(dalloc(ctx, &ctx->rope_cos, ct.size()));
    TRY(dalloc(ctx, &ctx->rope_sin, st.size()));
    TRY(cudaMemcpy(ctx->rope_cos, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(ctx->rope_sin, st.data(), st.size() * 4, cudaMemcpyHostToDevice));
  }
  // LSH hyperplanes (lsh_init, ops_lsh.c:40-85; table t seeded 42 + t)
  ec::LshLayout& lsh = ctx->lsh;
  lsh.tables = c.lsh_tables;
  lsh.bits = c.lsh_bits;
  lsh.unit = c.lsh_unit;
  lsh.max_units = c.lsh_max_units;
  lsh.radius = c.lsh_radius;
  lsh.max_cand = c.lsh_max_cand;
  if (lsh.tables > 0) {
    const std::vector<float> hp = ec::lsh_hyperplanes(lsh.tables, lsh.bits, hd);
    TRY(dalloc(ctx, &ctx->hp, hp.size()));
    TRY(cudaMemcpy(ctx->hp, hp.data(), hp.size() * 4, cudaMemcpyHostToDevice));
    lsh.hp = ctx->hp;
    TRY(dalloc(ctx, &lsh.acc, (size_t)S * hd));
    TRY(dalloc(ctx, &lsh.meta, (size_t)S * 4));
    TRY(dalloc(ctx, &lsh.unit_hash, (size_t)S * lsh.tables * lsh.max_units));
    TRY(dalloc(ctx, &lsh.unit_start, (size_t)S * lsh.max_units));
    TRY(dalloc(ctx, &lsh.unit_len, (size_t)S * lsh.max_units));
    TRY(dalloc(ctx, &lsh.heads, ((size_t)S * lsh.tables) << lsh.bits));
    TRY(dalloc(ctx, &lsh.next, (size_t)S * lsh.tables * lsh.max_units));
    TRY(dalloc(ctx, &lsh.counters, (size_t)S * 2));
  }
  TRY(dalloc(ctx, &ctx->tok_hist, (size_t)S * c.seq_len));
  // GEMV plans
  const int wk = c.weight_kind;
  const int fr = gemv_force_r();
  {
    // the chain needs one packed chunk width for all of a layer's matrices
    ec::ChainParams P{};
    const int ks[5] = {H * hd, D, F, D, D};
    for (int i = 0; i < 5; i++) P.ph[i].K = ks[i];
    P.nph = 5;
    const char* nc = getenv("EC_NO_CHAIN");
    ctx->chain = ec::chain_kce(P) != 0 && !(nc && atoi(nc));
    ctx->chain_kce = ctx->chain ? ec::chain_kce(P) : 0;
  }
  // co-resident plans measured slower (the block scheduler may place two CTAs
  // of one GEMV on an SM whose previous CTA has finished): opt-in only
  const bool co = getenv("EC_GEMV_SMEM_KB") != nullptr;
  if (!ec::packed_plan(wk, (H + 2 * KV) * hd, D, ctx->n_sm, fr, co, &ctx->p_qkv) ||
      !ec::packed_plan(wk, D, H * hd, ctx->n_sm, fr, co, &ctx->p_o) ||
      !ec::packed_plan(wk, 2 * F, D, ctx->n_sm, fr, co, &ctx->p_w13) ||
      !ec::packed_plan(wk, D, F, ctx->n_sm, fr, co, &ctx->p_w2) ||
      !ec::packed_plan(wk, V, D, ctx->n_sm, fr, false, &ctx->p_lm)) {
    ec_destroy(ctx);
    return fail(EC_ERR_UNSUPPORTED, "no GEMV plan for this shape");
  }
  // tensor-core GEMMs for large batched steps (INT8, K a multiple of 128)
  if (c.tensor_min_batch > 0 && wk == EC_W_INT8 && D % ec::kTcKb == 0 && F % ec::kTcKb == 0 &&
      (H * hd) % ec::kTcKb == 0) {
    ctx->tc = true;
    const int pb = S < ec::kTcMaxRows ? S : ec::kTcMaxRows;
    size_t wsb = 0;
    auto tc_alloc = [&](Mat& m) -> cudaError_t {
      cudaError_t e2 = dalloc(ctx, &m.tc, ec::tc_weight_bytes(m.rows, m.cols));
      if (e2 == cudaSuccess) e2 = cudaMemset(m.tc, 0, ec::tc_weight_bytes(m.rows, m.cols));
      const size_t w = ec::tc_ws_bytes(m.rows, m.cols, pb, ctx->n_sm);
      if (w > wsb) wsb = w;
      return e2;
    };
    for (int l = 0; l < L; l++) {
      TRY(tc_alloc(ctx->qkv[l]));
      TRY(tc_alloc(ctx->wo[l]));
      TRY(tc_alloc(ctx->w13[l]));
      TRY(tc_alloc(ctx->w2[l]));
    }
    TRY(tc_alloc(ctx->lm));
    const int kmax = F > D ? (F > H * hd ? F : H * hd) : (D > H * hd ? D : H * hd);
    TRY(dalloc(ctx, &ctx->tc_digits, ec::tc_digit_bytes(pb, kmax)));
    TRY(dalloc(ctx, &ctx->tc_sx, (size_t)ec::kTcMaxRows));
    TRY(dalloc(ctx, &ctx->tc_ws, wsb / 4));
    TRY(ec::tc_prepare());
  }
  {
    ec::StepBuffers sb{};
    sb.sparse_k = c.sparse_k;
    sb.window = c.window;
    sb.sparse_blocks_k = c.sparse_blocks_k;
    TRY(ec::gemv_prepare());
    TRY(ec::packed_prepare());
    TRY(ec::chain_prepare());
    TRY(ec::attn_prepare(ctx->kv, ctx->lsh, sb));
  }
  if (ctx->chain) {
    // the chain's grid-wide phase counters need every CTA resident at once
    int kmax = D > F ? D : F;
    if (H * hd > kmax) kmax = H * hd;
    if (ec::chain_blocks_per_sm(c.weight_kind, ctx->chain_kce, kmax, D) < 1) {
      ec_destroy(ctx);
      return fail(EC_ERR_UNSUPPORTED, "the GEMV chain kernel cannot keep one CTA per SM resident "
                                      "on this device");
    }
  }
  if (c.attention_mode != EC_ATTN_REFERENCE && ctx->kv.paged) {
    if (!ec::fast_attention_supported(ctx->kv, c.sparse_blocks_k)) {
      ec_destroy(ctx);
      return fail(EC_ERR_UNSUPPORTED, "split attention: head_dim <= 128 (multiple of 16), <= 8 "
                                      "KV heads, 1/2/4/8 query heads per KV head");
    }
    ctx->fast = c.attention_mode;
    TRY(ec::fast_attention_prepare(ctx->kv));
  }
  if (world > 1) {
    const ec_model_config& g = ctx->cg;
    const int cap = ctx->kv.paged ? 0 : ctx->cap_c;
    TRY(dalloc(ctx, &ctx->tp_q, (size_t)g.n_heads * hd));
    TRY(dalloc(ctx, &ctx->tp_k, (size_t)g.n_kv_heads * hd));
    TRY(dalloc(ctx, &ctx->tp_part, (size_t)D));
    TRY(dalloc(ctx, &ctx->tp_parts, (size_t)world * D));
    TRY(dalloc(ctx, &ctx->tp_lg, (size_t)V));
    if (cap) {
      TRY(dalloc(ctx, &ctx->tp_sp, (size_t)cap * KV));
      TRY(dalloc(ctx, &ctx->tp_sps, (size_t)world * cap * KV));
    }
  }
#undef TRY
  *out = ctx;
  for (int s = 0; s < S; s++) ec_reset(ctx, s);
  return cudaDeviceSynchronize() == cudaSuccess ? EC_OK : EC_ERR_CUDA;
}

}  // namespace

extern "C" int ec_create(const ec_model_config* cfg, int device, ec_ctx** out) {
  if (!cfg || !out) return fail(EC_ERR_ARG, "null argument");
  return create_ctx(*cfg, device, nullptr, 0, 1, out);
}

extern "C" int ec_tp_unique_id(void* out, size_t n) {
  const char* why = nullptr;
  const ec::NcclApi* api = ec::nccl_api(&why);
  if (!api) return fail(EC_ERR_UNSUPPORTED, why);
  if (!out || n < sizeof(ncclUniqueId)) return fail(EC_ERR_ARG, "id buffer smaller than 128 bytes");
  ncclUniqueId id;
  const ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) return fail(EC_ERR_CUDA, api->error_string(r));
  memcpy(out, &id, sizeof(id));
  return EC_OK;
}

extern "C" int ec_create_tp(const ec_model_config* cfg, int device, int rank, int world,
                            const void* id, ec_ctx** out) {
  if (!cfg || !out || !id) return fail(EC_ERR_ARG, "null argument");
  if (world < 1 || rank < 0 || rank >= world) return fail(EC_ERR_ARG, "bad rank or world size");
  const ec_model_config& g = *cfg;
  if (g.n_heads % world || g.n_kv_heads % world || g.hidden_dim % world || g.vocab_size % world ||
      (g.hidden_dim / world) % 32)
    return fail(EC_ERR_UNSUPPORTED, "heads, KV heads, hidden_dim and vocab_size must divide by the "
                                    "number of ranks");
  if (g.attention_mode != EC_ATTN_REFERENCE || g.tensor_min_batch > 0)
    return fail(EC_ERR_UNSUPPORTED, "tensor parallelism runs the reference-order attention and "
                                    "the exact GEMV chain");
  const char* why = nullptr;
  const ec::NcclApi* api = ec::nccl_api(&why);
  if (!api) return fail(EC_ERR_UNSUPPORTED, why);
  ec_model_config c = g;  // this rank's shard
  c.n_heads = g.n_heads / world;
  c.n_kv_heads = g.n_kv_heads / world;
  c.hidden_dim = g.hidden_dim / world;
  c.vocab_size = g.vocab_size / world;
  ec_ctx* ctx = nullptr;
  int rc = create_ctx(c, device, &g, rank, world, &ctx);
  if (rc) return rc;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  cudaSetDevice(device);
  const ncclResult_t r = api->comm_init_rank(&comm, world, uid, rank);
  if (r != ncclSuccess) {
    ec_destroy(ctx);
    return fail(EC_ERR_CUDA, api->error_string(r));
  }
  ctx->nccl = comm;
  // one collective of each kind outside any stream capture: NCCL sets up its
  // connections on first use, which a captured step must not do
  ec::NcclApi const* a = api;
  ncclResult_t w = a->all_gather(ctx->tp_part, ctx->tp_parts, (size_t)c.dim, ncclFloat32, comm,
                                 ctx->stream);
  if (w == ncclSuccess) w = a->broadcast(ctx->nsel, ctx->nsel, 1, ncclInt32, 0, comm, ctx->stream);
  if (w != ncclSuccess || cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    ec_destroy(ctx);
    return fail(EC_ERR_CUDA, w != ncclSuccess ? a->error_string(w) : "NCCL warm-up failed");
  }
  *out = ctx;
  return EC_OK;
}

extern "C" int ec_set_weight(ec_ctx* ctx, int layer, int which, const void* data,
                             const float* scales, int on_device) {
  if (!ctx || !data) return fail(EC_ERR_ARG, "null argument");
  const ec_model_config& c = ctx->c;
  cudaSetDevice(ctx->device);
  // device data may still be in flight on the caller's streams (ctx->stream
  // does not wait for them): let every prior device operation finish first
  if (on_device) {
    const cudaError_t e0 = cudaDeviceSynchronize();
    if (e0 != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e0));
  }
  const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  const cudaMemcpyKind skind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  const int D = c.dim, F = c.hidden_dim, hd = c.head_dim, H = c.n_heads, KV = c.n_kv_heads;
  const bool fp8 = c.weight_kind == EC_W_FP8;
  // tensor parallelism: this rank takes rows [r0, r0 + n) of a column-split
  // matrix (QKV, gate/up, LM head) or columns [c0, c0 + n) of a row-split one
  // (o, down); per-row scales follow the rows
  const int R = ctx->tp_rank;
  const ec_model_config& g = ctx->cg;
  // FP8 per-tensor scale -> per-row scale vector (same value on every row)
  auto put_scales_from = [&](float* dst, const float* src, int rows, int stride) -> cudaError_t {
    if (!src) return cudaErrorInvalidValue;
    if (!fp8) return cudaMemcpy2D(dst, stride * 4, src, 4, 4, rows, skind);
    float s = 0.0f;
    cudaError_t e = cudaMemcpy(&s, src, 4, on_device ? cudaMemcpyDeviceToHost : cudaMemcpyHostToHost);
    if (e != cudaSuccess) return e;
    std::vector<float> v(rows, s);
    return cudaMemcpy2D(dst, stride * 4, v.data(), 4, 4, rows, cudaMemcpyHostToDevice);
  };
  // scales of local rows [0, rows) = global rows [row0, row0 + rows)
  auto put_scales = [&](float* dst, int rows, int stride, long row0 = 0) -> cudaError_t {
    if (!scales) return cudaErrorInvalidValue;
    return put_scales_from(dst, fp8 ? scales : scales + row0, rows, stride);
  };
  // nr row-major rows of m.cols bytes -> packed rows row_base + row_stride*i;
  // src_cols > m.cols: the rows of src are src_cols bytes long and this
  // rank takes bytes [col0, col0 + m.cols) of each (a row-split shard)
  auto put_rows = [&](Mat& m, const void* src, int nr, int row_base, int row_stride,
                      int src_cols = 0, int col0 = 0) -> cudaError_t {
    const size_t bytes = (size_t)nr * m.cols;
    const uint8_t* d = static_cast<const uint8_t*>(src);
    void* tmp = nullptr;
    cudaError_t e2;
    if (!on_device || (src_cols && src_cols != m.cols)) {
      if ((e2 = cudaMalloc(&tmp, bytes)) != cudaSuccess) return e2;
      // same stream as the pack: a pageable cudaMemcpy may return before its
      // DMA has landed, and ctx->stream does not wait for the legacy stream
      if (src_cols && src_cols != m.cols)
        e2 = cudaMemcpy2DAsync(tmp, m.cols, d + col0, src_cols, m.cols, nr, kind, ctx->stream);
      else
        e2 = cudaMemcpyAsync(tmp, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
      if (e2 != cudaSuccess) {
        cudaFree(tmp);
        return e2;
      }
      d = static_cast<const uint8_t*>(tmp);
    }
    e2 = ec::packed_pack(d, m.w, m.rows, m.cols, nr, row_base, row_stride, ctx->stream);
    if (e2 == cudaSuccess && m.tc)
      e2 = ec::tc_pack(d, m.tc, m.rows, m.cols, nr, row_base, row_stride, ctx->stream);
    if (e2 == cudaSuccess) e2 = cudaStreamSynchronize(ctx->stream);
    if (tmp) cudaFree(tmp);
    return e2;
  };
  cudaError_t e = cudaSuccess;
  if (layer < 0) {
    switch (which) {
      case EC_EMBEDDING:
        e = cudaMemcpy(ctx->emb, data, (size_t)ctx->cg.vocab_size * D * 2, kind);
        break;
      case EC_FINAL_NORM:
        e = cudaMemcpy(ctx->final_norm, data, (size_t)D * 2, kind);
        break;
      case EC_LM_HEAD: {
        const long r0 = (long)R * c.vocab_size;
        e = put_rows(ctx->lm, static_cast<const uint8_t*>(data) + r0 * D, c.vocab_size, 0, 1);
        if (e == cudaSuccess) e = put_scales(ctx->lm.scale, c.vocab_size, 1, r0);
        break;
      }
      case EC_FINAL_ADAPTER:
      case EC_LOGIT_BIAS: {
        if (ctx->tp_world > 1)
          return fail(EC_ERR_UNSUPPORTED, "final adapter / logit bias with tensor parallelism");
        // optional tensors: kept only when not all zero (the reference's
        // zero-initialised adapter and bias change nothing)
        const bool ad = which == EC_FINAL_ADAPTER;
        const size_t n = ad ? (size_t)D * D : (size_t)c.vocab_size;
        void** dst = ad ? reinterpret_cast<void**>(&ctx->adapter)
                        : reinterpret_cast<void**>(&ctx->logit_bias);
        if (!*dst) {
          e = ad ? dalloc(ctx, &ctx->adapter, n) : dalloc(ctx, &ctx->logit_bias, n);
          if (e == cudaSuccess && ad && !ctx->xa) e = dalloc(ctx, &ctx->xa, (size_t)c.max_batch * D);
        }
        if (e == cudaSuccess) e = cudaMemcpy(*dst, data, n * (ad ? 2 : 4), kind);
        int* flag = nullptr;
        if (e == cudaSuccess) e = dalloc(ctx, &flag, 1);
        if (e == cudaSuccess) e = cudaMemset(flag, 0, 4);
        if (e == cudaSuccess) e = ec::launch_nonzero(*dst, (long)n, ad ? 16 : 32, flag, nullptr);
        int any = 0;
        if (e == cudaSuccess) e = cudaMemcpy(&any, flag, 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) (ad ? ctx->adapter_on : ctx->bias_on) = any != 0;
        // the captured step changes shape: capture again on the next step
        if (ctx->gexec) {
          cudaGraphExecDestroy(ctx->gexec);
          ctx->gexec = nullptr;
        }
        break;
      }
      default:
        return fail(EC_ERR_ARG, "unknown global tensor id");
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
    if (which <= EC_LM_HEAD) ctx->have_global |= 1u << (which - EC_EMBEDDING);
    return EC_OK;
  }
  if (layer >= c.n_layers) return fail(EC_ERR_ARG, "layer out of range");
  const uint8_t* src8 = static_cast<const uint8_t*>(data);
  switch (which) {
    case EC_WQ: case EC_WK: case EC_WV: {
      const int r0 = which == EC_WQ ? 0 : (which == EC_WK ? H * hd : (H + KV) * hd);
      const int nr = which == EC_WQ ? H * hd : KV * hd;
      const long g0 = (long)R * nr;  // this rank's heads within the whole matrix
      Mat& m = ctx->qkv[layer];
      e = put_rows(m, src8 + g0 * D, nr, r0, 1);
      if (e == cudaSuccess) e = put_scales(m.scale + r0, nr, 1, g0);
      break;
    }
    case EC_WO:
      e = put_rows(ctx->wo[layer], data, D, 0, 1, g.n_heads * hd, R * H * hd);
      if (e == cudaSuccess) e = put_scales(ctx->wo[layer].scale, D, 1);
      break;
    case EC_W1: case EC_W3: {
      // interleave: row 2i = gate i, row 2i+1 = up i
      Mat& m = ctx->w13[layer];
      const int off = which == EC_W1 ? 0 : 1;
      const long g0 = (long)R * F;
      e = put_rows(m, src8 + g0 * D, F, off, 2);
      if (e == cudaSuccess) e = put_scales(m.scale + off, F, 2, g0);
      break;
    }
    case EC_W2:
      e = put_rows(ctx->w2[layer], data, D, 0, 1, g.hidden_dim, R * F);
      if (e == cudaSuccess) e = put_scales(ctx->w2[layer].scale, D, 1);
      break;
    case EC_ATTN_NORM:
      e = cudaMemcpy(ctx->attn_norm[layer], data, (size_t)D * 2, kind);
      break;
    case EC_FFN_NORM:
      e = cudaMemcpy(ctx->ffn_norm[layer], data, (size_t)D * 2, kind);
      break;
    default:
      return fail(EC_ERR_ARG, "unknown layer tensor id");
  }
  // every copy above complete before the decode stream can read it
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
  ctx->have[layer] |= 1u << which;
  return EC_OK;
}

extern "C" int ec_set_context_bias(ec_ctx* ctx, const uint64_t* keys, const int* tokens,
                                   const float* biases, int size) {
  if (!ctx || size < 0 || (size > 0 && (!keys || !tokens || !biases)))
    return fail(EC_ERR_ARG, "bad context bias table");
  if (ctx->tp_world > 1)
    return fail(EC_ERR_UNSUPPORTED, "context bias with tensor parallelism");
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  bool any = false;
  for (int i = 0; i < size && !any; i++) any = keys[i] != 0;
  if (e == cudaSuccess && any) {
    if (size > ctx->cb_cap) {
      // a larger table: new buffers (the old ones are freed with the context)
      e = dalloc(ctx, &ctx->cb_keys, (size_t)size);
      if (e == cudaSuccess) e = dalloc(ctx, &ctx->cb_tokens, (size_t)size);
      if (e == cudaSuccess) e = dalloc(ctx, &ctx->cb_biases, (size_t)size);
      if (e == cudaSuccess) ctx->cb_cap = size;
    }
    if (e == cudaSuccess) e = cudaMemcpy(ctx->cb_keys, keys, (size_t)size * 8, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
      e = cudaMemcpy(ctx->cb_tokens, tokens, (size_t)size * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
      e = cudaMemcpy(ctx->cb_biases, biases, (size_t)size * 4, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
  // an all-zero (or empty) table changes nothing: the step stays without it
  ctx->cbias_on = any;
  ctx->cbias.keys = any ? ctx->cb_keys : nullptr;
  ctx->cbias.tokens = any ? ctx->cb_tokens : nullptr;
  ctx->cbias.biases = any ? ctx->cb_biases : nullptr;
  ctx->cbias.size = any ? size : 0;
  if (ctx->gexec) {
    // the captured step changes shape: capture again on the next step
    cudaGraphExecDestroy(ctx->gexec);
    ctx->gexec = nullptr;
  }
  return EC_OK;
}

extern "C" int ec_set_weight_bf16(ec_ctx* ctx, int layer, int which, const uint16_t* data,
                                  int on_device) {
  if (!ctx || !data) return fail(EC_ERR_ARG, "null argument");
  const ec_model_config& c = ctx->cg;  // the whole matrix comes in (a shard is taken later)
  const int D = c.dim, F = c.hidden_dim, QD = c.n_heads * c.head_dim, KVD = c.n_kv_heads * c.head_dim;
  int rows = 0, cols = 0;
  if (layer < 0 && which == EC_LM_HEAD) {
    rows = c.vocab_size;
    cols = D;
  } else if (layer >= 0) {
    switch (which) {
      case EC_WQ: rows = QD; cols = D; break;
      case EC_WK: case EC_WV: rows = KVD; cols = D; break;
      case EC_WO: rows = D; cols = QD; break;
      case EC_W1: case EC_W3: rows = F; cols = D; break;
      case EC_W2: rows = D; cols = F; break;
      default: break;
    }
  }
  if (!rows) return ec_set_weight(ctx, layer, which, data, nullptr, on_device);
  cudaSetDevice(ctx->device);
  if (on_device) EC_CUDA_TRY(cudaDeviceSynchronize());
  const size_t n = (size_t)rows * cols;
  uint16_t* bf = nullptr;
  uint8_t* q = nullptr;
  float* sc = nullptr;
  unsigned* amax = nullptr;
  auto release = [&]() {
    if (!on_device) cudaFree(bf);
    cudaFree(q);
    cudaFree(sc);
    cudaFree(amax);
  };
  cudaError_t e = cudaSuccess;
  if (!on_device) {
    e = cudaMalloc(&bf, n * 2);
    // on the stream the quantisation runs on: a pageable cudaMemcpy may
    // return before its DMA has landed, and ctx->stream does not wait for it
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(bf, data, n * 2, cudaMemcpyHostToDevice, ctx->stream);
  } else {
    bf = const_cast<uint16_t*>(data);
  }
  if (e == cudaSuccess) e = cudaMalloc(&q, n);
  if (e == cudaSuccess) e = cudaMalloc(&sc, (size_t)rows * 4);
  if (e == cudaSuccess) {
    if (c.weight_kind == EC_W_INT8) {
      e = ec::launch_quant_rows_int8(bf, reinterpret_cast<int8_t*>(q), sc, rows, cols, ctx->stream);
    } else {
      e = cudaMalloc(&amax, 4);
      if (e == cudaSuccess) e = cudaMemsetAsync(amax, 0, 4, ctx->stream);
      if (e == cudaSuccess) e = ec::launch_absmax_bf16(bf, (long)n, amax, ctx->stream);
      unsigned bits = 0;
      if (e == cudaSuccess) e = cudaMemcpyAsync(&bits, amax, 4, cudaMemcpyDeviceToHost, ctx->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
      if (e == cudaSuccess) {
        float m = 0.0f;
        memcpy(&m, &bits, 4);
        const float s = m > 0.0f ? (float)exp2(ceil(log2((double)m / 448.0))) : 1.0f;
        e = ec::launch_quant_fp8(bf, q, (long)n, s, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e == cudaSuccess) e = cudaMemcpy(sc, &s, 4, cudaMemcpyHostToDevice);
      }
    }
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    release();
    return fail(EC_ERR_CUDA, cudaGetErrorString(e));
  }
  const int rc = ec_set_weight(ctx, layer, which, q, sc, 1);
  release();
  return rc;
}

extern "C" int ec_reset(ec_ctx* ctx, int seq) {
  if (!ctx || seq < 0 || seq >= ctx->c.max_batch) return fail(EC_ERR_ARG, "bad sequence");
  cudaSetDevice(ctx->device);
  const ec::KvLayout& kv = ctx->kv;
  const size_t per = (size_t)kv.n_layers * kv.max_blocks;
  if (kv.paged) {
    EC_CUDA_TRY(cudaMemsetAsync(kv.centroid + seq * per * kv.head_dim, 0,
                                per * kv.head_dim * 4, ctx->stream));
  }
  const ec::LshLayout& l = ctx->lsh;
  if (l.tables > 0) {
    EC_CUDA_TRY(cudaMemsetAsync(l.acc + (size_t)seq * kv.head_dim, 0, kv.head_dim * 4, ctx->stream));
    EC_CUDA_TRY(cudaMemsetAsync(l.meta + seq * 4, 0, 16, ctx->stream));
    EC_CUDA_TRY(cudaMemsetAsync(l.heads + (((size_t)seq * l.tables) << l.bits), 0xFF,
                                ((size_t)l.tables << l.bits) * 4, ctx->stream));
    EC_CUDA_TRY(cudaMemsetAsync(l.counters + seq * 2, 0, 16, ctx->stream));
  }
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return EC_OK;
}

namespace {

double gemv_bytes(const Mat& m, int pro, int epi) {
  return (double)m.rows * m.cols + 4.0 * m.rows + 4.0 * m.cols +
         (pro == ec::PRO_RMSNORM ? 2.0 * m.cols : 0.0) +
         (epi == ec::EPI_SWIGLU ? 2.0 * m.rows : 4.0 * m.rows) +
         (epi == ec::EPI_RESID ? 4.0 * m.rows : 0.0);
}

cudaError_t gemv(ec_ctx* ctx, int kind, const Mat& m, const ec::PackedPlan& plan, int pro,
                 int epi, const float* x, const uint16_t* nw, float* y) {
  // algorithmic bytes: weights + row scales + x (+ norm weight) + y (+ y read)
  ProfScope ps(ctx, kind, gemv_bytes(m, pro, epi));
  ec::GemvParams p{};
  p.w = m.w;
  p.scale = m.scale;
  p.scale_stride = 1;
  p.x = x;
  p.norm_w = nw;
  p.eps = ctx->c.norm_eps;
  p.y = y;
  p.N = m.rows;
  p.K = m.cols;
  p.silu_vec_limit = (m.rows / 2) & ~7;
  p.err = ctx->err;
  ctx->launches++;
  return ec::packed_launch(ctx->c.weight_kind, pro, epi, plan, p, ctx->stream, true);
}

ec::ChainPhase chain_phase(const Mat& m, int pro, int epi, const float* x, const uint16_t* nw,
                           float* y) {
  ec::ChainPhase ph{};
  ph.w = m.w;
  ph.scale = m.scale;
  ph.x = x;
  ph.norm_w = nw;
  ph.y = y;
  ph.N = m.rows;
  ph.K = m.cols;
  ph.pro = pro;
  ph.epi = epi;
  ph.silu_vec_limit = (m.rows / 2) & ~7;
  return ph;
}

// The end of the step after the last layer's down projection when a final
// adapter or logit bias is registered (inference.c:580-651): RMSNorm of x
// (rows of D floats) into xn, the adapter xn -> xa, the LM head on it
// (lm(in, out, rows) issues the caller's GEMV), the logit bias.
// The embedding launch's token history: rows of sequences seq0.. or, in a
// prefill, rows of one sequence.
ec::TokenHistory token_history(ec_ctx* ctx, const int* pos, int seq0, int prefill_seq = -1) {
  ec::TokenHistory th;
  th.pos = pos;
  th.hist = ctx->tok_hist;
  th.seq_len = ctx->c.seq_len;
  th.seq0 = seq0;
  th.seq_plus1 = prefill_seq >= 0 ? prefill_seq + 1 : 0;
  return th;
}

// The context bias (inference.c:657-693) on B rows of logits, when a table
// with a key is registered; before the argmax, which advances positions.
cudaError_t enqueue_context_bias(ec_ctx* ctx, float* logits, int V, int B,
                                 const ec::TokenHistory& th) {
  if (!ctx->cbias_on) return cudaSuccess;
  ctx->launches++;
  return ec::launch_context_bias(logits, V, B, th, ctx->cbias, ctx->stream);
}

template <typename LM>
cudaError_t enqueue_final_extras(ec_ctx* ctx, const float* x, float* xn, float* xa, int B,
                                 float* logits, LM lm) {
  const ec_model_config& c = ctx->c;
  cudaError_t e;
  if ((e = ec::launch_rmsnorm_rows(xn, x, ctx->final_norm, c.dim, c.norm_eps, B, c.dim,
                                   ctx->stream)))
    return e;
  ctx->launches++;
  const float* in = xn;
  if (ctx->adapter_on) {
    if ((e = ec::launch_adapter(ctx->adapter, xn, xa, c.dim, B, ctx->stream))) return e;
    ctx->launches++;
    in = xa;
  }
  if ((e = lm(in, logits, B))) return e;
  if (ctx->bias_on) {
    if ((e = ec::launch_logit_bias(logits, ctx->logit_bias, c.vocab_size, B, ctx->stream)))
      return e;
    ctx->launches++;
  }
  return cudaSuccess;
}

// One layer's attention block after the QKV projection: the split path
// (append + rank selection, split attention) or the reference-order path
// (append + heap selection | linear-mode selection, attention).
cudaError_t enqueue_attention(ec_ctx* ctx, const ec::KvLayout& kv, const ec::LshLayout& lsh,
                              ec::StepBuffers& sb, int l, int B, bool split) {
  cudaError_t e;
  if (split) {
    {
      ProfScope ps(ctx, EC_K_KV_APPEND, 0.0);
      if ((e = ec::launch_fast_select(kv, lsh, sb, l, B, ctx->stream, true))) return e;
    }
    ProfScope ps(ctx, EC_K_ATTENTION, 0.0);
    if ((e = ec::launch_fast_attend(kv, sb, l, B, ctx->stream, true)))
      return e;
    ctx->launches += 2;
    return cudaSuccess;
  }
  {
    ProfScope ps(ctx, EC_K_KV_APPEND, 0.0);
    if ((e = ec::launch_kv_append(kv, lsh, sb, l, B, ctx->stream, true))) return e;
  }
  ctx->launches++;
  if (!kv.paged) {
    ProfScope ps(ctx, EC_K_SELECT, 0.0);
    if ((e = ec::launch_linear_select(kv, lsh, sb, l, B, ctx->stream, true))) return e;
    ctx->launches += ec::kLinearSelectLaunches;
  }
  ProfScope ps(ctx, EC_K_ATTENTION, 0.0);
  if ((e = ec::launch_attention(kv, sb, l, B, ctx->stream, true))) return e;
  ctx->launches++;
  return cudaSuccess;
}

// The batched step (B > 1 with the chain): every sequence-parallel kernel runs
// once for all B sequences; the weight-streaming GEMVs run as one batched
// chain per layer per pack of up to kPack sequences.
cudaError_t enqueue_step_batched(ec_ctx* ctx, const int* tokens, const int* pos, int B,
                                 bool feedback, int prefill_seq = -1, int prefill_pos0 = 0) {
  const ec_model_config& c = ctx->c;
  const int H = c.n_heads, KV = c.n_kv_heads, hd = c.head_dim, D = c.dim, F = c.hidden_dim;
  const int V = c.vocab_size, L = c.n_layers, QW = (H + 2 * KV) * hd;
  const bool extras = ctx->adapter_on || ctx->bias_on;
  cudaError_t e;
  ctx->launches = 0;
  ec::StepBuffers sb{};
  sb.rope_cos = ctx->rope_cos;
  sb.rope_sin = ctx->rope_sin;
  sb.sparse_k = c.sparse_k;
  sb.window = c.window;
  sb.sparse_blocks_k = c.sparse_blocks_k;
  sb.err = ctx->err;
  sb.max_sel = ctx->max_sel;
  sb.pos = pos;
  sb.qkv = ctx->qkvb;
  sb.qrot = ctx->qrot;
  sb.att = ctx->att;
  sb.sel = ctx->sel;
  sb.selp = ctx->selp;
  sb.nsel = ctx->nsel;
  sb.lcand = ctx->lcand;
  sb.lscore = ctx->lscore;
  sb.lnc = ctx->lnc;
  // prefill: the B rows are consecutive tokens of one sequence (paged KV)
  ec::KvLayout kv = ctx->kv;
  if (prefill_seq >= 0) {
    kv.seq_plus1 = prefill_seq + 1;
    sb.defer_centroid = 1;
  }
  auto phase = [&](const Mat& m, int pro, int epi, const float* x, int xs, const uint16_t* nw,
                   float* y, int ys) {
    ec::ChainPhase ph = chain_phase(m, pro, epi, x, nw, y);
    ph.x_stride = xs;
    ph.y_stride = ys;
    return ph;
  };
  auto norm = [&](const float* x, const uint16_t* nw, float* y) {
    ec::ChainPhase ph{};
    ph.x = x;
    ph.norm_w = nw;
    ph.y = y;
    ph.K = D;
    ph.pro = ec::PRO_NORM_ROWS;
    ph.x_stride = D;
    ph.y_stride = D;
    return ph;
  };
  auto run = [&](ec::ChainParams& P, int layer_slot, int pack, int nb) -> cudaError_t {
    P.ctr = ctx->chain_ctr +
            ((size_t)layer_slot * ctx->npacks + pack) * (ec::kMaxChainPhases + 1);
    P.err = ctx->err;
    P.eps = c.norm_eps;
    P.wait_iters = c.wait_limit < 0 ? -c.wait_limit : c.wait_limit;
    P.wait_extra = c.wait_limit < 0 ? 1 : 0;
    double by = 0;
    for (int i = 0; i < P.nph; i++)
      if (P.ph[i].pro != ec::PRO_NORM_ROWS) by += (double)P.ph[i].N * P.ph[i].K;
    ProfScope ps(ctx, EC_K_GEMV_CHAIN, by);
    ctx->launches++;
    if (nb == 1) return ec::chain_launch(c.weight_kind, P, ctx->n_sm, ctx->stream, true);
    return ec::chain_launch_nb(c.weight_kind, P, nb, ctx->n_sm, ctx->stream, true);
  };
  {
    ProfScope ps(ctx, EC_K_EMBED, (2.0 + 4.0) * D * B);
    const ec::TokenHistory th = token_history(ctx, pos, 0, prefill_seq);
    if ((e = ec::launch_embed(ctx->emb, tokens, ctx->x, D, c.vocab_size, B, ctx->stream, true,
                              &th)))
      return e;
    ctx->launches++;
  }
  // layer 0's QKV (its own counter block: slot L)
  for (int b0 = 0, pk = 0; b0 < B; b0 += kPack, pk++) {
    const int nb = B - b0 < kPack ? B - b0 : kPack;
    ec::ChainParams P{};
    if (nb == 1) {
      P.ph[0] = chain_phase(ctx->qkv[0], ec::PRO_RMSNORM, ec::EPI_STORE, ctx->x + (size_t)b0 * D,
                            ctx->attn_norm[0], ctx->qkvb + (size_t)b0 * QW);
      P.nph = 1;
    } else {
      P.ph[0] = norm(ctx->x + (size_t)b0 * D, ctx->attn_norm[0], ctx->xn + (size_t)b0 * D);
      P.ph[1] = phase(ctx->qkv[0], ec::PRO_NONE, ec::EPI_STORE, ctx->xn + (size_t)b0 * D, D, nullptr,
                      ctx->qkvb + (size_t)b0 * QW, QW);
      P.nph = 2;
    }
    if ((e = run(P, L, pk, nb))) return e;
  }
  const bool split = ctx->fast && prefill_seq < 0 && !ec::use_group_attention(kv, sb, B);
  for (int l = 0; l < L; l++) {
    if (split) {
      if ((e = enqueue_attention(ctx, kv, ctx->lsh, sb, l, B, true))) return e;
    } else {
      ProfScope ps(ctx, EC_K_KV_APPEND, 0.0);
      if ((e = ec::launch_kv_append(kv, ctx->lsh, sb, l, B, ctx->stream, true))) return e;
      ctx->launches++;
    }
    if (prefill_seq >= 0) {
      // every row's token is in the cache: the centroids of the blocks this
      // chunk filled, the layer-0 LSH update in row order, then (paged) each
      // row's block selection; linear mode selects below, each row seeing
      // the LSH units that end by its own position
      ProfScope ps(ctx, EC_K_SELECT, 0.0);
      if (kv.paged) {
        if ((e = ec::launch_paged_centroids(kv, l, prefill_seq, prefill_pos0, B, ctx->stream)))
          return e;
        ctx->launches++;
      }
      if (l == 0) {
        if ((e = ec::launch_lsh_update_rows(kv, ctx->lsh, sb, B, ctx->stream))) return e;
        if (ctx->lsh.tables > 0) ctx->launches++;
      }
      if (kv.paged) {
        if ((e = ec::launch_paged_select_rows(kv, sb, l, B, ctx->stream))) return e;
        ctx->launches++;
      }
    }
    if (!kv.paged && !split) {
      ProfScope ps(ctx, EC_K_SELECT, 0.0);
      if ((e = ec::launch_linear_select(kv, ctx->lsh, sb, l, B, ctx->stream, true))) return e;
      ctx->launches += ec::kLinearSelectLaunches;
    }
    if (!split) {
      ProfScope ps(ctx, EC_K_ATTENTION, 0.0);
      if ((e = ec::launch_attention(kv, sb, l, B, ctx->stream, true))) return e;
      ctx->launches++;
    }
    const bool last = l + 1 == L;
    for (int b0 = 0, pk = 0; b0 < B; b0 += kPack, pk++) {
      const int nb = B - b0 < kPack ? B - b0 : kPack;
      float* x = ctx->x + (size_t)b0 * D;
      float* xn = ctx->xn + (size_t)b0 * D;
      float* hb = ctx->hbuf + (size_t)b0 * F;
      float* att = ctx->att + (size_t)b0 * H * hd;
      ec::ChainParams P{};
      if (nb == 1) {
        P.ph[0] = chain_phase(ctx->wo[l], ec::PRO_NONE, ec::EPI_RESID, att, nullptr, x);
        P.ph[1] = chain_phase(ctx->w13[l], ec::PRO_RMSNORM, ec::EPI_SWIGLU, x, ctx->ffn_norm[l], hb);
        P.ph[2] = chain_phase(ctx->w2[l], ec::PRO_NONE, ec::EPI_RESID, hb, nullptr, x);
        P.ph[3] = last ? chain_phase(ctx->lm, ec::PRO_RMSNORM, ec::EPI_STORE, x, ctx->final_norm,
                                     ctx->logits + (size_t)b0 * V)
                       : chain_phase(ctx->qkv[l + 1], ec::PRO_RMSNORM, ec::EPI_STORE, x,
                                     ctx->attn_norm[l + 1], ctx->qkvb + (size_t)b0 * QW);
        P.nph = (last && extras) ? 3 : 4;
      } else {
        P.ph[0] = phase(ctx->wo[l], ec::PRO_NONE, ec::EPI_RESID, att, H * hd, nullptr, x, D);
        P.ph[1] = norm(x, ctx->ffn_norm[l], xn);
        P.ph[2] = phase(ctx->w13[l], ec::PRO_NONE, ec::EPI_SWIGLU, xn, D, nullptr, hb, F);
        P.ph[3] = phase(ctx->w2[l], ec::PRO_NONE, ec::EPI_RESID, hb, F, nullptr, x, D);
        P.ph[4] = norm(x, last ? ctx->final_norm : ctx->attn_norm[l + 1], xn);
        P.ph[5] = last ? phase(ctx->lm, ec::PRO_NONE, ec::EPI_STORE, xn, D, nullptr,
                               ctx->logits + (size_t)b0 * V, V)
                       : phase(ctx->qkv[l + 1], ec::PRO_NONE, ec::EPI_STORE, xn, D, nullptr,
                               ctx->qkvb + (size_t)b0 * QW, QW);
        P.nph = (last && extras) ? 4 : 6;
      }
      if ((e = run(P, l, pk, nb))) return e;
    }
  }
  if (extras) {
    // final RMSNorm, adapter, then the LM head as one-phase chains per pack
    auto lm = [&](const float* in, float* out, int rows) -> cudaError_t {
      for (int b0 = 0, pk = 0; b0 < rows; b0 += kPack, pk++) {
        const int nb = rows - b0 < kPack ? rows - b0 : kPack;
        ec::ChainParams P{};
        P.ph[0] = phase(ctx->lm, ec::PRO_NONE, ec::EPI_STORE, in + (size_t)b0 * D, D, nullptr,
                        out + (size_t)b0 * V, V);
        P.nph = 1;
        cudaError_t e2 = run(P, L, pk, nb);
        if (e2) return e2;
      }
      return cudaSuccess;
    };
    if ((e = enqueue_final_extras(ctx, ctx->x, ctx->xn, ctx->xa, B, ctx->logits, lm))) return e;
  }
  if ((e = enqueue_context_bias(ctx, ctx->logits, V, B, token_history(ctx, pos, 0, prefill_seq))))
    return e;
  {
    ProfScope ps(ctx, EC_K_ARGMAX, 4.0 * V * B);
    // one launch for all B sequences (scratch slice b per sequence)
    if ((e = ec::launch_argmax_split(ctx->logits, V, B, ctx->argmax,
                                     feedback ? const_cast<int*>(tokens) : nullptr,
                                     feedback ? const_cast<int*>(pos) : nullptr, ctx->amax,
                                     ctx->stream, true)))
      return e;
    ctx->launches++;
  }
  return cudaSuccess;
}

// The batched step on the tensor cores (B >= tensor_min_batch, INT8): the
// sequence-parallel kernels as in enqueue_step_batched; every projection is
// tc_quant (RMSNorm when the reference has one, digit planes) -> tc_gemm
// (tcgen05, whole tiles finished in its epilogue) -> tc_combine (tiles split
// between CTAs), per pass of up to kTcMaxRows sequences.
cudaError_t enqueue_step_tc(ec_ctx* ctx, const int* tokens, const int* pos, int B, bool feedback,
                            int prefill_seq = -1, int prefill_pos0 = 0) {
  const ec_model_config& c = ctx->c;
  const int H = c.n_heads, KV = c.n_kv_heads, hd = c.head_dim, D = c.dim, F = c.hidden_dim;
  const int V = c.vocab_size, L = c.n_layers, QW = (H + 2 * KV) * hd;
  const bool extras = ctx->adapter_on || ctx->bias_on;
  cudaError_t e;
  ctx->launches = 0;
  ec::StepBuffers sb{};
  sb.rope_cos = ctx->rope_cos;
  sb.rope_sin = ctx->rope_sin;
  sb.sparse_k = c.sparse_k;
  sb.window = c.window;
  sb.sparse_blocks_k = c.sparse_blocks_k;
  sb.err = ctx->err;
  sb.max_sel = ctx->max_sel;
  sb.pos = pos;
  sb.qkv = ctx->qkvb;
  sb.qrot = ctx->qrot;
  sb.att = ctx->att;
  sb.sel = ctx->sel;
  sb.selp = ctx->selp;
  sb.nsel = ctx->nsel;
  sb.lcand = ctx->lcand;
  sb.lscore = ctx->lscore;
  sb.lnc = ctx->lnc;
  // one projection of nb rows: x [nb][K] (x_stride apart) -> y per epi
  auto proj = [&](const Mat& m, const float* x, int xs, const uint16_t* nw, float* y, int ys,
                  int epi, int nb) -> cudaError_t {
    ec::TcQuant q{};
    q.x = x;
    q.x_stride = xs;
    q.norm_w = nw;
    q.eps = c.norm_eps;
    q.digits = ctx->tc_digits;
    q.sx = ctx->tc_sx;
    q.B = nb;
    q.K = m.cols;
    ec::TcGemm g{};
    g.w = m.tc;
    g.digits = ctx->tc_digits;
    g.ws = ctx->tc_ws;
    g.N = m.rows;
    g.K = m.cols;
    g.B = nb;
    g.grid = ctx->n_sm;
    g.err = ctx->err;
    g.out.sx = ctx->tc_sx;
    g.out.scale = m.scale;
    g.out.y = y;
    g.out.y_stride = ys;
    g.out.epi = epi;
    g.out.silu_vec_limit = (m.rows / 2) & ~7;
    cudaError_t e2;
    {
      ProfScope ps(ctx, EC_K_TC_QUANT, 4.0 * nb * m.cols + (double)ec::tc_digit_bytes(nb, m.cols));
      if ((e2 = ec::tc_quant(q, ctx->stream, true))) return e2;
    }
    {
      ProfScope ps(ctx, EC_K_TC_GEMM, (double)m.rows * m.cols + 4.0 * m.rows);
      if ((e2 = ec::tc_gemm(g, ctx->stream, true))) return e2;
    }
    ProfScope ps(ctx, EC_K_TC_COMBINE, 0.0);
    ctx->launches += 3;
    return ec::tc_combine(g, ctx->stream, true);
  };
  {
    ProfScope ps(ctx, EC_K_EMBED, (2.0 + 4.0) * D * B);
    const ec::TokenHistory th = token_history(ctx, pos, 0, prefill_seq);
    if ((e = ec::launch_embed(ctx->emb, tokens, ctx->x, D, c.vocab_size, B, ctx->stream, true,
                              &th)))
      return e;
    ctx->launches++;
  }
  for (int b0 = 0; b0 < B; b0 += ec::kTcMaxRows) {
    const int nb = B - b0 < ec::kTcMaxRows ? B - b0 : ec::kTcMaxRows;
    if ((e = proj(ctx->qkv[0], ctx->x + (size_t)b0 * D, D, ctx->attn_norm[0],
                  ctx->qkvb + (size_t)b0 * QW, QW, ec::EPI_STORE, nb)))
      return e;
  }
  // prefill (ec_prefill): the B rows are consecutive tokens of one sequence,
  // as in enqueue_step_batched
  ec::KvLayout kv = ctx->kv;
  if (prefill_seq >= 0) {
    kv.seq_plus1 = prefill_seq + 1;
    sb.defer_centroid = 1;
  }
  for (int l = 0; l < L; l++) {
    if (prefill_seq < 0) {
      if ((e = enqueue_attention(ctx, kv, ctx->lsh, sb, l, B,
                                 ctx->fast && !ec::use_group_attention(kv, sb, B))))
        return e;
    } else {
      {
        ProfScope ps(ctx, EC_K_KV_APPEND, 0.0);
        if ((e = ec::launch_kv_append(kv, ctx->lsh, sb, l, B, ctx->stream, true))) return e;
      }
      // every row's token is in the cache: the chunk's block centroids, the
      // layer-0 LSH update in row order, each row's selection (paged blocks,
      // or linear candidates from the LSH units that end by the row's
      // position)
      ProfScope ps(ctx, EC_K_SELECT, 0.0);
      if (kv.paged &&
          (e = ec::launch_paged_centroids(kv, l, prefill_seq, prefill_pos0, B, ctx->stream)))
        return e;
      if (l == 0 && (e = ec::launch_lsh_update_rows(kv, ctx->lsh, sb, B, ctx->stream))) return e;
      if (kv.paged) {
        if ((e = ec::launch_paged_select_rows(kv, sb, l, B, ctx->stream))) return e;
      } else if ((e = ec::launch_linear_select(kv, ctx->lsh, sb, l, B, ctx->stream, true))) {
        return e;
      }
      if ((e = ec::launch_attention(kv, sb, l, B, ctx->stream, true))) return e;
      ctx->launches += (kv.paged ? 4 : 2 + ec::kLinearSelectLaunches) +
                       (l == 0 && ctx->lsh.tables > 0);
    }
    const bool last = l + 1 == L;
    for (int b0 = 0; b0 < B; b0 += ec::kTcMaxRows) {
      const int nb = B - b0 < ec::kTcMaxRows ? B - b0 : ec::kTcMaxRows;
      float* x = ctx->x + (size_t)b0 * D;
      float* hb = ctx->hbuf + (size_t)b0 * F;
      const float* att = ctx->att + (size_t)b0 * H * hd;
      if ((e = proj(ctx->wo[l], att, H * hd, nullptr, x, D, ec::EPI_RESID, nb))) return e;
      if ((e = proj(ctx->w13[l], x, D, ctx->ffn_norm[l], hb, F, ec::EPI_SWIGLU, nb))) return e;
      if ((e = proj(ctx->w2[l], hb, F, nullptr, x, D, ec::EPI_RESID, nb))) return e;
      if (last && extras)
        e = cudaSuccess;  // the LM head runs after the adapter and bias below
      else if (last)
        e = proj(ctx->lm, x, D, ctx->final_norm, ctx->logits + (size_t)b0 * V, V, ec::EPI_STORE, nb);
      else
        e = proj(ctx->qkv[l + 1], x, D, ctx->attn_norm[l + 1], ctx->qkvb + (size_t)b0 * QW, QW,
                 ec::EPI_STORE, nb);
      if (e) return e;
    }
  }
  if (extras) {
    auto lm = [&](const float* in, float* out, int rows) -> cudaError_t {
      for (int b0 = 0; b0 < rows; b0 += ec::kTcMaxRows) {
        const int nb = rows - b0 < ec::kTcMaxRows ? rows - b0 : ec::kTcMaxRows;
        cudaError_t e2 = proj(ctx->lm, in + (size_t)b0 * D, D, nullptr, out + (size_t)b0 * V, V,
                              ec::EPI_STORE, nb);
        if (e2) return e2;
      }
      return cudaSuccess;
    };
    if ((e = enqueue_final_extras(ctx, ctx->x, ctx->xn, ctx->xa, B, ctx->logits, lm))) return e;
  }
  if ((e = enqueue_context_bias(ctx, ctx->logits, V, B, token_history(ctx, pos, 0, prefill_seq))))
    return e;
  {
    ProfScope ps(ctx, EC_K_ARGMAX, 4.0 * V * B);
    // one launch for all B sequences (scratch slice b per sequence)
    if ((e = ec::launch_argmax_split(ctx->logits, V, B, ctx->argmax,
                                     feedback ? const_cast<int*>(tokens) : nullptr,
                                     feedback ? const_cast<int*>(pos) : nullptr, ctx->amax,
                                     ctx->stream, true)))
      return e;
    ctx->launches++;
  }
  return cudaSuccess;
}

// Tensor-parallel decode step (ec_create_tp): this rank holds heads, KV
// heads, hidden rows and vocabulary rows [rank * n, (rank + 1) * n).  Per
// sequence and layer:
//   QKV (this rank's heads) -> RoPE + append (its KV heads) -> [layer 0:
//   keys gathered, LSH update of KV head 0 on every rank] -> paged: the block
//   selection of rank 0 (query head 0, KV head 0's centroids) broadcast |
//   linear: queries gathered for the LSH query mean, per-head candidate dots
//   gathered and added in head order, heap on every rank -> attention (its
//   heads) -> o partial -> gather, x += partials in rank order -> gate/up
//   (RMSNorm of the replicated x) + down partial -> gather, x += -> next QKV;
//   after the last layer the LM head rows, gathered into the whole logits.
// Every rank keeps identical x, selections and logits.  Collectives are
// NCCL all-gathers / broadcasts on the context stream (captured in the
// step graph); the sums over ranks run in rank order in the engine's own
// kernels, so the result does not depend on NCCL's reduction order.
cudaError_t enqueue_step_tp(ec_ctx* ctx, const int* tokens, const int* pos, int B, bool feedback) {
  const ec_model_config& c = ctx->c;
  const ec_model_config& g = ctx->cg;
  const int H = c.n_heads, KV = c.n_kv_heads, hd = c.head_dim, D = c.dim, F = c.hidden_dim;
  const int W = ctx->tp_world, Vg = g.vocab_size, L = c.n_layers;
  const ec::NcclApi* api = ec::nccl_api(nullptr);
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl);
  cudaError_t e;
  ctx->launches = 0;
  auto gather = [&](const void* send, void* recv, size_t count) -> cudaError_t {
    const ncclResult_t r = api->all_gather(send, recv, count, ncclFloat32, comm, ctx->stream);
    if (r != ncclSuccess) {
      ec_set_last_error(api->error_string(r));
      return cudaErrorUnknown;
    }
    return cudaSuccess;
  };
  auto bcast = [&](void* buf, size_t count) -> cudaError_t {
    const ncclResult_t r = api->broadcast(buf, buf, count, ncclInt32, 0, comm, ctx->stream);
    if (r != ncclSuccess) {
      ec_set_last_error(api->error_string(r));
      return cudaErrorUnknown;
    }
    return cudaSuccess;
  };
  // one or more GEMV phases: the chain kernel, or one launch per matrix
  auto phases = [&](ec::ChainParams& P, int slot, const ec::PackedPlan* plans[],
                    int kinds[]) -> cudaError_t {
    if (ctx->chain) {
      P.ctr = ctx->chain_ctr + (size_t)slot * ctx->npacks * (ec::kMaxChainPhases + 1);
      P.err = ctx->err;
      P.eps = c.norm_eps;
      double by = 0.0;  // weights, row scales and vectors of the phases
      for (int i = 0; i < P.nph; i++)
        by += (double)P.ph[i].N * P.ph[i].K + 8.0 * P.ph[i].N + 4.0 * P.ph[i].K;
      ProfScope ps(ctx, EC_K_GEMV_CHAIN, by);
      ctx->launches++;
      return ec::chain_launch(c.weight_kind, P, ctx->n_sm, ctx->stream, true);
    }
    for (int i = 0; i < P.nph; i++) {
      const ec::ChainPhase& ph = P.ph[i];
      Mat m;
      m.w = const_cast<uint8_t*>(ph.w);
      m.scale = const_cast<float*>(ph.scale);
      m.rows = ph.N;
      m.cols = ph.K;
      cudaError_t e2 = gemv(ctx, kinds[i], m, *plans[i], ph.pro, ph.epi, ph.x, ph.norm_w, ph.y);
      if (e2) return e2;
    }
    return cudaSuccess;
  };
  ec::StepBuffers sb{};
  sb.rope_cos = ctx->rope_cos;
  sb.rope_sin = ctx->rope_sin;
  sb.sparse_k = c.sparse_k;
  sb.window = c.window;
  sb.sparse_blocks_k = c.sparse_blocks_k;
  sb.err = ctx->err;
  sb.max_sel = ctx->max_sel;
  for (int b = 0; b < B; b++) {
    float* x = ctx->x + (size_t)b * D;
    sb.pos = pos + b;
    sb.qkv = ctx->qkvb + (size_t)b * (H + 2 * KV) * hd;
    sb.qrot = ctx->qrot + (size_t)b * H * hd;
    sb.att = ctx->att + (size_t)b * H * hd;
    sb.sel = ctx->sel + (size_t)b * ctx->max_sel;
    sb.selp = ctx->selp + (size_t)b * ctx->max_sel;
    sb.nsel = ctx->nsel + b;
    if (ctx->lcand) {
      sb.lcand = ctx->lcand + (size_t)b * ctx->cap_c;
      sb.lscore = ctx->lscore + (size_t)b * ctx->cap_c;
      sb.lnc = ctx->lnc + b;
    }
    ec::KvLayout kv = ctx->kv;
    ec::LshLayout lsh = ctx->lsh;
    const size_t per = (size_t)kv.n_layers * kv.max_blocks;
    if (kv.paged) {
      kv.kq += b * per * KV * 16 * hd;
      kv.vq += b * per * KV * 16 * hd;
      kv.ks += b * per * KV * 16;
      kv.vs += b * per * KV * 16;
      kv.centroid += b * per * hd;
      kv.page_table += b * per;
    } else {
      kv.lk += (size_t)b * kv.n_layers * kv.seq_len * KV * hd;
      kv.lv += (size_t)b * kv.n_layers * kv.seq_len * KV * hd;
    }
    if (lsh.tables > 0) {
      lsh.acc += (size_t)b * hd;
      lsh.meta += b * 4;
      lsh.unit_hash += (size_t)b * lsh.tables * lsh.max_units;
      lsh.unit_start += (size_t)b * lsh.max_units;
      lsh.unit_len += (size_t)b * lsh.max_units;
      lsh.heads += ((size_t)b * lsh.tables) << lsh.bits;
      lsh.next += (size_t)b * lsh.tables * lsh.max_units;
      lsh.counters += b * 2;
    }
    ec::LshLayout no_lsh = lsh;  // the append leaves the LSH update to the gathered keys
    no_lsh.tables = 0;
    const ec::TokenHistory th = token_history(ctx, pos + b, b);
    if ((e = ec::launch_embed(ctx->emb, tokens + b, x, D, Vg, 1, ctx->stream, true, &th))) return e;
    ctx->launches++;
    float* hb = ctx->hbuf + (size_t)b * F;
    int kinds[2];
    const ec::PackedPlan* plans[2];
    for (int l = 0; l < L; l++) {
      if (l == 0) {
        ec::ChainParams P{};
        P.ph[0] = chain_phase(ctx->qkv[0], ec::PRO_RMSNORM, ec::EPI_STORE, x, ctx->attn_norm[0],
                              sb.qkv);
        P.nph = 1;
        kinds[0] = EC_K_GEMV_QKV;
        plans[0] = &ctx->p_qkv;
        if ((e = phases(P, L, plans, kinds))) return e;
      }
      {
        ProfScope ps(ctx, EC_K_KV_APPEND, 0.0);
        if ((e = ec::launch_kv_append(kv, no_lsh, sb, l, 1, ctx->stream, true))) return e;
        ctx->launches++;
      }
      if (l == 0 && lsh.tables > 0) {
        // lsh_update of KV head 0 (rank 0's first head) on every rank
        if ((e = gather(sb.qkv + H * hd, ctx->tp_k, (size_t)KV * hd))) return e;
        if ((e = ec::launch_lsh_update_key(lsh, sb, ctx->tp_k, hd, ctx->stream))) return e;
        ctx->launches++;
      }
      if (kv.paged) {
        // rank 0 scored the blocks with query head 0 and KV head 0's centroids
        if ((e = bcast(sb.sel, (size_t)ctx->max_sel))) return e;
        if ((e = bcast(sb.nsel, 1))) return e;
      } else {
        ProfScope ps(ctx, EC_K_SELECT, 0.0);
        if ((e = gather(sb.qrot, ctx->tp_q, (size_t)H * hd))) return e;
        ec::StepBuffers s2 = sb;
        s2.q_all = ctx->tp_q;
        s2.h_all = g.n_heads;
        s2.score_parts = ctx->tp_sp;
        if ((e = ec::launch_linear_candidates(kv, lsh, s2, l, 1, ctx->stream))) return e;
        if ((e = ec::launch_linear_score_parts(kv, lsh, s2, l, 1, ctx->stream))) return e;
        if ((e = gather(ctx->tp_sp, ctx->tp_sps, (size_t)ctx->cap_c * KV))) return e;
        if ((e = ec::launch_linear_sum_heap(lsh, sb, ctx->tp_sps, W, KV, 1, ctx->stream))) return e;
        ctx->launches += 4;
      }
      {
        ProfScope ps(ctx, EC_K_ATTENTION, 0.0);
        if ((e = ec::launch_attention(kv, sb, l, 1, ctx->stream, false))) return e;
        ctx->launches++;
      }
      {
        // o: this rank's head columns, then the sum over ranks
        ec::ChainParams P{};
        P.ph[0] = chain_phase(ctx->wo[l], ec::PRO_NONE, ec::EPI_STORE, sb.att, nullptr, ctx->tp_part);
        P.nph = 1;
        kinds[0] = EC_K_GEMV_O;
        plans[0] = &ctx->p_o;
        if ((e = phases(P, l, plans, kinds))) return e;
        if ((e = gather(ctx->tp_part, ctx->tp_parts, (size_t)D))) return e;
        if ((e = ec::launch_tp_resid(x, ctx->tp_parts, W, D, ctx->stream))) return e;
        ctx->launches++;
      }
      {
        // gate/up (its hidden rows) + down (its hidden columns), then the sum
        ec::ChainParams P{};
        P.ph[0] = chain_phase(ctx->w13[l], ec::PRO_RMSNORM, ec::EPI_SWIGLU, x, ctx->ffn_norm[l], hb);
        P.ph[1] = chain_phase(ctx->w2[l], ec::PRO_NONE, ec::EPI_STORE, hb, nullptr, ctx->tp_part);
        P.nph = 2;
        kinds[0] = EC_K_GEMV_GATEUP;
        kinds[1] = EC_K_GEMV_DOWN;
        plans[0] = &ctx->p_w13;
        plans[1] = &ctx->p_w2;
        if ((e = phases(P, l, plans, kinds))) return e;
        if ((e = gather(ctx->tp_part, ctx->tp_parts, (size_t)D))) return e;
        if ((e = ec::launch_tp_resid(x, ctx->tp_parts, W, D, ctx->stream))) return e;
        ctx->launches++;
      }
      {
        ec::ChainParams P{};
        if (l + 1 < L) {
          P.ph[0] = chain_phase(ctx->qkv[l + 1], ec::PRO_RMSNORM, ec::EPI_STORE, x,
                                ctx->attn_norm[l + 1], sb.qkv);
          kinds[0] = EC_K_GEMV_QKV;
          plans[0] = &ctx->p_qkv;
        } else {
          P.ph[0] = chain_phase(ctx->lm, ec::PRO_RMSNORM, ec::EPI_STORE, x, ctx->final_norm,
                                ctx->tp_lg);
          kinds[0] = EC_K_GEMV_LM;
          plans[0] = &ctx->p_lm;
        }
        P.nph = 1;
        if ((e = phases(P, l, plans, kinds))) return e;
      }
    }
    float* lg = ctx->logits + (size_t)b * Vg;
    if ((e = gather(ctx->tp_lg, lg, (size_t)c.vocab_size))) return e;
    ProfScope ps(ctx, EC_K_ARGMAX, 4.0 * Vg);
    if ((e = ec::launch_argmax_split(lg, Vg, 1, ctx->argmax + b,
                                     feedback ? const_cast<int*>(tokens) + b : nullptr,
                                     feedback ? const_cast<int*>(pos) + b : nullptr,
                                     static_cast<uint8_t*>(ctx->amax) +
                                         (size_t)b * (ec::argmax_scratch_bytes(1)),
                                     ctx->stream, false)))
      return e;
    ctx->launches++;
  }
  return cudaSuccess;
}

// Enqueue one decode step for B sequences (tokens/pos in device memory).
cudaError_t enqueue_step(ec_ctx* ctx, const int* tokens, const int* pos, int B, bool feedback) {
  if (ctx->tp_world > 1) return enqueue_step_tp(ctx, tokens, pos, B, feedback);
  if (ctx->tc && B >= ctx->c.tensor_min_batch)
    return enqueue_step_tc(ctx, tokens, pos, B, feedback);
  if (ctx->chain && B > 1) return enqueue_step_batched(ctx, tokens, pos, B, feedback);
  const ec_model_config& c = ctx->c;
  const int H = c.n_heads, KV = c.n_kv_heads, hd = c.head_dim, D = c.dim, F = c.hidden_dim;
  cudaError_t e;
  ctx->launches = 0;
  ec::StepBuffers sb{};
  sb.rope_cos = ctx->rope_cos;
  sb.rope_sin = ctx->rope_sin;
  sb.sparse_k = c.sparse_k;
  sb.window = c.window;
  sb.sparse_blocks_k = c.sparse_blocks_k;
  sb.err = ctx->err;
  sb.max_sel = ctx->max_sel;
  const bool extras = ctx->adapter_on || ctx->bias_on;
  for (int b = 0; b < B; b++) {
    // Batch-1 kernels: sequence b's state lives at offset b of every buffer.
    float* x = ctx->x + (size_t)b * D;
    sb.pos = pos + b;
    sb.qkv = ctx->qkvb + (size_t)b * (H + 2 * KV) * hd;
    sb.qrot = ctx->qrot + (size_t)b * H * hd;
    sb.att = ctx->att + (size_t)b * H * hd;
    sb.sel = ctx->sel + (size_t)b * ctx->max_sel;
    sb.selp = ctx->selp + (size_t)b * ctx->max_sel;
    sb.nsel = ctx->nsel + b;
    if (ctx->lcand) {
      sb.lcand = ctx->lcand + (size_t)b * ctx->cap_c;
      sb.lscore = ctx->lscore + (size_t)b * ctx->cap_c;
      sb.lnc = ctx->lnc + b;
    }
    ec::KvLayout kv = ctx->kv;
    ec::LshLayout lsh = ctx->lsh;
    const size_t per = (size_t)kv.n_layers * kv.max_blocks;
    if (kv.paged) {
      kv.kq += b * per * KV * 16 * hd;
      kv.vq += b * per * KV * 16 * hd;
      kv.ks += b * per * KV * 16;
      kv.vs += b * per * KV * 16;
      kv.centroid += b * per * hd;
      kv.page_table += b * per;
    } else {
      kv.lk += (size_t)b * kv.n_layers * kv.seq_len * KV * hd;
      kv.lv += (size_t)b * kv.n_layers * kv.seq_len * KV * hd;
    }
    if (lsh.tables > 0) {
      lsh.acc += (size_t)b * hd;
      lsh.meta += b * 4;
      lsh.unit_hash += (size_t)b * lsh.tables * lsh.max_units;
      lsh.unit_start += (size_t)b * lsh.max_units;
      lsh.unit_len += (size_t)b * lsh.max_units;
      lsh.heads += ((size_t)b * lsh.tables) << lsh.bits;
      lsh.next += (size_t)b * lsh.tables * lsh.max_units;
      lsh.counters += b * 2;
    }
    {
      ProfScope ps(ctx, EC_K_EMBED, 2.0 * D + 4.0 * D);
      const ec::TokenHistory th = token_history(ctx, pos + b, b);
      if ((e = ec::launch_embed(ctx->emb, tokens + b, x, D, ctx->cg.vocab_size, 1, ctx->stream,
                                true, &th)))
        return e;
    }
    ctx->launches++;
    const bool chain = ctx->chain;
    float* lg = ctx->logits + (size_t)b * c.vocab_size;
    float* hb = ctx->hbuf + (size_t)b * F;
    for (int l = 0; l < c.n_layers; l++) {
      // with the chain, layer l's QKV ran at the end of layer l-1's chain
      if (!chain || l == 0) {
        if ((e = gemv(ctx, EC_K_GEMV_QKV, ctx->qkv[l], ctx->p_qkv, ec::PRO_RMSNORM, ec::EPI_STORE, x,
                      ctx->attn_norm[l], sb.qkv)))
          return e;
      }
      if ((e = enqueue_attention(ctx, kv, lsh, sb, l, 1, ctx->fast != 0))) return e;
      if (chain) {
        // o (+x), gate/up (RMSNorm, SwiGLU), down (+x), then the next layer's
        // QKV or the LM head: one persistent kernel
        ec::ChainParams P{};
        P.ph[0] = chain_phase(ctx->wo[l], ec::PRO_NONE, ec::EPI_RESID, sb.att, nullptr, x);
        P.ph[1] = chain_phase(ctx->w13[l], ec::PRO_RMSNORM, ec::EPI_SWIGLU, x, ctx->ffn_norm[l], hb);
        P.ph[2] = chain_phase(ctx->w2[l], ec::PRO_NONE, ec::EPI_RESID, hb, nullptr, x);
        if (l + 1 < c.n_layers)
          P.ph[3] = chain_phase(ctx->qkv[l + 1], ec::PRO_RMSNORM, ec::EPI_STORE, x,
                                ctx->attn_norm[l + 1], sb.qkv);
        else
          P.ph[3] = chain_phase(ctx->lm, ec::PRO_RMSNORM, ec::EPI_STORE, x, ctx->final_norm, lg);
        // with a final adapter or logit bias the LM head runs after them
        P.nph = (l + 1 == c.n_layers && extras) ? 3 : 4;
        P.ctr = ctx->chain_ctr + (size_t)l * ctx->npacks * (ec::kMaxChainPhases + 1);
        P.err = ctx->err;
        P.eps = c.norm_eps;
        P.mark = l == 1;
        P.wait_iters = c.wait_limit < 0 ? -c.wait_limit : c.wait_limit;
        P.wait_extra = c.wait_limit < 0 ? 1 : 0;
        const double by = gemv_bytes(ctx->wo[l], ec::PRO_NONE, ec::EPI_RESID) +
                          gemv_bytes(ctx->w13[l], ec::PRO_RMSNORM, ec::EPI_SWIGLU) +
                          gemv_bytes(ctx->w2[l], ec::PRO_NONE, ec::EPI_RESID) +
                          (P.nph == 4 ? gemv_bytes(l + 1 < c.n_layers ? ctx->qkv[l + 1] : ctx->lm,
                                                   ec::PRO_RMSNORM, ec::EPI_STORE)
                                      : 0.0);
        ProfScope ps(ctx, EC_K_GEMV_CHAIN, by);
        if ((e = ec::chain_launch(c.weight_kind, P, ctx->n_sm, ctx->stream, true))) return e;
        ctx->launches++;
        continue;
      }
      if ((e = gemv(ctx, EC_K_GEMV_O, ctx->wo[l], ctx->p_o, ec::PRO_NONE, ec::EPI_RESID, sb.att, nullptr, x)))
        return e;
      if ((e = gemv(ctx, EC_K_GEMV_GATEUP, ctx->w13[l], ctx->p_w13, ec::PRO_RMSNORM, ec::EPI_SWIGLU, x,
                    ctx->ffn_norm[l], hb)))
        return e;
      if ((e = gemv(ctx, EC_K_GEMV_DOWN, ctx->w2[l], ctx->p_w2, ec::PRO_NONE, ec::EPI_RESID, hb,
                    nullptr, x)))
        return e;
    }
    if (extras) {
      auto lm = [&](const float* in, float* out, int) -> cudaError_t {
        return gemv(ctx, EC_K_GEMV_LM, ctx->lm, ctx->p_lm, ec::PRO_NONE, ec::EPI_STORE, in, nullptr,
                    out);
      };
      if ((e = enqueue_final_extras(ctx, x, ctx->xn + (size_t)b * D,
                                    ctx->xa ? ctx->xa + (size_t)b * D : nullptr, 1, lg, lm)))
        return e;
    } else if (!chain) {
      if ((e = gemv(ctx, EC_K_GEMV_LM, ctx->lm, ctx->p_lm, ec::PRO_RMSNORM, ec::EPI_STORE, x,
                    ctx->final_norm, lg)))
        return e;
    }
    if ((e = enqueue_context_bias(ctx, lg, c.vocab_size, 1, token_history(ctx, pos + b, b))))
      return e;
    ProfScope ps(ctx, EC_K_ARGMAX, 4.0 * c.vocab_size);
    // sequence b's partials and counter live at offset b of the scratch
    if ((e = ec::launch_argmax_split(lg, c.vocab_size, 1, ctx->argmax + b,
                                     feedback ? const_cast<int*>(tokens) + b : nullptr,
                                     feedback ? const_cast<int*>(pos) + b : nullptr,
                                     static_cast<uint8_t*>(ctx->amax) +
                                         (size_t)b * (ec::argmax_scratch_bytes(1)),
                                     ctx->stream, true)))
      return e;
    ctx->launches++;
  }
  return cudaSuccess;
}

int check_weights(ec_ctx* ctx) {
  const unsigned need = (1u << EC_WQ) | (1u << EC_WK) | (1u << EC_WV) | (1u << EC_WO) |
                        (1u << EC_W1) | (1u << EC_W2) | (1u << EC_W3) | (1u << EC_ATTN_NORM) |
                        (1u << EC_FFN_NORM);
  for (int l = 0; l < ctx->c.n_layers; l++)
    if ((ctx->have[l] & need) != need) return fail(EC_ERR_STATE, "layer weights missing");
  if ((ctx->have_global & 7u) != 7u) return fail(EC_ERR_STATE, "global weights missing");
  return EC_OK;
}

int run_step(ec_ctx* ctx, const int* tokens_dev, const int* pos_dev, int B, int feedback) {
  if (B <= 0 || B > ctx->c.max_batch) return fail(EC_ERR_ARG, "B out of range");
  int rc = check_weights(ctx);
  if (rc) return rc;
  const bool use_graph = getenv("EC_NO_GRAPH") == nullptr && !ctx->prof;
  if (!use_graph) {
    cudaError_t e = enqueue_step(ctx, tokens_dev, pos_dev, B, feedback != 0);
    if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
    return EC_OK;
  }
  if (!ctx->gexec || ctx->g_B != B || ctx->g_fb != feedback || ctx->g_tok != tokens_dev ||
      ctx->g_pos != pos_dev) {
    if (ctx->gexec) {
      cudaGraphExecDestroy(ctx->gexec);
      ctx->gexec = nullptr;
    }
    cudaGraph_t g;
    EC_CUDA_TRY(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_step(ctx, tokens_dev, pos_dev, B, feedback != 0);
    cudaError_t e2 = cudaStreamEndCapture(ctx->stream, &g);
    if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
    if (e2 != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e2));
    e = cudaGraphInstantiate(&ctx->gexec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
    ctx->g_B = B;
    ctx->g_fb = feedback;
    ctx->g_tok = tokens_dev;
    ctx->g_pos = pos_dev;
  }
  EC_CUDA_TRY(cudaGraphLaunch(ctx->gexec, ctx->stream));
  return EC_OK;
}

int check_err(ec_ctx* ctx) {
  int h = 0;
  EC_CUDA_TRY(cudaMemcpy(&h, ctx->err, 4, cudaMemcpyDeviceToHost));
  if (h) {
    cudaMemset(ctx->err, 0, 4);
    return fail(h, "a bounded device wait timed out");
  }
  return EC_OK;
}

}  // namespace

extern "C" int ec_decode_step_device(ec_ctx* ctx, int* tokens_dev, int* pos_dev, int B,
                                     int greedy_feedback) {
  if (!ctx || !tokens_dev || !pos_dev) return fail(EC_ERR_ARG, "null argument");
  cudaSetDevice(ctx->device);
  return run_step(ctx, tokens_dev, pos_dev, B, greedy_feedback);
}

extern "C" int ec_decode_step(ec_ctx* ctx, const int* tokens, const int* pos, int B,
                              float* logits_host, int* argmax_host) {
  if (!ctx || !tokens || !pos) return fail(EC_ERR_ARG, "null argument");
  if (B <= 0 || B > ctx->c.max_batch) return fail(EC_ERR_ARG, "B out of range");
  cudaSetDevice(ctx->device);
  for (int b = 0; b < B; b++)
    if (tokens[b] < 0 || tokens[b] >= ctx->cg.vocab_size || pos[b] < 0)
      return fail(EC_ERR_ARG, "token or position out of range");
  EC_CUDA_TRY(cudaMemcpyAsync(ctx->tokens, tokens, B * 4, cudaMemcpyHostToDevice, ctx->stream));
  EC_CUDA_TRY(cudaMemcpyAsync(ctx->pos, pos, B * 4, cudaMemcpyHostToDevice, ctx->stream));
  int rc = run_step(ctx, ctx->tokens, ctx->pos, B, 0);
  if (rc) return rc;
  if (logits_host)
    EC_CUDA_TRY(cudaMemcpyAsync(logits_host, ctx->logits, (size_t)B * ctx->cg.vocab_size * 4,
                                cudaMemcpyDeviceToHost, ctx->stream));
  if (argmax_host)
    EC_CUDA_TRY(cudaMemcpyAsync(argmax_host, ctx->argmax, B * 4, cudaMemcpyDeviceToHost, ctx->stream));
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (ctx->prof) prof_collect(ctx);
  return check_err(ctx);
}

namespace {

// The rows of ec_prefill / ec_verify: n tokens of sequence seq from pos0, in
// chunks of max_batch rows; the greedy token of every row to argmax_all when
// given, the last row's logits / greedy token to the two others.
int prefill_rows(ec_ctx* ctx, int seq, const int* tokens, int n, int pos0, float* logits_host,
                 int* argmax_host, int* argmax_all) {
  if (!ctx || !tokens || n <= 0) return fail(EC_ERR_ARG, "null argument or n <= 0");
  const ec_model_config& c = ctx->c;
  if (seq < 0 || seq >= c.max_batch) return fail(EC_ERR_ARG, "bad sequence");
  if (pos0 < 0 || (long)pos0 + n > c.seq_len) return fail(EC_ERR_ARG, "positions past seq_len");
  if (!ctx->chain || ctx->tp_world > 1)
    return fail(EC_ERR_UNSUPPORTED, "prefill needs the chain GEMV layout (one rank)");
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= c.vocab_size) return fail(EC_ERR_ARG, "token out of range");
  cudaSetDevice(ctx->device);
  const int S = c.max_batch;
  std::vector<int> pos(S);
  int last_rows = 0;
  for (int c0 = 0; c0 < n; c0 += S) {
    const int C = n - c0 < S ? n - c0 : S;
    for (int i = 0; i < C; i++) pos[i] = pos0 + c0 + i;
    EC_CUDA_TRY(cudaMemcpyAsync(ctx->tokens, tokens + c0, C * 4, cudaMemcpyHostToDevice, ctx->stream));
    EC_CUDA_TRY(cudaMemcpyAsync(ctx->pos, pos.data(), C * 4, cudaMemcpyHostToDevice, ctx->stream));
    // chunks of at least tensor_min_batch rows run their projections on the
    // tensor cores (within tolerance), smaller ones on the exact chain
    cudaError_t e = (ctx->tc && C >= c.tensor_min_batch)
                        ? enqueue_step_tc(ctx, ctx->tokens, ctx->pos, C, false, seq, pos0 + c0)
                        : enqueue_step_batched(ctx, ctx->tokens, ctx->pos, C, false, seq, pos0 + c0);
    if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
    if (argmax_all)
      EC_CUDA_TRY(cudaMemcpyAsync(argmax_all + c0, ctx->argmax, C * 4, cudaMemcpyDeviceToHost,
                                  ctx->stream));
    // the host vectors above are read before the next chunk overwrites them
    EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    last_rows = C;
  }
  if (logits_host)
    EC_CUDA_TRY(cudaMemcpyAsync(logits_host, ctx->logits + (size_t)(last_rows - 1) * c.vocab_size,
                                (size_t)c.vocab_size * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (argmax_host)
    EC_CUDA_TRY(cudaMemcpyAsync(argmax_host, ctx->argmax + (last_rows - 1), 4,
                                cudaMemcpyDeviceToHost, ctx->stream));
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (ctx->prof) prof_collect(ctx);
  return check_err(ctx);
}

}  // namespace

extern "C" int ec_prefill(ec_ctx* ctx, int seq, const int* tokens, int n, int pos0,
                          float* logits_host, int* argmax_host) {
  return prefill_rows(ctx, seq, tokens, n, pos0, logits_host, argmax_host, nullptr);
}

extern "C" int ec_verify(ec_ctx* ctx, int seq, const int* tokens, int n, int pos0,
                         int* greedy_out) {
  if (!greedy_out) return fail(EC_ERR_ARG, "null argument");
  return prefill_rows(ctx, seq, tokens, n, pos0, nullptr, nullptr, greedy_out);
}

extern "C" float* ec_logits_device(ec_ctx* ctx) { return ctx ? ctx->logits : nullptr; }
extern "C" int* ec_argmax_device(ec_ctx* ctx) { return ctx ? ctx->argmax : nullptr; }
extern "C" void* ec_stream(ec_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

extern "C" int ec_synchronize(ec_ctx* ctx) {
  if (!ctx) return fail(EC_ERR_ARG, "null argument");
  cudaSetDevice(ctx->device);
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (ctx->prof) prof_collect(ctx);
  return check_err(ctx);
}

extern "C" int ec_profile_enable(ec_ctx* ctx, int on) {
  if (!ctx) return fail(EC_ERR_ARG, "null argument");
  cudaSetDevice(ctx->device);
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  prof_collect(ctx);
  ctx->prof = on != 0;
  for (int k = 0; k < EC_K_COUNT; k++) {
    ctx->prof_ms[k] = 0;
    ctx->prof_n[k] = 0;
    ctx->prof_bytes[k] = 0;
  }
  return EC_OK;
}

extern "C" int ec_profile_read(ec_ctx* ctx, int kind, double* ms, int* launches, double* bytes) {
  if (!ctx || kind < 0 || kind >= EC_K_COUNT) return fail(EC_ERR_ARG, "bad argument");
  cudaSetDevice(ctx->device);
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  prof_collect(ctx);
  if (ms) *ms = ctx->prof_ms[kind];
  if (launches) *launches = ctx->prof_n[kind];
  if (bytes) *bytes = ctx->prof_bytes[kind];
  return EC_OK;
}

extern "C" int ec_launches_per_step(ec_ctx* ctx, int B) {
  if (!ctx) return 0;
  // embed, [QKV(0)], per layer: QKV, append, [select], attention, o, gate/up,
  // down -- or with the chain: append, [select], attention, chain -- then
  // [LM head] and argmax
  const int sel = ctx->kv.paged ? 0 : ec::kLinearSelectLaunches;
  if (ctx->tp_world > 1) {
    // per sequence: embed, QKV(0), per layer append, [LSH update on layer 0],
    // [linear: candidates, dots, sum, heap], attention, o, sum, gate/up+down
    // (one chain, else two), sum, next QKV or LM head; argmax.  NCCL's own
    // kernels are not counted.
    const int ffn = ctx->chain ? 1 : 2;
    const int lsh0 = ctx->lsh.tables > 0 ? 1 : 0;
    return B * (3 + lsh0 + ctx->c.n_layers * ((ctx->kv.paged ? 0 : 4) + 6 + ffn));
  }
  // a registered final adapter / logit bias: final RMSNorm, [adapter], the
  // LM head on its own, [bias]
  const bool extras = ctx->adapter_on || ctx->bias_on;
  const int ex = extras ? 1 + ctx->adapter_on + ctx->bias_on : 0;
  // a registered context bias table: one launch before the argmax
  const int cb = ctx->cbias_on ? 1 : 0;
  if (ctx->tc && B >= ctx->c.tensor_min_batch) {
    // embed, per pass QKV(0) (quant, GEMM, combine), per layer append,
    // [select], attention and 4 projections per pass, argmax per sequence
    const int passes = (B + ec::kTcMaxRows - 1) / ec::kTcMaxRows;
    return 1 + 3 * passes + ctx->c.n_layers * (2 + sel + 12 * passes) + 1 + ex + cb;
  }
  if (ctx->chain && B > 1) {
    const int packs = (B + kPack - 1) / kPack;
    return 1 + packs + ctx->c.n_layers * (2 + sel + packs) + 1 + (extras ? ex + packs : 0) + cb;
  }
  if (ctx->chain) return B * (2 + ctx->c.n_layers * (3 + sel) + 1 + (extras ? ex + 1 : 0) + cb);
  return B * (1 + ctx->c.n_layers * (6 + sel) + 2 + ex + cb);
}

extern "C" int ec_read_state(ec_ctx* ctx, int which, int seq, float* out, size_t n) {
  if (!ctx || !out || seq < 0 || seq >= ctx->c.max_batch) return fail(EC_ERR_ARG, "bad argument");
  cudaSetDevice(ctx->device);
  // the copies below run on the legacy stream, which does not wait for ctx->stream
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  const ec_model_config& c = ctx->c;
  const int qkvw = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
  const float* src = nullptr;
  size_t cnt = 0;
  switch (which) {
    case 0: src = ctx->x + (size_t)seq * c.dim; cnt = c.dim; break;
    case 2: src = ctx->qrot + (size_t)seq * c.n_heads * c.head_dim;
            cnt = (size_t)c.n_heads * c.head_dim; break;
    case 3: src = ctx->qkvb + (size_t)seq * qkvw + c.n_heads * c.head_dim;
            cnt = (size_t)c.n_kv_heads * c.head_dim; break;
    case 4: src = ctx->qkvb + (size_t)seq * qkvw + (c.n_heads + c.n_kv_heads) * c.head_dim;
            cnt = (size_t)c.n_kv_heads * c.head_dim; break;
    case 5: src = ctx->att + (size_t)seq * c.n_heads * c.head_dim;
            cnt = (size_t)c.n_heads * c.head_dim; break;
    case 6: src = ctx->logits + (size_t)seq * ctx->cg.vocab_size; cnt = ctx->cg.vocab_size; break;
    case 7: src = ctx->hbuf + (size_t)seq * c.hidden_dim; cnt = c.hidden_dim; break;
    case 8: {
      // attended selection of the last attention launch: [n, ids...] as floats
      int ns = 0;
      EC_CUDA_TRY(cudaMemcpy(&ns, ctx->nsel + seq, 4, cudaMemcpyDeviceToHost));
      std::vector<int> ids(ctx->max_sel);
      EC_CUDA_TRY(cudaMemcpy(ids.data(), ctx->sel + (size_t)seq * ctx->max_sel,
                             ctx->max_sel * 4, cudaMemcpyDeviceToHost));
      if (n < 1) return fail(EC_ERR_ARG, "buffer too small");
      out[0] = (float)ns;
      for (int i = 0; i < ns && (size_t)(i + 1) < n; i++) out[i + 1] = (float)ids[i];
      return EC_OK;
    }
    case 9: {
      // paged KV: block centroids of the last layer in logical block order
      // ([max_blocks][head_dim]), for checking the block selection
      if (!ctx->kv.paged) return fail(EC_ERR_UNSUPPORTED, "centroids exist in paged mode only");
      const size_t mb = ctx->kv.max_blocks, hd = c.head_dim;
      if (n < mb * hd) return fail(EC_ERR_ARG, "buffer too small");
      const size_t base = ((size_t)seq * c.n_layers + c.n_layers - 1) * mb;
      std::vector<int> pt(mb);
      std::vector<float> cen(mb * hd);
      EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
      EC_CUDA_TRY(cudaMemcpy(pt.data(), ctx->kv.page_table + base, mb * 4, cudaMemcpyDeviceToHost));
      EC_CUDA_TRY(cudaMemcpy(cen.data(), ctx->kv.centroid + base * hd, mb * hd * 4,
                             cudaMemcpyDeviceToHost));
      for (size_t lb = 0; lb < mb; lb++)
        memcpy(out + lb * hd, cen.data() + (size_t)pt[lb] * hd, hd * 4);
      return EC_OK;
    }
    default: return fail(EC_ERR_ARG, "unknown state id");
  }
  if (n < cnt) return fail(EC_ERR_ARG, "buffer too small");
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  EC_CUDA_TRY(cudaMemcpy(out, src, cnt * 4, cudaMemcpyDeviceToHost));
  return EC_OK;
}

extern "C" int ec_read_lsh(ec_ctx* ctx, int seq, int* n_units, uint32_t* unit_hash,
                           int* unit_start, int* unit_len, int* heads, int* next) {
  if (!ctx || seq < 0 || seq >= ctx->c.max_batch) return fail(EC_ERR_ARG, "bad argument");
  const ec::LshLayout& l = ctx->lsh;
  if (l.tables <= 0) return fail(EC_ERR_STATE, "LSH disabled");
  cudaSetDevice(ctx->device);
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  int meta[4];
  EC_CUDA_TRY(cudaMemcpy(meta, l.meta + seq * 4, 16, cudaMemcpyDeviceToHost));
  if (n_units) *n_units = meta[2];
  const size_t mu = l.max_units, tb = (size_t)seq * l.tables;
  if (unit_hash)
    EC_CUDA_TRY(cudaMemcpy(unit_hash, l.unit_hash + tb * mu, l.tables * mu * 4, cudaMemcpyDeviceToHost));
  if (unit_start)
    EC_CUDA_TRY(cudaMemcpy(unit_start, l.unit_start + seq * mu, mu * 4, cudaMemcpyDeviceToHost));
  if (unit_len)
    EC_CUDA_TRY(cudaMemcpy(unit_len, l.unit_len + seq * mu, mu * 4, cudaMemcpyDeviceToHost));
  if (heads)
    EC_CUDA_TRY(cudaMemcpy(heads, l.heads + (tb << l.bits), ((size_t)l.tables << l.bits) * 4,
                           cudaMemcpyDeviceToHost));
  if (next) EC_CUDA_TRY(cudaMemcpy(next, l.next + tb * mu, l.tables * mu * 4, cudaMemcpyDeviceToHost));
  return EC_OK;
}

extern "C" int ec_read_counters(ec_ctx* ctx, int seq, unsigned long long* out2) {
  if (!ctx || !out2 || seq < 0 || seq >= ctx->c.max_batch) return fail(EC_ERR_ARG, "bad argument");
  if (ctx->lsh.tables <= 0) {
    out2[0] = out2[1] = 0;
    return EC_OK;
  }
  cudaSetDevice(ctx->device);
  EC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  EC_CUDA_TRY(cudaMemcpy(out2, ctx->lsh.counters + seq * 2, 16, cudaMemcpyDeviceToHost));
  return EC_OK;
}

// ------------------------------------------------------------------------
// per-op entry points
// ------------------------------------------------------------------------
extern "C" int ec_op_gemv(int wkind, const void* w, const float* scale, const float* x, float* y,
                          int m, int k, void* stream) {
  if (!w || !x || !y || m <= 0 || k <= 0) return fail(EC_ERR_ARG, "bad argument");
  if (wkind != EC_W_BF16 && !scale) return fail(EC_ERR_ARG, "scale required");
  if (k % 32) return fail(EC_ERR_UNSUPPORTED, "k must be a multiple of 32");
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  EC_CUDA_TRY(ec::gemv_prepare());
  ec::GemvPlan plan;
  if (!ec::gemv_plan(wkind, m, k, ec::EPI_STORE, nsm, &plan))
    return fail(EC_ERR_UNSUPPORTED, "no GEMV plan for this shape");
  ec::GemvParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.scale = scale;
  p.scale_stride = (wkind == EC_W_INT8) ? 1 : 0;
  p.x = x;
  p.y = y;
  p.N = m;
  p.K = k;
  EC_CUDA_TRY(ec::gemv_launch(wkind, ec::PRO_NONE, ec::EPI_STORE, plan, p,
                              static_cast<cudaStream_t>(stream), false));
  return EC_OK;
}

extern "C" size_t ec_gemv_packed_bytes(int m, int k) {
  return (m > 0 && k > 0) ? ec::packed_bytes(m, k) : 0;
}

extern "C" int ec_gemv_pack(const void* w_rowmajor, void* w_packed, int m, int k, void* stream) {
  if (!w_rowmajor || !w_packed || m <= 0 || k <= 0) return fail(EC_ERR_ARG, "bad argument");
  if (k % 32) return fail(EC_ERR_UNSUPPORTED, "k must be a multiple of 32");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // padding rows of the last quad read as zero
  EC_CUDA_TRY(cudaMemsetAsync(w_packed, 0, ec::packed_bytes(m, k), s));
  EC_CUDA_TRY(ec::packed_pack(static_cast<const uint8_t*>(w_rowmajor),
                              static_cast<uint8_t*>(w_packed), m, k, m, 0, 1, s));
  return EC_OK;
}

extern "C" int ec_op_gemv_packed(int wkind, const void* w, const float* scale, const float* x,
                                 float* y, int m, int k, void* stream) {
  if (!w || !x || !y || !scale || m <= 0 || k <= 0) return fail(EC_ERR_ARG, "bad argument");
  if (wkind != EC_W_INT8 && wkind != EC_W_FP8) return fail(EC_ERR_ARG, "INT8 or FP8 weights");
  if (k % 32) return fail(EC_ERR_UNSUPPORTED, "k must be a multiple of 32");
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  EC_CUDA_TRY(ec::packed_prepare());
  ec::PackedPlan plan;
  if (!ec::packed_plan(wkind, m, k, nsm, gemv_force_r(), false, &plan))
    return fail(EC_ERR_UNSUPPORTED, "no GEMV plan for this shape");
  ec::GemvParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.scale = scale;
  p.scale_stride = (wkind == EC_W_INT8) ? 1 : 0;
  p.x = x;
  p.y = y;
  p.N = m;
  p.K = k;
  EC_CUDA_TRY(ec::packed_launch(wkind, ec::PRO_NONE, ec::EPI_STORE, plan, p,
                                static_cast<cudaStream_t>(stream), false));
  return EC_OK;
}

extern "C" int ec_op_gemv_packed_batch(int wkind, const void* w, const float* scale,
                                       const float* x, float* y, int m, int k, int nb,
                                       void* stream) {
  if (!w || !x || !y || !scale || m <= 0 || k <= 0 || nb <= 0) return fail(EC_ERR_ARG, "bad argument");
  if (wkind != EC_W_INT8 && wkind != EC_W_FP8) return fail(EC_ERR_ARG, "INT8 or FP8 weights");
  if (nb > 1 && k % 512) return fail(EC_ERR_UNSUPPORTED, "batched GEMV needs k % 512 == 0");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  EC_CUDA_TRY(ec::chain_prepare());
  int* ctr = nullptr;
  const size_t cb = (ec::kMaxChainPhases + 2) * sizeof(int);  // counters + error word
  EC_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&ctr), cb, s));
  int rc = EC_OK;
  cudaError_t e = cudaMemsetAsync(ctr, 0, cb, s);
  for (int b0 = 0; b0 < nb && e == cudaSuccess; b0 += kPack) {
    const int n = nb - b0 < kPack ? nb - b0 : kPack;
    ec::ChainParams P{};
    ec::ChainPhase& ph = P.ph[0];
    ph.w = static_cast<const uint8_t*>(w);
    ph.scale = scale;
    ph.x = x + (size_t)b0 * k;
    ph.y = y + (size_t)b0 * m;
    ph.N = m;
    ph.K = k;
    ph.pro = ec::PRO_NONE;
    ph.epi = ec::EPI_STORE;
    ph.x_stride = k;
    ph.y_stride = m;
    P.nph = 1;
    P.ctr = ctr;
    P.err = ctr + ec::kMaxChainPhases + 1;
    if (wkind == EC_W_FP8) {
      // the chain reads one scale per row: per-tensor FP8 scale -> per-op packed kernel
      rc = ec_op_gemv_packed(wkind, w, scale, ph.x, ph.y, m, k, stream);
      for (int i = 1; i < n && rc == EC_OK; i++)
        rc = ec_op_gemv_packed(wkind, w, scale, ph.x + (size_t)i * k, ph.y + (size_t)i * m, m, k, stream);
      if (rc != EC_OK) break;
      continue;
    }
    e = n == 1 ? ec::chain_launch(wkind, P, nsm, s, false)
               : ec::chain_launch_nb(wkind, P, n, nsm, s, false);
  }
  cudaFreeAsync(ctr, s);
  if (rc != EC_OK) return rc;
  EC_CUDA_TRY(e);
  return EC_OK;
}

extern "C" int ec_op_rmsnorm(float* out, const float* x, const uint16_t* w, int n, float eps,
                             void* stream) {
  if (!out || !x || !w || n <= 0) return fail(EC_ERR_ARG, "bad argument");
  EC_CUDA_TRY(ec::launch_rmsnorm(out, x, w, n, eps, static_cast<cudaStream_t>(stream)));
  return EC_OK;
}

extern "C" int ec_op_rope(float* data, int n_heads, int head_dim, int pos, const float* cos_t,
                          const float* sin_t, int max_seq, void* stream) {
  if (!data || !cos_t || !sin_t || head_dim % 2 || n_heads <= 0) return fail(EC_ERR_ARG, "bad argument");
  EC_CUDA_TRY(ec::launch_rope(data, n_heads, head_dim, pos, cos_t, sin_t, max_seq,
                              static_cast<cudaStream_t>(stream)));
  return EC_OK;
}

extern "C" int ec_op_silu_mul(float* out, const float* gate, const float* up, int n, void* stream) {
  if (!out || !gate || !up || n <= 0) return fail(EC_ERR_ARG, "bad argument");
  EC_CUDA_TRY(ec::launch_silu(out, gate, up, n, static_cast<cudaStream_t>(stream)));
  return EC_OK;
}

extern "C" int ec_op_quant_int8(int8_t* out, float* scales, const float* in, int rows, int n,
                                void* stream) {
  if (!out || !scales || !in || rows <= 0 || n <= 0) return fail(EC_ERR_ARG, "bad argument");
  EC_CUDA_TRY(ec::launch_quant(out, scales, in, rows, n, static_cast<cudaStream_t>(stream)));
  return EC_OK;
}

extern "C" int ec_op_argmax(const float* logits, int n, int B, int* out, void* stream) {
  if (!logits || !out || n <= 0 || B <= 0) return fail(EC_ERR_ARG, "bad argument");
  EC_CUDA_TRY(ec::launch_argmax(logits, n, B, out, nullptr, nullptr,
                                static_cast<cudaStream_t>(stream), false));
  return EC_OK;
}

namespace {

// KvLayout of a caller's one-layer view.
bool view_layout(const ec_paged_view* pv, ec::KvLayout* kv) {
  if (!pv || !pv->k || !pv->v || !pv->k_scale || !pv->v_scale || !pv->centroid ||
      !pv->page_table || pv->n_kv_heads <= 0 || pv->max_blocks <= 0 ||
      (pv->head_dim != 32 && pv->head_dim != 64 && pv->head_dim != 128))
    return false;
  *kv = ec::KvLayout{};
  kv->n_layers = 1;
  kv->n_kv_heads = pv->n_kv_heads;
  kv->head_dim = pv->head_dim;
  kv->max_blocks = pv->max_blocks;
  kv->seq_len = pv->max_blocks * 16;
  kv->paged = 1;
  kv->kq = pv->k;
  kv->vq = pv->v;
  kv->ks = pv->k_scale;
  kv->vs = pv->v_scale;
  kv->centroid = pv->centroid;
  kv->page_table = const_cast<int*>(pv->page_table);
  return true;
}

}  // namespace

extern "C" int ec_op_paged_append(const ec_paged_view* pv, const float* k, const float* v, int pos,
                                  void* stream) {
  ec::KvLayout kv;
  if (!view_layout(pv, &kv) || !k || !v) return fail(EC_ERR_ARG, "bad paged view or vectors");
  if (pos < 0 || pos >= pv->max_blocks * 16) return fail(EC_ERR_ARG, "position beyond the view");
  EC_CUDA_TRY(ec::launch_paged_append_view(kv, k, v, pos, nullptr, static_cast<cudaStream_t>(stream)));
  return EC_OK;
}

namespace {

// Shared body of the per-op paged attention: `scratch` holds
// [sel: max_sel ints][nsel][err], max_sel = paged_attention_max_sel(...).
int paged_attention_run(const ec_paged_view* pv, const float* q, float* out, int n_heads,
                        int n_tokens, int sparse_blocks_k, int* selected_out,
                        int* n_selected_out, int* scratch, int max_sel, cudaStream_t s) {
  ec::KvLayout kv;
  view_layout(pv, &kv);
  kv.n_heads = n_heads;
  ec::StepBuffers sb{};
  sb.pos = nullptr;
  sb.pos_fixed = n_tokens - 1;
  sb.qrot = const_cast<float*>(q);
  sb.att = out;
  sb.sel = scratch;
  sb.nsel = scratch + max_sel;
  sb.err = scratch + max_sel + 1;
  sb.max_sel = max_sel;
  sb.sparse_blocks_k = sparse_blocks_k > 0 ? sparse_blocks_k : 1 << 30;
  sb.q_rotated = 1;
  sb.list_dense = 1;
  const int nb = (n_tokens + 15) / 16;
  const int max_tok = (sparse_blocks_k > 0 && nb > sparse_blocks_k) ? 16 * sparse_blocks_k
                                                                   : ((n_tokens + 15) & ~15);
  EC_CUDA_TRY(cudaMemsetAsync(sb.err, 0, sizeof(int), s));
  EC_CUDA_TRY(ec::launch_paged_select(kv, sb, s));
  EC_CUDA_TRY(ec::launch_attention_n(kv, sb, max_tok, s));
  if (selected_out)
    EC_CUDA_TRY(cudaMemcpyAsync(selected_out, sb.sel, (size_t)(sparse_blocks_k > 0 && nb > sparse_blocks_k ? sparse_blocks_k : nb) * 4,
                                cudaMemcpyDeviceToDevice, s));
  if (n_selected_out)
    EC_CUDA_TRY(cudaMemcpyAsync(n_selected_out, sb.nsel, 4, cudaMemcpyDeviceToDevice, s));
  return EC_OK;
}

int paged_attention_check(const ec_paged_view* pv, const float* q, float* out, int n_heads,
                          int n_tokens, int sparse_blocks_k) {
  ec::KvLayout kv;
  if (!view_layout(pv, &kv) || !q || !out) return fail(EC_ERR_ARG, "bad paged view or vectors");
  if (n_heads <= 0 || n_heads % pv->n_kv_heads) return fail(EC_ERR_ARG, "n_heads");
  if (n_tokens <= 0 || n_tokens > pv->max_blocks * 16) return fail(EC_ERR_ARG, "n_tokens");
  if (sparse_blocks_k < 0 || sparse_blocks_k > 64)
    return fail(EC_ERR_UNSUPPORTED, "sparse_blocks_k must be 0..64");
  const int nb = (n_tokens + 15) / 16;
  if (nb > 2048) return fail(EC_ERR_UNSUPPORTED, "at most 2048 blocks");
  const bool dense = !(sparse_blocks_k > 0 && nb > sparse_blocks_k);
  const int max_tok = dense ? ((n_tokens + 15) & ~15) : 16 * sparse_blocks_k;
  if ((dense && (long)max_tok * pv->head_dim > 131072) ||
      ec::attention_smem_bytes(max_tok, pv->head_dim, true) > 226 * 1024)
    return fail(EC_ERR_UNSUPPORTED, "dense attention over more than 131072 K bytes");
  return EC_OK;
}

}  // namespace

extern "C" int ec_op_paged_attention(const ec_paged_view* pv, const float* q, float* out,
                                     int n_heads, int n_tokens, int sparse_blocks_k,
                                     int* selected_out, int* n_selected_out, void* stream) {
  int rc = paged_attention_check(pv, q, out, n_heads, n_tokens, sparse_blocks_k);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nb = (n_tokens + 15) / 16;
  const int max_sel = nb > 66 ? nb : 66;
  int* scratch = nullptr;
  EC_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&scratch), (size_t)(max_sel + 2) * 4, s));
  rc = paged_attention_run(pv, q, out, n_heads, n_tokens, sparse_blocks_k, selected_out,
                           n_selected_out, scratch, max_sel, s);
  cudaFreeAsync(scratch, s);
  return rc;
}

// ---------------------------------------------------------------------------
// ec_op_paged_attention_static: the same operation for callers that cannot
// allocate device memory -- code running inside another runtime's memory
// pool or allocator hooks, code that is forbidden to call cudaMalloc after
// start-up, or hosts whose own allocator owns the whole device.  Its scratch
// (the selected-block list, its count and an error word) is a fixed array in
// this library's device memory instead of a stream-ordered allocation.

namespace {

// Largest context the fixed scratch serves: 2048 blocks of 16 tokens.
constexpr int kStaticMaxBlocks = 2048;
constexpr int kStaticMaxSel = kStaticMaxBlocks;  // >= 66 for the sparse path

// [sel: kStaticMaxSel][nsel][err].  Every device that loads the library holds
// one copy (about 8 KB) until the process exits.  Host code may not use this
// name as a device address; it takes the address from cudaGetSymbolAddress.
static __device__ __align__(256) int g_paged_scratch[kStaticMaxSel + 2];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
int* g_scratch_addr[kMaxDevices] = {};

// Device address of g_paged_scratch on the current device, looked up once per
// device (the first call on each device does it).
int static_scratch(int** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(EC_ERR_UNSUPPORTED, "device ordinal too large");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_paged_scratch);
    if (e != cudaSuccess) return fail(EC_ERR_CUDA, cudaGetErrorString(e));
    g_scratch_addr[dev] = static_cast<int*>(p);
  }
  *out = g_scratch_addr[dev];
  return EC_OK;
}

}  // namespace

extern "C" int ec_op_paged_attention_static(const ec_paged_view* pv, const float* q, float* out,
                                            int n_heads, int n_tokens, int sparse_blocks_k,
                                            int* selected_out, int* n_selected_out,
                                            void* stream) {
  if (n_tokens > kStaticMaxBlocks * 16)
    return fail(EC_ERR_UNSUPPORTED,
                "n_tokens beyond the fixed scratch of ec_op_paged_attention_static "
                "(at most 32768 tokens = 2048 blocks)");
  int rc = paged_attention_check(pv, q, out, n_heads, n_tokens, sparse_blocks_k);
  if (rc) return rc;
  int* scratch = nullptr;
  rc = static_scratch(&scratch);
  if (rc) return rc;
  // paged_attention_run zeroes the error word; the list and count are always
  // written by the selection before the attention reads them.
  return paged_attention_run(pv, q, out, n_heads, n_tokens, sparse_blocks_k, selected_out,
                             n_selected_out, scratch, kStaticMaxSel,
                             static_cast<cudaStream_t>(stream));
}
