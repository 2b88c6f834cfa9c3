// gemv_packed.cu -- the decode step's GEMV: the same arithmetic as gemv.cu
// (matvec_bf16_f32_blocked, src/compute/ops_matmul.c:57-141, bit for bit)
// over weights repacked once, at upload, into a layout built for streaming.
//
// Packed layout, for a matrix of N rows and K columns and a chunk of KCE
// columns (KCE = 512 when K % 512 == 0, else 32):
//
//     [chunk c < K/KCE][row quad q < ceil(N/4)][piece p < KCE/32][row r < 4][32 bytes]
//
// i.e. byte (row 4q+r, column j) lives at
//     ((c * nq + q) * (KCE/32) + p) * 128 + r * 32 + (j % 32),  c = j / KCE,
//     p = (j % KCE) / 32.
// Rows beyond N are zero.  Consequences:
//   * one pipeline stage (a run of consecutive quads of one chunk) is ONE
//     contiguous range, moved by ONE cp.async.bulk;
//   * a warp (4 rows x 8 lane quads) reads 128 contiguous bytes of shared
//     memory per weight load: no bank conflicts, no padding.
//
// Per thread: lanes 4s..4s+3 (s = lane & 7) of the reference's 32 lanes for
// R rows (one row of each of R quads), so every lane's FMA chain runs in the
// reference's order in one thread and one load of x feeds R rows.  INT8 bytes
// become floats with one byte permute each (2^23 + 128 + v, exact) and a
// paired subtraction; products accumulate with paired FMAs (fma.rn.f32x2:
// two independent fma.rn, the same rounding as the scalar form).
#include <cstdlib>

#include "ec_internal.cuh"
#include "gemv.cuh"

namespace ec {

namespace {

// -(2^23 + 128), twice: the INT8 decode bias
constexpr uint64_t kBias2 = 0xCB000080CB000080ull;
constexpr int kMaxStages = 8;
constexpr int kMaxWarps = 16;  // consumer warps

template <int WK, int PRO, int EPI, int R, int KCE>
__global__ void __launch_bounds__(32 + 32 * kMaxWarps, 1) gemv_packed_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* xbar = empty + kMaxStages;
  float* red = reinterpret_cast<float*>(xbar + 2);  // 16 floats
  float* xs = red + 16;                              // [K]
  uint8_t* stages = reinterpret_cast<uint8_t*>(xs + p.K);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int W = (blockDim.x >> 5) - 1;  // consumer warps
  const int QS = W * R;                 // quads per stage
  const int stage_bytes = QS * 4 * KCE;

  const int nq = (p.N + 3) >> 2;
  const int q0 = (int)((long)nq * blockIdx.x / gridDim.x);
  const int q1 = (int)((long)nq * (blockIdx.x + 1) / gridDim.x);
  const int ngroups = (q1 - q0 + QS - 1) / QS;
  const int nchunks = p.K / KCE;
  const int ntasks = ngroups * nchunks;

  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int t = 0; t < ntasks; t++) {
        const int s = t % S;
        if (t >= S && !mbar_wait(&empty[s], ((t / S) - 1) & 1, p.err)) return;
        const int g = t / nchunks;
        const int c = t - g * nchunks;
        const int gq0 = q0 + g * QS;
        const int gn = min(QS, q1 - gq0);
        const uint32_t bytes = (uint32_t)gn * 4 * KCE;
        mbar_expect_tx(&full[s], bytes);
        bulk_g2s(stages + (size_t)s * stage_bytes, p.w + ((long)c * nq + gq0) * 4 * KCE, bytes,
                 &full[s]);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int ct = tid - 32;
  const int wc = warp - 1;
  pdl_wait();
  if (ct == 0) {
    mbar_expect_tx(xbar, (uint32_t)(p.K * 4));
    bulk_g2s(xs, p.x, (uint32_t)(p.K * 4), xbar);
  }
  bool ok = mbar_wait(xbar, 0, p.err);
  if constexpr (PRO == PRO_RMSNORM) rmsnorm_smem(xs, p.norm_w, p.K, p.eps, red, ct, W * 32);

  const int rq = lane >> 3;  // row within the quad
  const int sl = lane & 7;   // lane quad: reference lanes 4*sl .. 4*sl+3
  uint64_t acc01[R], acc23[R];

  for (int t = 0; t < ntasks; t++) {
    const int s = t % S;
    const int g = t / nchunks;
    const int c = t - g * nchunks;
    const int gq0 = q0 + g * QS;
    const int gn = min(QS, q1 - gq0);
    if (c == 0) {
#pragma unroll
      for (int i = 0; i < R; i++) acc01[i] = acc23[i] = 0;
    }
    if (ok) ok = mbar_wait(&full[s], (t / S) & 1, p.err);
    if (ok) {
      const uint8_t* base = stages + (size_t)s * stage_bytes + rq * 32 + sl * 4;
      const float* xc = xs + c * KCE + sl * 4;
      const bool live[2] = {wc * R < gn, wc * R + 1 < gn};
      if (live[0]) {
#pragma unroll
        for (int pc = 0; pc < KCE / 32; pc++) {
          const ulonglong2 xv = *reinterpret_cast<const ulonglong2*>(xc + pc * 32);
#pragma unroll
          for (int i = 0; i < R; i++) {
            if (i > 0 && !live[1]) break;
            const uint32_t wv = *reinterpret_cast<const uint32_t*>(
                base + (size_t)(wc * R + i) * 4 * KCE + pc * 128);
            if constexpr (WK == EC_W_INT8) {
              fma4_i8(wv, xv.x, xv.y, kBias2, acc01[i], acc23[i]);
            } else {
              uint64_t w01, w23;
              decode_pairs<WK>(wv, w01, w23);
              fma2(acc01[i], w01, xv.x);
              fma2(acc23[i], w23, xv.y);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    if (c == nchunks - 1) {
#pragma unroll
      for (int i = 0; i < R; i++) {
        // combine lanes: (g0+g1)+(g2+g3) per 8-lane position, then hsum8
        float v[4] = {lo_f(acc01[i]), hi_f(acc01[i]), lo_f(acc23[i]), hi_f(acc23[i])};
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float t1 = __fadd_rn(v[k], __shfl_xor_sync(0xffffffffu, v[k], 2));
          v[k] = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 4));
        }
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = __fadd_rn(v[k], __shfl_xor_sync(0xffffffffu, v[k], 1));
        float sum = __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
        const int ql = wc * R + i;
        const int gr = (gq0 + ql) * 4 + rq;
        const bool valid = ok && ql < gn && gr < p.N;
        if (valid) sum = __fmul_rn(sum, p.scale[(long)gr * p.scale_stride]);
        if constexpr (EPI == EPI_SWIGLU) {
          const float up = __shfl_down_sync(0xffffffffu, sum, 8);
          if (valid && sl == 0 && (rq & 1) == 0) {
            const int o = gr >> 1;
            float sig;
            if (o < p.silu_vec_limit)
              sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf_vec(__fsub_rn(0.0f, sum))));
            else
              sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf(-sum)));
            p.y[o] = __fmul_rn(__fmul_rn(sum, sig), up);
          }
        } else if constexpr (EPI == EPI_RESID) {
          if (valid && sl == 0) p.y[gr] = __fadd_rn(p.y[gr], sum);
        } else {
          if (valid && sl == 0) p.y[gr] = sum;
        }
      }
    }
  }
}

// Row-major rows -> packed positions.  Source row i goes to packed row
// row_base + row_stride * i.  Each thread moves 16 bytes.
__global__ void gemv_pack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                 int N, int K, int kce, int nr, int row_base, int row_stride) {
  const long per_row = K / 16;
  const long total = (long)nr * per_row;
  const int nq = (N + 3) >> 2;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total;
       i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / per_row);
    const int j = (int)(i - (long)r * per_row) * 16;
    const int row = row_base + row_stride * r;
    const int c = j / kce, pc = (j % kce) / 32;
    const long off = (((long)c * nq + (row >> 2)) * (kce / 32) + pc) * 128 + (row & 3) * 32 + (j & 31);
    *reinterpret_cast<uint4*>(dst + off) =
        *reinterpret_cast<const uint4*>(src + (long)r * K + j);
  }
}

template <int WK, int PRO, int EPI, int R, int KCE>
cudaError_t launch_one(const PackedPlan& plan, const GemvParams& p, cudaStream_t stream,
                       bool pdl) {
  auto fn = gemv_packed_kernel<WK, PRO, EPI, R, KCE>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(32 + 32 * plan.warps);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  GemvParams q = p;
  q.stages = plan.stages;
  return cudaLaunchKernelEx(&cfg, fn, q);
}

template <int WK, int PRO, int EPI, int R, int KCE>
cudaError_t set_attr_one() {
  return cudaFuncSetAttribute(gemv_packed_kernel<WK, PRO, EPI, R, KCE>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
}

// The prologue/epilogue combinations the decode step and the per-op entry
// use: (RMSNorm, store) for QKV and the LM head, (none, +residual) for O and
// down, (RMSNorm, SwiGLU) for gate/up, (none, store) for ec_op_gemv_packed.
template <int WK, int R, int KCE>
cudaError_t dispatch_pe(int pro, int epi, const PackedPlan& plan, const GemvParams& p,
                        cudaStream_t s, bool pdl, bool attr_only) {
  if (pro == PRO_RMSNORM && epi == EPI_STORE)
    return attr_only ? set_attr_one<WK, PRO_RMSNORM, EPI_STORE, R, KCE>()
                     : launch_one<WK, PRO_RMSNORM, EPI_STORE, R, KCE>(plan, p, s, pdl);
  if (pro == PRO_RMSNORM && epi == EPI_SWIGLU)
    return attr_only ? set_attr_one<WK, PRO_RMSNORM, EPI_SWIGLU, R, KCE>()
                     : launch_one<WK, PRO_RMSNORM, EPI_SWIGLU, R, KCE>(plan, p, s, pdl);
  if (pro == PRO_NONE && epi == EPI_RESID)
    return attr_only ? set_attr_one<WK, PRO_NONE, EPI_RESID, R, KCE>()
                     : launch_one<WK, PRO_NONE, EPI_RESID, R, KCE>(plan, p, s, pdl);
  if (pro == PRO_NONE && epi == EPI_STORE)
    return attr_only ? set_attr_one<WK, PRO_NONE, EPI_STORE, R, KCE>()
                     : launch_one<WK, PRO_NONE, EPI_STORE, R, KCE>(plan, p, s, pdl);
  return cudaErrorInvalidValue;
}

template <int WK>
cudaError_t dispatch_w(int pro, int epi, const PackedPlan& plan, const GemvParams& p,
                       cudaStream_t s, bool pdl, bool attr_only) {
  if (plan.kce == 512)
    return plan.rows_per_thread == 2 ? dispatch_pe<WK, 2, 512>(pro, epi, plan, p, s, pdl, attr_only)
                                     : dispatch_pe<WK, 1, 512>(pro, epi, plan, p, s, pdl, attr_only);
  return plan.rows_per_thread == 2 ? dispatch_pe<WK, 2, 32>(pro, epi, plan, p, s, pdl, attr_only)
                                   : dispatch_pe<WK, 1, 32>(pro, epi, plan, p, s, pdl, attr_only);
}

cudaError_t dispatch(int wkind, int pro, int epi, const PackedPlan& plan, const GemvParams& p,
                     cudaStream_t s, bool pdl, bool attr_only) {
  if (wkind == EC_W_INT8) return dispatch_w<EC_W_INT8>(pro, epi, plan, p, s, pdl, attr_only);
  if (wkind == EC_W_FP8) return dispatch_w<EC_W_FP8>(pro, epi, plan, p, s, pdl, attr_only);
  return cudaErrorInvalidValue;
}

}  // namespace

int packed_kce(int K) { return (K % 512 == 0) ? 512 : 32; }

size_t packed_bytes(int N, int K) { return (size_t)((N + 3) / 4) * 4 * (size_t)K; }

bool packed_plan(int wkind, int N, int K, int n_sm, int force_r, bool co_resident,
                 PackedPlan* plan) {
  if ((wkind != EC_W_INT8 && wkind != EC_W_FP8) || N <= 0 || K <= 0 || K % 32 != 0) return false;
  const int kce = packed_kce(K);
  const int nq = (N + 3) / 4;
  const int grid = nq < n_sm ? nq : n_sm;
  const int qpc = (nq + grid - 1) / grid;  // quads of the busiest CTA
  // co_resident: leave room on every SM for the next kernel's CTA (shared
  // memory, threads and registers), so that under programmatic dependent
  // launch it starts streaming its own weights while this one drains
  int R = (!co_resident && qpc * 4 >= 256) ? 2 : 1;
  if (force_r == 1 || force_r == 2) R = force_r;
  const int max_warps = co_resident ? kMaxWarps - 1 : kMaxWarps;
  // spread the CTA's quads evenly over the fewest groups of <= max_warps*R
  const int ngroups = (qpc + max_warps * R - 1) / (max_warps * R);
  const int qs = (qpc + ngroups - 1) / ngroups;
  int warps = (qs + R - 1) / R;
  const int fixed = (2 * kMaxStages + 2) * 8 + 16 * 4 + K * 4;
  int budget = 220 * 1024;
  if (co_resident) {
    const char* v = getenv("EC_GEMV_SMEM_KB");
    budget = (v ? atoi(v) : 110) * 1024;
    if (budget < fixed + 2 * 4 * kce) budget = fixed + 2 * 4 * kce;
  }
  int stages = 0;
  for (;;) {
    const int sb = warps * R * 4 * kce;
    stages = (budget - fixed) / sb;
    if (stages >= 2 || warps == 1) break;
    warps--;
  }
  if (stages < 2) return false;
  const int nchunks = K / kce;
  const int tasks_max = ((qpc + warps * R - 1) / (warps * R)) * nchunks;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages > tasks_max) stages = tasks_max < 2 ? 2 : tasks_max;
  plan->grid = grid;
  plan->warps = warps;
  plan->rows_per_thread = R;
  plan->kce = kce;
  plan->stages = stages;
  plan->smem = fixed + stages * warps * R * 4 * kce;
  return true;
}

cudaError_t packed_prepare() {
  const int kinds[2] = {EC_W_INT8, EC_W_FP8};
  const int pe[4][2] = {{PRO_RMSNORM, EPI_STORE}, {PRO_RMSNORM, EPI_SWIGLU},
                        {PRO_NONE, EPI_RESID}, {PRO_NONE, EPI_STORE}};
  GemvParams p{};
  for (int wk : kinds)
    for (int r = 1; r <= 2; r++)
      for (int kce : {32, 512})
        for (auto& x : pe) {
          PackedPlan plan{};
          plan.rows_per_thread = r;
          plan.kce = kce;
          cudaError_t e = dispatch(wk, x[0], x[1], plan, p, nullptr, false, true);
          if (e != cudaSuccess) return e;
        }
  return cudaSuccess;
}

cudaError_t packed_launch(int wkind, int pro, int epi, const PackedPlan& plan,
                          const GemvParams& p, cudaStream_t stream, bool pdl) {
  return dispatch(wkind, pro, epi, plan, p, stream, pdl, false);
}

cudaError_t packed_pack(const uint8_t* src, uint8_t* dst, int N, int K, int nr, int row_base,
                        int row_stride, cudaStream_t stream) {
  if (K % 32 || nr <= 0) return cudaErrorInvalidValue;
  const long total = (long)nr * (K / 16);
  const int threads = 256;
  long blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  gemv_pack_kernel<<<(int)blocks, threads, 0, stream>>>(src, dst, N, K, packed_kce(K), nr,
                                                         row_base, row_stride);
  return cudaGetLastError();
}

}  // namespace ec
