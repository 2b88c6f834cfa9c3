// tc_gemm.cu -- batched decode GEMMs on the 5th-generation tensor cores.
//
// Layouts (both K-major, no swizzle; a "core matrix" is 8 rows x 16 bytes
// stored as 128 contiguous bytes):
//   weights  [tile of 128 rows][K block of 128 bytes][slab of 32 bytes (4)]
//            [row group of 8 (16)][16-byte half of the slab (2)][8 rows][16 B]
//            so one 16 KB block is one pipeline unit and one bulk copy;
//   digits   [K block][slab (4)][row group of 8 (NP / 8)][half (2)][8][16 B],
//            digit row c = plane * Bpad + b (planes 0..2 = d0, d1, d2).
// Within a slab the MMA's descriptor steps 128 bytes between the two K halves
// (leading byte offset) and 256 bytes between row groups (stride byte offset).
//
// Kernel: one CTA per SM; the flattened (tile, K block) units are split
// evenly over the CTAs (stream-K), so every SM streams the same number of
// weight bytes.  A CTA's run of units is cut into segments at tile
// boundaries; each segment accumulates into one of two TMEM buffers (int32,
// 128 lanes x NP columns) while the epilogue warps drain the other into the
// workspace [CTA][segment][digit row][128 rows] -- or, when the segment is
// the whole tile, straight into the outputs.  Warp 0 streams units with
// cp.async.bulk onto mbarriers, warp 1 issues tcgen05.mma (kind::i8, M 128,
// N NP, K 32 per instruction) and tcgen05.commit, warps 2..5 read TMEM with
// tcgen05.ld.  tc_combine_kernel then adds the segments of the tiles split
// between CTAs in int64 and applies the epilogue.  Every wait is bounded (error word, then exit).
#include "tc_gemm.cuh"
#include "ec_internal.cuh"
#include "gemv.cuh"

namespace ec {
namespace {

constexpr int kThreads = 192;
constexpr int kStagesMax = 8;
constexpr int kUnitA = kTcRows * kTcKb;  // 16 KB of weights per unit
constexpr int kHdr = 1024;               // barriers etc. before the stages
constexpr int kSmemMax = 227 * 1024;

__host__ __device__ inline long unit_start(int i, long W, int G) { return (long)i * W / G; }

__host__ __device__ inline int max_segments(long W, int G, int Kb) {
  const long per = (W + G - 1) / G;
  return (int)((per + Kb - 1) / Kb) + 1;
}

// ------------------------------------------------------- tcgen05 helpers --

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  // start >> 4 | LBO 128 B >> 4 | SBO 256 B >> 4 | version 1 (sm_100) | no swizzle
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) |
         ((uint64_t)(256 >> 4) << 32) | (1ull << 46);
}

__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p; }" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// One result v of row n for sequence b -> the epilogue.  All 32 lanes of a
// warp call it with the same b and consecutive rows (SWIGLU pairs lanes 2i,
// 2i + 1 = gate, up).
__device__ __forceinline__ void emit(const TcOut& o, int N, int n, int b, float v) {
  float* y = o.y + (size_t)b * o.y_stride;
  if (o.epi == EPI_SWIGLU) {
    const float up = __shfl_down_sync(0xffffffffu, v, 1);
    if ((n & 1) == 0 && n < N) {
      const int i = n >> 1;
      float sig;
      if (i < o.silu_vec_limit)
        sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf_vec(__fsub_rn(0.0f, v))));
      else
        sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf(-v)));
      y[i] = __fmul_rn(__fmul_rn(v, sig), up);
    }
  } else if (n < N) {
    y[n] = o.epi == EPI_RESID ? __fadd_rn(y[n], v) : v;
  }
}

__device__ __forceinline__ float finish(long long tot, double sx, float sc) {
  return (float)((double)tot * (sx * (double)sc));
}

// ------------------------------------------------------------- kernels --

__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(TcGemm g, int NP, int S, int maxseg) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStagesMax;
  uint64_t* tfull = empty + kStagesMax;
  uint64_t* tempty = tfull + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);
  uint8_t* stg = smem + kHdr;
  const int stage_bytes = kUnitA + NP * kTcKb;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Kb = g.K / kTcKb;
  const long W = (long)((g.N + kTcRows - 1) / kTcRows) * Kb;
  const int G = gridDim.x;
  const long u0 = unit_start(blockIdx.x, W, G), u1 = unit_start(blockIdx.x + 1, W, G);

  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tslot)), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      // weights do not depend on the previous kernel: the first stages'
      // weight copies go out before the wait for the digits
      const long pre = min((long)S, u1 - u0);
      for (long t = 0; t < pre; t++) {
        const long u = u0 + t;
        uint8_t* st = stg + (size_t)t * stage_bytes;
        mbar_expect_tx(&full[t], (uint32_t)stage_bytes);
        bulk_g2s(st, g.w + (size_t)u * kUnitA, kUnitA, &full[t]);
      }
      pdl_wait();
      bool ok = true;
      for (long t = 0; t < u1 - u0 && ok; t++) {
        const long u = u0 + t;
        const int s = (int)(t % S);
        uint8_t* st = stg + (size_t)s * stage_bytes;
        const int kb = (int)(u % Kb);
        if (t >= pre) {
          ok = mbar_wait(&empty[s], (uint32_t)(((t / S) - 1) & 1), g.err);
          if (!ok) break;
          mbar_expect_tx(&full[s], (uint32_t)stage_bytes);
          bulk_g2s(st, g.w + (size_t)u * kUnitA, kUnitA, &full[s]);
        }
        bulk_g2s(st + kUnitA, g.digits + (size_t)kb * NP * kTcKb, (uint32_t)(NP * kTcKb), &full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // kind::i8: D s32 (bits 4-5 = 2), A and B signed (bits 7-9, 10-12 = 1),
      // both K-major, N >> 3 at bit 17, M >> 4 at bit 24
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NP >> 3) << 17) |
                             ((uint32_t)(kTcRows >> 4) << 24);
      bool ok = true;
      long t = 0;
      int seg = 0;
      for (long u = u0; u < u1 && ok; seg++) {
        const long tile = u / Kb;
        const long uend = min(u1, (tile + 1) * Kb);
        const int buf = seg & 1;
        if (seg >= 2) {
          ok = mbar_wait(&tempty[buf], (uint32_t)(((seg >> 1) - 1) & 1), g.err);
          if (!ok) break;
        }
        tc_fence_after();
        const uint32_t d = tbase + (uint32_t)(buf * 256);
        const long useg = u;
        for (; u < uend; u++, t++) {
          const int s = (int)(t % S);
          ok = mbar_wait(&full[s], (uint32_t)((t / S) & 1), g.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(stg + (size_t)s * stage_bytes);
          const uint32_t b0 = a0 + kUnitA;
#pragma unroll
          for (int j = 0; j < kTcKb / 32; j++)
            mma_i8(d, smem_desc(a0 + j * 4096), smem_desc(b0 + j * NP * 32), idesc,
                   (u > useg || j > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&tfull[buf]);
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lanes 32q .. 32q + 31 (this warp's quadrant)
    const int row = q * 32 + lane;
    pdl_wait();  // the workspace and y may still be read by the previous kernel
    const int Bp = tc_bpad(g.B);
    bool ok = true;
    int seg = 0;
    for (long u = u0; u < u1 && ok; seg++) {
      const long tile = u / Kb, us = u;
      u = min(u1, (tile + 1) * Kb);
      const bool whole = us == tile * Kb && u == (tile + 1) * Kb;
      const int buf = seg & 1;
      ok = mbar_wait(&tfull[buf], (uint32_t)((seg >> 1) & 1), g.err);
      if (!ok) break;
      tc_fence_after();
      const uint32_t ta = tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 256);
      if (whole) {
        // the tile is this CTA's alone: digit planes -> int64 -> outputs
        const int n = (int)tile * kTcRows + row;
        const float sc = n < g.N ? g.out.scale[n] : 0.0f;
        for (int b0 = 0; b0 < g.B; b0 += 16) {
          int p0[16], p1[16], p2[16];
          tmem_ld16(ta + b0, p0);
          tmem_ld16(ta + Bp + b0, p1);
          tmem_ld16(ta + 2 * Bp + b0, p2);
#pragma unroll
          for (int c = 0; c < 16; c++) {
            const int b = b0 + c;
            if (b < g.B) {
              const long long tot =
                  (long long)p0[c] * 16384 + (long long)p1[c] * 128 + (long long)p2[c];
              emit(g.out, g.N, n, b, finish(tot, g.out.sx[b], sc));
            }
          }
        }
      } else {
        int* dst = g.ws + ((size_t)(blockIdx.x * maxseg + seg) * NP) * kTcRows + row;
        for (int c0 = 0; c0 < NP; c0 += 16) {
          int r[16];
          tmem_ld16(ta + c0, r);
#pragma unroll
          for (int c = 0; c < 16; c++) dst[(size_t)(c0 + c) * kTcRows] = r[c];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(512)
                 : "memory");
  }
}

// Tiles split between CTAs: CTA (i, y) finishes sequences 4y .. 4y + 3 of
// the tile in which GEMM CTA i starts, when that start is inside the tile and
// no earlier CTA starts inside it too.  Thread r owns row tile * 128 + r; its
// loads of one segment are independent, so a CTA waits about one memory
// round trip per segment.
constexpr int kCombSeq = 4;

__global__ void __launch_bounds__(kTcRows) tc_combine_kernel(TcGemm g, int NP, int maxseg) {
  pdl_wait();
  pdl_launch_dependents();
  const int Kb = g.K / kTcKb;
  const long W = (long)((g.N + kTcRows - 1) / kTcRows) * Kb;
  const int G = g.grid < W ? g.grid : (int)W;
  const int i = blockIdx.x, r = threadIdx.x, b0 = blockIdx.y * kCombSeq;
  if (i == 0) return;
  const long si = unit_start(i, W, G);
  const long t = si / Kb, ub = t * Kb, ue = ub + Kb;
  if (si == ub || unit_start(i - 1, W, G) > ub) return;
  const int n = (int)t * kTcRows + r;
  const int Bp = tc_bpad(g.B);
  const float sc = n < g.N ? g.out.scale[n] : 0.0f;
  long long tot[kCombSeq];
#pragma unroll
  for (int k = 0; k < kCombSeq; k++) tot[k] = 0;
  // this tile's partial sums: CTAs i - 1, i, ... while they start inside it
  for (int j = i - 1; j < G; j++) {
    const long sj = unit_start(j, W, G);
    if (sj >= ue) break;
    const int* p = g.ws + ((size_t)(j * maxseg + (int)(t - sj / Kb)) * NP) * kTcRows + r;
#pragma unroll
    for (int k = 0; k < kCombSeq; k++) {
      const int b = b0 + k;
      if (b < g.B)
        tot[k] += (long long)__ldcg(p + (size_t)b * kTcRows) * 16384 +
                  (long long)__ldcg(p + (size_t)(Bp + b) * kTcRows) * 128 +
                  (long long)__ldcg(p + (size_t)(2 * Bp + b) * kTcRows);
    }
  }
#pragma unroll
  for (int k = 0; k < kCombSeq; k++)
    if (b0 + k < g.B) emit(g.out, g.N, n, b0 + k, finish(tot[k], g.out.sx[b0 + k], sc));
}

// One CTA per sequence: (RMSNorm,) max |x|, digit planes.
constexpr int kQThreads = 512;

__global__ void __launch_bounds__(kQThreads) tc_quant_kernel(TcQuant q) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  __shared__ float s_max;
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x, tid = threadIdx.x, K = q.K;
  const float* x = q.x + (size_t)b * q.x_stride;
  for (int j = tid; j < K; j += kQThreads) xs[j] = x[j];
  __syncthreads();
  if (q.norm_w) {
    rmsnorm_smem(xs, q.norm_w, K, q.eps, red, tid, kQThreads);
    if (q.xn)
      for (int j = tid; j < K; j += kQThreads) q.xn[(size_t)b * q.x_stride + j] = xs[j];
  }
  float m = 0.0f;
  for (int j = tid; j < K; j += kQThreads) m = fmaxf(m, fabsf(xs[j]));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = m;
  __syncthreads();
  if (tid < 32) {
    float v = tid < kQThreads / 32 ? red[tid] : 0.0f;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (tid == 0) {
      s_max = v;
      q.sx[b] = v > 0.0f ? (double)v / (double)kTcDigitMax : 0.0;
    }
  }
  __syncthreads();
  const float mx = s_max;
  const double inv = mx > 0.0f ? (double)kTcDigitMax / (double)mx : 0.0;
  const int NP = tc_np(q.B), Bp = tc_bpad(q.B);
  for (int ch = tid; ch < K / 16; ch += kQThreads) {
    const int k0 = ch * 16, kb = k0 >> 7, kk = k0 & 127;
    uint32_t w[3][4];
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      uint32_t p0 = 0, p1 = 0, p2 = 0;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const long long xv = llrint((double)xs[k0 + e + i] * inv);
        const long long d0 = llrint((double)xv * (1.0 / 16384.0));
        const long long r0 = xv - d0 * 16384;
        const long long d1 = llrint((double)r0 * (1.0 / 128.0));
        const long long d2 = r0 - d1 * 128;
        p0 |= (uint32_t)(uint8_t)(int8_t)d0 << (8 * i);
        p1 |= (uint32_t)(uint8_t)(int8_t)d1 << (8 * i);
        p2 |= (uint32_t)(uint8_t)(int8_t)d2 << (8 * i);
      }
      w[0][e >> 2] = p0;
      w[1][e >> 2] = p1;
      w[2][e >> 2] = p2;
    }
    const size_t base = (size_t)kb * NP * kTcKb + (size_t)(kk >> 5) * NP * 32 + ((kk >> 4) & 1) * 128;
#pragma unroll
    for (int pl = 0; pl < 3; pl++) {
      const int c = pl * Bp + b;
      *reinterpret_cast<uint4*>(q.digits + base + (c >> 3) * 256 + (c & 7) * 16) =
          make_uint4(w[pl][0], w[pl][1], w[pl][2], w[pl][3]);
    }
  }
}

// 16 bytes of one source row per thread.
__global__ void tc_pack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int K,
                               int nr, int row_base, int row_stride) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per = K / 16;
  if (i >= (long)nr * per) return;
  const int rr = (int)(i / per), ch = (int)(i % per);
  const int n = row_base + row_stride * rr;
  const int tile = n / kTcRows, r = n % kTcRows, k0 = ch * 16, kb = k0 >> 7, kk = k0 & 127;
  const size_t off = ((size_t)tile * (K / kTcKb) + kb) * kUnitA + (size_t)(kk >> 5) * 4096 +
                     (r >> 3) * 256 + ((kk >> 4) & 1) * 128 + (r & 7) * 16;
  *reinterpret_cast<uint4*>(dst + off) = *reinterpret_cast<const uint4*>(src + (size_t)rr * K + k0);
}

template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
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

int stages_for(int NP) {
  const int sb = kUnitA + NP * kTcKb;
  int S = (kSmemMax - kHdr) / sb;
  return S > kStagesMax ? kStagesMax : S;
}

}  // namespace

size_t tc_weight_bytes(int N, int K) { return (size_t)((N + kTcRows - 1) / kTcRows) * kTcRows * K; }

size_t tc_digit_bytes(int B, int K) { return (size_t)tc_np(B) * K; }

size_t tc_ws_bytes(int N, int K, int B, int grid) {
  const int Kb = K / kTcKb;
  const long W = (long)((N + kTcRows - 1) / kTcRows) * Kb;
  const int G = grid < W ? grid : (int)W;
  return (size_t)G * max_segments(W, G, Kb) * tc_np(B) * kTcRows * 4;
}

cudaError_t tc_prepare() {
  cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSmemMax);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tc_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemMax - 1024);
  return e;
}

cudaError_t tc_pack(const uint8_t* src, uint8_t* dst, int N, int K, int nr, int row_base,
                    int row_stride, cudaStream_t s) {
  if (K % kTcKb || row_base + (long)row_stride * (nr - 1) >= N) return cudaErrorInvalidValue;
  const long n = (long)nr * (K / 16);
  if (n == 0) return cudaSuccess;
  tc_pack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, dst, K, nr, row_base, row_stride);
  return cudaGetLastError();
}

cudaError_t tc_quant(const TcQuant& q, cudaStream_t s, bool pdl) {
  if (q.K % kTcKb || q.B < 1 || q.B > kTcMaxRows || (size_t)q.K * 4 > (size_t)kSmemMax - 2048)
    return cudaErrorInvalidValue;
  return launch_ex(tc_quant_kernel, dim3(q.B), dim3(kQThreads), (size_t)q.K * 4, s, pdl, q);
}

cudaError_t tc_gemm(const TcGemm& g, cudaStream_t s, bool pdl) {
  if (g.K % kTcKb || g.B < 1 || g.B > kTcMaxRows || g.N < 1) return cudaErrorInvalidValue;
  const int NP = tc_np(g.B), Kb = g.K / kTcKb;
  const long W = (long)((g.N + kTcRows - 1) / kTcRows) * Kb;
  const int G = g.grid < W ? g.grid : (int)W;
  const int S = stages_for(NP);
  const size_t smem = kHdr + (size_t)S * (kUnitA + NP * kTcKb);
  return launch_ex(tc_gemm_kernel, dim3(G), dim3(kThreads), smem, s, pdl, g, NP, S,
                   max_segments(W, G, Kb));
}

cudaError_t tc_combine(const TcGemm& g, cudaStream_t s, bool pdl) {
  if (g.K % kTcKb || g.B < 1 || g.B > kTcMaxRows) return cudaErrorInvalidValue;
  const int Kb = g.K / kTcKb;
  const long W = (long)((g.N + kTcRows - 1) / kTcRows) * Kb;
  const int G = g.grid < W ? g.grid : (int)W;
  return launch_ex(tc_combine_kernel, dim3(G, (g.B + kCombSeq - 1) / kCombSeq), dim3(kTcRows), 0,
                   s, pdl, g, tc_np(g.B),
                   max_segments(W, G, Kb));
}

}  // namespace ec

// ------------------------------------------------------------- C ABI ----

extern "C" size_t ec_gemm_tc_bytes(int m, int k) {
  return (m > 0 && k > 0 && k % ec::kTcKb == 0) ? ec::tc_weight_bytes(m, k) : 0;
}

extern "C" int ec_gemm_tc_pack(const void* w_rowmajor, void* w_tc, int m, int k, void* stream) {
  if (!w_rowmajor || !w_tc || m <= 0 || k <= 0 || k % ec::kTcKb) {
    ec_set_last_error("ec_gemm_tc_pack: null pointer, or k not a multiple of 128");
    return EC_ERR_ARG;
  }
  EC_CUDA_TRY(ec::tc_pack(static_cast<const uint8_t*>(w_rowmajor), static_cast<uint8_t*>(w_tc), m,
                          k, m, 0, 1, static_cast<cudaStream_t>(stream)));
  return EC_OK;
}

extern "C" int ec_op_gemm_tc(const void* w_tc, const float* scale, const float* x, float* y,
                             int m, int k, int nb, void* stream) {
  if (!w_tc || !scale || !x || !y || m <= 0 || k <= 0 || nb <= 0 || k % ec::kTcKb ||
      (size_t)k * 4 > 200 * 1024) {
    ec_set_last_error("ec_op_gemm_tc: null pointer, k not a multiple of 128, or k > 51200");
    return EC_ERR_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0, n_sm = 148;
  EC_CUDA_TRY(cudaGetDevice(&dev));
  EC_CUDA_TRY(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
  EC_CUDA_TRY(ec::tc_prepare());
  const int pb = nb < ec::kTcMaxRows ? nb : ec::kTcMaxRows;
  const size_t dig = (ec::tc_digit_bytes(pb, k) + 255) & ~(size_t)255;
  const size_t sxb = 1024;
  const size_t wsb = ec::tc_ws_bytes(m, k, pb, n_sm);
  uint8_t* buf = nullptr;
  EC_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&buf), dig + sxb + wsb + 256, s));
  int8_t* digits = reinterpret_cast<int8_t*>(buf);
  double* sx = reinterpret_cast<double*>(buf + dig);
  int* ws = reinterpret_cast<int*>(buf + dig + sxb);
  int* err = reinterpret_cast<int*>(buf + dig + sxb + wsb);
  cudaError_t e = cudaMemsetAsync(err, 0, 4, s);
  for (int b0 = 0; b0 < nb && e == cudaSuccess; b0 += ec::kTcMaxRows) {
    const int B = nb - b0 < ec::kTcMaxRows ? nb - b0 : ec::kTcMaxRows;
    ec::TcQuant q{};
    q.x = x + (size_t)b0 * k;
    q.x_stride = k;
    q.digits = digits;
    q.sx = sx;
    q.B = B;
    q.K = k;
    ec::TcGemm g{};
    g.w = static_cast<const uint8_t*>(w_tc);
    g.digits = digits;
    g.ws = ws;
    g.N = m;
    g.K = k;
    g.B = B;
    g.grid = n_sm;
    g.err = err;
    g.out.sx = sx;
    g.out.scale = scale;
    g.out.y = y + (size_t)b0 * m;
    g.out.y_stride = m;
    g.out.epi = ec::EPI_STORE;
    e = ec::tc_quant(q, s, false);
    if (e == cudaSuccess) e = ec::tc_gemm(g, s, true);
    if (e == cudaSuccess) e = ec::tc_combine(g, s, true);
  }
  int h = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&h, err, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFreeAsync(buf, s);
  if (e != cudaSuccess) {
    ec_set_last_error(cudaGetErrorString(e));
    return EC_ERR_CUDA;
  }
  if (h) {
    ec_set_last_error("ec_op_gemm_tc: a bounded device wait timed out");
    return h;
  }
  return EC_OK;
}
