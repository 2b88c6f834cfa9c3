// gemv.cuh -- batch-1 weight-streaming GEMV (INT8 / FP8-E4M3 / BF16 weights).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace ec {

enum GemvPro { PRO_NONE = 0, PRO_RMSNORM = 1 };
enum GemvEpi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2 };

struct GemvParams {
  const uint8_t* w;        // [N][K] elements of the weight kind, row-major
  const float* scale;      // per row: scale[row * scale_stride] (BF16: unused)
  int scale_stride;        // 1: one scale per row; 0: one scale per matrix
  const float* x;          // [K] fp32 input
  const uint16_t* norm_w;  // [K] bf16 RMSNorm weight (PRO_RMSNORM)
  float eps;
  float* y;                // STORE: [N]; RESID: [N] (y += W.x); SWIGLU: [N/2]
  int N;
  int K;
  int rg;                  // rows per group (consumer threads = 8 * rg)
  int kcb;                 // bytes of one row streamed per pipeline stage
  int silu_vec_limit;      // SWIGLU: outputs below this index use the vector form
  int* err;
  int stages;              // packed kernel: pipeline stages (set from the plan)
};

// Host-side launch description for one GEMV shape.
struct GemvPlan {
  int grid;
  int block;
  int smem;
  int rg;
  int kcb;
};

// Build a plan for `n_sm` SMs; returns false if the shape is unsupported.
bool gemv_plan(int wkind, int N, int K, int epi, int n_sm, GemvPlan* plan);

// Set the kernels' shared-memory attribute on the current device.
cudaError_t gemv_prepare();

// Launch (PDL attribute set when `pdl` is true).
cudaError_t gemv_launch(int wkind, int pro, int epi, const GemvPlan& plan, const GemvParams& p,
                        cudaStream_t stream, bool pdl);

// ---------------------------------------------------------------------------
// Packed-layout GEMV (gemv_packed.cu): the decode step's weight matrices are
// repacked once at upload into [chunk][row quad][32-column piece][4 rows][32 B]
// so that one bulk copy fills each pipeline stage.
struct PackedPlan {
  int grid;
  int warps;            // consumer warps (block = 32 * (warps + 1))
  int rows_per_thread;  // 1 or 2
  int kce;              // columns per chunk: 512 or 32
  int stages;
  int smem;
};

int packed_kce(int K);
size_t packed_bytes(int N, int K);
// force_r: 0 = choose, 1 or 2 = rows per thread.  co_resident: at most
// about half an SM (shared memory, threads), so the next kernel fits beside.
bool packed_plan(int wkind, int N, int K, int n_sm, int force_r, bool co_resident,
                 PackedPlan* plan);
cudaError_t packed_prepare();
cudaError_t packed_launch(int wkind, int pro, int epi, const PackedPlan& plan,
                          const GemvParams& p, cudaStream_t stream, bool pdl);
// Pack nr row-major rows of K bytes (device) into packed rows
// row_base + row_stride * i of an N-row packed matrix (device).
cudaError_t packed_pack(const uint8_t* src, uint8_t* dst, int N, int K, int nr, int row_base,
                        int row_stride, cudaStream_t stream);

}  // namespace ec
