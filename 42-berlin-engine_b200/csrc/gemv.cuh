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

}  // namespace ec
