// tc_gemm.cuh -- batched decode GEMMs on the tensor cores (tcgen05, kind::i8).
//
// y[b][n] = scale[n] * sum_k W[n][k] x[b][k] for B sequences at once, INT8
// weights.  The activation rows are written as three signed 8-bit digit
// planes (x ~= m_b * (d0 * 2^14 + d1 * 2^7 + d2) / (127 * 2^14), m_b the
// row's max |x|), so the tensor cores multiply INT8 by INT8 into exact int32
// accumulators in TMEM; the digit planes are recombined in int64 and scaled
// once in double.  The only approximation is the 21-bit fixed-point rounding
// of each activation (relative error <= 2^-22 of the row's max |x|); the
// result does not depend on the tiling, the split or the launch.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ec {

constexpr int kTcRows = 128;        // weight rows per tile (the MMA's M)
constexpr int kTcKb = 128;          // K bytes per pipeline unit
constexpr int kTcDigitMax = 2080768;  // 127 * 2^14: full-scale fixed-point value
constexpr int kTcMaxRows = 80;      // sequences per pass (3 digit planes <= 240 columns)

// 3 * B rounded up to 16 sequences: the MMA's N (digit rows)
__host__ __device__ inline int tc_np(int B) { return 3 * ((B + 15) / 16) * 16; }
__host__ __device__ inline int tc_bpad(int B) { return (B + 15) / 16 * 16; }
// weights in the tensor-core layout: ceil(N / 128) tiles of 128 rows x K
size_t tc_weight_bytes(int N, int K);
size_t tc_digit_bytes(int B, int K);
// int32 partial sums of one GEMM launched on `grid` CTAs
size_t tc_ws_bytes(int N, int K, int B, int grid);
cudaError_t tc_prepare();

// rows i < nr of a row-major [nr][K] byte matrix (device) -> rows
// row_base + row_stride * i of the tensor-core layout of an N x K matrix
cudaError_t tc_pack(const uint8_t* src, uint8_t* dst, int N, int K, int nr, int row_base,
                    int row_stride, cudaStream_t s);

// activation rows -> digit planes (+ per-row scale m_b / kTcDigitMax)
struct TcQuant {
  const float* x;
  int x_stride;
  const uint16_t* norm_w;  // RMSNorm first (the reference's op_rmsnorm) when set
  float eps;
  float* xn;               // optional: the normalised rows [B][K] (x_stride apart)
  int8_t* digits;
  double* sx;              // [B]
  int B, K;
};
cudaError_t tc_quant(const TcQuant& q, cudaStream_t s, bool pdl);

// where and how results land (gemv.cuh EPI_*): STORE y[b][n] = v; RESID
// y[b][n] += v; SWIGLU (rows 2i gate, 2i+1 up) y[b][i] = silu(gate) * up
struct TcOut {
  const double* sx;  // tc_quant's per-row scales
  const float* scale;
  float* y;
  int y_stride;
  int epi;
  int silu_vec_limit;
};

struct TcGemm {
  const uint8_t* w;        // tensor-core layout
  const int8_t* digits;    // tc_quant output for the same B, K
  int* ws;                 // tc_ws_bytes: partial sums of tiles split between CTAs
  int N, K, B;
  int grid;                // CTAs (normally the SM count)
  int* err;
  TcOut out;               // tiles one CTA owns whole are finished in the GEMM
};
cudaError_t tc_gemm(const TcGemm& g, cudaStream_t s, bool pdl);

// the tiles split between CTAs: partial sums -> outputs (same TcGemm)
cudaError_t tc_combine(const TcGemm& g, cudaStream_t s, bool pdl);

}  // namespace ec
