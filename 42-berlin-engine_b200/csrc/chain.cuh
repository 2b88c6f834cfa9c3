// chain.cuh -- one layer's weight-streaming GEMVs as one persistent kernel.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "gemv.cuh"

namespace ec {

constexpr int kMaxChainPhases = 6;

// One GEMV of the chain: y = W . prologue(x) with the given epilogue, W in
// the packed layout of gemv_packed.cu with one fp32 scale per row.
struct ChainPhase {
  const uint8_t* w;
  const float* scale;
  const float* x;          // [K], complete when the previous phase is
  const uint16_t* norm_w;  // PRO_RMSNORM: [K] bf16
  float* y;
  int N, K;
  int pro, epi;
  int silu_vec_limit;
  int x_stride, y_stride;  // batched chain: floats between sequences
};

// Batched chain: one more phase kind, the RMSNorm of NB rows into y (no
// weights; CTA b normalises row b), so that the GEMV phases read normalised
// vectors chunk by chunk.
constexpr int PRO_NORM_ROWS = 2;

struct ChainParams {
  ChainPhase ph[kMaxChainPhases];
  int nph;
  int* ctr;  // [kMaxChainPhases + 1] zeroed counters, owned by this chain
  int* err;
  float eps;
  int mark;    // record phase timestamps (builds with EC_PHASE_TIMING)
  int kmax;    // set by chain_launch
  int knorm;   // set by chain_launch: the largest K of an RMSNorm phase
  int stages;  // set by chain_launch
  // Grid-counter waits between phases: iterations before EC_ERR_TIMEOUT
  // (0: the default limit, about a second); wait_extra > 0 makes the first
  // such wait look for a count no CTA reaches (a test of the timeout path).
  int wait_iters;
  int wait_extra;
};

// 512 or 32 when every phase has the same packed chunk width, else 0 (the
// chain cannot run; launch the phases one by one).
int chain_kce(const ChainParams& P);
cudaError_t chain_prepare();
// CTAs of the batch-1 chain kernel one SM holds at once (every CTA of the
// chain must be resident together: the grid is the SM count).
// knorm: the largest K of an RMSNorm phase (the model dimension).
int chain_blocks_per_sm(int wkind, int kce, int kmax, int knorm);
// grid = the SM count (every CTA resident at once).
cudaError_t chain_launch(int wkind, ChainParams P, int grid, cudaStream_t s, bool pdl);
// The same chain over nb sequences (2..8) at once: each weight byte is
// decoded once and accumulated for every sequence in the reference's order.
// Phases with pro == PRO_NORM_ROWS normalise (x -> y, norm_w, K columns).
cudaError_t chain_launch_nb(int wkind, ChainParams P, int nb, int grid, cudaStream_t s, bool pdl);

}  // namespace ec
