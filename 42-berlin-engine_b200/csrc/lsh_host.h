// lsh_host.h -- host side of the LSH hyperplanes, shared by the decode
// context and the isolated LSH attention.
#pragma once
#include <cmath>
#include <vector>

namespace ec {

// rand_gaussian, src/compute/ops_lsh.c:22-34 (host libm, same formula)
inline float rand_gaussian(unsigned* seed) {
  *seed = *seed * 1103515245u + 12345u;
  float u1 = (float)((*seed >> 16) & 0x7FFF) / 32767.0f;
  *seed = *seed * 1103515245u + 12345u;
  float u2 = (float)((*seed >> 16) & 0x7FFF) / 32767.0f;
  if (u1 < 1e-6f) u1 = 1e-6f;
  return sqrtf(-2.0f * logf(u1)) * cosf(2.0f * 3.14159265f * u2);
}

// lsh_init (ops_lsh.c:40-85) for L tables of `bits` hyperplanes over `dim`
// dimensions, L2-normalised: table t is seeded 42 + t.  [t][bit][dim].
inline std::vector<float> lsh_hyperplanes(int tables, int bits, int dim) {
  std::vector<float> hp((size_t)tables * bits * dim);
  for (int t = 0; t < tables; t++) {
    unsigned seed = 42u + (unsigned)t;
    for (int b = 0; b < bits; b++) {
      float* row = &hp[((size_t)t * bits + b) * dim];
      float norm = 0.0f;
      for (int d = 0; d < dim; d++) {
        row[d] = rand_gaussian(&seed);
        norm = norm + row[d] * row[d];
      }
      norm = sqrtf(norm);
      if (norm > 1e-6f)
        for (int d = 0; d < dim; d++) row[d] = row[d] / norm;
    }
  }
  return hp;
}

}  // namespace ec
