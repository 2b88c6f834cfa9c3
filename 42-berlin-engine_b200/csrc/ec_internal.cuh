// ec_internal.cuh -- shared device helpers for libengine_cuda (sm_100a).
//
// Numerics contract: this library is compiled with -fmad=false, so no
// multiply-add is fused unless written here as __fmaf_rn.  Every FMA below sits
// where the reference engine's AVX2 code (or its compiler's contraction of
// scalar C) fuses one, so the decode step reproduces the reference's floating
// point results bit for bit.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "engine_cuda.h"

namespace ec {

// ---------------------------------------------------------------- numerics --

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __int_as_float(((uint32_t)b) << 16);
}

// round-to-nearest-even on the bit pattern (src/tensor/tensor.c:67-76)
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// Schraudolph's exponential (Neural Computation 11(4), 1999), scalar form of
// src/compute/ops_math_fast.h:48-64: below -87 -> 0, above 87 clamped, then
// (int)(2^23/ln2 * x + 127<<23) truncated toward zero, read as float bits.
__device__ __forceinline__ float fast_expf(float x) {
  if (x < -87.0f) return 0.0f;
  if (x > 87.0f) x = 87.0f;
  return __int_as_float(__float2int_rz(__fmaf_rn(12102203.0f, x, 1065353216.0f)));
}

// Vector form (ops_math_fast.h:105-126): max/min clamp (NaN takes the clamp
// value), one FMA, conversion with round-to-nearest-even.
__device__ __forceinline__ float fast_expf_vec(float x) {
  x = (x > -87.0f) ? x : -87.0f;
  x = (x < 87.0f) ? x : 87.0f;
  return __int_as_float(__float2int_rn(__fmaf_rn(x, 12102203.0f, 1065353216.0f)));
}

// ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)): the AVX 8-lane horizontal sum
__device__ __forceinline__ float hsum8(const float* v) {
  float a = __fadd_rn(__fadd_rn(v[0], v[4]), __fadd_rn(v[1], v[5]));
  float b = __fadd_rn(__fadd_rn(v[2], v[6]), __fadd_rn(v[3], v[7]));
  return __fadd_rn(a, b);
}

// 8-lane FMA dot product + horizontal sum + FMA tail (simd_dot_f32_f32,
// simd_kernels.h:162-191), one thread.
__device__ __forceinline__ float dot8_f32(const float* a, const float* b, int n) {
  float acc[8];
#pragma unroll
  for (int l = 0; l < 8; l++) acc[l] = 0.0f;
  int i = 0;
  for (; i + 7 < n; i += 8) {
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = __fmaf_rn(a[i + l], b[i + l], acc[l]);
  }
  float s = hsum8(acc);
  for (; i < n; i++) s = __fmaf_rn(a[i], b[i], s);
  return s;
}

// ---------------------------------------------------- int8 / fp8 decoding --

// Four signed bytes of w -> four exact floats.  (byte ^ 0x80) is placed in the
// low mantissa byte of 2^23 (0x4B000000); subtracting 2^23 + 128 recovers the
// signed value exactly.
__device__ __forceinline__ void dec_i8x4(uint32_t w, float* f) {
  uint32_t u = w ^ 0x80808080u;
  f[0] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)), 8388736.0f);
  f[1] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)), 8388736.0f);
  f[2] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)), 8388736.0f);
  f[3] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)), 8388736.0f);
}

// E4M3 byte -> float with the reference's semantics (ops_quant.c:27-50): the
// 7 low bits placed at bit 20 give 2^(e-127)(1+m/8) for e>0 and m*2^-129 for
// e==0; one multiply by 2^120 rescales both exactly; 0x7F decodes to 480.
__device__ __forceinline__ float dec_fp8(uint32_t byte) {
  float mag = __uint_as_float((byte & 0x7Fu) << 20) * 0x1p120f;
  return (byte & 0x80u) ? -mag : mag;
}

__device__ __forceinline__ void dec_fp8x4(uint32_t w, float* f) {
  f[0] = dec_fp8(w & 0xFF);
  f[1] = dec_fp8((w >> 8) & 0xFF);
  f[2] = dec_fp8((w >> 16) & 0xFF);
  f[3] = dec_fp8(w >> 24);
}

// two BF16 in w -> two floats
__device__ __forceinline__ void dec_bf16x2(uint32_t w, float* f) {
  f[0] = __uint_as_float(w << 16);
  f[1] = __uint_as_float(w & 0xFFFF0000u);
}

// --------------------------------------------------------- bulk copies --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000; "
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a phase (no suspension): for loops that have other
// work to do while they wait.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; "
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait with an iteration limit (each try_wait may suspend the thread for up
// to 1 us until the phase completes, so the limit is about a second).  On
// timeout the error word is set and false is returned; callers then skip
// their work and exit instead of hanging the GPU.
constexpr uint32_t kWaitLimit = 1u << 20;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kWaitLimit; i++)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicCAS(err, 0, EC_ERR_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src and bytes must be multiples of 16.
// 16-byte asynchronous copy global -> shared through L2 (cp.async.cg).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed
// (the arrival is not counted up front: init the barrier with the number of
// arriving threads).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 16-byte read-only global load that skips L1.
__device__ __forceinline__ uint4 ldg_nc16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Prefetch [src, src + bytes) into L2 (no shared memory, no completion).
// src and bytes multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue now / wait until the previous kernel's memory is visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Four INT8 weights (one 32-bit word, elements 0..3) times x (pairs 0,1 and
// 2,3) accumulated into two f32x2 accumulators: each byte v becomes the exact
// float 2^23 + 128 + v by one byte permute, the bias is subtracted in pairs,
// then paired fma.rn -- four independent fma.rn chains.  bias2 holds
// -(2^23 + 128) twice.
__device__ __forceinline__ void fma4_i8(uint32_t w, uint64_t x01, uint64_t x23, uint64_t bias2,
                                        uint64_t& acc01, uint64_t& acc23) {
  asm("{\n\t.reg .b32 u, a, b, c, d;\n\t.reg .b64 p, q;\n\t"
      "xor.b32 u, %4, 0x80808080;\n\t"
      "prmt.b32 a, u, 0x4B000000, 0x7540;\n\t"
      "prmt.b32 b, u, 0x4B000000, 0x7541;\n\t"
      "prmt.b32 c, u, 0x4B000000, 0x7542;\n\t"
      "prmt.b32 d, u, 0x4B000000, 0x7543;\n\t"
      "mov.b64 p, {a, b};\n\t"
      "mov.b64 q, {c, d};\n\t"
      "add.rn.f32x2 p, p, %5;\n\t"
      "add.rn.f32x2 q, q, %5;\n\t"
      "fma.rn.f32x2 %0, p, %2, %0;\n\t"
      "fma.rn.f32x2 %1, q, %3, %1;\n\t}"
      : "+l"(acc01), "+l"(acc23)
      : "l"(x01), "l"(x23), "r"(w), "l"(bias2));
}

// ------------------------------------------------ paired f32 arithmetic --
// add/mul/fma.rn.f32x2 (sm_100): two independent IEEE operations, the same
// rounding as the scalar forms.
__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ void fma2(uint64_t& acc, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// Four weight bytes -> two float pairs (elements 0,1 and 2,3), exact.
template <int WK>
__device__ __forceinline__ void decode_pairs(uint32_t w, uint64_t& p01, uint64_t& p23) {
  if constexpr (WK == EC_W_INT8) {
    // 0x4B0000xx with xx = v ^ 0x80 is 2^23 + 128 + v
    const uint32_t u = w ^ 0x80808080u;
    const uint64_t bias = pack2(__float_as_uint(-8388736.0f), __float_as_uint(-8388736.0f));
    p01 = add2(pack2(__byte_perm(u, 0x4B000000u, 0x7540), __byte_perm(u, 0x4B000000u, 0x7541)),
               bias);
    p23 = add2(pack2(__byte_perm(u, 0x4B000000u, 0x7542), __byte_perm(u, 0x4B000000u, 0x7543)),
               bias);
  } else {
    // E4M3 with the reference's semantics (fp8_to_float, ops_quant.c:27-50):
    // byte k moved to the top byte, an arithmetic shift by 4 leaves the sign
    // in bit 31 and the 7 magnitude bits at 20..26; times 2^120 exactly
    auto bits = [](uint32_t t) { return (uint32_t)(((int)t) >> 4) & 0x87F00000u; };
    const uint64_t s120 = pack2(__float_as_uint(0x1p120f), __float_as_uint(0x1p120f));
    p01 = mul2(pack2(bits(w << 24), bits(w << 16)), s120);
    p23 = mul2(pack2(bits(w << 8), bits(w)), s120);
  }
}

// RMSNorm of xs[0..K) in place (consumer threads only; `nc` of them).
__device__ __forceinline__ void rmsnorm_smem(float* xs, const uint16_t* __restrict__ w, int K,
                                             float eps, float* red, int ct, int nc) {
  if (ct < 8) {
    float acc = 0.0f;
    int j = ct;
    const int k8 = K & ~7;
#pragma unroll 8
    for (; j < k8; j += 8) acc = __fmaf_rn(xs[j], xs[j], acc);
    red[ct] = acc;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nc));
  if (ct == 0) {
    float ss = hsum8(red);
    for (int j = K & ~7; j < K; j++) ss = __fmaf_rn(xs[j], xs[j], ss);
    ss = __fdiv_rn(ss, (float)K);
    red[8] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, eps)));
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nc));
  const float inv = red[8];
  for (int j = ct; j < K; j += nc) xs[j] = __fmul_rn(__fmul_rn(xs[j], inv), bf16_to_f32(w[j]));
  asm volatile("bar.sync 1, %0;" ::"r"(nc));
}

}  // namespace ec

// ------------------------------------------------------------- host side --
#define EC_CUDA_TRY(expr)                          \
  do {                                             \
    cudaError_t e_ = (expr);                       \
    if (e_ != cudaSuccess) {                       \
      ec_set_last_error(cudaGetErrorString(e_));   \
      return EC_ERR_CUDA;                          \
    }                                              \
  } while (0)

extern "C" void ec_set_last_error(const char* msg);
