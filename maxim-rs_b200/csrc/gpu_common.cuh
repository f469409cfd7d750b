// Shared device-side helpers for the executor's kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "common.h"

namespace mx {

#define MX_CUDA(call)                                                                                      \
  do {                                                                                                     \
    cudaError_t e_ = (call);                                                                               \
    if (e_ != cudaSuccess)                                                                                 \
      throw ::mx::Error(std::string(#call) + ": " + cudaGetErrorString(e_), MX_E_CUDA);                   \
  } while (0)

// A strided NHWC view of one plan buffer: pixel p, channel c lives at
// ptr[p * stride + c]. `stride` is the channel count of the buffer that owns
// the storage (a channel view of a wider buffer keeps its parent's stride).
struct View {
  float* ptr;
  int64_t stride;
  int64_t c;  // channels of this buffer
  int64_t npix;
};

inline unsigned blocks_for(int64_t n, int threads) { return unsigned((n + threads - 1) / threads); }

#ifdef __CUDACC__
// The activations, shared by the standalone elementwise kernels and the
// tensor-core epilogue so a fused step computes exactly what the separate
// op would (src/exec_cpu.rs: gelu with erf, the logistic sigmoid).
//
// GELU in its erf form, x * Phi(x), evaluated as
//   x Phi(x) = max(x, 0) - u Phi(-u),   u = |x|,
//   Phi(-u)  = exp(-u^2 / 2) * R(u),     R(u) = erfcx(u / sqrt 2) / 2,
// with R a degree-11 polynomial in u fitted for this kernel set (least squares
// on [0, 5.6] weighted by exp(-u^2 / 2), reweighted toward minimax) and u
// clamped to 5.6 inside R, past which the term is below 2^-24 |x|. No
// subtraction cancels: for x < 0 the result is the product itself. The
// exponential is one ex2.approx. Including fp32 evaluation, the error over
// [-12, 12] stays within about 1.3 ulp of |x| and, for x > -0.7, 3 ulp of the
// result (checked against a double-precision erf by tests/test_gelu_poly.py;
// the erf form loses about as much to the rounding of 1 + erf). It costs 18
// instructions, where
// 0.5 x (1 + erff(x / sqrt 2)) costs about 28, and the tensor-core epilogue
// of a GELU step is bound by its instruction issue.
__device__ __forceinline__ float ex2_approx(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}
__device__ __forceinline__ float gelu_f(float x) {
  constexpr float kGeluR[12] = {
      0.4999999701976776f,
      -0.3989405930042267f,
      0.24997256696224213f,
      -0.13280577957630157f,
      0.06192392110824585f,
      -0.025471799075603485f,
      0.009003829210996628f,
      -0.0025900795590132475f,
      0.0005636486457660794f,
      -8.47700794111006e-05f,
      7.708666089456528e-06f,
      -3.155372496621567e-07f};
  const float u = fminf(fabsf(x), 5.6f);
  float p = kGeluR[11];
#pragma unroll
  for (int k = 10; k >= 0; --k) p = fmaf(p, u, kGeluR[k]);
  const float e = ex2_approx(__fmul_rn(__fmul_rn(x, -0.72134752f), x));  // 2^(-x^2 log2(e) / 2)
  return fmaf(-__fmul_rn(u, e), p, fmaxf(x, 0.0f));
}
__device__ __forceinline__ float sigmoid_f(float a) { return 1.0f / (1.0f + expf(-a)); }

// Paired fp32 arithmetic (the f32x2 instructions of sm_100): one instruction
// carries out the same IEEE round-to-nearest operation on two lanes, each
// lane rounded exactly as the scalar instruction rounds it, so a paired
// evaluation is bit-identical to the scalar one and halves the instructions
// the epilogue issues for it.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// The sum t + b where t is the result of a paired multiply. Written as the
// paired add, it is fused with that multiply by the assembler (measured on
// B200: mul.rn.f32x2 followed by add.rn.f32x2 comes out as one fused
// multiply-add, its rounding differing from the two roundings in about a
// quarter of cases, whatever the contraction flag says). A fused
// multiply-add of t by a one the assembler cannot see is exactly one rounded
// addition (t * 1 is exact), so it keeps the separate rounding.
static __constant__ float kOnePair[2] = {1.0f, 1.0f};
__device__ __forceinline__ uint64_t f2_add_after_mul(uint64_t t, uint64_t b) {
  return f2_fma(t, *reinterpret_cast<const uint64_t*>(kOnePair), b);
}
// a += b and c += d as one paired add.
__device__ __forceinline__ void f2_add_to(float& a, float& c, float b, float d) {
  f2_unpack(f2_add(f2_pack(a, c), f2_pack(b, d)), a, c);
}

// gelu_f on two values at once, bit-identical to gelu_f on each. With
// w = -u = max(-|x|, -5.6) and kGeluRw[k] = (-1)^k kGeluR[k] (the magnitudes:
// R's coefficients alternate in sign), Horner over w gives (-1)^k times every
// partial sum of Horner over u - the same magnitudes, rounded the same way -
// and ends on exactly R(u); w e is then exactly -(u e), the scalar form's
// first factor.
__device__ __forceinline__ void gelu_f2(float& a, float& b) {
  constexpr float kGeluRw[12] = {
      0.4999999701976776f,
      0.3989405930042267f,
      0.24997256696224213f,
      0.13280577957630157f,
      0.06192392110824585f,
      0.025471799075603485f,
      0.009003829210996628f,
      0.0025900795590132475f,
      0.0005636486457660794f,
      8.47700794111006e-05f,
      7.708666089456528e-06f,
      3.155372496621567e-07f};
  const uint64_t w = f2_pack(fmaxf(-fabsf(a), -5.6f), fmaxf(-fabsf(b), -5.6f));
  uint64_t p = f2_pack(kGeluRw[11], kGeluRw[11]);
#pragma unroll
  for (int k = 10; k >= 0; --k) p = f2_fma(p, w, f2_pack(kGeluRw[k], kGeluRw[k]));
  const uint64_t x = f2_pack(a, b);
  float ta, tb;
  f2_unpack(f2_mul(f2_mul(x, f2_pack(-0.72134752f, -0.72134752f)), x), ta, tb);
  const uint64_t s = f2_mul(w, f2_pack(ex2_approx(ta), ex2_approx(tb)));
  f2_unpack(f2_fma(s, p, f2_pack(fmaxf(a, 0.0f), fmaxf(b, 0.0f))), a, b);
}
#endif

}  // namespace mx
