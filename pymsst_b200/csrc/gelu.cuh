// GELU (exact erf form, torch.nn.GELU()) and its derivative as device
// functions, shared by the elementwise GELU passes (gelu.cu) and the GEMM
// epilogues of the fused feed-forward block (feed_forward.cu).  Internal
// linkage: every translation unit that includes this gets its own copy.
#pragma once

#include "common.cuh"

namespace pmb {
namespace {

__device__ __forceinline__ float phi_cdf(float v) { return 0.5f * (1.0f + erff(v * 0.70710678118654752f)); }
__device__ __forceinline__ float phi_pdf(float v) { return 0.39894228040143268f * expf(-0.5f * v * v); }

// 16-bit paths.  Phi(x) = 1 / (1 + 2^(-x H(x^2 / 5.5^2))) with H the degree-9
// polynomial fitted by pymsst_b200/gelu_fit.py to log2(Phi / (1 - Phi)) / x
// on [0, 5.5] (uniform relative error of the exponent, so of x Phi(x) on both
// sides of zero); beyond |x| = 5.5 Phi saturates to 0 / 1, as fp32 erf has
// already rounded to -1 / 1 there.  Two MUFU operations (ex2.approx,
// rcp.approx) and 14 FMA-pipe ones per value instead of erff's longer
// sequence, which made these passes issue-bound.  Over every finite bf16
// input the rounded GELU equals the exact one (float64) rounded; fp16 differs
// in 32 of 63488 inputs by one unit in the last place.  fp32 keeps erff.
__constant__ float kPhiH[10] = {2.302230358e+00f, 3.169386864e+00f, -3.889901191e-02f, -4.928254604e+00f,
                                1.236330509e+01f, -1.772161293e+01f, 1.614952087e+01f, -9.167760849e+00f,
                                2.937237978e+00f, -4.014779925e-01f};

__device__ __forceinline__ float ex2_approx(float v) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ float rcp_approx(float v) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ float phi_cdf_fast(float x) {
  const float t = x * x;
  const float s = t * (1.0f / 30.25f);
  float h = kPhiH[9];
#pragma unroll
  for (int i = 8; i >= 0; --i) h = fmaf(h, s, kPhiH[i]);
  h = t > 30.25f ? 1e4f : h;  // |x| > 5.5: the exponent overflows to +-inf, Phi to 0 / 1
  return rcp_approx(1.0f + ex2_approx(-x * h));
}

// phi(x) = exp(-x^2 / 2) / sqrt(2 pi) through ex2.approx
__device__ __forceinline__ float phi_pdf_fast(float x) {
  return 0.39894228040143268f * ex2_approx(x * x * -0.72134752044448170f);  // -log2(e) / 2
}

// Pairs of fp32 values in one 64-bit register for the sm_100a packed
// instructions fma / mul / add .rn.f32x2: each half is the IEEE fp32
// operation of the scalar form, rounded the same way, so the paired
// evaluation below gives the scalar functions' results bit for bit with half
// the FMA-pipe instructions (the 16-bit GELU passes are issue-bound).
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// phi_cdf_fast of two values; t = x^2 is returned for the derivative's density term
__device__ __forceinline__ void phi_cdf_fast2(float x0, float x1, float& p0, float& p1, uint64_t& t) {
  const uint64_t x = pk2(x0, x1);
  t = mul2(x, x);
  const uint64_t sc = mul2(t, pk2(1.0f / 30.25f, 1.0f / 30.25f));
  uint64_t h = pk2(kPhiH[9], kPhiH[9]);
#pragma unroll
  for (int i = 8; i >= 0; --i) h = fma2(h, sc, pk2(kPhiH[i], kPhiH[i]));
  float h0, h1, t0, t1;
  unpk2(h, h0, h1);
  unpk2(t, t0, t1);
  h0 = t0 > 30.25f ? 1e4f : h0;
  h1 = t1 > 30.25f ? 1e4f : h1;
  float a0, a1;
  unpk2(mul2(pk2(-x0, -x1), pk2(h0, h1)), a0, a1);
  float d0, d1;
  unpk2(add2(pk2(1.0f, 1.0f), pk2(ex2_approx(a0), ex2_approx(a1))), d0, d1);
  p0 = rcp_approx(d0);
  p1 = rcp_approx(d1);
}

// 16-bit path, two values at a time: Phi(x) + x phi(x)
__device__ __forceinline__ void gelu_grad_fast2(float x0, float x1, float& g0, float& g1) {
  float p0, p1;
  uint64_t t;
  phi_cdf_fast2(x0, x1, p0, p1, t);
  float u0, u1;
  unpk2(mul2(t, pk2(-0.72134752044448170f, -0.72134752044448170f)), u0, u1);  // -log2(e) / 2
  const uint64_t pdf = mul2(pk2(0.39894228040143268f, 0.39894228040143268f), pk2(ex2_approx(u0), ex2_approx(u1)));
  unpk2(fma2(pk2(x0, x1), pdf, pk2(p0, p1)), g0, g1);
}

template <typename T>
__device__ __forceinline__ float gelu_of(float v) {
  if constexpr (sizeof(T) == 2) return v * phi_cdf_fast(v);
  else return v * phi_cdf(v);
}

template <typename T>
__device__ __forceinline__ float gelu_grad_of(float v) {
  if constexpr (sizeof(T) == 2) return phi_cdf_fast(v) + v * phi_pdf_fast(v);
  else return phi_cdf(v) + v * phi_pdf(v);
}

}  // namespace
}  // namespace pmb
