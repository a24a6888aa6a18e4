// Activation functions shared by the GeGLU kernels (norm.cu) and the GEMM epilogues (gemm.cu).
#pragma once

#include "common.cuh"

namespace me {

// gelu_tanh(x) = 0.5 x (1 + tanh(y)), y = k0 (x + k1 x^3), evaluated as x * s with
// s = 0.5 (1 + tanh(y)) = 1 / (1 + e^{-2y}): one exponential and one division per element
// (and s -> 0 without cancellation for very negative x). Its derivative:
// s + x * 0.5 (1 - tanh^2 y) y' = s + 2 x s (1 - s) k0 (1 + 3 k1 x^2).
ME_DEVICE float gelu_gate(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float y = k0 * (x + k1 * x * x * x);
  return __fdividef(1.f, 1.f + __expf(-2.f * y));
}
ME_DEVICE float gelu_tanh(float x) { return x * gelu_gate(x); }
ME_DEVICE float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float s = gelu_gate(x);
  return s + 2.f * x * s * (1.f - s) * k0 * (1.f + 3.f * k1 * x * x);
}

// 2^x on the SFU (ex2.approx.ftz: relative error about 2^-22, denormal results flush to 0).
ME_DEVICE float exp2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 1/x on the SFU (rcp.approx.ftz; 1/inf = 0).
ME_DEVICE float rcp_fast(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// Final-logit softcap c * tanh(z / c), with tanh(y) = 1 - 2 / (e^{2y} + 1) evaluated on the SFU
// (one ex2, one rcp): saturates cleanly to +-c for large |z| (e^{2y} -> inf gives 1, -> 0 gives
// -1); absolute error of the result about c * 2^-21.
ME_DEVICE float softcap_fast(float z, float cap) {
  const float e = exp2_fast(z * (2.f * kLog2e) / cap);
  return cap * (1.f - 2.f * rcp_fast(e + 1.f));
}

}  // namespace me
