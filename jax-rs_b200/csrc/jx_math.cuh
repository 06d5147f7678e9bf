// jx_math.cuh -- per-element semantics of the elementwise ops, shared by the
// plain elementwise kernels and the generated op-tape kernels.
//
// Every op follows the reference's f32 operation order with explicit
// round-to-nearest intrinsics (no FMA contraction), so ops without a
// transcendental are bit-identical to jax-rs's CPU path.  exp and tanh (and
// through them sigmoid and gelu) are evaluated on the multi-function unit with
// the compensated methods below, a few ulp from glibc; log/sin/cos/pow call
// CUDA's own functions.
#pragma once

#ifndef __CUDACC_RTC__  // NVRTC builds of op-tape kernels get the JX_* codes from their prelude
#include <math.h>

#include "../../include/jaxrs_cuda.h"
#endif

namespace jxm {

constexpr float PI_F = 3.14159265358979323846f;

// --- exp / tanh on the multi-function unit ------------------------------------
// exp(x) = 2^(x*log2(e)).  hi = fl(x*L2E) goes to ex2.approx, which covers the
// whole f32 range itself (overflow to +inf, flush to zero below 2^-126, NaN
// through); the product's rounding error lo = fma(x, L2E, -hi) is applied as
// the first-order factor (1 + lo*ln2).  Relative error about 2e-7 for
// |x| <= 30 and below 1.3e-6 across the range (log2(e)'s own f32 rounding
// contributes |x|*1.3e-8).  Beyond |hi| = 128 the result is +inf or 0 and is
// returned as is (the correction would turn inf into inf - inf, and lo is NaN
// for infinite x).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float jx_exp(float x) {
  const float L2E = 1.44269502162933349609375f;  // log2(e) rounded to f32
  const float LN2 = 0.693147180559945309417f;
  const float hi = x * L2E;
  const float lo = fmaf(x, L2E, -hi);
  const float e = ex2_approx(hi);
  return fabsf(hi) < 128.0f ? fmaf(e, lo * LN2, e) : e;
}
// tanh: odd Taylor series x - x^3/3 + 2x^5/15 for |x| < 0.05 (next term below
// 5e-11 relative), else 1 - 2/(e^{2|x|} + 1) with the sign restored.  Both are
// evaluated and one is selected, so warps whose lanes fall on both sides do
// not diverge.  Absolute error about 2e-7, relative error a few ulp for
// |x| < 0.05 and above 0.5.
__device__ __forceinline__ float tanh_series(float x) {
  const float x2 = x * x;
  return fmaf(x * x2, fmaf(x2, 2.0f / 15.0f, -1.0f / 3.0f), x);
}
__device__ __forceinline__ float jx_tanh(float x) {
  const float ax = fabsf(x);
  const float e = ex2_approx(ax * 2.88539004325866699219f);  // 2|x|*log2(e); error damped by 2/(e+1)^2
  const float big = copysignf(1.0f - 2.0f * rcp_approx(e + 1.0f), x);
  return ax < 0.05f ? tanh_series(x) : big;
}

// sigmoid(x) and tanh(x) of the same x from one exponential and one
// reciprocal.  With E = exp(-|x|) in (0, 1]:
//   sigmoid(x) = (x >= 0 ? 1 : E) / (1 + E),   tanh(|x|) = (1 - E^2) / (1 + E^2),
// and both quotients share r = 1 / ((1 + E)(1 + E^2)).  For |x| < 0.05 tanh
// takes the odd series (1 - E^2 cancels there).  Used by op-tapes that apply
// both functions to one value.  E is jx_exp's compensated exponential of
// -min(|x|, 104): exp(-104) is below 2^-149 and flushes to zero, so the
// clamp changes no result, keeps the exponent finite (infinite x would make
// the correction term NaN), and min.NaN lets a NaN argument through.
__device__ __forceinline__ float min_nan(float a, float b) {
  float y;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(y) : "f"(a), "f"(b));
  return y;
}
__device__ __forceinline__ void sigmoid_tanh(float x, float& s, float& t) {
  const float L2E = 1.44269502162933349609375f;  // log2(e) rounded to f32
  const float LN2 = 0.693147180559945309417f;
  const float ax = fabsf(x);
  const float a_c = min_nan(ax, 104.0f);
  const float hi = a_c * -L2E;
  const float lo = fmaf(a_c, -L2E, -hi);
  const float e = ex2_approx(hi);
  const float E = fmaf(e, lo * LN2, e);
  const float E2 = E * E;
  const float a = 1.0f + E, b = 1.0f + E2;
  const float r = rcp_approx(a * b);
  s = (x >= 0.0f ? 1.0f : E) * b * r;
  const float big = copysignf((1.0f - E2) * a * r, x);
  t = ax < 0.05f ? tanh_series(x) : big;
}

// CUDA's accurate functions for the ops off the hot path, kept out of line so
// the op-tape interpreter's cases stay small.
static __device__ __noinline__ float jx_logf(float x) { return logf(x); }
static __device__ __noinline__ float jx_sinf(float x) { return sinf(x); }
static __device__ __noinline__ float jx_cosf(float x) { return cosf(x); }
static __device__ __noinline__ float jx_powf(float a, float b) { return powf(a, b); }
// The remaining unary methods (src/ops/unary.rs:82-541), CUDA's functions;
// the rounding family and sign are exact.
static __device__ __noinline__ float jx_unary_more(int op, float x) {
  switch (op) {
    case JX_UN_TAN: return tanf(x);
    case JX_UN_SINH: return sinhf(x);
    case JX_UN_COSH: return coshf(x);
    case JX_UN_ASIN: return asinf(x);
    case JX_UN_ACOS: return acosf(x);
    case JX_UN_ATAN: return atanf(x);
    case JX_UN_ASINH: return asinhf(x);
    case JX_UN_ACOSH: return acoshf(x);
    case JX_UN_ATANH: return atanhf(x);
    case JX_UN_EXPM1: return expm1f(x);
    case JX_UN_LOG1P: return log1pf(x);
    case JX_UN_CBRT: return cbrtf(x);
    default: return log2f(x);
  }
}
// Array::sign (src/ops/unary.rs:117-127): 1, -1, else 0 (NaN gives 0 too).
__device__ __forceinline__ float sign_f(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

// nn::gelu (src/nn.rs:111-122): coeff = sqrt(2/pi); inner = coeff*(v + 0.044715*v^3);
// 0.5*v*(1 + tanh(inner)).  coeff is the f32 value of sqrtf(2.0f / PI)
// (0x3f4c4229), as the reference computes it per element.  The identity
// 0.5*(1 + tanh(z)) = 1/(1 + e^{-2z}) takes one exponential and one
// reciprocal instead of tanh's two paths, and the exponent -2*inner*log2(e)
// is formed as v*(K + KC1*v^2) with K = fl(-2*log2(e)*coeff) and
// KC1 = fl(K*0.044715) (one multiply, one FMA, one multiply).  That argument
// is within a few ulp of the reference's rounded inner times -2*log2(e); the
// relative error it puts on e, |arg|*ln2*2.4e-7, matters only while
// 1/(1 + e) is not negligible, and the result stays within 2e-6 relative
// (3e-7 absolute near zero) of the reference's evaluation.  Large negative v
// gives -0 or a tiny negative value as in the reference.
__device__ __forceinline__ float gelu_coeff() { return __int_as_float(0x3f4c4229); }
__device__ __forceinline__ float gelu_k() { return __int_as_float(0xc0135760); }    // fl(-2*fl(log2 e)*coeff)
__device__ __forceinline__ float gelu_kc1() { return __int_as_float(0xbdd2d3e6); }  // fl(K*0.044715)
__device__ __forceinline__ float gelu_c3() { return __int_as_float(0x3ddb33b5); }   // fl(3*0.044715*coeff)
// log2 of e^{-2 inner(v)}
__device__ __forceinline__ float gelu_arg(float v, float v2) { return __fmul_rn(v, fmaf(v2, gelu_kc1(), gelu_k())); }
__device__ __forceinline__ float gelu_f(float v) {
  const float e = ex2_approx(gelu_arg(v, __fmul_rn(v, v)));
  return v * rcp_approx(1.0f + e);
}

// d/du of gelu_f (restated adjoint; the reference leaves gelu untraced):
// 0.5*(1+t) + 0.5*u*(1-t^2)*dinner with t = tanh(inner),
// dinner = coeff*(1 + 3*0.044715*u^2) = coeff + C3*u^2.  With s = 0.5*(1+t)
// = 1/(1+e), e = e^{-2 inner}: 0.5*(1 - t^2) = 2 s (1 - s), and 1 - s = e*s
// without cancellation while e <= 1 (1 - s is exact enough above that,
// s <= 1/2).  gelu_pair returns gelu_f and gelu_grad_f of one u from one
// exponential and one reciprocal (op-tapes that apply both to one value).
__device__ __forceinline__ void gelu_pair(float u, float& g, float& dg) {
  const float u2 = __fmul_rn(u, u);
  const float e = ex2_approx(gelu_arg(u, u2));
  const float s = rcp_approx(1.0f + e);
  const float oms = e <= 1.0f ? e * s : 1.0f - s;
  const float dinner = fmaf(u2, gelu_c3(), gelu_coeff());
  g = u * s;
  dg = s + 2.0f * u * s * oms * dinner;
}
__device__ __forceinline__ float gelu_grad_f(float u) {
  float g, dg;
  gelu_pair(u, g, dg);
  return dg;
}

// nn::sigmoid (src/nn.rs:135-140): 1 / (1 + exp(-v))
__device__ __forceinline__ float sigmoid_f(float v) { return rcp_approx(1.0f + jx_exp(-v)); }

template <int OP>
__device__ __forceinline__ float unary_t(float x) {
  if constexpr (OP == JX_UN_NEG) return -x;
  else if constexpr (OP == JX_UN_ABS) return fabsf(x);
  else if constexpr (OP == JX_UN_SIN) return jx_sinf(x);
  else if constexpr (OP == JX_UN_COS) return jx_cosf(x);
  else if constexpr (OP == JX_UN_TANH) return jx_tanh(x);
  else if constexpr (OP == JX_UN_EXP) return jx_exp(x);
  else if constexpr (OP == JX_UN_LOG) return jx_logf(x);
  else if constexpr (OP == JX_UN_SQRT) return __fsqrt_rn(x);
  else if constexpr (OP == JX_UN_RECIP) return __fdiv_rn(1.0f, x);
  else if constexpr (OP == JX_UN_SQUARE) return __fmul_rn(x, x);
  else if constexpr (OP == JX_UN_RELU) return fmaxf(x, 0.0f);  // Rust f32::max ignores NaN like fmaxf
  else if constexpr (OP == JX_UN_GELU) return gelu_f(x);
  else if constexpr (OP == JX_UN_SIGMOID) return sigmoid_f(x);
  else if constexpr (OP == JX_UN_GELU_GRAD) return gelu_grad_f(x);
  else if constexpr (OP == JX_UN_SIGN) return sign_f(x);
  else if constexpr (OP == JX_UN_CEIL) return ceilf(x);
  else if constexpr (OP == JX_UN_FLOOR) return floorf(x);
  else if constexpr (OP == JX_UN_ROUND) return roundf(x);  // half away from zero, as f32::round
  else if constexpr (OP == JX_UN_TRUNC) return truncf(x);
  else if constexpr (OP >= JX_UN_TAN && OP <= JX_UN_LOG2) return jx_unary_more(OP, x);
  else return x;
}

// Binary ops; JX_BIN_SELECT_GT (7) is the tape's mask op: a > 0 ? b : 0.
template <int OP>
__device__ __forceinline__ float binary_t(float a, float b) {
  if constexpr (OP == JX_BIN_ADD) return __fadd_rn(a, b);
  else if constexpr (OP == JX_BIN_SUB) return __fsub_rn(a, b);
  else if constexpr (OP == JX_BIN_MUL) return __fmul_rn(a, b);
  else if constexpr (OP == JX_BIN_DIV) return __fdiv_rn(a, b);
  else if constexpr (OP == JX_BIN_POW) return jx_powf(a, b);
  else if constexpr (OP == JX_BIN_MIN) return fminf(a, b);
  else if constexpr (OP == JX_BIN_MAX) return fmaxf(a, b);
  else return a > 0.0f ? b : 0.0f;
}

__device__ __forceinline__ float unary_f(int op, float x) {
  switch (op) {
    case JX_UN_NEG: return unary_t<JX_UN_NEG>(x);
    case JX_UN_ABS: return unary_t<JX_UN_ABS>(x);
    case JX_UN_SIN: return unary_t<JX_UN_SIN>(x);
    case JX_UN_COS: return unary_t<JX_UN_COS>(x);
    case JX_UN_TANH: return unary_t<JX_UN_TANH>(x);
    case JX_UN_EXP: return unary_t<JX_UN_EXP>(x);
    case JX_UN_LOG: return unary_t<JX_UN_LOG>(x);
    case JX_UN_SQRT: return unary_t<JX_UN_SQRT>(x);
    case JX_UN_RECIP: return unary_t<JX_UN_RECIP>(x);
    case JX_UN_SQUARE: return unary_t<JX_UN_SQUARE>(x);
    case JX_UN_RELU: return unary_t<JX_UN_RELU>(x);
    case JX_UN_GELU: return unary_t<JX_UN_GELU>(x);
    case JX_UN_SIGMOID: return unary_t<JX_UN_SIGMOID>(x);
    case JX_UN_GELU_GRAD: return unary_t<JX_UN_GELU_GRAD>(x);
    case JX_UN_SIGN: return unary_t<JX_UN_SIGN>(x);
    case JX_UN_CEIL: return unary_t<JX_UN_CEIL>(x);
    case JX_UN_FLOOR: return unary_t<JX_UN_FLOOR>(x);
    case JX_UN_ROUND: return unary_t<JX_UN_ROUND>(x);
    case JX_UN_TRUNC: return unary_t<JX_UN_TRUNC>(x);
    default:
      if (op >= JX_UN_TAN && op <= JX_UN_LOG2) return jx_unary_more(op, x);
      return x;
  }
}

__device__ __forceinline__ float binary_f(int op, float a, float b) {
  switch (op) {
    case JX_BIN_ADD: return binary_t<JX_BIN_ADD>(a, b);
    case JX_BIN_SUB: return binary_t<JX_BIN_SUB>(a, b);
    case JX_BIN_MUL: return binary_t<JX_BIN_MUL>(a, b);
    case JX_BIN_DIV: return binary_t<JX_BIN_DIV>(a, b);
    case JX_BIN_POW: return binary_t<JX_BIN_POW>(a, b);
    case JX_BIN_MIN: return binary_t<JX_BIN_MIN>(a, b);
    case JX_BIN_MAX: return binary_t<JX_BIN_MAX>(a, b);
    default: return binary_t<7>(a, b);
  }
}

}  // namespace jxm
