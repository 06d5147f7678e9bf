// nn_common.cuh -- per-row and per-element pieces shared by the nn kernels
// (nn.cu) and the fused training step (mlp.cu), so both compile the same
// arithmetic and give the same bits.
#pragma once

#include <math.h>

#include "jx_common.cuh"
#include "jx_math.cuh"

namespace jxn {

constexpr float XENT_EPS = 1e-7f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// one_hot's class of a label (src/nn.rs:214-218): `idx as usize` saturates
// negatives and NaN to 0 and truncates toward zero; out-of-range classes mark nothing.
__device__ __forceinline__ long long label_class(float v) {
  if (!(v > 0.0f)) return 0;  // negative, zero, NaN
  if (v >= 9.2e18f) return 0x7fffffffffffffffLL;
  return (long long)v;
}

template <int ACT>
__device__ __forceinline__ float act_f(float x) {
  if constexpr (ACT == 1) return fmaxf(x, 0.0f);
  else if constexpr (ACT == 2) return jxm::gelu_f(x);
  else return x;
}
template <int ACT>
__device__ __forceinline__ float act_grad(float x) {
  if constexpr (ACT == 1) return x > 0.0f ? 1.0f : 0.0f;  // relu'(0) taken as 0
  else if constexpr (ACT == 2) return jxm::gelu_grad_f(x);
  else return 1.0f;
}

// Runtime activation code (0 none, 1 relu, 2 gelu).
__device__ __forceinline__ float act_apply(int act, float x) {
  return act == 1 ? act_f<1>(x) : act == 2 ? act_f<2>(x) : x;
}
__device__ __forceinline__ float act_grad_rt(int act, float x) {
  return act == 1 ? act_grad<1>(x) : act == 2 ? act_grad<2>(x) : 1.0f;
}

// Fused softmax + cross-entropy of one row, by one warp: probabilities
// (optional output), dL/dlogits (optional) with the reference's normaliser
// `count` (rows*cols for one call; the global element count when the batch is
// split across data-parallel ranks), and the row's loss contribution
// -ln(p_y + eps) (the other classes contribute -0 * ln(p + eps) = 0),
// returned on lane 0.
__device__ __forceinline__ float softmax_xent_row(const float* __restrict__ in, float label, int cols, float count,
                                                  float* __restrict__ probs_row, float* __restrict__ dl_row,
                                                  int lane) {
  const long long y = label_class(label);
  float m = -INFINITY;
  for (int c = lane; c < cols; c += 32) m = fmaxf(m, in[c]);
  m = warp_max(m);
  float s = 0.0f;
  for (int c = lane; c < cols; c += 32) s += jxm::jx_exp(in[c] - m);
  s = warp_sum(s);
  const bool has = y < cols;
  const float py = has ? __fdiv_rn(jxm::jx_exp(in[y] - m), s) : 0.0f;
  // dL/dp_y and sum_k p_k dL/dp_k (only the label term is non-zero)
  const float dpy = has ? -__fdiv_rn(1.0f, __fmul_rn(__fadd_rn(py, XENT_EPS), count)) : 0.0f;
  const float sdot = __fmul_rn(py, dpy);
  for (int c = lane; c < cols; c += 32) {
    const float p = __fdiv_rn(jxm::jx_exp(in[c] - m), s);
    if (probs_row) probs_row[c] = p;
    if (dl_row) {
      const float dp = (has && c == y) ? dpy : 0.0f;
      dl_row[c] = __fmul_rn(p, __fsub_rn(dp, sdot));
    }
  }
  return has ? -logf(__fadd_rn(py, XENT_EPS)) : 0.0f;
}

}  // namespace jxn
