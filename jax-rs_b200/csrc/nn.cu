// nn.cu -- the nn/optim pieces of a Dense training step.
//
//   softmax per row              nn::softmax src/nn.rs:155-168 (1-D there; applied per row)
//   fused softmax + cross-entropy forward/backward
//                                nn::one_hot :205-221, nn::cross_entropy_loss :300-318
//   bias add + activation        broadcast_to src/ops/manipulation.rs:919-946, nn::relu :22-26,
//                                nn::gelu :111-122
//   activation backward, column sums (bias gradient)
//   Adam                         optim::adam_update src/optim.rs:138-189
//
// The reference has no gradient for softmax/cross-entropy or the activations
// (they are untraced).  The backward kernels are the exact derivatives of the
// reference's forward formulas, epsilon included:
//   L = -sum_k t_k ln(p_k + 1e-7) / count,  dL/dp_k = -t_k / ((p_k + 1e-7) count),
//   dL/dz_j = p_j (dL/dp_j - sum_k p_k dL/dp_k).
#include <math.h>

#include <vector>

#include "jx_common.cuh"
#include "jx_math.cuh"
#include "nn_common.cuh"

namespace {

using jxn::act_f;
using jxn::act_grad;
using jxn::label_class;
using jxn::warp_max;
using jxn::warp_sum;
using jxn::XENT_EPS;

// One warp per row.  Softmax: m = max (fold with max, order-free), e_c =
// exp(x_c - m), s = sum e_c, p_c = e_c / s.
__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ y, long long rows, int cols) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* in = x + r * cols;
    float* out = y + r * cols;
    float m = -INFINITY;
    for (int c = lane; c < cols; c += 32) m = fmaxf(m, in[c]);
    m = warp_max(m);
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) s += jxm::jx_exp(in[c] - m);
    s = warp_sum(s);
    for (int c = lane; c < cols; c += 32) out[c] = __fdiv_rn(jxm::jx_exp(in[c] - m), s);
  }
}

// Fused softmax + cross-entropy with one-hot labels, one warp per row
// (jxn::softmax_xent_row).
__global__ void softmax_xent_kernel(const float* __restrict__ logits, const float* __restrict__ labels,
                                    float* __restrict__ probs, float* __restrict__ dlogits,
                                    float* __restrict__ row_loss, long long rows, int cols, float count) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float l = jxn::softmax_xent_row(logits + r * cols, labels[r], cols, count, probs ? probs + r * cols : nullptr,
                                          dlogits ? dlogits + r * cols : nullptr, lane);
    if (lane == 0) row_loss[r] = l;
  }
}

// loss = (sum of row losses) / count, one block, fixed order.
__global__ void sum_div_kernel(const float* __restrict__ v, long long n, float count, float* __restrict__ out) {
  __shared__ float sm[32];
  float acc = 0.0f;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) acc += v[i];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.0f;
    acc = warp_sum(acc);
    if (threadIdx.x == 0) out[0] = __fdiv_rn(acc, count);
  }
}

// y = act(y + bias[c]) over [rows, cols]; pre (optional) keeps y + bias.
template <int ACT>
__global__ void bias_act_kernel(float* __restrict__ y, const float* __restrict__ bias, float* __restrict__ pre,
                                long long rows, int cols) {
  const long long n = rows * cols;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const bool vec = ((cols & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0) &&
                   (!pre || (reinterpret_cast<uintptr_t>(pre) & 15) == 0);
  if (vec) {
    const long long n4 = n >> 2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
      float4 v = reinterpret_cast<float4*>(y)[i];
      const int c = (int)((i << 2) % cols);
      const float4 b = bias ? *reinterpret_cast<const float4*>(bias + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      v.x = __fadd_rn(v.x, b.x); v.y = __fadd_rn(v.y, b.y); v.z = __fadd_rn(v.z, b.z); v.w = __fadd_rn(v.w, b.w);
      if (pre) reinterpret_cast<float4*>(pre)[i] = v;
      v.x = act_f<ACT>(v.x); v.y = act_f<ACT>(v.y); v.z = act_f<ACT>(v.z); v.w = act_f<ACT>(v.w);
      reinterpret_cast<float4*>(y)[i] = v;
    }
  } else {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
      float v = __fadd_rn(y[i], bias ? bias[i % cols] : 0.0f);
      if (pre) pre[i] = v;
      y[i] = act_f<ACT>(v);
    }
  }
}

// dz = dy * act'(pre)
template <int ACT>
__global__ void act_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ pre, float* __restrict__ dz,
                               long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    dz[i] = __fmul_rn(dy[i], act_grad<ACT>(pre[i]));
}

// Column sums of dy[rows, cols] in two deterministic passes: row chunks of
// CS rows produce partial sums (coalesced across columns), then the chunks are
// added in chunk order.
constexpr int CS = 256;
__global__ void col_partial_kernel(const float* __restrict__ dy, float* __restrict__ part, long long rows, int cols) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const long long r0 = (long long)blockIdx.y * CS;
  if (c >= cols) return;
  const long long r1 = r0 + CS < rows ? r0 + CS : rows;
  float acc = 0.0f;
  for (long long r = r0; r < r1; r += 16) {  // 16 loads in flight, added in row order
    float vals[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) vals[j] = r + j < r1 ? dy[(r + j) * cols + c] : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (r + j < r1) acc += vals[j];
  }
  part[(long long)blockIdx.y * cols + c] = acc;
}
__global__ void col_final_kernel(const float* __restrict__ part, float* __restrict__ db, int chunks, int cols) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float acc = 0.0f;
  for (int k = 0; k < chunks; ++k) acc += part[(long long)k * cols + c];
  db[c] = acc;
}

// optim::adam_update (src/optim.rs:138-189) in the reference's op order:
//   m = m*b1 + g*(1-b1)   (first step: g*(1-b1))
//   v = v*b2 + (g*g)*(1-b2)
//   p = p - (m*(1/bc1) / (sqrt(v*(1/bc2)) + eps)) * lr
// bc1 = 1 - b1^t and bc2 = 1 - b2^t come from the host (powf in f32), so every
// rounding step matches the reference: bit-identical results.
struct AdamScalars {
  float lr, b1, b2, eps, omb1, omb2, r1, r2;
  int first;
};
__global__ void adam_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                            float* __restrict__ v, long long n, const AdamScalars a) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gi = g[i];
    const float mi = a.first ? __fmul_rn(gi, a.omb1) : __fadd_rn(__fmul_rn(m[i], a.b1), __fmul_rn(gi, a.omb1));
    const float g2 = __fmul_rn(gi, gi);
    const float vi = a.first ? __fmul_rn(g2, a.omb2) : __fadd_rn(__fmul_rn(v[i], a.b2), __fmul_rn(g2, a.omb2));
    const float mh = __fmul_rn(mi, a.r1);
    const float vh = __fmul_rn(vi, a.r2);
    const float upd = __fmul_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), a.eps)), a.lr);
    p[i] = __fsub_rn(p[i], upd);
    m[i] = mi;
    v[i] = vi;
  }
}

int grid_rows(long long rows, int warps_per_block) {
  long long blocks = (rows + warps_per_block - 1) / warps_per_block;
  long long cap = (long long)jx::num_sms() * 16;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}
int grid_elems(long long n) {
  long long blocks = (n + 255) / 256;
  long long cap = (long long)jx::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

}  // namespace

namespace jx {
int col_sum(const float* dy, float* db, long long rows, int cols, cudaStream_t st) {
  const int chunks = (int)((rows + CS - 1) / CS);
  JX_REQUIRE(chunks < 65536, "col_sum: too many rows");
  void* part = nullptr;
  int rc = scratch_get(sizeof(float) * (size_t)chunks * cols, &part, st);
  if (rc) return rc;
  float* pp = reinterpret_cast<float*>(part);
  col_partial_kernel<<<dim3((cols + 255) / 256, chunks), 256, 0, st>>>(dy, pp, rows, cols);
  col_final_kernel<<<(cols + 255) / 256, 256, 0, st>>>(pp, db, chunks, cols);
  cudaError_t e = cudaGetLastError();
  scratch_release(part, st);
  if (e != cudaSuccess) return check_cuda(e, "col_sum kernels");
  return JX_OK;
}

void adam_scalars(float lr, float b1, float b2, float eps, long long step, void* out) {
  AdamScalars a;
  const float t = (float)step;
  const float bc1 = 1.0f - powf(b1, t);  // host powf: the reference computes beta.powf(t) on the host too
  const float bc2 = 1.0f - powf(b2, t);
  a.lr = lr;
  a.b1 = b1;
  a.b2 = b2;
  a.eps = eps;
  a.omb1 = 1.0f - b1;
  a.omb2 = 1.0f - b2;
  a.r1 = 1.0f / bc1;
  a.r2 = 1.0f / bc2;
  a.first = step == 1;
  *reinterpret_cast<AdamScalars*>(out) = a;
}
}  // namespace jx

extern "C" {

int jx_softmax_rows_f32(const float* x, float* y, int64_t rows, int64_t cols, jx_stream_t stream) {
  JX_TRACE("jx_softmax_rows_f32");
  JX_REQUIRE(rows >= 0 && cols >= 1 && cols < (1LL << 31), "softmax: bad size");
  if (rows == 0) return JX_OK;
  JX_REQUIRE(x && y, "softmax: NULL pointer");
  softmax_rows_kernel<<<grid_rows(rows, 8), 256, 0, jx::as_stream(stream)>>>(x, y, rows, (int)cols);
  JX_LAUNCH_CHECK("softmax_rows_kernel");
  return JX_OK;
}

int jx_softmax_xent_f32(const float* logits, const float* labels, float* probs, float* dlogits, float* loss_out,
                        int64_t rows, int64_t cols, int64_t count, jx_stream_t stream) {
  JX_TRACE("jx_softmax_xent_f32");
  JX_REQUIRE(rows >= 1 && cols >= 1 && cols < (1LL << 31), "cross_entropy: bad size");
  JX_REQUIRE(count >= 1, "cross_entropy: count must be positive");
  JX_REQUIRE(logits && labels && loss_out, "cross_entropy: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  void* rl = nullptr;
  int rc = jx::scratch_get(sizeof(float) * rows, &rl, st);
  if (rc) return rc;
  float* row_loss = reinterpret_cast<float*>(rl);
  softmax_xent_kernel<<<grid_rows(rows, 8), 256, 0, st>>>(logits, labels, probs, dlogits, row_loss, rows, (int)cols,
                                                          (float)count);
  sum_div_kernel<<<1, 1024, 0, st>>>(row_loss, rows, (float)count, loss_out);
  cudaError_t e = cudaGetLastError();
  jx::scratch_release(rl, st);
  if (e != cudaSuccess) return jx::check_cuda(e, "softmax_xent kernels");
  return JX_OK;
}

int jx_bias_act_f32(float* y, const float* bias, float* pre, int64_t rows, int64_t cols, int act, jx_stream_t stream) {
  JX_TRACE("jx_bias_act_f32");
  JX_REQUIRE(rows >= 0 && cols >= 1 && cols < (1LL << 31), "bias_act: bad size");
  JX_REQUIRE(act >= 0 && act <= 2, "bias_act: act must be 0 (none), 1 (relu) or 2 (gelu)");
  if (rows == 0) return JX_OK;
  JX_REQUIRE(y, "bias_act: NULL pointer");
  JX_REQUIRE(!bias || (reinterpret_cast<uintptr_t>(bias) & 15) == 0 || (cols & 3) != 0,
             "bias_act: bias must be 16-byte aligned");
  cudaStream_t st = jx::as_stream(stream);
  const int g = grid_elems(rows * cols / 4 + 1);
  if (act == 0) bias_act_kernel<0><<<g, 256, 0, st>>>(y, bias, pre, rows, (int)cols);
  else if (act == 1) bias_act_kernel<1><<<g, 256, 0, st>>>(y, bias, pre, rows, (int)cols);
  else bias_act_kernel<2><<<g, 256, 0, st>>>(y, bias, pre, rows, (int)cols);
  JX_LAUNCH_CHECK("bias_act_kernel");
  return JX_OK;
}

int jx_act_bwd_f32(const float* dy, const float* pre, float* dz, float* db, int64_t rows, int64_t cols, int act,
                   jx_stream_t stream) {
  JX_TRACE("jx_act_bwd_f32");
  JX_REQUIRE(rows >= 0 && cols >= 1 && cols < (1LL << 31), "act_bwd: bad size");
  JX_REQUIRE(act >= 0 && act <= 2, "act_bwd: act must be 0, 1 or 2");
  if (rows == 0) return JX_OK;
  JX_REQUIRE(dy && dz && (act == 0 || pre), "act_bwd: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  const long long n = rows * cols;
  if (act == 0) {
    if (dz != dy) JX_CUDA(cudaMemcpyAsync(dz, dy, sizeof(float) * n, cudaMemcpyDeviceToDevice, st));
  } else if (act == 1) {
    act_bwd_kernel<1><<<grid_elems(n), 256, 0, st>>>(dy, pre, dz, n);
  } else {
    act_bwd_kernel<2><<<grid_elems(n), 256, 0, st>>>(dy, pre, dz, n);
  }
  JX_LAUNCH_CHECK("act_bwd_kernel");
  if (db) return jx::col_sum(dz, db, rows, (int)cols, st);
  return JX_OK;
}

int jx_col_sum_f32(const float* dy, float* db, int64_t rows, int64_t cols, jx_stream_t stream) {
  JX_TRACE("jx_col_sum_f32");
  JX_REQUIRE(rows >= 0 && cols >= 1 && cols < (1LL << 31), "col_sum: bad size");
  JX_REQUIRE(dy && db, "col_sum: NULL pointer");
  if (rows == 0) {
    JX_CUDA(cudaMemsetAsync(db, 0, sizeof(float) * cols, jx::as_stream(stream)));
    return JX_OK;
  }
  return jx::col_sum(dy, db, rows, (int)cols, jx::as_stream(stream));
}

int jx_adam_step_f32(float* const* params, const float* const* grads, float* const* m, float* const* v,
                     const int64_t* sizes, int count, float lr, float beta1, float beta2, float eps, int64_t step,
                     jx_stream_t stream) {
  JX_TRACE("jx_adam_step_f32");
  JX_REQUIRE(count >= 0, "adam: negative tensor count");
  JX_REQUIRE(step >= 1, "adam: step must be >= 1 (the state's step after increment)");
  if (count == 0) return JX_OK;
  JX_REQUIRE(params && grads && m && v && sizes, "adam: NULL array");
  AdamScalars a;
  jx::adam_scalars(lr, beta1, beta2, eps, step, &a);
  cudaStream_t st = jx::as_stream(stream);
  for (int i = 0; i < count; ++i) {
    JX_REQUIRE(sizes[i] >= 0, "adam: tensor %d has negative size", i);
    if (sizes[i] == 0) continue;
    JX_REQUIRE(params[i] && grads[i] && m[i] && v[i], "adam: tensor %d has a NULL pointer", i);
    adam_kernel<<<grid_elems(sizes[i]), 256, 0, st>>>(params[i], grads[i], m[i], v[i], sizes[i], a);
  }
  JX_LAUNCH_CHECK("adam_kernel");
  return JX_OK;
}

}  // extern "C"
