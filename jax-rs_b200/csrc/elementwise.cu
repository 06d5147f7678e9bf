// elementwise.cu -- broadcasting binary ops and unary ops.
//
// Replaces gpu_binary_op (src/backend/ops.rs:21-149, same-shape only) with a
// broadcasting kernel (binary_op src/ops/binary.rs:7-74, broadcast_index
// :134-168), and the CPU-only unary_op (src/ops/unary.rs:30-49) and nn
// activations (src/nn.rs:22-26,111-140) with device kernels.  Per-element
// semantics live in jx_math.cuh (shared with the op-tape in tape.cu).
#include <string.h>

#include "jx_common.cuh"
#include "jx_math.cuh"

namespace {

using jxm::binary_f;
using jxm::unary_f;

// --- plain kernels --------------------------------------------------------------
__global__ void unary_kernel(int op, const float* __restrict__ x, float* __restrict__ y, long long n, int vec_ok) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  if (vec_ok) {
    const long long n4 = n / 4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
      float4 q = reinterpret_cast<const float4*>(x)[i];
      q.x = unary_f(op, q.x); q.y = unary_f(op, q.y); q.z = unary_f(op, q.z); q.w = unary_f(op, q.w);
      reinterpret_cast<float4*>(y)[i] = q;
    }
    for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
      y[i] = unary_f(op, x[i]);
  } else {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) y[i] = unary_f(op, x[i]);
  }
}

constexpr int BMAX_DIMS = 8;
struct BroadcastArgs {
  int nd;
  long long n;
  long long out_dims[BMAX_DIMS];
  long long sa[BMAX_DIMS];  // element strides of a in output index space (0 = broadcast)
  long long sb[BMAX_DIMS];
};

__global__ void binary_bcast_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                                    float* __restrict__ out, const __grid_constant__ BroadcastArgs g) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < g.n; i += stride) {
    long long rem = i, ia = 0, ib = 0;
    for (int d = g.nd - 1; d >= 0; --d) {
      const long long idx = rem % g.out_dims[d];
      rem /= g.out_dims[d];
      ia += idx * g.sa[d];
      ib += idx * g.sb[d];
    }
    out[i] = binary_f(op, a[ia], b[ib]);
  }
}

__global__ void binary_same_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                                   float* __restrict__ out, long long n, int vec_ok) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  if (vec_ok) {
    const long long n4 = n / 4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
      float4 p = reinterpret_cast<const float4*>(a)[i], q = reinterpret_cast<const float4*>(b)[i];
      reinterpret_cast<float4*>(out)[i] =
          make_float4(binary_f(op, p.x, q.x), binary_f(op, p.y, q.y), binary_f(op, p.z, q.z), binary_f(op, p.w, q.w));
    }
    for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
      out[i] = binary_f(op, a[i], b[i]);
  } else {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
      out[i] = binary_f(op, a[i], b[i]);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int grid_for(long long work, int threads) {
  long long blocks = (work + threads - 1) / threads;
  long long cap = (long long)jx::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

}  // namespace

extern "C" {

int jx_unary_f32(int op, const float* x, float* y, int64_t n, jx_stream_t stream) {
  JX_TRACE("jx_unary_f32");
  JX_REQUIRE(op >= 0 && op <= JX_UN_LOG2, "unary: unknown op %d", op);
  JX_REQUIRE(n >= 0, "unary: negative size");
  if (n == 0) return JX_OK;
  JX_REQUIRE(x && y, "unary: NULL pointer");
  unary_kernel<<<grid_for((n + 3) / 4, 256), 256, 0, jx::as_stream(stream)>>>(op, x, y, n,
                                                                              aligned16(x) && aligned16(y));
  JX_LAUNCH_CHECK("unary_kernel");
  return JX_OK;
}

int jx_binary_f32(int op, const float* a, const int64_t* a_shape, int a_ndim, const float* b, const int64_t* b_shape,
                  int b_ndim, float* out, jx_stream_t stream) {
  JX_TRACE("jx_binary_f32");
  JX_REQUIRE(op >= 0 && op <= JX_BIN_MAX, "binary: unknown op %d", op);
  JX_REQUIRE(a_ndim >= 0 && a_ndim <= BMAX_DIMS && b_ndim >= 0 && b_ndim <= BMAX_DIMS, "binary: rank > %d",
             BMAX_DIMS);
  JX_REQUIRE((a_ndim == 0 || a_shape) && (b_ndim == 0 || b_shape), "binary: NULL shape");
  const int nd = a_ndim > b_ndim ? a_ndim : b_ndim;
  BroadcastArgs g;
  memset(&g, 0, sizeof(g));
  g.nd = nd;
  long long total = 1;
  bool same = a_ndim == b_ndim;
  // NumPy broadcasting (src/shape.rs:87-113): align trailing dims.
  long long stride_a = 1, stride_b = 1;
  for (int d = nd - 1; d >= 0; --d) {
    const int ia = d - (nd - a_ndim), ib = d - (nd - b_ndim);
    const long long da = ia >= 0 ? a_shape[ia] : 1, db = ib >= 0 ? b_shape[ib] : 1;
    JX_REQUIRE(da >= 0 && db >= 0, "binary: negative dimension");
    if (da != db && da != 1 && db != 1)
      return jx::fail(JX_EINVAL, "Shapes are not broadcast-compatible (dim %d: %lld vs %lld)", d, da, db);
    if (da != db) same = false;
    const long long od = da == 1 ? db : da;
    g.out_dims[d] = od;
    g.sa[d] = (da == 1) ? 0 : stride_a;
    g.sb[d] = (db == 1) ? 0 : stride_b;
    stride_a *= da;
    stride_b *= db;
    total *= od;
  }
  g.n = total;
  if (total == 0) return JX_OK;
  JX_REQUIRE(a && b && out, "binary: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  if (same) {
    binary_same_kernel<<<grid_for((total + 3) / 4, 256), 256, 0, st>>>(op, a, b, out, total,
                                                                       aligned16(a) && aligned16(b) && aligned16(out));
  } else {
    binary_bcast_kernel<<<grid_for(total, 256), 256, 0, st>>>(op, a, b, out, g);
  }
  JX_LAUNCH_CHECK("binary kernel");
  return JX_OK;
}

}  // extern "C"
