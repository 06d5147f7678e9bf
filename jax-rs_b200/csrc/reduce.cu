// reduce.cu -- reductions and their VJPs.
//
// Replaces gpu_reduce_all (src/backend/ops.rs:639-787, two passes whose second
// pass is one 256-wide workgroup, wrong for n > 65536) and the CPU-only
// reduce_axis (src/ops/reduce.rs:53-135), argmax/argmin (:281-309) and the
// grad rules transpose_sum_axis / transpose_max_all
// (src/trace/transpose_rules.rs:409-418, 444-469).
//
// HBM-bound: 128-bit loads, several loads in flight per thread, warp shuffles
// then shared memory.  Sums are tree-ordered (not the reference's sequential
// fold), max/min/argmax are order-independent and bit-exact.
#include <float.h>
#include <math.h>

#include "jx_common.cuh"

namespace {

__device__ __forceinline__ float red_init(int op) {
  return op == JX_RED_SUM ? 0.0f : op == JX_RED_MAX ? -INFINITY : op == JX_RED_MIN ? INFINITY : 1.0f;
}
__device__ __forceinline__ float red_f(int op, float a, float x) {
  // Rust f32::max/min ignore a NaN operand, like fmaxf/fminf.
  return op == JX_RED_SUM ? a + x : op == JX_RED_MAX ? fmaxf(a, x) : op == JX_RED_MIN ? fminf(a, x) : a * x;
}
__device__ __forceinline__ float warp_red(int op, float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = red_f(op, v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp per row of a [rows, cols] array (inner == 1).
template <int OP>
__global__ void __launch_bounds__(256) reduce_rows_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                          long long rows, int cols) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const bool vec = ((cols & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* row = x + r * cols;
    float acc = red_init(OP);
    if (vec) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      const int n4 = cols >> 2;
      int i = lane;
      for (; i + 96 < n4; i += 128) {
        float4 a = __ldcs(r4 + i), b = __ldcs(r4 + i + 32), c = __ldcs(r4 + i + 64), d = __ldcs(r4 + i + 96);
        float s0 = red_f(OP, red_f(OP, a.x, a.y), red_f(OP, a.z, a.w));
        float s1 = red_f(OP, red_f(OP, b.x, b.y), red_f(OP, b.z, b.w));
        float s2 = red_f(OP, red_f(OP, c.x, c.y), red_f(OP, c.z, c.w));
        float s3 = red_f(OP, red_f(OP, d.x, d.y), red_f(OP, d.z, d.w));
        acc = red_f(OP, acc, red_f(OP, red_f(OP, s0, s1), red_f(OP, s2, s3)));
      }
      for (; i < n4; i += 32) {
        float4 a = __ldcs(r4 + i);
        acc = red_f(OP, acc, red_f(OP, red_f(OP, a.x, a.y), red_f(OP, a.z, a.w)));
      }
    } else {
      for (int i = lane; i < cols; i += 32) acc = red_f(OP, acc, row[i]);
    }
    acc = warp_red(OP, acc);
    if (lane == 0) out[r] = acc;
  }
}

// x viewed as [outer, len, inner] with inner > 1: one thread per (outer, inner)
// output, coalesced across inner.
__global__ void reduce_strided_kernel(const float* __restrict__ x, float* __restrict__ out, long long outer,
                                      long long len, long long inner, int op) {
  const long long total = outer * inner;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long o = t / inner, in = t - o * inner;
    const float* p = x + o * len * inner + in;
    float acc = red_init(op);
    for (long long a = 0; a < len; ++a) acc = red_f(op, acc, p[a * inner]);
    out[t] = acc;
  }
}

// Full reduction, pass 1: grid-stride partials; pass 2: one block folds them.
template <int OP>
__global__ void __launch_bounds__(512) reduce_all_pass1(const float* __restrict__ x, float* __restrict__ part,
                                                        long long n) {
  __shared__ float sm[32];
  float acc = red_init(OP);
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  long long tail = 0;
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const long long n4 = n >> 2;
    long long i = tid;
    for (; i + 3 * stride < n4; i += 4 * stride) {
      float4 a = __ldcs(x4 + i), b = __ldcs(x4 + i + stride), c = __ldcs(x4 + i + 2 * stride),
             d = __ldcs(x4 + i + 3 * stride);
      float s0 = red_f(OP, red_f(OP, a.x, a.y), red_f(OP, a.z, a.w));
      float s1 = red_f(OP, red_f(OP, b.x, b.y), red_f(OP, b.z, b.w));
      float s2 = red_f(OP, red_f(OP, c.x, c.y), red_f(OP, c.z, c.w));
      float s3 = red_f(OP, red_f(OP, d.x, d.y), red_f(OP, d.z, d.w));
      acc = red_f(OP, acc, red_f(OP, red_f(OP, s0, s1), red_f(OP, s2, s3)));
    }
    for (; i < n4; i += stride) {
      float4 a = __ldcs(x4 + i);
      acc = red_f(OP, acc, red_f(OP, red_f(OP, a.x, a.y), red_f(OP, a.z, a.w)));
    }
    tail = n4 << 2;
  }
  for (long long i = tail + tid; i < n; i += stride) acc = red_f(OP, acc, x[i]);
  acc = warp_red(OP, acc);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sm[w] = acc;
  __syncthreads();
  if (w == 0) {
    acc = l < (blockDim.x >> 5) ? sm[l] : red_init(OP);
    acc = warp_red(OP, acc);
    if (l == 0) part[blockIdx.x] = acc;
  }
}

__global__ void reduce_all_pass2(const float* __restrict__ part, float* __restrict__ out, int n, int op) {
  __shared__ float sm[32];
  float acc = red_init(op);
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc = red_f(op, acc, part[i]);
  acc = warp_red(op, acc);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sm[w] = acc;
  __syncthreads();
  if (w == 0) {
    acc = l < (blockDim.x >> 5) ? sm[l] : red_init(op);
    acc = warp_red(op, acc);
    if (l == 0) out[0] = acc;
  }
}

// Per-row argmax/argmin.  Candidate order: argmax prefers the larger value,
// then the LARGER index (max_by keeps the last maximum); argmin prefers the
// smaller value, then the SMALLER index (min_by keeps the first minimum).
template <bool IS_MAX>
__device__ __forceinline__ void arg_merge(float& v, int& i, float v2, int i2) {
  if (IS_MAX) {
    if (v2 > v || (v2 == v && i2 > i)) { v = v2; i = i2; }
  } else {
    if (v2 < v || (v2 == v && i2 < i)) { v = v2; i = i2; }
  }
}

template <bool IS_MAX>
__global__ void __launch_bounds__(256) argreduce_rows_kernel(const float* __restrict__ x, int32_t* __restrict__ idx,
                                                             float* __restrict__ val, long long rows, int cols,
                                                             unsigned int* err) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const bool vec = ((cols & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* row = x + r * cols;
    float bv = IS_MAX ? -INFINITY : INFINITY;
    int bi = IS_MAX ? -1 : 0x7fffffff;
    bool nan = false;
    if (vec) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      for (int i = lane; i < (cols >> 2); i += 32) {
        float4 a = __ldcs(r4 + i);
        const int c = i << 2;
        nan |= (a.x != a.x) | (a.y != a.y) | (a.z != a.z) | (a.w != a.w);
        arg_merge<IS_MAX>(bv, bi, a.x, c);
        arg_merge<IS_MAX>(bv, bi, a.y, c + 1);
        arg_merge<IS_MAX>(bv, bi, a.z, c + 2);
        arg_merge<IS_MAX>(bv, bi, a.w, c + 3);
      }
    } else {
      for (int c = lane; c < cols; c += 32) {
        const float a = row[c];
        nan |= (a != a);
        arg_merge<IS_MAX>(bv, bi, a, c);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      arg_merge<IS_MAX>(bv, bi, v2, i2);
    }
    nan = __any_sync(0xffffffffu, nan);
    if (lane == 0) {
      if (nan) atomicOr(err, JX_DEVERR_NAN);
      // A row of all +-inf ties on the sentinel; the reference's fold then keeps
      // index cols-1 (argmax) or 0 (argmin).
      if (bi < 0 || bi >= cols) bi = IS_MAX ? cols - 1 : 0;
      idx[r] = bi;
      if (val) val[r] = row[bi];
    }
  }
}

__global__ void sum_rows_vjp_kernel(const float* __restrict__ ct, float* __restrict__ dx, long long rows, int cols) {
  // dx[r, c] = ct[r]: one 128-bit store per thread when aligned.
  const bool vec = ((cols & 3) == 0) && ((reinterpret_cast<uintptr_t>(dx) & 15) == 0);
  const long long stride = (long long)gridDim.x * blockDim.x;
  if (vec) {
    const long long c4 = cols >> 2, total = rows * c4;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total; t += stride) {
      const float v = __ldg(ct + t / c4);
      __stcs(reinterpret_cast<float4*>(dx) + t, make_float4(v, v, v, v));
    }
  } else {
    const long long total = rows * cols;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total; t += stride)
      dx[t] = ct[t / cols];
  }
}

// transpose_max_all applied per row: mask = (x == max); count = sum(mask);
// scale = count > 1 ? 1/count : 1; dx = mask*scale*ct.  One warp per row: the
// row is read twice (max+count, then write), the second read hits L2.
__global__ void __launch_bounds__(256) max_rows_vjp_kernel(const float* __restrict__ x, const float* __restrict__ ct,
                                                           float* __restrict__ dx, long long rows, int cols) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const bool vec = ((cols & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(dx) & 15) == 0);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* row = x + r * cols;
    float* drow = dx + r * cols;
    float m = -INFINITY;
    if (vec) {
      for (int i = lane; i < (cols >> 2); i += 32) {
        float4 a = reinterpret_cast<const float4*>(row)[i];
        m = fmaxf(m, fmaxf(fmaxf(a.x, a.y), fmaxf(a.z, a.w)));
      }
    } else {
      for (int c = lane; c < cols; c += 32) m = fmaxf(m, row[c]);
    }
    m = warp_red(JX_RED_MAX, m);
    int cnt = 0;
    for (int c = lane; c < cols; c += 32) cnt += (row[c] == m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    const float count = (float)cnt;  // exact: counts < 2^24
    const float g = ct[r];
    const float scale = count > 1.0f ? __fdiv_rn(1.0f, count) : 1.0f;
    if (vec) {
      for (int i = lane; i < (cols >> 2); i += 32) {
        float4 a = __ldcs(reinterpret_cast<const float4*>(row) + i);
        float4 o;
        o.x = __fmul_rn((a.x == m) ? (count > 1.0f ? scale : 1.0f) : 0.0f, g);
        o.y = __fmul_rn((a.y == m) ? (count > 1.0f ? scale : 1.0f) : 0.0f, g);
        o.z = __fmul_rn((a.z == m) ? (count > 1.0f ? scale : 1.0f) : 0.0f, g);
        o.w = __fmul_rn((a.w == m) ? (count > 1.0f ? scale : 1.0f) : 0.0f, g);
        __stcs(reinterpret_cast<float4*>(drow) + i, o);
      }
    } else {
      for (int c = lane; c < cols; c += 32)
        drow[c] = __fmul_rn((row[c] == m) ? (count > 1.0f ? scale : 1.0f) : 0.0f, g);
    }
  }
}

// Rows of up to 8192 floats (a multiple of 4, 16-byte aligned): one block
// per row, the row held in registers (V4 float4 per thread), so it is read
// once: block max, block count of the maxima, then the write.
template <int V4>
__global__ void __launch_bounds__(256) max_rows_vjp_reg_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ ct, float* __restrict__ dx,
                                                               long long rows, int cols) {
  __shared__ float sm_max[8];
  __shared__ int sm_cnt[8];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c4 = cols >> 2;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const float4* row = reinterpret_cast<const float4*>(x + r * cols);
    float4 v[V4];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < V4; ++k) {
      const int i = threadIdx.x + 256 * k;
      v[k] = i < c4 ? __ldcs(row + i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
    }
    m = warp_red(JX_RED_MAX, m);
    if (lane == 0) sm_max[w] = m;
    __syncthreads();
    m = sm_max[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, sm_max[i]);
    int cnt = 0;
#pragma unroll
    for (int k = 0; k < V4; ++k)
      if (threadIdx.x + 256 * k < c4) cnt += (v[k].x == m) + (v[k].y == m) + (v[k].z == m) + (v[k].w == m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) sm_cnt[w] = cnt;
    __syncthreads();
    cnt = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) cnt += sm_cnt[i];
    const float count = (float)cnt;  // exact: counts < 2^24
    const float g = ct[r];
    const float hit = count > 1.0f ? __fdiv_rn(1.0f, count) : 1.0f;
    float4* drow = reinterpret_cast<float4*>(dx + r * cols);
#pragma unroll
    for (int k = 0; k < V4; ++k) {
      const int i = threadIdx.x + 256 * k;
      if (i < c4) {
        float4 o;
        o.x = __fmul_rn(v[k].x == m ? hit : 0.0f, g);
        o.y = __fmul_rn(v[k].y == m ? hit : 0.0f, g);
        o.z = __fmul_rn(v[k].z == m ? hit : 0.0f, g);
        o.w = __fmul_rn(v[k].w == m ? hit : 0.0f, g);
        __stcs(drow + i, o);
      }
    }
    __syncthreads();  // sm_max / sm_cnt are reused by the next row
  }
}

int grid_rows(long long rows, int warps_per_block) {
  long long blocks = (rows + warps_per_block - 1) / warps_per_block;
  long long cap = (long long)jx::num_sms() * 16;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

}  // namespace

extern "C" {

int jx_reduce_all_f32(const float* x, float* out, int64_t n, int op, jx_stream_t stream) {
  JX_TRACE("jx_reduce_all_f32");
  JX_REQUIRE(op >= JX_RED_SUM && op <= JX_RED_PROD, "reduce: unknown op %d", op);
  JX_REQUIRE(n >= 0, "reduce: negative size");
  JX_REQUIRE(out && (n == 0 || x), "reduce: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  const int threads = 512;
  long long blocks = (n / 4 + threads - 1) / threads;
  const long long cap = (long long)jx::num_sms() * 4;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  void* part = nullptr;
  int rc = jx::scratch_get(sizeof(float) * blocks, &part, st);
  if (rc) return rc;
  float* p = reinterpret_cast<float*>(part);
  switch (op) {
    case JX_RED_SUM: reduce_all_pass1<JX_RED_SUM><<<(int)blocks, threads, 0, st>>>(x, p, n); break;
    case JX_RED_MAX: reduce_all_pass1<JX_RED_MAX><<<(int)blocks, threads, 0, st>>>(x, p, n); break;
    case JX_RED_MIN: reduce_all_pass1<JX_RED_MIN><<<(int)blocks, threads, 0, st>>>(x, p, n); break;
    default: reduce_all_pass1<JX_RED_PROD><<<(int)blocks, threads, 0, st>>>(x, p, n); break;
  }
  reduce_all_pass2<<<1, 1024, 0, st>>>(p, out, (int)blocks, op);
  cudaError_t e = cudaGetLastError();
  jx::scratch_release(part, st);
  if (e != cudaSuccess) return jx::check_cuda(e, "reduce_all kernels");
  return JX_OK;
}

int jx_reduce_axis_f32(const float* x, float* out, int64_t outer, int64_t len, int64_t inner, int op,
                       jx_stream_t stream) {
  JX_TRACE("jx_reduce_axis_f32");
  JX_REQUIRE(op >= JX_RED_SUM && op <= JX_RED_PROD, "reduce: unknown op %d", op);
  JX_REQUIRE(outer >= 0 && len >= 0 && inner >= 0, "reduce: negative size");
  if (outer == 0 || inner == 0) return JX_OK;
  JX_REQUIRE(x && out, "reduce: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  if (inner == 1 && len > 0 && len < (1LL << 31)) {
    const int g = grid_rows(outer, 8);
    switch (op) {
      case JX_RED_SUM: reduce_rows_kernel<JX_RED_SUM><<<g, 256, 0, st>>>(x, out, outer, (int)len); break;
      case JX_RED_MAX: reduce_rows_kernel<JX_RED_MAX><<<g, 256, 0, st>>>(x, out, outer, (int)len); break;
      case JX_RED_MIN: reduce_rows_kernel<JX_RED_MIN><<<g, 256, 0, st>>>(x, out, outer, (int)len); break;
      default: reduce_rows_kernel<JX_RED_PROD><<<g, 256, 0, st>>>(x, out, outer, (int)len); break;
    }
  } else {
    long long total = outer * inner;
    long long blocks = (total + 255) / 256;
    if (blocks > (long long)jx::num_sms() * 16) blocks = (long long)jx::num_sms() * 16;
    reduce_strided_kernel<<<(int)blocks, 256, 0, st>>>(x, out, outer, len, inner, op);
  }
  JX_LAUNCH_CHECK("reduce_axis kernel");
  return JX_OK;
}

int jx_argreduce_rows_f32(const float* x, int32_t* out_idx, float* out_val, int64_t rows, int64_t cols, int is_max,
                          jx_stream_t stream) {
  JX_TRACE("jx_argreduce_rows_f32");
  JX_REQUIRE(rows >= 0, "argreduce: negative rows");
  JX_REQUIRE(cols >= 1 && cols < (1LL << 31), "argreduce: cols must be in [1, 2^31)");
  if (rows == 0) return JX_OK;
  JX_REQUIRE(x && out_idx, "argreduce: NULL pointer");
  unsigned int* err = jx::device_error_word();
  JX_REQUIRE(err, "argreduce: device not initialised (call jx_init)");
  cudaStream_t st = jx::as_stream(stream);
  const int g = grid_rows(rows, 8);
  if (is_max)
    argreduce_rows_kernel<true><<<g, 256, 0, st>>>(x, out_idx, out_val, rows, (int)cols, err);
  else
    argreduce_rows_kernel<false><<<g, 256, 0, st>>>(x, out_idx, out_val, rows, (int)cols, err);
  JX_LAUNCH_CHECK("argreduce_rows_kernel");
  return JX_OK;
}

int jx_sum_rows_vjp_f32(const float* ct, float* dx, int64_t rows, int64_t cols, jx_stream_t stream) {
  JX_TRACE("jx_sum_rows_vjp_f32");
  JX_REQUIRE(rows >= 0 && cols >= 0 && cols < (1LL << 31), "sum vjp: bad size");
  if (rows == 0 || cols == 0) return JX_OK;
  JX_REQUIRE(ct && dx, "sum vjp: NULL pointer");
  long long total = rows * cols / 4 + 1;
  long long blocks = (total + 255) / 256;
  if (blocks > (long long)jx::num_sms() * 16) blocks = (long long)jx::num_sms() * 16;
  sum_rows_vjp_kernel<<<(int)blocks, 256, 0, jx::as_stream(stream)>>>(ct, dx, rows, (int)cols);
  JX_LAUNCH_CHECK("sum_rows_vjp_kernel");
  return JX_OK;
}

int jx_max_rows_vjp_f32(const float* x, const float* ct, float* dx, int64_t rows, int64_t cols, jx_stream_t stream) {
  JX_TRACE("jx_max_rows_vjp_f32");
  JX_REQUIRE(rows >= 0 && cols >= 1 && cols < (1LL << 31), "max vjp: bad size");
  if (rows == 0) return JX_OK;
  JX_REQUIRE(x && ct && dx, "max vjp: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  const bool vec = (cols & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(dx) & 15) == 0;
  const int blocks = (int)std::min<long long>(rows, (long long)jx::num_sms() * 8);
  if (vec && cols <= 1024)
    max_rows_vjp_reg_kernel<1><<<blocks, 256, 0, st>>>(x, ct, dx, rows, (int)cols);
  else if (vec && cols <= 2048)
    max_rows_vjp_reg_kernel<2><<<blocks, 256, 0, st>>>(x, ct, dx, rows, (int)cols);
  else if (vec && cols <= 4096)
    max_rows_vjp_reg_kernel<4><<<blocks, 256, 0, st>>>(x, ct, dx, rows, (int)cols);
  else if (vec && cols <= 8192)
    max_rows_vjp_reg_kernel<8><<<blocks, 256, 0, st>>>(x, ct, dx, rows, (int)cols);
  else
    max_rows_vjp_kernel<<<grid_rows(rows, 8), 256, 0, st>>>(x, ct, dx, rows, (int)cols);
  JX_LAUNCH_CHECK("max_rows_vjp_kernel");
  return JX_OK;
}

}  // extern "C"
