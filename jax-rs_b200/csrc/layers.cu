// layers.cu -- conv1d, 2-D pooling, global pooling and batch / layer
// normalisation: the ops the reference runs only as WGSL kernels or CPU loops.
//
//   conv1d        gpu_conv1d src/backend/ops.rs:1014-1200 with conv1d_shader
//                 src/backend/shaders.rs:449-519; nn::conv1d src/nn.rs:1662-1722
//   pooling       gpu_maxpool2d / gpu_avgpool2d src/backend/ops.rs:1204-1514 with
//                 the shaders at src/backend/shaders.rs:524-667; nn::maxpool2d /
//                 avgpool2d src/nn.rs:2164-2280; max_pool2d / avg_pool2d
//                 :1121-1261; max_pool1d / avg_pool1d :1002-1100
//   global pool   nn::global_avg_pool2d / global_max_pool2d src/nn.rs:2383-2455
//   batchnorm     gpu_batchnorm src/backend/ops.rs:1516-1693 (its bind group does
//                 not match its shader, src/backend/shaders.rs:672-727, so that
//                 path never ran); nn::batch_norm_2d src/nn.rs:2303-2360,
//                 batch_norm :656-699, layer_norm :712-725
//
// Parity.  conv1d and pooling run the reference's loops in its order, one
// output per accumulator, with unfused f32 multiply and add, so they are
// bit-identical to the CPU loops.  Global average pooling and the
// normalisation statistics are tree reductions (tolerance-checked); the
// normalisation itself, (x - mean) / std * gamma + beta, is evaluated with
// the reference's operations in its order.
//
// Layout and bounds.  Everything is NCHW / [outer, channels, inner] row-major
// f32, as in the reference.  Pooling and global pooling are HBM-bound (one
// read of x, one write of y).  Normalisation needs the statistics before the
// first output, so it reads x twice and writes y once; the second read walks
// the tensor backwards so that the part the statistics pass left in L2 is
// read from there.  conv1d is FP32-issue-bound: each multiply-add is an FMUL
// and an FADD (no contraction, as the reference's Rust arithmetic).
#include <math.h>

#include <algorithm>

#include "jx_common.cuh"

namespace {

// ---------------------------------------------------------------------------
// conv1d
// ---------------------------------------------------------------------------
// Block tile: 64 output channels x 128 output positions, 256 threads.  Warp w
// owns output channels [8w, 8w+8) of the tile, lane l owns positions
// l + 32j (j < 4), so each thread keeps 32 accumulators.  Input channels
// stream through shared memory in chunks of `icc`:
//   xs[ic][XW]        the input window of the tile's 128 positions
//                     (XW = 127*S + K), zero outside [0, L)
//   ws[ic][k][64]     the chunk's filter taps, output channel fastest
// Per output the sum runs over ic, then k, as the shader's loop.  A tap that
// falls into the padding is skipped, as the shader's bounds check does; a
// thread whose taps are all in range takes the unchecked loop.
constexpr int C1_OC = 64, C1_POS = 128, C1_THREADS = 256;

struct Conv1dArgs {
  const float* x;
  const float* w;
  float* y;
  long long B, C, L, O, K, S, P, OL;
  int icc, xw;
};

template <bool CHECKED>
__device__ __forceinline__ void conv1d_chunk(const float* __restrict__ xs, const float* __restrict__ ws,
                                             float (&acc)[8][4], int nic, int K, int S, int xw, int og, int lane,
                                             long long in0, long long L) {
  for (int ic = 0; ic < nic; ++ic) {
    const float* xr = xs + ic * xw;
    for (int k = 0; k < K; ++k) {
      const float4* wp = reinterpret_cast<const float4*>(ws + (ic * K + k) * C1_OC + og * 8);
      const float4 w0 = wp[0], w1 = wp[1];
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int off = (lane + 32 * j) * S + k;
        if (CHECKED) {
          const long long ip = in0 + off;
          if (ip < 0 || ip >= L) continue;
        }
        const float xv = xr[off];
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[r][j] = __fadd_rn(acc[r][j], __fmul_rn(xv, wv[r]));
      }
    }
  }
}

__global__ void __launch_bounds__(C1_THREADS) conv1d_kernel(Conv1dArgs a) {
  extern __shared__ __align__(16) float c1_smem[];
  float* ws = c1_smem;                                  // icc * K * 64
  float* xs = c1_smem + (size_t)a.icc * a.K * C1_OC;    // icc * xw
  const int tid = threadIdx.x, lane = tid & 31, og = tid >> 5;
  const long long p0 = (long long)blockIdx.x * C1_POS;
  const long long o0 = (long long)blockIdx.y * C1_OC;
  const long long b = blockIdx.z;
  const long long in0 = p0 * a.S - a.P;  // input position of xs[.][0]
  const int K = (int)a.K, S = (int)a.S;

  // Whether every tap of this thread's valid outputs is inside [0, L).
  const long long p_first = p0 + lane;
  long long p_last = p0 + lane + 96;
  if (p_last >= a.OL) p_last = p0 + lane + 32 * ((a.OL - 1 - p0 - lane) / 32);
  const bool interior = p_first >= a.OL || (p_first * a.S - a.P >= 0 && p_last * a.S - a.P + a.K <= a.L);
  const bool warp_interior = __all_sync(0xffffffffu, interior);

  float acc[8][4];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[r][j] = 0.0f;

  for (long long c0 = 0; c0 < a.C; c0 += a.icc) {
    const int nic = (int)min((long long)a.icc, a.C - c0);
    __syncthreads();
    // filter taps: w[o][c0+ic][k] -> ws[(ic*K + k)*64 + o_local]; reads run
    // along (ic, k), contiguous in w for a fixed o
    const int wn = nic * K;
    for (int i = tid; i < C1_OC * wn; i += C1_THREADS) {
      const int ol = i / wn, r = i - ol * wn;
      const long long o = o0 + ol;
      ws[r * C1_OC + ol] = o < a.O ? __ldg(a.w + (o * a.C + c0) * a.K + r) : 0.0f;
    }
    // input window, zero outside [0, L)
    const float* xb = a.x + (b * a.C + c0) * a.L;
    for (int i = tid; i < nic * a.xw; i += C1_THREADS) {
      const int ic = i / a.xw, off = i - ic * a.xw;
      const long long ip = in0 + off;
      xs[i] = (ip >= 0 && ip < a.L) ? __ldg(xb + ic * a.L + ip) : 0.0f;
    }
    __syncthreads();
    if (warp_interior)
      conv1d_chunk<false>(xs, ws, acc, nic, K, S, a.xw, og, lane, in0, a.L);
    else
      conv1d_chunk<true>(xs, ws, acc, nic, K, S, a.xw, og, lane, in0, a.L);
  }

#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const long long o = o0 + og * 8 + r;
    if (o >= a.O) break;
    float* yr = a.y + (b * a.O + o) * a.OL;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const long long p = p0 + lane + 32 * j;
      if (p < a.OL) yr[p] = acc[r][j];
    }
  }
}

// ---------------------------------------------------------------------------
// 2-D pooling: one output per thread, taps in (row, column) order.
// ---------------------------------------------------------------------------
struct PoolArgs {
  const float* x;
  float* y;
  long long N, H, W, OH, OW;
  int kh, kw, sh, sw, ph, pw;
};

// IDX is the index type: 32-bit when every index fits (cheaper division).
template <bool MAX, typename IDX>
__global__ void __launch_bounds__(256) pool2d_kernel(PoolArgs a) {
  const IDX total = (IDX)(a.N * a.OH * a.OW), OW = (IDX)a.OW, OH = (IDX)a.OH;
  const IDX stride = (IDX)gridDim.x * blockDim.x;
  for (IDX idx = (IDX)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const IDX t = idx / OW;
    const IDX ow = idx - t * OW;
    const IDX n = t / OH;
    const IDX oh = t - n * OH;
    const float* plane = a.x + (long long)n * a.H * a.W;
    const long long ih0 = (long long)oh * a.sh - a.ph, iw0 = (long long)ow * a.sw - a.pw;
    float acc = MAX ? -INFINITY : 0.0f;
    int count = 0;
    for (int r = 0; r < a.kh; ++r) {
      const long long ih = ih0 + r;
      if (ih < 0 || ih >= a.H) continue;
      const float* row = plane + ih * a.W;
      for (int c = 0; c < a.kw; ++c) {
        const long long iw = iw0 + c;
        if (iw < 0 || iw >= a.W) continue;
        const float v = __ldg(row + iw);
        acc = MAX ? fmaxf(acc, v) : __fadd_rn(acc, v);
        ++count;
      }
    }
    a.y[idx] = MAX ? acc : (count ? __fdiv_rn(acc, (float)count) : 0.0f);
  }
}

// ---------------------------------------------------------------------------
// Global pooling: one warp per [S] row.
// ---------------------------------------------------------------------------
template <bool MAX>
__global__ void __launch_bounds__(256) global_pool_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                           long long N, long long S) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const bool vec = (S & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (long long n = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
    const float* row = x + n * S;
    float acc = MAX ? -INFINITY : 0.0f;
    if (vec) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      for (long long i = lane; i < S / 4; i += 32) {
        const float4 v = __ldg(r4 + i);
        if (MAX)
          acc = fmaxf(fmaxf(acc, v.x), fmaxf(v.y, fmaxf(v.z, v.w)));
        else
          acc += (v.x + v.y) + (v.z + v.w);
      }
    } else {
      for (long long i = lane; i < S; i += 32) {
        const float v = __ldg(row + i);
        acc = MAX ? fmaxf(acc, v) : acc + v;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, acc, o);
      acc = MAX ? fmaxf(acc, t) : acc + t;
    }
    if (lane == 0) y[n] = MAX ? acc : __fdiv_rn(acc, (float)S);
  }
}

// ---------------------------------------------------------------------------
// Normalisation of x viewed as [outer, C, inner], statistics per channel.
// ---------------------------------------------------------------------------
// Statistics are shifted sums in f64: with p = x[0, c, 0], s1 = sum (x - p)
// and s2 = sum (x - p)^2 over the channel, mean = p + s1/n and var = s2/n -
// (s1/n)^2, accurate for any ratio of mean to spread that matters in f32.
// Partials are written in a fixed layout and combined in a fixed order, so
// results are reproducible run to run.
//
// Wide rows (inner >= 128): the channel's outer*inner elements, in (o, i)
// order, are cut into G chunks of `chunk` elements; block (c, g) sums chunk
// g, row segment by row segment, with float4 loads where aligned.
// Narrow rows: block covers 256 consecutive columns of the [outer, C*inner]
// matrix for rows g, g+G, ...; thread = one column.
struct NormArgs {
  const float* x;
  long long outer, C, inner;
  long long chunk;  // wide: elements per chunk (a multiple of 4)
  int G;            // wide: chunks per channel; narrow: row groups
};

__device__ __forceinline__ double2 add2(double2 a, double2 b) { return make_double2(a.x + b.x, a.y + b.y); }

__device__ __forceinline__ double2 block_sum2(double2 v, double2* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
    v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : make_double2(0.0, 0.0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
      v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
    }
  }
  return v;
}

__global__ void __launch_bounds__(256) norm_stats_wide(NormArgs a, double2* __restrict__ part) {
  __shared__ double2 red[8];
  const long long c = blockIdx.x;
  const int g = blockIdx.y;
  const float p = __ldg(a.x + c * a.inner);
  const bool vec = (a.inner & 3) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
  const long long per = a.outer * a.inner;
  long long t = (long long)g * a.chunk;
  const long long t_end = min(per, t + a.chunk);
  double2 s = make_double2(0.0, 0.0);
  while (t < t_end) {
    const long long o = t / a.inner, i0 = t - o * a.inner, i1 = min(a.inner, i0 + (t_end - t));
    const float* row = a.x + (o * a.C + c) * a.inner;
    if (vec) {  // i0 and i1 are multiples of 4 here
      const float4* r4 = reinterpret_cast<const float4*>(row);
      for (long long i = i0 / 4 + threadIdx.x; i < i1 / 4; i += blockDim.x) {
        const float4 v = __ldg(r4 + i);
        const double d0 = (double)v.x - p, d1 = (double)v.y - p, d2 = (double)v.z - p, d3 = (double)v.w - p;
        s.x += (d0 + d1) + (d2 + d3);
        s.y += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
      }
    } else {
      for (long long i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const double d = (double)__ldg(row + i) - p;
        s.x += d;
        s.y += d * d;
      }
    }
    t += i1 - i0;
  }
  s = block_sum2(s, red);
  if (threadIdx.x == 0) part[(long long)g * a.C + c] = s;
}

__global__ void __launch_bounds__(256) norm_stats_narrow(NormArgs a, double2* __restrict__ part) {
  const long long cols = a.C * a.inner;
  const long long col = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int g = blockIdx.y;
  if (col >= cols) return;
  const long long c = col / a.inner;
  const float p = __ldg(a.x + c * a.inner);
  double2 s = make_double2(0.0, 0.0);
  for (long long o = g; o < a.outer; o += a.G) {
    const double d = (double)__ldg(a.x + o * cols + col) - p;
    s.x += d;
    s.y += d * d;
  }
  part[(long long)g * cols + col] = s;
}

// One warp per channel: combine the partials, then mean, var and
// std = sqrt(var + eps) in f32 as the reference computes std.
__global__ void __launch_bounds__(256) norm_finalize(NormArgs a, const double2* __restrict__ part, bool wide,
                                                     float eps, float2* __restrict__ ms, float* __restrict__ mean_out,
                                                     float* __restrict__ var_out) {
  const int lane = threadIdx.x & 31;
  const long long c = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (c >= a.C) return;
  double2 s = make_double2(0.0, 0.0);
  if (wide) {
    for (int g = lane; g < a.G; g += 32) s = add2(s, part[(long long)g * a.C + c]);
  } else {
    const long long cols = a.C * a.inner, m = (long long)a.G * a.inner;
    for (long long t = lane; t < m; t += 32) {
      const long long g = t / a.inner, i = t - g * a.inner;
      s = add2(s, part[g * cols + c * a.inner + i]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s.x += __shfl_xor_sync(0xffffffffu, s.x, o);
    s.y += __shfl_xor_sync(0xffffffffu, s.y, o);
  }
  if (lane == 0) {
    const double n = (double)a.outer * (double)a.inner;
    const double p = (double)__ldg(a.x + c * a.inner);
    const double d = s.x / n;
    const double var = fmax(s.y / n - d * d, 0.0);
    const float mean_f = (float)(p + d), var_f = (float)var;
    ms[c] = make_float2(mean_f, sqrtf(var_f + eps));
    if (mean_out) mean_out[c] = mean_f;
    if (var_out) var_out[c] = var_f;
  }
}

// y = (x - mean) / std * gamma + beta, unfused, in the reference's order.
// The grid sweeps the tensor from its end to its start, so the statistics
// pass's most recent reads (still in L2) are read first.
template <bool AFFINE>
__device__ __forceinline__ float norm1(float v, float2 m, float g, float b) {
  const float z = __fdiv_rn(__fsub_rn(v, m.x), m.y);
  return AFFINE ? __fadd_rn(__fmul_rn(z, g), b) : z;
}

template <bool AFFINE, bool VEC, typename IDX>
__global__ void __launch_bounds__(256) norm_apply(const float* __restrict__ x, float* __restrict__ y,
                                                  const float2* __restrict__ ms, const float* __restrict__ gamma,
                                                  const float* __restrict__ beta, long long n, long long C_,
                                                  long long inner_) {
  const IDX units = (IDX)(VEC ? n / 4 : n), C = (IDX)C_, inner = (IDX)inner_;
  const IDX nthreads = (IDX)gridDim.x * blockDim.x;
  const IDX tid = (IDX)blockIdx.x * blockDim.x + threadIdx.x;
  for (IDX sweep = (units + nthreads - 1) / nthreads; sweep-- > 0;) {
    const IDX u = sweep * nthreads + tid;
    if (u >= units) continue;
    const IDX e = VEC ? u * 4 : u;
    const IDX c = (e / inner) % C;
    const float2 m = ms[c];
    const float g = AFFINE ? __ldg(gamma + c) : 1.0f, b = AFFINE ? __ldg(beta + c) : 0.0f;
    if (VEC) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(x) + u);
      float4 r;
      r.x = norm1<AFFINE>(v.x, m, g, b);
      r.y = norm1<AFFINE>(v.y, m, g, b);
      r.z = norm1<AFFINE>(v.z, m, g, b);
      r.w = norm1<AFFINE>(v.w, m, g, b);
      reinterpret_cast<float4*>(y)[u] = r;
    } else {
      y[u] = norm1<AFFINE>(__ldg(x + u), m, g, b);
    }
  }
}

int grid_for(long long work, int per_block, int cap_per_sm) {
  const long long want = (work + per_block - 1) / per_block;
  const long long cap = (long long)jx::num_sms() * cap_per_sm;
  return (int)std::max(1LL, std::min(want, cap));
}

}  // namespace

extern "C" {

int jx_conv1d_f32(const float* x, const float* w, float* y, int64_t batch, int64_t in_channels,
                  int64_t out_channels, int64_t input_len, int64_t kernel_len, int64_t stride, int64_t padding,
                  jx_stream_t stream) {
  JX_REQUIRE(batch >= 0 && in_channels >= 1 && out_channels >= 0 && input_len >= 1,
             "jx_conv1d_f32: bad dims (batch %lld, in %lld, out %lld, len %lld)", (long long)batch,
             (long long)in_channels, (long long)out_channels, (long long)input_len);
  JX_REQUIRE(kernel_len >= 1 && stride >= 1 && padding >= 0, "jx_conv1d_f32: kernel %lld stride %lld padding %lld",
             (long long)kernel_len, (long long)stride, (long long)padding);
  JX_REQUIRE(kernel_len <= input_len + 2 * padding, "Kernel size must be <= input size");
  JX_REQUIRE(stride <= 64 && kernel_len <= 512, "jx_conv1d_f32: stride <= 64 and kernel_len <= 512 (got %lld, %lld)",
             (long long)stride, (long long)kernel_len);
  const long long OL = (input_len + 2 * padding - kernel_len) / stride + 1;
  if (batch == 0 || out_channels == 0) return JX_OK;
  JX_REQUIRE(x && w && y, "jx_conv1d_f32: NULL buffer");
  JX_REQUIRE(batch <= 65535 && (out_channels + C1_OC - 1) / C1_OC <= 65535,
             "jx_conv1d_f32: batch <= 65535 and out_channels <= %d", 65535 * C1_OC);
  Conv1dArgs a;
  a.x = x;
  a.w = w;
  a.y = y;
  a.B = batch;
  a.C = in_channels;
  a.L = input_len;
  a.O = out_channels;
  a.K = kernel_len;
  a.S = stride;
  a.P = padding;
  a.OL = OL;
  a.xw = (int)((C1_POS - 1) * stride + kernel_len);
  const long long per_ic = (long long)kernel_len * C1_OC + a.xw;  // floats per input channel of a chunk
  const long long budget = 48 * 1024 / 4;
  a.icc = (int)std::max(1LL, std::min({16LL, (long long)in_channels, budget / per_ic}));
  const size_t smem = (size_t)a.icc * per_ic * 4;
  JX_REQUIRE(smem <= 200 * 1024, "jx_conv1d_f32: window too large for shared memory");
  if (smem > 48 * 1024) JX_CUDA(cudaFuncSetAttribute(conv1d_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)smem));
  const dim3 grid((unsigned)((OL + C1_POS - 1) / C1_POS), (unsigned)((out_channels + C1_OC - 1) / C1_OC),
                  (unsigned)batch);
  conv1d_kernel<<<grid, C1_THREADS, smem, jx::as_stream(stream)>>>(a);
  JX_LAUNCH_CHECK("conv1d_kernel");
  return JX_OK;
}

int jx_pool2d_f32(const float* x, float* y, int64_t batch, int64_t channels, int64_t input_h, int64_t input_w,
                  int64_t pool_h, int64_t pool_w, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
                  int op, jx_stream_t stream) {
  JX_REQUIRE(op == JX_POOL_MAX || op == JX_POOL_AVG, "jx_pool2d_f32: unknown op %d", op);
  JX_REQUIRE(pool_h > 0 && pool_w > 0, "Pool size must be positive");
  JX_REQUIRE(stride_h > 0 && stride_w > 0, "Stride must be positive");
  JX_REQUIRE(batch >= 0 && channels >= 0 && input_h >= 1 && input_w >= 1 && pad_h >= 0 && pad_w >= 0,
             "jx_pool2d_f32: bad dims");
  JX_REQUIRE(pool_h <= input_h + 2 * pad_h && pool_w <= input_w + 2 * pad_w,
             "jx_pool2d_f32: window %lldx%lld larger than the padded input %lldx%lld", (long long)pool_h,
             (long long)pool_w, (long long)(input_h + 2 * pad_h), (long long)(input_w + 2 * pad_w));
  JX_REQUIRE(pool_h <= (1 << 20) && pool_w <= (1 << 20) && stride_h <= (1 << 30) && stride_w <= (1 << 30) &&
                 pad_h <= (1 << 30) && pad_w <= (1 << 30),
             "jx_pool2d_f32: window, stride or padding out of range");
  PoolArgs a;
  a.x = x;
  a.y = y;
  a.N = batch * channels;
  a.H = input_h;
  a.W = input_w;
  a.OH = (input_h + 2 * pad_h - pool_h) / stride_h + 1;
  a.OW = (input_w + 2 * pad_w - pool_w) / stride_w + 1;
  a.kh = (int)pool_h;
  a.kw = (int)pool_w;
  a.sh = (int)stride_h;
  a.sw = (int)stride_w;
  a.ph = (int)pad_h;
  a.pw = (int)pad_w;
  const long long total = a.N * a.OH * a.OW;
  if (total == 0) return JX_OK;
  JX_REQUIRE(x && y, "jx_pool2d_f32: NULL buffer");
  const int grid = grid_for(total, 256, 16);
  const bool small = total + 256LL * grid < (1LL << 31) && a.N * a.H * a.W < (1LL << 31);
  cudaStream_t st = jx::as_stream(stream);
  if (op == JX_POOL_MAX) {
    if (small)
      pool2d_kernel<true, unsigned><<<grid, 256, 0, st>>>(a);
    else
      pool2d_kernel<true, long long><<<grid, 256, 0, st>>>(a);
  } else {
    if (small)
      pool2d_kernel<false, unsigned><<<grid, 256, 0, st>>>(a);
    else
      pool2d_kernel<false, long long><<<grid, 256, 0, st>>>(a);
  }
  JX_LAUNCH_CHECK("pool2d_kernel");
  return JX_OK;
}

int jx_maxpool2d_f32(const float* x, float* y, int64_t batch, int64_t channels, int64_t input_h, int64_t input_w,
                     int64_t pool_h, int64_t pool_w, int64_t stride, int64_t padding, jx_stream_t stream) {
  return jx_pool2d_f32(x, y, batch, channels, input_h, input_w, pool_h, pool_w, stride, stride, padding, padding,
                       JX_POOL_MAX, stream);
}

int jx_avgpool2d_f32(const float* x, float* y, int64_t batch, int64_t channels, int64_t input_h, int64_t input_w,
                     int64_t pool_h, int64_t pool_w, int64_t stride, int64_t padding, jx_stream_t stream) {
  return jx_pool2d_f32(x, y, batch, channels, input_h, input_w, pool_h, pool_w, stride, stride, padding, padding,
                       JX_POOL_AVG, stream);
}

int jx_global_pool2d_f32(const float* x, float* y, int64_t batch, int64_t channels, int64_t height, int64_t width,
                         int op, jx_stream_t stream) {
  JX_REQUIRE(op == JX_POOL_MAX || op == JX_POOL_AVG, "jx_global_pool2d_f32: unknown op %d", op);
  JX_REQUIRE(batch >= 0 && channels >= 0 && height >= 1 && width >= 1, "jx_global_pool2d_f32: bad dims");
  const long long N = batch * channels, S = height * width;
  if (N == 0) return JX_OK;
  JX_REQUIRE(x && y, "jx_global_pool2d_f32: NULL buffer");
  const int grid = grid_for(N * 32, 256, 16);
  if (op == JX_POOL_MAX)
    global_pool_kernel<true><<<grid, 256, 0, jx::as_stream(stream)>>>(x, y, N, S);
  else
    global_pool_kernel<false><<<grid, 256, 0, jx::as_stream(stream)>>>(x, y, N, S);
  JX_LAUNCH_CHECK("global_pool_kernel");
  return JX_OK;
}

int jx_batchnorm_f32(const float* x, const float* gamma, const float* beta, float* y, int64_t batch,
                     int64_t channels, int64_t spatial, float epsilon, float* mean_out, float* var_out,
                     jx_stream_t stream) {
  JX_REQUIRE(batch >= 1 && channels >= 1 && spatial >= 1, "jx_batchnorm_f32: bad dims (%lld, %lld, %lld)",
             (long long)batch, (long long)channels, (long long)spatial);
  JX_REQUIRE((gamma == nullptr) == (beta == nullptr), "jx_batchnorm_f32: gamma and beta go together");
  JX_REQUIRE(x && y, "jx_batchnorm_f32: NULL buffer");
  cudaStream_t st = jx::as_stream(stream);
  NormArgs a;
  a.x = x;
  a.outer = batch;
  a.C = channels;
  a.inner = spatial;
  const bool wide = spatial >= 128;
  const long long target = 4LL * jx::num_sms();  // blocks for the statistics pass
  long long parts;
  a.chunk = 0;
  if (wide) {
    const long long per = batch * spatial;
    const long long g = std::max(1LL, std::min({(target + channels - 1) / channels, (per + 4095) / 4096, 4096LL}));
    a.chunk = ((per + g - 1) / g + 3) / 4 * 4;
    a.G = (int)((per + a.chunk - 1) / a.chunk);
    JX_REQUIRE(channels <= 0x7fffffffLL, "jx_batchnorm_f32: too many channels");
    parts = (long long)a.G * channels;
  } else {
    const long long cols = channels * spatial, col_blocks = (cols + 255) / 256;
    JX_REQUIRE(col_blocks <= 0x7fffffffLL, "jx_batchnorm_f32: too many columns");
    a.G = (int)std::max(1LL, std::min({(long long)batch, (target + col_blocks - 1) / col_blocks, 1024LL}));
    parts = (long long)a.G * cols;
  }
  void* ws = nullptr;
  const size_t part_bytes = (size_t)parts * sizeof(double2);
  if (int rc = jx::scratch_get(part_bytes + (size_t)channels * sizeof(float2), &ws, st)) return rc;
  double2* part = static_cast<double2*>(ws);
  float2* ms = reinterpret_cast<float2*>(static_cast<char*>(ws) + part_bytes);
  int rc = JX_OK;
  if (wide)
    norm_stats_wide<<<dim3((unsigned)channels, (unsigned)a.G), 256, 0, st>>>(a, part);
  else
    norm_stats_narrow<<<dim3((unsigned)((channels * spatial + 255) / 256), (unsigned)a.G), 256, 0, st>>>(a, part);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    norm_finalize<<<(unsigned)((channels + 7) / 8), 256, 0, st>>>(a, part, wide, epsilon, ms, mean_out, var_out);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    const long long n = batch * channels * spatial;
    const bool vec = (spatial & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    const int grid = grid_for(vec ? n / 4 : n, 256, 8);
    const bool small = n + 256LL * grid < (1LL << 31);
#define JX_NORM_APPLY(AFF, VEC)                                                                   \
  do {                                                                                            \
    if (small)                                                                                    \
      norm_apply<AFF, VEC, unsigned><<<grid, 256, 0, st>>>(x, y, ms, gamma, beta, n, channels, spatial);  \
    else                                                                                          \
      norm_apply<AFF, VEC, long long><<<grid, 256, 0, st>>>(x, y, ms, gamma, beta, n, channels, spatial); \
  } while (0)
    if (gamma) {
      if (vec)
        JX_NORM_APPLY(true, true);
      else
        JX_NORM_APPLY(true, false);
    } else {
      if (vec)
        JX_NORM_APPLY(false, true);
      else
        JX_NORM_APPLY(false, false);
    }
#undef JX_NORM_APPLY
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) rc = jx::check_cuda(e, "batchnorm kernels");
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

}  // extern "C"
