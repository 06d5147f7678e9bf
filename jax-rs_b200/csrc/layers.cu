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
// the reference's operations in its order, with the mean carried as two f32
// parts.
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

int grid_for(long long work, int per_block, int cap_per_sm) {
  const long long want = (work + per_block - 1) / per_block;
  const long long cap = (long long)jx::num_sms() * cap_per_sm;
  return (int)std::max(1LL, std::min(want, cap));
}

// ---------------------------------------------------------------------------
// conv1d
// ---------------------------------------------------------------------------
// Block tile: 64 output channels x 256 output positions, 256 threads.  Warp w
// owns output channels [8w, 8w+8) of the tile, lane l owns positions
// l + 32j (j < 8), so each thread keeps 64 accumulators.  Input channels
// stream through shared memory in chunks of `icc`:
//   xs[ic][XW]        the input window of the tile's 256 positions
//                     (XW = 255*S + K), zero outside [0, L)
//   ws[ic][k][64]     the chunk's filter taps, output channel fastest
// Per output the sum runs over ic, then k, as the shader's loop, each step an
// unfused __fmul_rn then __fadd_rn (the reference's Rust arithmetic), so the
// result is bit-identical.  A tap that falls into the padding is skipped, as
// the shader's bounds check does; a warp whose taps are all in range takes
// the unchecked loop.  The stride and the common tap count 3 are compile-time
// constants where they can be, so tap addresses are immediate offsets.
constexpr int C1_OC = 64, C1_NJ = 8, C1_POS = 32 * C1_NJ, C1_THREADS = 256;

struct Conv1dArgs {
  const float* x;
  const float* wt;  // filter as [C*K][Opad], output channel fastest, zero past O
  float* y;
  long long B, C, L, O, K, S, P, OL, Opad;
  int icc, xw;
  int buf_floats;  // one of the two shared-memory buffers: icc*K*64 taps + icc*xw inputs, padded to 4
  float one;       // 1.0, a kernel argument so that the compiler cannot fold it
};

// w [O][C][K] -> wt [C*K][Opad] (Opad = O rounded up to the 64-channel tile).
__global__ void __launch_bounds__(256) conv1d_filter_kernel(const float* __restrict__ w, float* __restrict__ wt,
                                                             long long O, long long CK, long long Opad) {
  const long long total = CK * Opad;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / Opad, o = i - r * Opad;
    wt[i] = o < O ? __ldg(w + o * CK + r) : 0.0f;
  }
}

// acc.{x,y} = rn(rn(x * w.{x,y}) + acc.{x,y}) with packed f32x2 operations:
// one mul.f32x2 and one fma.f32x2 for two multiply-adds, half the
// instructions of the scalar FMUL + FADD pairs.  The add is an FMA by a
// run-time 1.0 that the compiler cannot see, so the product keeps its own
// rounding (a plain add.f32x2 after the mul.f32x2 is contracted into one
// fma.f32x2 even under --fmad=false, which is 1 ulp off the reference's
// separately rounded multiply and add).
__device__ __forceinline__ void mac2(float2& acc, float x, float2 w, float one) {
  asm("{\n\t.reg .b64 xa, wa, ca, oa, pa;\n\t"
      "mov.b64 xa, {%2, %2};\n\t"
      "mov.b64 wa, {%3, %4};\n\t"
      "mov.b64 ca, {%0, %1};\n\t"
      "mov.b64 oa, {%5, %5};\n\t"
      "mul.rn.f32x2 pa, xa, wa;\n\t"
      "fma.rn.f32x2 ca, pa, oa, ca;\n\t"
      "mov.b64 {%0, %1}, ca;\n\t}"
      : "+f"(acc.x), "+f"(acc.y)
      : "f"(x), "f"(w.x), "f"(w.y), "f"(one));
}

template <int SS, int KK, bool CHECKED>
__device__ __forceinline__ void conv1d_chunk(const float* __restrict__ xs, const float* __restrict__ ws,
                                             float (&acc)[8][C1_NJ], int nic, int K_rt, int S_rt, int xw, int og,
                                             int lane, long long in0, long long L, float one) {
  const int S = SS > 0 ? SS : S_rt;
  const int K = KK > 0 ? KK : K_rt;
  for (int ic = 0; ic < nic; ++ic) {
    const float* xr = xs + ic * xw + lane * S;
    const float* wr = ws + ic * K * C1_OC + og * 8;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float4 w0 = *reinterpret_cast<const float4*>(wr + k * C1_OC);
      const float4 w1 = *reinterpret_cast<const float4*>(wr + k * C1_OC + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int j = 0; j < C1_NJ; ++j) {
        if (CHECKED) {
          const long long ip = in0 + (long long)(lane + 32 * j) * S + k;
          if (ip < 0 || ip >= L) continue;
        }
        const float xv = xr[32 * j * S + k];
#pragma unroll
        for (int r = 0; r < 8; r += 2) {
          float2 a2 = make_float2(acc[r][j], acc[r + 1][j]);
          mac2(a2, xv, make_float2(wv[r], wv[r + 1]), one);
          acc[r][j] = a2.x;
          acc[r + 1][j] = a2.y;
        }
      }
    }
  }
}

__device__ __forceinline__ void c1_cp4(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(jxd::smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void c1_cp16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(jxd::smem_u32(dst)), "l"(src) : "memory");
}

// Input channels stream through two shared-memory buffers filled by
// cp.async: chunk i+1 lands while chunk i is summed.
template <int SS, int KK>
__global__ void __launch_bounds__(C1_THREADS) conv1d_kernel(Conv1dArgs a) {
  extern __shared__ __align__(16) float c1_smem[];
  const int tid = threadIdx.x, lane = tid & 31, og = tid >> 5;
  const long long p0 = (long long)blockIdx.x * C1_POS;
  const long long o0 = (long long)blockIdx.y * C1_OC;
  const long long b = blockIdx.z;
  const long long in0 = p0 * a.S - a.P;  // input position of xs[.][0]
  const int K = (int)a.K, S = (int)a.S;

  // Whether every tap of this thread's valid outputs is inside [0, L).
  const long long p_first = p0 + lane;
  long long p_last = p0 + lane + 32 * (C1_NJ - 1);
  if (p_last >= a.OL) p_last = p0 + lane + 32 * ((a.OL - 1 - p0 - lane) / 32);
  const bool interior = p_first >= a.OL || (p_first * a.S - a.P >= 0 && p_last * a.S - a.P + a.K <= a.L);
  const bool warp_interior = __all_sync(0xffffffffu, interior);

  // fill(buf, c0): taps of input channels [c0, c0 + nic) (rows (c0+ic)*K + k
  // of wt, the tile's 64 channels each, 16-byte copies) and their input
  // windows (zero outside [0, L))
  auto fill = [&](int buf, long long c0) {
    float* ws = c1_smem + (size_t)buf * a.buf_floats;
    float* xs = ws + (size_t)a.icc * a.K * C1_OC;
    const int nic = (int)min((long long)a.icc, a.C - c0);
    const int wn4 = nic * K * (C1_OC / 4);
    const float* wsrc = a.wt + c0 * a.K * a.Opad + o0;
    for (int i = tid; i < wn4; i += C1_THREADS) c1_cp16(ws + 4 * i, wsrc + (long long)(i >> 4) * a.Opad + 4 * (i & 15));
    const float* xb = a.x + (b * a.C + c0) * a.L;
    int ic = tid / a.xw, off = tid - ic * a.xw;
    for (int i = tid; i < nic * a.xw; i += C1_THREADS) {
      const long long ip = in0 + off;
      const bool v = ip >= 0 && ip < a.L;
      c1_cp4(xs + i, v ? xb + (long long)ic * a.L + ip : a.x, v);
      off += C1_THREADS;
      while (off >= a.xw) {
        off -= a.xw;
        ++ic;
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float acc[8][C1_NJ];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int j = 0; j < C1_NJ; ++j) acc[r][j] = 0.0f;

  fill(0, 0);
  int buf = 0;
  for (long long c0 = 0; c0 < a.C; c0 += a.icc, buf ^= 1) {
    const int nic = (int)min((long long)a.icc, a.C - c0);
    if (c0 + a.icc < a.C) {
      fill(buf ^ 1, c0 + a.icc);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // chunk c0 has landed for every thread
    const float* ws = c1_smem + (size_t)buf * a.buf_floats;
    const float* xs = ws + (size_t)a.icc * a.K * C1_OC;
    if (warp_interior)
      conv1d_chunk<SS, KK, false>(xs, ws, acc, nic, K, S, a.xw, og, lane, in0, a.L, a.one);
    else
      conv1d_chunk<SS, KK, true>(xs, ws, acc, nic, K, S, a.xw, og, lane, in0, a.L, a.one);
    __syncthreads();  // done with this buffer before it is refilled
  }

#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const long long o = o0 + og * 8 + r;
    if (o >= a.O) break;
    float* yr = a.y + (b * a.O + o) * a.OL;
#pragma unroll
    for (int j = 0; j < C1_NJ; ++j) {
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
  unsigned ow_m, oh_m;  // division by OW and OH as multiply-high (fast_div), 32-bit index path
  int ow_l, oh_l;
};

// n / d for n < 2^31 by the multiply-high method of Granlund and Montgomery
// ("Division by invariant integers using multiplication", 1994): with
// l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// n / d = (umulhi(n, m) + n) >> l (the sum stays below 2^32 for n < 2^31).
void fast_div_params(unsigned d, unsigned& m, int& l) {
  l = 0;
  while ((1ull << l) < d) ++l;
  m = (unsigned)((((1ull << l) - d) << 32) / d + 1);
}
__device__ __forceinline__ unsigned fast_div(unsigned n, unsigned m, int l) { return (__umulhi(n, m) + n) >> l; }

// IDX is the index type: 32-bit when every index fits (cheaper division).
// KH, KW > 0 fix the window at compile time (fully unrolled); 0 reads it from
// the arguments.  Out-of-range taps load the fold's neutral value (-inf for
// max, +0 for the sum) instead of being skipped: the sum starts at +0 and so
// never holds -0, which makes adding +0 an identity, and max(acc, -inf) = acc,
// so the result is the reference's bit for bit while every tap's load is
// issued at once.
template <bool MAX>
__device__ __forceinline__ float pool_fold(float acc, float v) {
  return MAX ? fmaxf(acc, v) : __fadd_rn(acc, v);
}

template <bool MAX, typename IDX, int KH, int KW>
__global__ void __launch_bounds__(256) pool2d_kernel(PoolArgs a) {
  const IDX total = (IDX)(a.N * a.OH * a.OW), OW = (IDX)a.OW, OH = (IDX)a.OH;
  const IDX stride = (IDX)gridDim.x * blockDim.x;
  const float neutral = MAX ? -INFINITY : 0.0f;
  const int kh = KH > 0 ? KH : a.kh, kw = KW > 0 ? KW : a.kw;
  constexpr bool SMALL = sizeof(IDX) == 4;
  for (IDX idx = (IDX)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const IDX t = SMALL ? (IDX)fast_div((unsigned)idx, a.ow_m, a.ow_l) : idx / OW;
    const IDX ow = idx - t * OW;
    const IDX n = SMALL ? (IDX)fast_div((unsigned)t, a.oh_m, a.oh_l) : t / OH;
    const IDX oh = t - n * OH;
    const float* plane = a.x + (long long)n * a.H * a.W;
    const long long ih0 = (long long)oh * a.sh - a.ph, iw0 = (long long)ow * a.sw - a.pw;
    float acc = neutral;
    int count = 0;
    if (KH > 0 && ih0 >= 0 && iw0 >= 0 && ih0 + kh <= a.H && iw0 + kw <= a.W) {
      // the whole window inside the plane: no tests
      const float* p0 = plane + ih0 * a.W + iw0;
      float v[KH > 0 ? KH : 1][KW > 0 ? KW : 1];
#pragma unroll
      for (int r = 0; r < kh; ++r)
#pragma unroll
        for (int c = 0; c < kw; ++c) v[r][c] = __ldg(p0 + r * a.W + c);
#pragma unroll
      for (int r = 0; r < kh; ++r)
#pragma unroll
        for (int c = 0; c < kw; ++c) acc = pool_fold<MAX>(acc, v[r][c]);
      count = kh * kw;
    } else if (KH > 0) {
      float v[KH > 0 ? KH : 1][KW > 0 ? KW : 1];
#pragma unroll
      for (int r = 0; r < kh; ++r) {
        const long long ih = ih0 + r;
        const bool rok = ih >= 0 && ih < a.H;
#pragma unroll
        for (int c = 0; c < kw; ++c) {
          const long long iw = iw0 + c;
          const bool ok = rok && iw >= 0 && iw < a.W;
          v[r][c] = ok ? __ldg(plane + ih * a.W + iw) : neutral;
          if (!MAX) count += ok;
        }
      }
#pragma unroll
      for (int r = 0; r < kh; ++r)
#pragma unroll
        for (int c = 0; c < kw; ++c) acc = pool_fold<MAX>(acc, v[r][c]);
    } else {
      for (int r = 0; r < kh; ++r) {
        const long long ih = ih0 + r;
        const bool rok = ih >= 0 && ih < a.H;
#pragma unroll 4
        for (int c = 0; c < kw; ++c) {
          const long long iw = iw0 + c;
          const bool ok = rok && iw >= 0 && iw < a.W;
          acc = pool_fold<MAX>(acc, ok ? __ldg(plane + ih * a.W + iw) : neutral);
          if (!MAX) count += ok;
        }
      }
    }
    a.y[idx] = MAX ? acc : (count ? __fdiv_rn(acc, (float)count) : 0.0f);
  }
}

template <bool MAX, typename IDX>
void launch_pool(const PoolArgs& a, cudaStream_t st) {
  const int grid = grid_for(a.N * a.OH * a.OW, 256, 16);
  if (a.kh == 2 && a.kw == 2)
    pool2d_kernel<MAX, IDX, 2, 2><<<grid, 256, 0, st>>>(a);
  else if (a.kh == 3 && a.kw == 3)
    pool2d_kernel<MAX, IDX, 3, 3><<<grid, 256, 0, st>>>(a);
  else
    pool2d_kernel<MAX, IDX, 0, 0><<<grid, 256, 0, st>>>(a);
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

// Wide rows: work items (chunk g, channel c), one warp each, in (g, c) order
// so the pass reads memory front to back.  A lane issues all U of its loads
// (float4 when rows are 16-byte aligned) before it sums; chunk is a multiple
// of the warp's sub-step of 32*U*E elements.
template <bool VEC>
__global__ void __launch_bounds__(256) norm_stats_items(NormArgs a, double2* __restrict__ part) {
  constexpr int U = 8, E = VEC ? 4 : 1, STEP = 32 * U * E;
  const int lane = threadIdx.x & 31;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long items = a.C * a.G, per = a.outer * a.inner;
  for (long long it = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < items; it += nw) {
    const long long g = it / a.C, c = it - g * a.C;
    const float p = __ldg(a.x + c * a.inner);
    const long long t0 = g * a.chunk, t1 = min(per, t0 + a.chunk);
    double sx = 0.0, sy = 0.0;
    for (long long ts = t0; ts < t1; ts += STEP) {
      long long t = ts + (long long)lane * E;
      long long o = t / a.inner, i = t - o * a.inner;
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float* ptr = a.x + (o * a.C + c) * a.inner + i;
        if (VEC)
          v[u] = t < t1 ? __ldg(reinterpret_cast<const float4*>(ptr)) : make_float4(p, p, p, p);
        else
          v[u].x = t < t1 ? __ldg(ptr) : p;
        t += 32 * E;
        i += 32 * E;
        while (i >= a.inner) {
          i -= a.inner;
          ++o;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        // shifted values summed in f32 (x - p is exact while x is within a
        // factor 2 of p), then carried in f64
        if (VEC) {
          const float d0 = v[u].x - p, d1 = v[u].y - p, d2 = v[u].z - p, d3 = v[u].w - p;
          sx += (double)((d0 + d1) + (d2 + d3));
          sy += (double)((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3));
        } else {
          const float d = v[u].x - p;
          sx += (double)d;
          sy += (double)(d * d);
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sx += __shfl_xor_sync(0xffffffffu, sx, off);
      sy += __shfl_xor_sync(0xffffffffu, sy, off);
    }
    if (lane == 0) part[it] = make_double2(sx, sy);
  }
}

__global__ void __launch_bounds__(256) norm_stats_narrow(NormArgs a, double2* __restrict__ part) {
  const long long cols = a.C * a.inner;
  const long long col = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int g = blockIdx.y;
  if (col >= cols) return;
  const long long c = col / a.inner;
  const float p = __ldg(a.x + c * a.inner);
  double2 s = make_double2(0.0, 0.0);
  for (long long o = g; o < a.outer; o += 4LL * a.G) {
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long r = o + (long long)u * a.G;
      v[u] = r < a.outer ? __ldg(a.x + r * cols + col) : p;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const double d = (double)v[u] - p;
      s.x += d;
      s.y += d * d;
    }
  }
  part[(long long)g * cols + col] = s;
}

// One block per channel: combine the partials in a fixed order, then mean,
// var and std = sqrt(var + eps) in f32 as the reference computes std.  The
// mean is kept as hi + lo (two f32 values) so that x - mean loses nothing to
// the mean's own rounding when the mean is large against the spread.
__global__ void __launch_bounds__(256) norm_finalize(NormArgs a, const double2* __restrict__ part, bool wide,
                                                     float eps, float4* __restrict__ ms, float* __restrict__ mean_out,
                                                     float* __restrict__ var_out) {
  __shared__ double2 red[8];
  const long long c = blockIdx.x;
  double2 s = make_double2(0.0, 0.0);
  if (wide) {
    for (long long g = threadIdx.x; g < a.G; g += blockDim.x) s = add2(s, part[g * a.C + c]);
  } else {
    const long long cols = a.C * a.inner, m = (long long)a.G * a.inner;
    for (long long t = threadIdx.x; t < m; t += blockDim.x) {
      const long long g = t / a.inner, i = t - g * a.inner;
      s = add2(s, part[g * cols + c * a.inner + i]);
    }
  }
  s = block_sum2(s, red);
  if (threadIdx.x == 0) {
    const double n = (double)a.outer * (double)a.inner;
    const double p = (double)__ldg(a.x + c * a.inner);
    const double d = s.x / n;
    const double var = fmax(s.y / n - d * d, 0.0);
    const double mean = p + d;
    const float mean_f = (float)mean, var_f = (float)var;
    ms[c] = make_float4(mean_f, (float)(mean - (double)mean_f), sqrtf(var_f + eps), 0.0f);
    if (mean_out) mean_out[c] = mean_f;
    if (var_out) var_out[c] = var_f;
  }
}

// y = (x - mean) / std * gamma + beta, unfused, in the reference's order
// (x - mean taken as (x - hi) - lo).  Each thread handles four units one grid
// apart per pass, loads first; the passes walk the tensor from its end to its
// start, so the statistics pass's most recent reads (still in L2) come first.
template <bool AFFINE>
__device__ __forceinline__ float norm1(float v, float4 m, float g, float b) {
  const float z = __fdiv_rn(__fsub_rn(__fsub_rn(v, m.x), m.y), m.z);
  return AFFINE ? __fadd_rn(__fmul_rn(z, g), b) : z;
}

template <bool AFFINE, bool VEC, typename IDX>
__global__ void __launch_bounds__(256) norm_apply(const float* __restrict__ x, float* __restrict__ y,
                                                  const float4* __restrict__ ms, const float* __restrict__ gamma,
                                                  const float* __restrict__ beta, long long n, long long C_,
                                                  long long inner_, unsigned in_m, int in_l, unsigned c_m, int c_l) {
  constexpr int U = 4;
  const IDX units = (IDX)(VEC ? n / 4 : n), C = (IDX)C_, inner = (IDX)inner_;
  const IDX nthreads = (IDX)gridDim.x * blockDim.x;
  const IDX tid = (IDX)blockIdx.x * blockDim.x + threadIdx.x;
  const IDX per = nthreads * U;
  for (IDX pass = (units + per - 1) / per; pass-- > 0;) {
    const IDX base = pass * per + tid;
    float4 v[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const IDX u = base + (IDX)k * nthreads;
      if (u < units) {
        if (VEC)
          v[k] = __ldg(reinterpret_cast<const float4*>(x) + u);
        else
          v[k].x = __ldg(x + u);
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const IDX u = base + (IDX)k * nthreads;
      if (u >= units) continue;
      const IDX e = VEC ? u * 4 : u;
      IDX c;
      if constexpr (sizeof(IDX) == 4) {  // e < 2^31: channel by multiply-high divisions
        const unsigned q = fast_div((unsigned)e, in_m, in_l);
        c = (IDX)(q - fast_div(q, c_m, c_l) * (unsigned)C);
      } else {
        c = (e / inner) % C;
      }
      const float4 m = ms[c];
      const float g = AFFINE ? __ldg(gamma + c) : 1.0f, b = AFFINE ? __ldg(beta + c) : 0.0f;
      if (VEC) {
        float4 r;
        r.x = norm1<AFFINE>(v[k].x, m, g, b);
        r.y = norm1<AFFINE>(v[k].y, m, g, b);
        r.z = norm1<AFFINE>(v[k].z, m, g, b);
        r.w = norm1<AFFINE>(v[k].w, m, g, b);
        reinterpret_cast<float4*>(y)[u] = r;
      } else {
        y[u] = norm1<AFFINE>(v[k].x, m, g, b);
      }
    }
  }
}

}  // namespace

extern "C" {

int jx_conv1d_f32(const float* x, const float* w, float* y, int64_t batch, int64_t in_channels,
                  int64_t out_channels, int64_t input_len, int64_t kernel_len, int64_t stride, int64_t padding,
                  jx_stream_t stream) {
  JX_TRACE("jx_conv1d_f32");
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
  a.y = y;
  a.B = batch;
  a.C = in_channels;
  a.L = input_len;
  a.O = out_channels;
  a.K = kernel_len;
  a.S = stride;
  a.P = padding;
  a.OL = OL;
  a.one = 1.0f;
  a.xw = (int)((C1_POS - 1) * stride + kernel_len);
  const long long per_ic = (long long)kernel_len * C1_OC + a.xw;  // floats per input channel of a chunk
  const long long budget = 48 * 1024 / 4;                          // floats per buffer
  a.icc = (int)std::max(1LL, std::min({16LL, (long long)in_channels, budget / per_ic}));
  a.buf_floats = (int)((a.icc * per_ic + 3) / 4 * 4);
  const size_t smem = (size_t)2 * a.buf_floats * 4;
  JX_REQUIRE(smem <= 220 * 1024, "jx_conv1d_f32: window too large for shared memory");
  void (*kern)(Conv1dArgs) = stride == 1 ? (kernel_len == 3 ? conv1d_kernel<1, 3> : conv1d_kernel<1, 0>)
                            : stride == 2 ? conv1d_kernel<2, 0> : conv1d_kernel<0, 0>;
  if (smem > 48 * 1024)
    JX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const dim3 grid((unsigned)((OL + C1_POS - 1) / C1_POS), (unsigned)((out_channels + C1_OC - 1) / C1_OC),
                  (unsigned)batch);
  cudaStream_t st = jx::as_stream(stream);
  a.Opad = (out_channels + C1_OC - 1) / C1_OC * C1_OC;
  const long long ck = in_channels * kernel_len;
  void* ws = nullptr;
  if (int rc = jx::scratch_get((size_t)(ck * a.Opad) * sizeof(float), &ws, st)) return rc;
  a.wt = static_cast<const float*>(ws);
  conv1d_filter_kernel<<<grid_for(ck * a.Opad, 256, 8), 256, 0, st>>>(w, static_cast<float*>(ws), out_channels, ck,
                                                                       a.Opad);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    kern<<<grid, C1_THREADS, smem, st>>>(a);
    e = cudaGetLastError();
  }
  const int rc = e == cudaSuccess ? JX_OK : jx::check_cuda(e, "conv1d kernels");
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

int jx_pool2d_f32(const float* x, float* y, int64_t batch, int64_t channels, int64_t input_h, int64_t input_w,
                  int64_t pool_h, int64_t pool_w, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
                  int op, jx_stream_t stream) {
  JX_TRACE("jx_pool2d_f32");
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
  const bool small = total + 256LL * 16 * jx::num_sms() < (1LL << 31) && a.N * a.H * a.W < (1LL << 31);
  if (small) {
    fast_div_params((unsigned)a.OW, a.ow_m, a.ow_l);
    fast_div_params((unsigned)a.OH, a.oh_m, a.oh_l);
  }
  cudaStream_t st = jx::as_stream(stream);
  if (op == JX_POOL_MAX) {
    if (small)
      launch_pool<true, unsigned>(a, st);
    else
      launch_pool<true, long long>(a, st);
  } else {
    if (small)
      launch_pool<false, unsigned>(a, st);
    else
      launch_pool<false, long long>(a, st);
  }
  JX_LAUNCH_CHECK("pool2d_kernel");
  return JX_OK;
}

int jx_maxpool2d_f32(const float* x, float* y, int64_t batch, int64_t channels, int64_t input_h, int64_t input_w,
                     int64_t pool_h, int64_t pool_w, int64_t stride, int64_t padding, jx_stream_t stream) {
  JX_TRACE("jx_maxpool2d_f32");
  return jx_pool2d_f32(x, y, batch, channels, input_h, input_w, pool_h, pool_w, stride, stride, padding, padding,
                       JX_POOL_MAX, stream);
}

int jx_avgpool2d_f32(const float* x, float* y, int64_t batch, int64_t channels, int64_t input_h, int64_t input_w,
                     int64_t pool_h, int64_t pool_w, int64_t stride, int64_t padding, jx_stream_t stream) {
  JX_TRACE("jx_avgpool2d_f32");
  return jx_pool2d_f32(x, y, batch, channels, input_h, input_w, pool_h, pool_w, stride, stride, padding, padding,
                       JX_POOL_AVG, stream);
}

int jx_global_pool2d_f32(const float* x, float* y, int64_t batch, int64_t channels, int64_t height, int64_t width,
                         int op, jx_stream_t stream) {
  JX_TRACE("jx_global_pool2d_f32");
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
  JX_TRACE("jx_batchnorm_f32");
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
  const bool vec_rows = (spatial & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  long long parts;
  a.chunk = 0;
  int stats_grid = 0;
  if (wide) {
    const long long per = batch * spatial, step = vec_rows ? 1024 : 256;
    const long long target_items = 256LL * jx::num_sms();  // about 4 per resident warp
    const long long m = std::max(1LL, (channels * ((per + step - 1) / step) + target_items - 1) / target_items);
    a.chunk = m * step;
    const long long G = (per + a.chunk - 1) / a.chunk;
    JX_REQUIRE(G <= 0x7fffffffLL && channels <= 0x7fffffffLL, "jx_batchnorm_f32: too many items");
    a.G = (int)G;
    parts = G * channels;
    stats_grid = grid_for(parts * 32, 256, 8);
  } else {
    const long long target = 8LL * jx::num_sms();
    const long long cols = channels * spatial, col_blocks = (cols + 255) / 256;
    JX_REQUIRE(col_blocks <= 0x7fffffffLL, "jx_batchnorm_f32: too many columns");
    a.G = (int)std::max(1LL, std::min({(long long)batch, (target + col_blocks - 1) / col_blocks, 1024LL}));
    parts = (long long)a.G * cols;
  }
  void* ws = nullptr;
  const size_t part_bytes = (size_t)parts * sizeof(double2);
  if (int rc = jx::scratch_get(part_bytes + (size_t)channels * sizeof(float4), &ws, st)) return rc;
  double2* part = static_cast<double2*>(ws);
  float4* ms = reinterpret_cast<float4*>(static_cast<char*>(ws) + part_bytes);
  int rc = JX_OK;
  if (wide && vec_rows)
    norm_stats_items<true><<<stats_grid, 256, 0, st>>>(a, part);
  else if (wide)
    norm_stats_items<false><<<stats_grid, 256, 0, st>>>(a, part);
  else
    norm_stats_narrow<<<dim3((unsigned)((channels * spatial + 255) / 256), (unsigned)a.G), 256, 0, st>>>(a, part);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    norm_finalize<<<(unsigned)channels, 256, 0, st>>>(a, part, wide, epsilon, ms, mean_out, var_out);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    const long long n = batch * channels * spatial;
    const bool vec = (spatial & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    const int grid = grid_for(vec ? n / 4 : n, 256, 8);
    const bool small = n + 4LL * 256 * grid < (1LL << 31);
    unsigned in_m = 0, c_m = 0;
    int in_l = 0, c_l = 0;
    if (small) {
      fast_div_params((unsigned)spatial, in_m, in_l);
      fast_div_params((unsigned)channels, c_m, c_l);
    }
#define JX_NORM_APPLY(AFF, VEC)                                                                                 \
  do {                                                                                                          \
    if (small)                                                                                                  \
      norm_apply<AFF, VEC, unsigned><<<grid, 256, 0, st>>>(x, y, ms, gamma, beta, n, channels, spatial, in_m, in_l, \
                                                           c_m, c_l);                                          \
    else                                                                                                        \
      norm_apply<AFF, VEC, long long><<<grid, 256, 0, st>>>(x, y, ms, gamma, beta, n, channels, spatial, 0, 0, 0, \
                                                            0);                                                 \
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
