// conv.cu -- conv2d forward, input gradient and weight gradient on the
// tcgen05 3xTF32 GEMM core.
//
// Replaces nn::conv2d_batched (src/nn.rs:2048-2144: NCHW input, OIHW weight,
// stride and zero padding, the CPU loop b -> oc -> oh -> ow -> ic -> kh -> kw)
// and gpu_conv2d (src/backend/ops.rs:815-998: one output per thread, no data
// reuse, forward only).  The reference has no conv backward; dX and dW here
// are the exact adjoints of its forward loop.
//
// Implicit GEMM (conv_gemm_kernel).  With K = C*KH*KW and P = OH*OW:
//   forward   Y[O, (b,p)]      = W[O, (c,kh,kw)]  . X gathered at (b,p),(c,kh,kw)
//   input     dX[C, (b,ih,iw)] = W'[C, (o,kh,kw)] . dY gathered at (b,ih,iw),(o,kh,kw)
//   weight    dW[O, (c,kh,kw)] = sum over slices of dY[O, (b,p)] . X gathered
// The A operand (filter, or dY for the weight gradient) is split into tf32
// hi/lo once and streamed by TMA.  The B operand is never stored: the eight
// epilogue warps of the GEMM gather it straight from the NCHW tensor every
// k-block (bounds and stride tests from a per-index offset table in shared
// memory), split it, and write the hi/lo tiles into the stage in the layout
// TMA would have produced, then publish them to the tensor core with
// fence.proxy.async before arriving on the stage's barrier.  The same warps
// drain the TMEM span partials and store the tile (NCHW for the forward and
// the input gradient).  The weight-gradient contraction over B*P is split in
// slices whose partial products are added in slice order.
//
// Shapes outside the implicit kernel's limits (table of more than 4096
// indices, more than 32 filter taps) take the explicit path:
// fused im2col+split producers into scratch, the plain GEMM, col2im.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "tc_gemm.cuh"

namespace jx {
int gemm_presplit_err(const float* Ah, const float* Al, const float* Bh, const float* Bl, float* C, int M, int N,
                      int Kp, long long ldc, long long strideC, int batch, cudaStream_t st, unsigned int* err,
                      bool a_bcast, bool b_bcast);
int gemm_split_operand(const float* src, float* hi, float* lo, int rows, int K, int Kp, long long ld, long long sb,
                       int batch, bool transposed, cudaStream_t st);
long long gemm_kpad(long long K);
}  // namespace jx

namespace {

struct Geo {
  int C, H, W, O, KH, KW, S, P, OH, OW;
  __host__ __device__ int K() const { return C * KH * KW; }
  __host__ __device__ int NP() const { return OH * OW; }
};

// Forward B operand: rows (b, p) of Kp values, element k = (c, kh, kw) is
// x[b, c, oh*S + kh - P, ow*S + kw - P] (0 outside the image and for k >= K).
__global__ void im2col_rows_split(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  long long rows, int Kp, const Geo g) {
  const int K = g.K(), kk = g.KH * g.KW, np = g.NP();
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const long long b = r / np;
    const int p = (int)(r - b * np);
    const int oh = p / g.OW, ow = p - (p / g.OW) * g.OW;
    const float* xb = x + b * g.C * g.H * g.W;
    float* hr = hi + r * Kp;
    float* lr = lo + r * Kp;
    for (int k = threadIdx.x; k < Kp; k += blockDim.x) {
      float v = 0.0f;
      if (k < K) {
        const int c = k / kk, rem = k - (k / kk) * kk;
        const int kh = rem / g.KW, kw = rem - (rem / g.KW) * g.KW;
        const int ih = oh * g.S + kh - g.P, iw = ow * g.S + kw - g.P;
        if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) v = __ldg(xb + ((long long)c * g.H + ih) * g.W + iw);
      }
      float h, l;
      jxd::split_tf32(v, h, l);
      hr[k] = h;
      lr[k] = l;
    }
  }
}

// Weight-gradient B operand: for slice s, row k holds x at q = s*Ks + j for
// j < Ksp (q = b*P + p over all images and output pixels; 0 past the end).
__global__ void im2col_cols_split(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  long long Q, long long Ks, int Ksp, int S_slices, const Geo g) {
  const int K = g.K(), kk = g.KH * g.KW, np = g.NP();
  const long long rows = (long long)S_slices * K;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const int s = (int)(r / K);
    const int k = (int)(r - (long long)s * K);
    const int c = k / kk, rem = k - (k / kk) * kk;
    const int kh = rem / g.KW, kw = rem - (rem / g.KW) * g.KW;
    float* hr = hi + r * Ksp;
    float* lr = lo + r * Ksp;
    for (int j = threadIdx.x; j < Ksp; j += blockDim.x) {
      const long long q = (long long)s * Ks + j;
      float v = 0.0f;
      if (j < Ks && q < Q) {
        const long long b = q / np;
        const int p = (int)(q - b * np);
        const int oh = p / g.OW, ow = p - (p / g.OW) * g.OW;
        const int ih = oh * g.S + kh - g.P, iw = ow * g.S + kw - g.P;
        if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W)
          v = __ldg(x + ((b * g.C + c) * g.H + ih) * (long long)g.W + iw);
      }
      float h, l;
      jxd::split_tf32(v, h, l);
      hr[j] = h;
      lr[j] = l;
    }
  }
}

// Weight-gradient A operand: for slice s, row o holds dY[b, o, p] at q = b*P + p.
// A thread writes 4 consecutive positions (16-byte hi and lo stores; Ksp is
// a multiple of 32) and divides once per 4: Q < 2^31, so 32-bit division.
__global__ void dy_rows_split(const float* __restrict__ dy, float* __restrict__ hi, float* __restrict__ lo,
                              long long Q, long long Ks, int Ksp, int S_slices, const Geo g) {
  const unsigned np = (unsigned)g.NP();
  const long long rows = (long long)S_slices * g.O;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const int s = (int)(r / g.O);
    const int o = (int)(r - (long long)s * g.O);
    float4* hr = reinterpret_cast<float4*>(hi + r * Ksp);
    float4* lr = reinterpret_cast<float4*>(lo + r * Ksp);
    const long long qs = (long long)s * Ks;
    for (int j4 = threadIdx.x; j4 < Ksp / 4; j4 += blockDim.x) {
      const int j0 = 4 * j4;
      const unsigned q0 = (unsigned)(qs + j0);
      unsigned b = q0 / np, p = q0 - b * np;
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const long long q = qs + j0 + e;
        v[e] = (j0 + e < Ks && q < Q) ? __ldg(dy + ((long long)b * g.O + o) * (long long)np + p) : 0.0f;
        if (++p == np) {
          p = 0;
          ++b;
        }
      }
      float4 h, l;
      jxd::split_tf32(v[0], h.x, l.x);
      jxd::split_tf32(v[1], h.y, l.y);
      jxd::split_tf32(v[2], h.z, l.z);
      jxd::split_tf32(v[3], h.w, l.w);
      hr[j4] = h;
      lr[j4] = l;
    }
  }
}

// dx[b, c, ih, iw] = sum over (kh, kw) with oh*S = ih + P - kh and
// ow*S = iw + P - kw in range of dcol[b, (c, kh, kw), (oh, ow)].
__global__ void col2im_gather(const float* __restrict__ dcol, float* __restrict__ dx, long long nb, const Geo g) {
  const long long total = nb * g.C * g.H * g.W;
  const int K = g.K(), np = g.NP();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int iw = (int)(i % g.W);
    const int ih = (int)((i / g.W) % g.H);
    const int c = (int)((i / ((long long)g.W * g.H)) % g.C);
    const long long b = i / ((long long)g.W * g.H * g.C);
    const float* db = dcol + b * (long long)K * np;
    float acc = 0.0f;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int th = ih + g.P - kh;
      if (th < 0 || th % g.S) continue;
      const int oh = th / g.S;
      if (oh >= g.OH) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int tw = iw + g.P - kw;
        if (tw < 0 || tw % g.S) continue;
        const int ow = tw / g.S;
        if (ow >= g.OW) continue;
        acc += db[((long long)(c * g.KH + kh) * g.KW + kw) * np + oh * g.OW + ow];
      }
    }
    dx[i] = acc;
  }
}

// out[i] = sum over s of part[s * n + i], in slice order.
__global__ void slice_sum(const float* __restrict__ part, float* __restrict__ out, long long n, int slices) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (int s = 0; s < slices; ++s) acc += part[(long long)s * n + i];
    out[i] = acc;
  }
}

// ---------------------------------------------------------------------------
// Implicit GEMM
// ---------------------------------------------------------------------------
using jxg::A_TILE;
using jxg::B_TILE;
using jxg::BK;
using jxg::BM;
using jxg::BN;
using jxg::EPI_COLS;
using jxg::EPI_WARPS;
using jxg::SPAN_KB;
using jxg::STAGE_BYTES;
using jxg::STAGES;
using jxg::TMEM_COLS;
using jxg::PAIR_OP;
using jxg::PAIR_ROWS;
using jxg::PAIR_TILE;
using jxg::TileInfo;
using jxg::pair_tile_coords;

// Warps: warpgroup 0 = TMA (warp 0), MMA issuer and TMEM owner (warp 1), two
// idle warps; warpgroups 1 and 2 (warps 4..11) gather, drain and store.  The
// block launches with 168 registers per thread (384 x 168 = 64,512); warpgroup
// 0 gives all but 40 back (setmaxnreg.dec) and the gathering warpgroups take
// 232 each (setmaxnreg.inc): 128 x 40 + 256 x 232 = 64,512, the launch total.
constexpr int CONV_THREADS = 384;
constexpr int CONV_FIRST_EPI = 4;
constexpr int CONV_LAUNCH_REGS = 168;
constexpr int CONV_LOW_REGS = 40;
constexpr int CONV_HIGH_REGS = 232;
static_assert(128 * CONV_LOW_REGS + 256 * CONV_HIGH_REGS <= CONV_THREADS * CONV_LAUNCH_REGS,
              "register split exceeds the launch allocation");
constexpr int TABLE_MAX = 4096;  // gather indices held in shared memory
constexpr int BAR_BYTES = 256;
constexpr size_t IMPLICIT_SMEM = (size_t)STAGES * STAGE_BYTES + BAR_BYTES + TABLE_MAX * 8 + 1024 /*align*/;

// Gather table entry for one index of the gathered dimension (k in rows
// mode, the GEMM column in cols mode):
//   x = element offset of the index from a position's base (channel plane + tap)
//   y = 1 << (kh * KW + kw), the index's filter tap; 0 for a padding entry.
// A position (a pixel, with its own base pointer) keeps a mask of the taps
// that land inside the gathered tensor; the element is base[x] when
// (mask & y) != 0, else 0.
struct ImplicitArgs {
  int M, N, num_kb;                  // GEMM rows, columns, contraction k-blocks
  int tiles_m, tiles_n, num_tiles;   // num_tiles = tiles_m * tiles_n * slices
  int a_bcast;                       // A has one batch entry (the filter)
  int table_n;
  int LH, LW;                        // spatial extent of the gathered tensor
  int KH, KW, S, P;                  // filter extent, stride, padding
  long long img_stride;              // elements per image of the gathered tensor
  // rows mode (forward, input gradient): B rows are pixels of a PH x PW grid
  int PW, NPpix, dx_mode;
  long long out_img_stride;          // M * NPpix: NCHW output
  // cols mode (weight gradient): B columns are output pixels q of all images
  int Q, Ks;                         // contraction length, per-slice length
  int OW, NPo;
  unsigned npo_m, ow_m;              // q / NPo and p / OW as multiply-high (Granlund-Montgomery)
  int npo_l, ow_l;
  long long ldc, strideC;            // row-major partial outputs per slice
  int Ksp;                           // per-slice stride of the contraction (k-blocks * BK)
  const uint2* pixtab;               // conv_pair_kernel, cols mode: per contraction position
                                     // (offset of its base from src, tap mask), [slices][Ksp]
};

// Table of the gathered index: TAB_FWD (c,kh,kw) over x; TAB_DX (o,kh,kw)
// over dY; entries [count, n) are padding.
enum { TAB_FWD = 0, TAB_DX = 1 };
__global__ void build_gather_table(uint2* __restrict__ tab, int n, int count, int mode, const Geo g) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int kk = g.KH * g.KW;
  if (i >= count) {
    tab[i] = make_uint2(0u, 0u);
    return;
  }
  const int ch = i / kk, r = i - (i / kk) * kk;
  const int kh = r / g.KW, kw = r - (r / g.KW) * g.KW;
  if (mode == TAB_FWD) {
    // x[b, c, oh*S - P + kh, ow*S - P + kw]: base at (oh*S - P, ow*S - P)
    tab[i] = make_uint2((uint32_t)(ch * g.H * g.W + kh * g.W + kw), 1u << r);
  } else {
    // dY[b, o, oh, ow] with oh*S = ih + P - kh: writing ih + P = S*qh + rh, tap
    // kh contributes iff kh % S == rh, at oh = qh - kh / S (base at (qh, qw))
    tab[i] = make_uint2((uint32_t)(ch * g.OH * g.OW - (kh / g.S) * g.OW - (kw / g.S)), 1u << r);
  }
}

// Taps of a position that read inside the gathered tensor.  Forward and
// weight gradient: input row qh + kh (qh = oh*S - P).  Input gradient: tap kh
// needs kh % S == rh and output row qh - kh / S.
__device__ __forceinline__ uint32_t tap_mask(int qh, int qw, int rh, int rw, const ImplicitArgs& a, bool dx) {
  uint32_t cols = 0;
  for (int kw = 0; kw < a.KW; ++kw) {
    const int w = dx ? qw - kw / a.S : qw + kw;
    const bool ok = (!dx || kw % a.S == rw) && (unsigned)w < (unsigned)a.LW;
    cols |= ok ? 1u << kw : 0u;
  }
  uint32_t m = 0;
  for (int kh = 0; kh < a.KH; ++kh) {
    const int h = dx ? qh - kh / a.S : qh + kh;
    const bool ok = (!dx || kh % a.S == rh) && (unsigned)h < (unsigned)a.LH;
    m |= ok ? cols << (kh * a.KW) : 0u;
  }
  return m;
}

// One predicated load: base[off] when ok != 0, else 0 (no branch).
__device__ __forceinline__ float gather_one(const float* base, int off, uint32_t ok) {
  float v = 0.0f;
  asm("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %2, 0;\n\t@p ld.global.nc.f32 %0, [%1];\n\t}"
      : "+f"(v)
      : "l"(base + off), "r"(ok));
  return v;
}

// Rows mode (forward, input gradient): the base pointer and tap mask of B
// row n, the flattened output pixel (forward) or input pixel (input
// gradient) n = b * NPpix + p.  Rows past N keep mask 0 (zeros).
__device__ __forceinline__ void row_position(const float* src, long long n, const ImplicitArgs& a, const float*& base,
                                             uint32_t& mask) {
  if (n >= a.N) return;
  const long long b = n / a.NPpix;
  const int p = (int)(n - b * a.NPpix);
  const int ph = p / a.PW, pw = p - (p / a.PW) * a.PW;
  int qh, qw, rh = 0, rw = 0;
  if (a.dx_mode) {
    const int th = ph + a.P, tw = pw + a.P;
    qh = th / a.S;
    rh = th - qh * a.S;
    qw = tw / a.S;
    rw = tw - qw * a.S;
  } else {
    qh = ph * a.S - a.P;
    qw = pw * a.S - a.P;
  }
  mask = tap_mask(qh, qw, rh, rw, a, a.dx_mode != 0);
  base = src + (b * a.img_stride + (long long)qh * a.LW + qw);
}

// Cols mode (weight gradient): the base pointer and tap mask of contraction
// position jq of slice `slice`, the output pixel q = slice * Ks + jq of all
// images; positions past the slice or past Q get mask 0.
__device__ __forceinline__ void col_offset(int jq, int slice, const ImplicitArgs& a, long long& off, uint32_t& gmask) {
  const long long q = (long long)slice * a.Ks + jq;
  gmask = 0;
  off = 0;
  if (jq < a.Ks && q < a.Q) {
    const int qi = (int)q;
    // qi < 2^31: n / d = (umulhi(n, m) + n) >> l with the host's (m, l)
    const int b = (int)((__umulhi((unsigned)qi, a.npo_m) + (unsigned)qi) >> a.npo_l);
    const int p = qi - b * a.NPo;
    const int oh = (int)((__umulhi((unsigned)p, a.ow_m) + (unsigned)p) >> a.ow_l), ow = p - oh * a.OW;
    const int qh = oh * a.S - a.P, qw = ow * a.S - a.P;
    gmask = tap_mask(qh, qw, 0, 0, a, false);
    off = (long long)b * a.img_stride + (long long)qh * a.LW + qw;
  }
}
__device__ __forceinline__ void col_position(const float* src, int jq, int slice, const ImplicitArgs& a,
                                             const float*& gbase, uint32_t& gmask) {
  long long off;
  col_offset(jq, slice, a, off, gmask);
  if (gmask) gbase = src + off;
}

// The cols-mode position table of conv_pair_kernel: entry s * Ksp + j =
// (offset from src of position j of slice s, its tap mask), mask 0 past the
// slice or past Q.  Offsets fit 32 bits (the host checks the whole tensor).
__global__ void build_pixel_table(uint2* __restrict__ tq, long long n, const ImplicitArgs a) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int s = (int)(i / a.Ksp), j = (int)(i - (long long)s * a.Ksp);
    long long off;
    uint32_t m;
    col_offset(j, s, a, off, m);
    tq[i] = make_uint2((uint32_t)(int)off, m);
  }
}

// Store one epilogue thread's EPI_COLS outputs of row m, columns n0.. of the
// GEMM.  Rows mode: NCHW, out[b, m, p] for the flattened pixel n = b * NPpix
// + p; cols mode: row-major partial output of slice b.
template <bool COLS>
__device__ __forceinline__ void store_tile(const float (&acc)[EPI_COLS], const ImplicitArgs& a, int m, long long n0,
                                           int slice, float* __restrict__ out) {
  if (m >= a.M) return;
  if constexpr (!COLS) {
    long long b = n0 / a.NPpix;
    int p = (int)(n0 - b * a.NPpix);
    float* ob = out + b * a.out_img_stride + (long long)m * a.NPpix;
    const long long nlim = a.N - n0;
    if ((a.NPpix & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
      for (int v4 = 0; v4 < EPI_COLS / 4; ++v4) {
        if (4 * v4 < nlim)
          *reinterpret_cast<float4*>(ob + p) = make_float4(acc[4 * v4], acc[4 * v4 + 1], acc[4 * v4 + 2], acc[4 * v4 + 3]);
        p += 4;
        if (p == a.NPpix) {
          p = 0;
          ob += a.out_img_stride;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) {
        if (j < nlim) ob[p] = acc[j];
        if (++p == a.NPpix) {
          p = 0;
          ob += a.out_img_stride;
        }
      }
    }
  } else {
    float* crow = out + (long long)slice * a.strideC + (long long)m * a.ldc;
    const long long nlim = a.N - n0;
    if ((a.ldc & 3) == 0 && (a.strideC & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
        nlim >= EPI_COLS) {
      float4* dst = reinterpret_cast<float4*>(crow + n0);
#pragma unroll
      for (int v4 = 0; v4 < EPI_COLS / 4; ++v4)
        dst[v4] = make_float4(acc[4 * v4], acc[4 * v4 + 1], acc[4 * v4 + 2], acc[4 * v4 + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j)
        if (j < nlim) crow[n0 + j] = acc[j];
    }
  }
}

// COLS = false: forward / input gradient (B rows = pixels, k = gathered index)
// COLS = true:  weight gradient (B rows = gathered index, k = output pixels)
template <bool COLS>
__global__ void __launch_bounds__(CONV_THREADS, 1)
    conv_gemm_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                     const float* __restrict__ src, const uint2* __restrict__ table, const ImplicitArgs a,
                     float* __restrict__ out, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = jxd::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;                     // [STAGES] A landed + B written
  uint64_t* empty = bars + STAGES;           // [STAGES] MMA done with the stage
  uint64_t* sfull = bars + 2 * STAGES;       // [2] span partial ready
  uint64_t* sempty = bars + 2 * STAGES + 2;  // [2] span partial drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint2* tab = reinterpret_cast<uint2*>(smem + STAGES * STAGE_BYTES + BAR_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = a.num_kb;

  for (int i = threadIdx.x; i < a.table_n; i += blockDim.x) tab[i] = table[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      jxd::mbar_init(&full[s], 1 + EPI_WARPS);  // TMA's expect_tx arrive + one per gathering warp
      jxd::mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      jxd::mbar_init(&sfull[s], 1);
      jxd::mbar_init(&sempty[s], EPI_WARPS);
    }
    *abort_flag = 0;
    jxd::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    jxd::tma_prefetch_desc(&tmAh);
    jxd::tma_prefetch_desc(&tmAl);
  }
  if (warp == 1) {
    jxd::tmem_alloc(tmem_slot, TMEM_COLS);
    jxd::tmem_relinquish();
  }
  jxd::tc_fence_before();
  __syncthreads();
  jxd::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < CONV_FIRST_EPI) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(CONV_LOW_REGS));
    // ---------------- TMA: A operand (hi, lo) ----------------
    if (warp == 0 && jxd::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < a.num_tiles && !*abort_flag; t += gridDim.x) {
        const jxg::TileInfo ti = jxg::tile_coords(t, a.tiles_m, a.tiles_n);
        const int ya = ti.m_blk * BM, za = a.a_bcast ? 0 : ti.b;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!jxg::wait_bounded(&empty[stage], phase ^ 1u, err)) { *abort_flag = 1; break; }
          uint8_t* st = smem + stage * STAGE_BYTES;
          jxd::mbar_arrive_expect_tx(&full[stage], 2 * A_TILE);
          jxd::tma_load_3d(st, &tmAh, &full[stage], kb * BK, ya, za);
          jxd::tma_load_3d(st + A_TILE, &tmAl, &full[stage], kb * BK, ya, za);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      for (int s = 0; s < STAGES; ++s) {
        if (!jxg::wait_bounded(&empty[stage], phase ^ 1u, err)) break;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
    // ---------------- MMA issuer ----------------
    if (warp == 1 && jxd::elect_one())
      jxg::mma_issuer(smem, full, empty, sfull, sempty, tmem_base, a.num_tiles, num_kb, abort_flag, err);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(CONV_HIGH_REGS));
    // ---------------- gather B, drain spans, store ----------------
    const int gw = warp - CONV_FIRST_EPI;  // 0..7
    const int q4 = warp & 3, half = gw >> 2;
    int stage = 0;
    uint32_t phase = 0;
    uint32_t span_ctr = 0;
    for (int t = blockIdx.x; t < a.num_tiles; t += gridDim.x) {
      const jxg::TileInfo ti = jxg::tile_coords(t, a.tiles_m, a.tiles_n);
      float acc[EPI_COLS];
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.0f;
      // rows mode: this thread's B row is one pixel for the whole tile
      const float* base = src;
      uint32_t mask = 0;
      if constexpr (!COLS) row_position(src, (long long)ti.n_blk * BN + gw * 32 + lane, a, base, mask);
      bool ok = true;
      int spans_done = 0;
      const int nspan = (num_kb + SPAN_KB - 1) / SPAN_KB;
      // gather(v, kb): issue k-block kb's 32 loads (no wait on the stage).
      auto gather = [&](float (&v)[32], int kb) {
        const float* gbase = base;
        uint32_t gmask = mask;
        if constexpr (COLS) col_position(src, kb * BK + lane, ti.b, a, gbase, gmask);
        const uint4* te = reinterpret_cast<const uint4*>(COLS ? tab + ti.n_blk * BN + gw * 32 : tab + kb * BK);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint4 e = te[i];
          v[2 * i] = gather_one(gbase, (int)e.x, e.y & gmask);
          v[2 * i + 1] = gather_one(gbase, (int)e.z, e.w & gmask);
        }
      };
      // publish(v, kb): wait for the stage, write v as tf32 hi/lo, hand the
      // stage to the tensor core, and drain a span partial when one is due.
      auto publish = [&](float (&v)[32], int kb) -> bool {
        if (*abort_flag || !jxg::wait_bounded(&empty[stage], phase ^ 1u, err)) {
          *abort_flag = 1;
          return false;
        }
        uint8_t* bh = smem + stage * STAGE_BYTES + 2 * A_TILE;
        if constexpr (!COLS) {
          // row gw*32+lane, 8 chunks of 4 k values, 128-byte swizzle
          const int row = gw * 32 + lane;
          uint8_t* rp = bh + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float4 h, l;
            jxd::split_tf32(v[4 * c], h.x, l.x);
            jxd::split_tf32(v[4 * c + 1], h.y, l.y);
            jxd::split_tf32(v[4 * c + 2], h.z, l.z);
            jxd::split_tf32(v[4 * c + 3], h.w, l.w);
            const int off = (c ^ (row & 7)) << 4;
            *reinterpret_cast<float4*>(rp + off) = h;
            *reinterpret_cast<float4*>(rp + B_TILE + off) = l;
          }
        } else {
          // rows gw*32 + r, this lane's k position within each 128-byte row
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const int row = gw * 32 + r;
            float h, l;
            jxd::split_tf32(v[r], h, l);
            const int off = row * 128 + (((lane >> 2) ^ (row & 7)) << 4) + ((lane & 3) << 2);
            *reinterpret_cast<float*>(bh + off) = h;
            *reinterpret_cast<float*>(bh + B_TILE + off) = l;
          }
        }
        jxd::fence_proxy_async_smem();  // make the generic-proxy writes visible to the tensor core
        __syncwarp();
        if (lane == 0) jxd::mbar_arrive(&full[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        // Once span i is fully written, drain span i-1 (its MMAs have been
        // issued before any of span i's could be).
        if ((kb % SPAN_KB == SPAN_KB - 1 || kb == num_kb - 1) && kb >= SPAN_KB) {
          if (!jxg::drain_span<32, CONV_FIRST_EPI>(acc, tmem_base, span_ctr, sfull, sempty, warp, lane, abort_flag,
                                                   err))
            return false;
          ++span_ctr;
          ++spans_done;
        }
        return true;
      };
      // Software pipeline: k-block kb+1's loads are in flight while k-block kb
      // waits for its stage and is written.
      float va[32], vb[32];
      if (num_kb > 0) gather(va, 0);
      for (int kb = 0; kb < num_kb; kb += 2) {
        if (kb + 1 < num_kb) gather(vb, kb + 1);
        if (!publish(va, kb)) { ok = false; break; }
        if (kb + 1 < num_kb) {
          if (kb + 2 < num_kb) gather(va, kb + 2);
          if (!publish(vb, kb + 1)) { ok = false; break; }
        }
      }
      while (ok && spans_done < nspan) {
        if (!jxg::drain_span<32, CONV_FIRST_EPI>(acc, tmem_base, span_ctr, sfull, sempty, warp, lane, abort_flag, err)) ok = false;
        ++span_ctr;
        ++spans_done;
      }
      if (!ok) break;
      // ---- store ----
      store_tile<COLS>(acc, a, ti.m_blk * BM + q4 * 32 + lane, (long long)ti.n_blk * BN + half * EPI_COLS, ti.b,
                       out);
    }
  }

  jxd::tc_fence_before();
  __syncthreads();
  jxd::tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    jxd::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Implicit GEMM on SM pairs
// ---------------------------------------------------------------------------
// conv_pair_kernel: the same three convolutions on the pair MMA
// (tcgen05.mma.cta_group::2, a 256 x 256 tile per cluster of two CTAs).
// CTA r of the pair holds rows 128r.. of the tile's A operand (the filter's
// or dY's hi and lo, by TMA) and gathers rows 128r.. of its B operand, so an
// SM gathers 128 B rows per k-block instead of conv_gemm_kernel's 256 for
// the same tensor-core work, and a stage takes 64 KB instead of 96, which
// leaves room for three stages instead of two.
//
//   warp 0 (each CTA)    TMA: this CTA's A hi / lo slices
//   warp 1 (even CTA)    TMEM (both CTAs) + the pair MMA issuer
//   warp 2 (each CTA)    forwards gfull[s] completions to the even CTA's full[s]
//   warp 3 (each CTA)    forwards gempty[p] completions to the even CTA's sempty[p]
//   warps 4..11 (each)   gather B, drain the TMEM spans, store
// The forwarders keep the gathering warps from ever waiting on their own
// group: a warp arrives locally and moves on to its next k-block.
//
// Rows mode: B row = one pixel; the two warps of a TMEM lane quarter share
// 32 pixels and take 16 of the k-block's 32 gathered indices each.  Cols
// mode: B row = one gathered index; a thread takes 4 rows at 4 consecutive
// output pixels of the k-block, whose base offsets and tap masks come from a
// table built once per call (build_pixel_table), and writes one 16-byte
// chunk per row.
//
// Handshakes (every wait bounded, about 4 s, then JX_DEVERR_TIMEOUT):
//   gfull[s]  (each CTA)  TMA's expect_tx arrival + one per gathering warp
//   full[s]   (even CTA)  one arrival per CTA, by its warp 2 once gfull[s]
//                         completes (cluster-scope release)
//   empty[s]  (each CTA)  the pair's MMAs on stage s retired (multicast commit)
//   sfull[p]  (each CTA)  span buffer p holds a finished partial (multicast)
//   gempty[p] (each CTA)  one arrival per draining warp; sempty[p] (even
//                         CTA) one per CTA, by its warp 3
constexpr int CP_STAGES = 3;
// k-blocks whose gathers are in flight ahead of the one being written
// (forward at [64,256,56,56]: 1.149 / 0.973 / 1.022 ms with 1 / 2 / 3 ahead;
// with 2 ahead the gathering warps spill a few dozen bytes, with 3 more)
constexpr int CP_AHEAD = 2;
constexpr int CP_STAGE = 4 * PAIR_OP;  // [A hi][A lo][B hi][B lo], 16 KB each
constexpr size_t CP_SMEM = (size_t)CP_STAGES * CP_STAGE + BAR_BYTES + TABLE_MAX * 8 + 1024 /*align*/;
static_assert(CP_SMEM <= 232448, "conv_pair_kernel shared memory exceeds the per-block limit");
static_assert(EPI_COLS == PAIR_TILE / 2, "two draining warps per TMEM lane quarter split the tile's columns");
static_assert(BN == PAIR_TILE, "gather tables are padded to whole tiles of either kernel");

template <bool COLS>
__global__ void __launch_bounds__(CONV_THREADS, 1)
    conv_pair_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                     const float* __restrict__ src, const uint2* __restrict__ table, const ImplicitArgs a,
                     float* __restrict__ out, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = jxd::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CP_STAGES * CP_STAGE);
  uint64_t* gfull = bars;                       // [CP_STAGES] local
  uint64_t* full = bars + CP_STAGES;            // [CP_STAGES] (even CTA)
  uint64_t* empty = bars + 2 * CP_STAGES;       // [CP_STAGES]
  uint64_t* sfull = bars + 3 * CP_STAGES;       // [2]
  uint64_t* sempty = bars + 3 * CP_STAGES + 2;  // [2] (even CTA)
  uint64_t* gempty = bars + 3 * CP_STAGES + 4;  // [2] local
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * CP_STAGES + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint2* tab = reinterpret_cast<uint2*>(smem + CP_STAGES * CP_STAGE + BAR_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = jxd::cluster_ctarank();  // 0 or 1 within the pair
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_kb = a.num_kb;

  for (int i = threadIdx.x; i < a.table_n; i += blockDim.x) tab[i] = table[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < CP_STAGES; ++s) {
      jxd::mbar_init(&gfull[s], 1 + EPI_WARPS);
      jxd::mbar_init(&full[s], 2);
      jxd::mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      jxd::mbar_init(&sfull[s], 1);
      jxd::mbar_init(&sempty[s], 2);
      jxd::mbar_init(&gempty[s], EPI_WARPS);
    }
    *abort_flag = 0;
    jxd::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    jxd::tma_prefetch_desc(&tmAh);
    jxd::tma_prefetch_desc(&tmAl);
  }
  if (warp == 1) {
    jxd::tmem_alloc_pair(tmem_slot, 2 * PAIR_TILE);
    jxd::tmem_relinquish_pair();
  }
  jxd::tc_fence_before();
  __syncthreads();
  jxd::cluster_sync_all();  // the peer's barriers are initialised before anyone signals them
  jxd::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full0 = jxd::mapa_shared(&full[0], 0), sempty0 = jxd::mapa_shared(&sempty[0], 0);

  if (warp < CONV_FIRST_EPI) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(CONV_LOW_REGS));
    if (warp == 0 && jxd::elect_one()) {
      // ---------------- TMA: this CTA's A hi / lo slices ----------------
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < a.num_tiles && !*abort_flag; t += npairs) {
        const TileInfo ti = pair_tile_coords(t, a.tiles_m, a.tiles_n);
        const int ya = ti.m_blk * PAIR_TILE + (int)rank * PAIR_ROWS, za = a.a_bcast ? 0 : ti.b;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!jxg::wait_bounded(&empty[stage], phase ^ 1u, err)) { *abort_flag = 1; break; }
          uint8_t* st = smem + stage * CP_STAGE;
          jxd::mbar_arrive_expect_tx(&gfull[stage], 2 * PAIR_OP);
          jxd::tma_load_3d(st, &tmAh, &gfull[stage], kb * BK, ya, za);
          jxd::tma_load_3d(st + PAIR_OP, &tmAl, &gfull[stage], kb * BK, ya, za);
          if (++stage == CP_STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      for (int s = 0; s < CP_STAGES; ++s) {
        if (!jxg::wait_bounded(&empty[stage], phase ^ 1u, err)) break;
        if (++stage == CP_STAGES) { stage = 0; phase ^= 1u; }
      }
    }
    if (warp == 1 && rank == 0 && jxd::elect_one())
      // ---------------- pair MMA issuer (even CTA) ----------------
      jxg::pair_mma_issuer<false, false, CP_STAGES, CP_STAGE>(jxd::smem_u32(smem), full, empty, sfull, sempty,
                                                              tmem_base, pair, a.num_tiles, npairs, num_kb, abort_flag,
                                                              err);
    if (warp == 2 && jxd::elect_one()) {
      // ---------------- forward "stage written" to the even CTA ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; ok && t < a.num_tiles; t += npairs)
        for (int kb = 0; kb < num_kb; ++kb) {
          if (*abort_flag || !jxg::wait_bounded(&gfull[stage], phase, err)) { *abort_flag = 1; ok = false; break; }
          jxd::mbar_arrive_cluster(full0 + stage * 8);
          if (++stage == CP_STAGES) { stage = 0; phase ^= 1u; }
        }
    }
    if (warp == 3 && jxd::elect_one()) {
      // ---------------- forward "span drained" to the even CTA ----------------
      const int nspan = (num_kb + SPAN_KB - 1) / SPAN_KB;
      uint32_t span_ctr = 0;
      bool ok = true;
      for (int t = pair; ok && t < a.num_tiles; t += npairs)
        for (int sp = 0; sp < nspan; ++sp, ++span_ctr) {
          const uint32_t p = span_ctr & 1u, ph = (span_ctr >> 1) & 1u;
          if (*abort_flag || !jxg::wait_bounded(&gempty[p], ph, err)) { *abort_flag = 1; ok = false; break; }
          jxd::mbar_arrive_cluster(sempty0 + p * 8);
        }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(CONV_HIGH_REGS));
    // ---------------- gather B, drain spans, store (warps 4..11) ----------------
    const int gw = warp - CONV_FIRST_EPI;  // 0..7
    const int q4 = warp & 3, half = gw >> 2;
    const int rg = gw * 4 + (lane >> 3), pg = lane & 7;  // cols mode: row group, position group
    int stage = 0;
    uint32_t phase = 0;
    uint32_t span_ctr = 0;
    bool ok = true;
    for (int t = pair; ok && t < a.num_tiles; t += npairs) {
      const TileInfo ti = pair_tile_coords(t, a.tiles_m, a.tiles_n);
      float acc[EPI_COLS];
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.0f;
      // rows mode: this thread's B row is one pixel for the whole tile
      const float* base = src;
      uint32_t mask = 0;
      if constexpr (!COLS)
        row_position(src, (long long)ti.n_blk * PAIR_TILE + (int)rank * PAIR_ROWS + q4 * 32 + lane, a, base, mask);
      int spans_done = 0;
      const int nspan = (num_kb + SPAN_KB - 1) / SPAN_KB;
      // gather(v, kb): issue k-block kb's 16 loads of this thread (no wait on the stage).
      auto gather = [&](float (&v)[16], int kb) {
        if constexpr (!COLS) {
          const uint4* te = reinterpret_cast<const uint4*>(tab + kb * BK + half * 16);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 e = te[i];
            v[2 * i] = gather_one(base, (int)e.x, e.y & mask);
            v[2 * i + 1] = gather_one(base, (int)e.z, e.w & mask);
          }
        } else {
          // rows 4 rg .. 4 rg + 3 at the k-block's positions 4 pg .. 4 pg + 3:
          // two 16-byte loads of the position table, two of the row table
          const uint4* pq = reinterpret_cast<const uint4*>(a.pixtab + (long long)ti.b * a.Ksp + kb * BK + 4 * pg);
          const uint4 p01 = __ldg(pq), p23 = __ldg(pq + 1);
          const uint4* te = reinterpret_cast<const uint4*>(tab + ti.n_blk * PAIR_TILE + (int)rank * PAIR_ROWS + 4 * rg);
          const uint4 r01 = te[0], r23 = te[1];
          const int po[4] = {(int)p01.x, (int)p01.z, (int)p23.x, (int)p23.z};
          const uint32_t pm[4] = {p01.y, p01.w, p23.y, p23.w};
          const uint32_t ro[4] = {r01.x, r01.z, r23.x, r23.z};
          const uint32_t rm[4] = {r01.y, r01.w, r23.y, r23.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) v[4 * i + j] = gather_one(src + po[j], (int)ro[i], rm[i] & pm[j]);
        }
      };
      // drain(): add span partial span_ctr into acc and hand its buffer back.
      auto drain = [&]() -> bool {
        const uint32_t p = span_ctr & 1u, ph = (span_ctr >> 1) & 1u;
        if (!jxg::warp_wait_bounded(&sfull[p], ph, abort_flag, err)) return false;
        jxd::tc_fence_after();
        const uint32_t t_addr =
            tmem_base + ((uint32_t)(q4 * 32) << 16) + p * (uint32_t)PAIR_TILE + (uint32_t)(half * EPI_COLS);
#pragma unroll
        for (int c = 0; c < EPI_COLS; c += 16) {
          uint32_t r[16];
          jxd::tmem_ld16(t_addr + c, r);
          jxd::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[c + j] = __fadd_rn(acc[c + j], __uint_as_float(r[j]));
        }
        jxd::tc_fence_before();
        ++span_ctr;
        ++spans_done;
        __syncwarp();
        if (lane == 0) jxd::mbar_arrive(&gempty[p]);  // warp 3 forwards the group's completion
        return true;
      };
      // publish(v, kb): wait for the stage, write v as tf32 hi/lo, hand the
      // stage to the pair (once TMA's A slices have landed too), and drain a
      // span partial when one is due.
      auto publish = [&](float (&v)[16], int kb) -> bool {
        if (!jxg::warp_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, err)) return false;
        uint8_t* bh = smem + stage * CP_STAGE + 2 * PAIR_OP;
        if constexpr (!COLS) {
          // row q4*32+lane, 16-byte chunks 4*half..4*half+3 of its 128-byte row, 128-byte swizzle
          const int row = q4 * 32 + lane;
          uint8_t* rp = bh + row * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float4 h, l;
            jxd::split_tf32(v[4 * c], h.x, l.x);
            jxd::split_tf32(v[4 * c + 1], h.y, l.y);
            jxd::split_tf32(v[4 * c + 2], h.z, l.z);
            jxd::split_tf32(v[4 * c + 3], h.w, l.w);
            const int off = ((4 * half + c) ^ (row & 7)) << 4;
            *reinterpret_cast<float4*>(rp + off) = h;
            *reinterpret_cast<float4*>(rp + PAIR_OP + off) = l;
          }
        } else {
          // rows 4 rg + i: positions 4 pg .. 4 pg + 3 are 16-byte chunk pg of the row
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int row = 4 * rg + i;
            float4 h, l;
            jxd::split_tf32(v[4 * i], h.x, l.x);
            jxd::split_tf32(v[4 * i + 1], h.y, l.y);
            jxd::split_tf32(v[4 * i + 2], h.z, l.z);
            jxd::split_tf32(v[4 * i + 3], h.w, l.w);
            const int off = row * 128 + ((pg ^ (row & 7)) << 4);
            *reinterpret_cast<float4*>(bh + off) = h;
            *reinterpret_cast<float4*>(bh + PAIR_OP + off) = l;
          }
        }
        jxd::fence_proxy_async_smem();  // make the generic-proxy writes visible to the tensor cores
        __syncwarp();
        if (lane == 0) jxd::mbar_arrive(&gfull[stage]);  // warp 2 forwards the stage's completion
        if (++stage == CP_STAGES) { stage = 0; phase ^= 1u; }
        // Once span i is fully written, drain span i-1 (its MMAs have been
        // issued before any of span i's could be).
        if ((kb % SPAN_KB == SPAN_KB - 1 || kb == num_kb - 1) && kb >= SPAN_KB)
          if (!drain()) return false;
        return true;
      };
      // Software pipeline over CP_AHEAD + 1 register buffers: the loads of
      // k-blocks kb+1 .. kb+CP_AHEAD are in flight while k-block kb waits
      // for its stage and is written (half-rows make a buffer 16 values, so
      // four of them cost what conv_gemm_kernel's two full rows do).
      float v[CP_AHEAD + 1][16];
#pragma unroll
      for (int j = 0; j < CP_AHEAD; ++j)
        if (j < num_kb) gather(v[j], j);
      for (int kb0 = 0; ok && kb0 < num_kb; kb0 += CP_AHEAD + 1) {
#pragma unroll
        for (int j = 0; j <= CP_AHEAD; ++j) {
          const int kb = kb0 + j;
          if (kb >= num_kb) break;
          if (kb + CP_AHEAD < num_kb) gather(v[(j + CP_AHEAD) % (CP_AHEAD + 1)], kb + CP_AHEAD);
          if (!publish(v[j], kb)) { ok = false; break; }
        }
      }
      while (ok && spans_done < nspan)
        if (!drain()) ok = false;
      if (!ok) break;
      store_tile<COLS>(acc, a, ti.m_blk * PAIR_TILE + (int)rank * PAIR_ROWS + q4 * 32 + lane,
                       (long long)ti.n_blk * PAIR_TILE + half * EPI_COLS, ti.b, out);
    }
  }

  jxd::tc_fence_before();
  __syncthreads();
  jxd::cluster_sync_all();  // neither CTA leaves while its peer may still signal it
  jxd::tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    jxd::tmem_dealloc_pair(tmem_base, 2 * PAIR_TILE);
  }
}

// A operand of the input gradient: Wt[c][(o, kh, kw)] = W[o][c][kh][kw],
// split into tf32 hi/lo, rows padded to Kp with zeros.
__global__ void split_filter_ocswap(const float* __restrict__ w, float* __restrict__ hi, float* __restrict__ lo,
                                    int Kp, const Geo g) {
  const int kk = g.KH * g.KW;
  const long long K = (long long)g.O * kk;
  const long long total = (long long)g.C * Kp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i / Kp), k = (int)(i - (long long)(i / Kp) * Kp);
    float x = 0.0f;
    if (k < K) {
      const int o = k / kk, r = k - (k / kk) * kk;
      x = w[((long long)o * g.C + c) * kk + r];
    }
    float h, l;
    jxd::split_tf32(x, h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

// Constants for n / d by multiply-high (Granlund and Montgomery, "Division
// by invariant integers using multiplication", 1994), valid for n < 2^31:
// l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1.
void magic_div(unsigned d, unsigned& m, int& l) {
  l = 0;
  while ((1ull << l) < d) ++l;
  m = (unsigned)((((1ull << l) - d) << 32) / d + 1);
}

int blocks_for(long long work, int cap_per_sm) {
  long long b = work;
  const long long cap = (long long)jx::num_sms() * cap_per_sm;
  if (b > cap) b = cap;
  return b < 1 ? 1 : (int)b;
}

int check_geo(long long B, long long C, long long H, long long W, long long O, long long KH, long long KW,
              long long stride, long long pad, Geo* g) {
  JX_REQUIRE(B >= 0 && C >= 1 && H >= 1 && W >= 1 && O >= 1 && KH >= 1 && KW >= 1, "conv2d: bad shape");
  JX_REQUIRE(stride > 0, "Stride must be positive");
  JX_REQUIRE(pad >= 0, "conv2d: negative padding");
  JX_REQUIRE(KH <= H + 2 * pad, "Kernel height too large");
  JX_REQUIRE(KW <= W + 2 * pad, "Kernel width too large");
  const long long OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  JX_REQUIRE(C * KH * KW < (1LL << 30) && OH * OW < (1LL << 30) && O < (1LL << 30) && H * W < (1LL << 30),
             "conv2d: dimensions too large");
  *g = Geo{(int)C, (int)H, (int)W, (int)O, (int)KH, (int)KW, (int)stride, (int)pad, (int)OH, (int)OW};
  return JX_OK;
}

// Images per pass so one pass's operand workspace stays under ~4 GiB.
long long images_per_pass(long long B, long long per_image_floats) {
  const long long budget = (4LL << 30) / 4;
  long long nb = per_image_floats > 0 ? budget / per_image_floats : B;
  if (nb < 1) nb = 1;
  return nb < B ? nb : B;
}

// ---- implicit GEMM host side ------------------------------------------------

// Shapes the implicit kernel covers: a gather table that fits shared memory,
// at most 32 filter taps (one mask bit each), and 32-bit element offsets
// within one image.
bool implicit_fits(const Geo& g, long long table_entries, long long n_cols, long long img_elems) {
  return table_entries <= TABLE_MAX && g.KH * g.KW <= 32 && n_cols < (1LL << 31) && img_elems < (1LL << 31);
}

std::atomic<int> g_conv_kernel{JX_CONV_AUTO};  // jx_conv_set_kernel
std::mutex g_conv_mu;                            // per-device kernel preparation

// Per device and mode, once: conv_gemm_kernel's shared-memory limit and the
// register count it was built with.  Two host threads making their first
// call on a device serialise on the mutex.
template <bool COLS>
int conv_gemm_prepare(int* regs_out) {
  static int regs[64];
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_conv_mu);
  if (!regs[dev & 63]) {
    cudaFuncAttributes fa;
    JX_CUDA(cudaFuncGetAttributes(&fa, conv_gemm_kernel<COLS>));
    JX_CUDA(cudaFuncSetAttribute(conv_gemm_kernel<COLS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)IMPLICIT_SMEM));
    regs[dev & 63] = fa.numRegs;
  }
  *regs_out = regs[dev & 63];
  return JX_OK;
}

template <bool COLS>
int launch_conv_gemm(const float* Ah, const float* Al, int a_batch, int Kp, const float* src, const uint2* tab,
                     const ImplicitArgs& a, float* out, cudaStream_t st) {
  CUtensorMap mAh, mAl;
  int rc = jx::gemm_make_kmajor_map(&mAh, Ah, Kp, a.M, a_batch, BM);
  if (!rc) rc = jx::gemm_make_kmajor_map(&mAl, Al, Kp, a.M, a_batch, BM);
  if (rc) return rc;
  int regs = 0;
  if ((rc = conv_gemm_prepare<COLS>(&regs))) return rc;
  // The register split inside the kernel assumes exactly CONV_LAUNCH_REGS per
  // thread at launch; with any other allocation setmaxnreg.inc could wait for
  // registers that never come, so refuse to launch.
  if (regs != CONV_LAUNCH_REGS)
    return jx::fail(JX_EUNSUPPORTED, "conv_gemm_kernel built with %d registers per thread, expected %d", regs,
                    CONV_LAUNCH_REGS);
  const int grid = std::min(a.num_tiles, jx::num_sms());
  conv_gemm_kernel<COLS><<<grid, CONV_THREADS, IMPLICIT_SMEM, st>>>(mAh, mAl, src, tab, a, out,
                                                                  jx::device_error_word());
  JX_LAUNCH_CHECK("conv_gemm_kernel");
  return JX_OK;
}

// ---- SM-pair launcher --------------------------------------------------------


// Whether a pass with `pair_tiles` 256 x 256 tiles runs on conv_pair_kernel:
// by default once they fill at least 90% of the SM pairs (below that the
// one-CTA kernel's 128 x 256 tiles spread over more SMs; at 72 tiles on 74
// pairs, the weight gradient of 8 images sliced 8 ways, both fill 97%).
bool conv_use_pair(long long pair_tiles) {
  const int k = g_conv_kernel.load();
  if (k == JX_CONV_ONE_CTA) return false;
  if (k == JX_CONV_PAIR) return true;
  return 10 * pair_tiles >= 9 * (long long)(jx::num_sms() / 2);
}

// Per device and mode, once: the shared-memory limit, the register count the
// kernel was built with, and how many pairs can be resident at once.
template <bool COLS>
int conv_pair_prepare(int* regs_out, int* max_pairs_out) {
  static int regs[64], max_pairs[64];
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_conv_mu);
  if (!regs[dev & 63]) {
    auto k = conv_pair_kernel<COLS>;
    cudaFuncAttributes fa;
    JX_CUDA(cudaFuncGetAttributes(&fa, k));
    JX_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CP_SMEM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)jx::num_sms());
    cfg.blockDim = dim3(CONV_THREADS);
    cfg.dynamicSmemBytes = CP_SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int clusters = 0;
    JX_CUDA(cudaOccupancyMaxActiveClusters(&clusters, (void*)k, &cfg));
    max_pairs[dev & 63] = clusters;
    regs[dev & 63] = fa.numRegs;
  }
  *regs_out = regs[dev & 63];
  *max_pairs_out = max_pairs[dev & 63];
  return JX_OK;
}

// a.tiles_m / tiles_n / num_tiles count 256 x 256 pair tiles.
template <bool COLS>
int launch_conv_pair(const float* Ah, const float* Al, int a_batch, int Kp, const float* src, const uint2* tab,
                     const ImplicitArgs& a, float* out, cudaStream_t st) {
  CUtensorMap mAh, mAl;
  int rc = jx::gemm_make_kmajor_map(&mAh, Ah, Kp, a.M, a_batch, PAIR_ROWS);
  if (!rc) rc = jx::gemm_make_kmajor_map(&mAl, Al, Kp, a.M, a_batch, PAIR_ROWS);
  if (rc) return rc;
  int regs = 0, max_pairs = 0;
  if ((rc = conv_pair_prepare<COLS>(&regs, &max_pairs))) return rc;
  // The register split inside the kernel assumes exactly CONV_LAUNCH_REGS per
  // thread at launch; with any other allocation setmaxnreg.inc could wait for
  // registers that never come, so refuse to launch.
  if (regs != CONV_LAUNCH_REGS)
    return jx::fail(JX_EUNSUPPORTED, "conv_pair_kernel built with %d registers per thread, expected %d", regs,
                    CONV_LAUNCH_REGS);
  if (max_pairs < 1) return jx::fail(JX_EUNSUPPORTED, "conv_pair_kernel: no SM pair can hold a cluster");
  if (a.num_tiles == 0) return JX_OK;
  const int pairs = std::min(a.num_tiles, max_pairs);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(CONV_THREADS);
  cfg.dynamicSmemBytes = CP_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  unsigned int* errw = jx::device_error_word();
  JX_CUDA(cudaLaunchKernelEx(&cfg, conv_pair_kernel<COLS>, mAh, mAl, src, tab, a, out, errw));
  return JX_OK;
}

// Tile counts of a pass with M GEMM rows, N columns and `slices` batch
// entries, for the kernel it runs on, then the launch.
template <bool COLS>
int launch_implicit(bool pair, const float* Ah, const float* Al, int a_batch, int Kp, const float* src,
                    const uint2* tab, ImplicitArgs a, int slices, float* out, cudaStream_t st) {
  const int tm = pair ? PAIR_TILE : BM, tn = pair ? PAIR_TILE : BN;
  a.tiles_m = (a.M + tm - 1) / tm;
  a.tiles_n = (a.N + tn - 1) / tn;
  a.num_tiles = a.tiles_m * a.tiles_n * slices;
  return pair ? launch_conv_pair<COLS>(Ah, Al, a_batch, Kp, src, tab, a, out, st)
              : launch_conv_gemm<COLS>(Ah, Al, a_batch, Kp, src, tab, a, out, st);
}

int table_build(uint2* tab, int n, int count, int mode, const Geo& g, cudaStream_t st) {
  build_gather_table<<<(n + 255) / 256, 256, 0, st>>>(tab, n, count, mode, g);
  JX_LAUNCH_CHECK("build_gather_table");
  return JX_OK;
}

int conv_fwd_implicit(const float* x, const float* w, float* y, long long B, const Geo& g, cudaStream_t st) {
  const long long K = g.K(), Kp = jx::gemm_kpad(K), NP = g.NP();
  void* ws = nullptr;
  int rc = jx::scratch_get(sizeof(float) * (size_t)(2 * g.O * Kp + 2 * Kp), &ws, st);
  if (rc) return rc;
  float* Wh = reinterpret_cast<float*>(ws);
  float* Wl = Wh + g.O * Kp;
  uint2* tab = reinterpret_cast<uint2*>(Wl + g.O * Kp);
  rc = jx::gemm_split_operand(w, Wh, Wl, g.O, (int)K, (int)Kp, K, 0, 1, false, st);
  if (!rc) rc = table_build(tab, (int)Kp, (int)K, TAB_FWD, g, st);
  if (!rc) {
    ImplicitArgs a{};
    a.M = g.O;
    a.N = (int)(B * NP);
    a.num_kb = (int)(Kp / BK);
    a.a_bcast = 1;
    a.table_n = (int)Kp;
    a.LH = g.H;
    a.LW = g.W;
    a.KH = g.KH;
    a.KW = g.KW;
    a.S = g.S;
    a.P = g.P;
    a.img_stride = (long long)g.C * g.H * g.W;
    a.PW = g.OW;
    a.NPpix = (int)NP;
    a.dx_mode = 0;
    a.out_img_stride = (long long)g.O * NP;
    const bool pair = conv_use_pair((long long)((a.M + PAIR_TILE - 1) / PAIR_TILE) * ((a.N + PAIR_TILE - 1) / PAIR_TILE));
    rc = launch_implicit<false>(pair, Wh, Wl, 1, (int)Kp, x, tab, a, 1, y, st);
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

int conv_bwd_data_implicit(const float* dy, const float* w, float* dx, long long B, const Geo& g, cudaStream_t st) {
  const long long Kd = (long long)g.O * g.KH * g.KW, Kdp = jx::gemm_kpad(Kd);
  void* ws = nullptr;
  int rc = jx::scratch_get(sizeof(float) * (size_t)(2 * g.C * Kdp + 2 * Kdp), &ws, st);
  if (rc) return rc;
  float* Ah = reinterpret_cast<float*>(ws);
  float* Al = Ah + g.C * Kdp;
  uint2* tab = reinterpret_cast<uint2*>(Al + g.C * Kdp);
  split_filter_ocswap<<<blocks_for((g.C * Kdp + 255) / 256, 8), 256, 0, st>>>(w, Ah, Al, (int)Kdp, g);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) rc = jx::check_cuda(e, "split_filter_ocswap");
  if (!rc) rc = table_build(tab, (int)Kdp, (int)Kd, TAB_DX, g, st);
  if (!rc) {
    ImplicitArgs a{};
    a.M = g.C;
    a.N = (int)(B * g.H * g.W);
    a.num_kb = (int)(Kdp / BK);
    a.a_bcast = 1;
    a.table_n = (int)Kdp;
    a.LH = g.OH;
    a.LW = g.OW;
    a.KH = g.KH;
    a.KW = g.KW;
    a.S = g.S;
    a.P = g.P;
    a.img_stride = (long long)g.O * g.OH * g.OW;
    a.PW = g.W;
    a.NPpix = g.H * g.W;
    a.dx_mode = 1;
    a.out_img_stride = (long long)g.C * g.H * g.W;
    const bool pair = conv_use_pair((long long)((a.M + PAIR_TILE - 1) / PAIR_TILE) * ((a.N + PAIR_TILE - 1) / PAIR_TILE));
    rc = launch_implicit<false>(pair, Ah, Al, 1, (int)Kdp, dy, tab, a, 1, dx, st);
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

// Slices of the weight-gradient contraction: the count in [1, 64] (each
// slice at least 1024 long) that minimises the estimated time
// waves x (k-blocks per tile + DW_TILE_COST), where `units` tiles run at once
// (SMs, or SM pairs) and DW_TILE_COST is a tile's fixed cost (pipeline fill,
// last span drain, partial store) in k-block times.  At [64,256,56,56] x
// [256,256,3,3] on SM pairs this takes 8 slices (72 tiles, one wave of 784
// k-blocks) over the 41 that fill the waves best (369 tiles, 5 waves of 153):
// whole conv step 237.2 against 234.1 TFLOP/s; 16 slices gave 235.8.
constexpr long long DW_TILE_COST = 13;
long long dw_slices(long long tiles, long long Q, long long units) {
  long long best = 1, best_cost = -1;
  for (long long S = 1; S <= 64; ++S) {
    if (S > 1 && Q / S < 1024) break;
    const long long waves = (tiles * S + units - 1) / units;
    const long long kb = ((Q + S - 1) / S + BK - 1) / BK;
    const long long cost = waves * (kb + DW_TILE_COST);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

int conv_bwd_filter_implicit(const float* x, const float* dy, float* dw, long long B, const Geo& g, cudaStream_t st) {
  const long long K = g.K(), NP = g.NP(), Q = B * NP;
  // SM pairs when their tiles, sliced to fill the pairs, reach one per pair
  const long long pair_tiles = (long long)((g.O + PAIR_TILE - 1) / PAIR_TILE) * ((K + PAIR_TILE - 1) / PAIR_TILE);
  const long long pair_slices = dw_slices(pair_tiles, Q, jx::num_sms() / 2);
  // the pair kernel's position table holds 32-bit offsets into the whole x
  const bool pair = B * g.C * g.H * g.W < (1LL << 31) && conv_use_pair(pair_tiles * pair_slices);
  const int tiles_m = (g.O + BM - 1) / BM, tiles_n = (int)((K + BN - 1) / BN);
  const long long S = pair ? pair_slices : dw_slices((long long)tiles_m * tiles_n, Q, jx::num_sms());
  const long long Ks = (Q + S - 1) / S, Ksp = jx::gemm_kpad(Ks);
  const long long tab_n = (long long)tiles_n * BN;  // BN = PAIR_TILE: whole tiles of either kernel
  void* ws = nullptr;
  const long long pix_n = pair ? S * Ksp : 0;  // position table entries
  const size_t floats = (size_t)(2 * S * g.O * Ksp + 2 * tab_n + 2 * pix_n + (S > 1 ? S * g.O * K : 0));
  int rc = jx::scratch_get(sizeof(float) * floats, &ws, st);
  if (rc) return rc;
  float* Ah = reinterpret_cast<float*>(ws);
  float* Al = Ah + S * g.O * Ksp;
  uint2* tab = reinterpret_cast<uint2*>(Al + S * g.O * Ksp);
  uint2* pixtab = tab + tab_n;  // 16-byte aligned: Ksp and tab_n are multiples of 32
  float* part = S > 1 ? reinterpret_cast<float*>(pixtab + pix_n) : dw;
  dy_rows_split<<<blocks_for(S * g.O, 16), 256, 0, st>>>(dy, Ah, Al, Q, Ks, (int)Ksp, (int)S, g);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) rc = jx::check_cuda(e, "dy_rows_split");
  if (!rc) rc = table_build(tab, (int)tab_n, (int)K, TAB_FWD, g, st);
  if (!rc) {
    ImplicitArgs a{};
    a.M = g.O;
    a.N = (int)K;
    a.num_kb = (int)(Ksp / BK);
    a.a_bcast = 0;
    a.table_n = (int)tab_n;
    a.LH = g.H;
    a.LW = g.W;
    a.KH = g.KH;
    a.KW = g.KW;
    a.S = g.S;
    a.P = g.P;
    a.img_stride = (long long)g.C * g.H * g.W;
    a.Q = (int)Q;
    a.Ks = (int)Ks;
    a.OW = g.OW;
    a.NPo = (int)NP;
    magic_div((unsigned)a.NPo, a.npo_m, a.npo_l);
    magic_div((unsigned)a.OW, a.ow_m, a.ow_l);
    a.ldc = K;
    a.strideC = (long long)g.O * K;
    a.Ksp = (int)Ksp;
    a.pixtab = pixtab;
    if (pair) {
      build_pixel_table<<<blocks_for((pix_n + 255) / 256, 8), 256, 0, st>>>(pixtab, pix_n, a);
      const cudaError_t e2 = cudaGetLastError();
      if (e2 != cudaSuccess) rc = jx::check_cuda(e2, "build_pixel_table");
    }
    if (!rc) rc = launch_implicit<true>(pair, Ah, Al, (int)S, (int)Ksp, x, tab, a, (int)S, part, st);
  }
  if (!rc && S > 1) {
    slice_sum<<<blocks_for((g.O * K + 255) / 256, 8), 256, 0, st>>>(part, dw, g.O * K, (int)S);
    e = cudaGetLastError();
    if (e != cudaSuccess) rc = jx::check_cuda(e, "slice_sum");
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

}  // namespace

extern "C" {

int jx_conv_set_kernel(int which) {
  JX_TRACE("jx_conv_set_kernel");
  JX_REQUIRE(which == JX_CONV_AUTO || which == JX_CONV_ONE_CTA || which == JX_CONV_PAIR,
             "jx_conv_set_kernel: unknown kernel %d", which);
  g_conv_kernel.store(which);
  return JX_OK;
}

int jx_conv2d_fwd_f32(const float* x, const float* w, float* y, int64_t B, int64_t C, int64_t H, int64_t W, int64_t O,
                      int64_t KH, int64_t KW, int64_t stride, int64_t pad, jx_stream_t stream) {
  JX_TRACE("jx_conv2d_fwd_f32");
  Geo g;
  int rc = check_geo(B, C, H, W, O, KH, KW, stride, pad, &g);
  if (rc) return rc;
  if (B == 0) return JX_OK;
  JX_REQUIRE(x && w && y, "conv2d: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  const long long K = g.K(), Kp = jx::gemm_kpad(K), NP = g.NP();
  if (implicit_fits(g, Kp, B * NP, C * H * W)) return conv_fwd_implicit(x, w, y, B, g, st);
  const long long nb = images_per_pass(B, 2 * NP * Kp);
  void* ws = nullptr;
  if ((rc = jx::scratch_get(sizeof(float) * (size_t)(2 * O * Kp + 2 * nb * NP * Kp), &ws, st))) return rc;
  float* Wh = reinterpret_cast<float*>(ws);
  float* Wl = Wh + O * Kp;
  float* Xh = Wl + O * Kp;
  float* Xl = Xh + nb * NP * Kp;
  rc = jx::gemm_split_operand(w, Wh, Wl, (int)O, (int)K, (int)Kp, K, 0, 1, false, st);
  for (long long b0 = 0; !rc && b0 < B; b0 += nb) {
    const long long n = std::min(nb, B - b0);
    im2col_rows_split<<<blocks_for(n * NP, 16), 256, 0, st>>>(x + b0 * C * H * W, Xh, Xl, n * NP, (int)Kp, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = jx::check_cuda(e, "im2col_rows_split");
    // Y_b[O, NP] = W . Xcol_b for each image of the pass
    if (!rc)
      rc = jx::gemm_presplit_err(Wh, Wl, Xh, Xl, y + b0 * O * NP, (int)O, (int)NP, (int)Kp, NP, O * NP, (int)n, st,
                                 jx::device_error_word(), true, false);
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

int jx_conv2d_bwd_data_f32(const float* dy, const float* w, float* dx, int64_t B, int64_t C, int64_t H, int64_t W,
                           int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad, jx_stream_t stream) {
  JX_TRACE("jx_conv2d_bwd_data_f32");
  Geo g;
  int rc = check_geo(B, C, H, W, O, KH, KW, stride, pad, &g);
  if (rc) return rc;
  if (B == 0) return JX_OK;
  JX_REQUIRE(dy && w && dx, "conv2d: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  if (implicit_fits(g, jx::gemm_kpad(O * KH * KW), B * H * W, O * (long long)g.OH * g.OW))
    return conv_bwd_data_implicit(dy, w, dx, B, g, st);
  const long long K = g.K(), Op = jx::gemm_kpad(O), NP = g.NP();
  const long long nb = images_per_pass(B, 2 * NP * Op + K * NP);
  void* ws = nullptr;
  if ((rc = jx::scratch_get(sizeof(float) * (size_t)(2 * K * Op + nb * (2 * NP * Op + K * NP)), &ws, st))) return rc;
  float* Ah = reinterpret_cast<float*>(ws);  // W^T split: rows k, contraction over o
  float* Al = Ah + K * Op;
  float* Bh = Al + K * Op;  // dY_b^T split: rows p, contraction over o
  float* Bl = Bh + nb * NP * Op;
  float* dcol = Bl + nb * NP * Op;
  rc = jx::gemm_split_operand(w, Ah, Al, (int)K, (int)O, (int)Op, K, 0, 1, true, st);
  for (long long b0 = 0; !rc && b0 < B; b0 += nb) {
    const long long n = std::min(nb, B - b0);
    rc = jx::gemm_split_operand(dy + b0 * O * NP, Bh, Bl, (int)NP, (int)O, (int)Op, NP, O * NP, (int)n, true, st);
    if (!rc)
      rc = jx::gemm_presplit_err(Ah, Al, Bh, Bl, dcol, (int)K, (int)NP, (int)Op, NP, K * NP, (int)n, st,
                                 jx::device_error_word(), true, false);
    if (!rc) {
      col2im_gather<<<blocks_for((n * C * H * W + 255) / 256, 8), 256, 0, st>>>(dcol, dx + b0 * C * H * W, n, g);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) rc = jx::check_cuda(e, "col2im_gather");
    }
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

int jx_conv2d_bwd_filter_f32(const float* x, const float* dy, float* dw, int64_t B, int64_t C, int64_t H, int64_t W,
                             int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad, jx_stream_t stream) {
  JX_TRACE("jx_conv2d_bwd_filter_f32");
  Geo g;
  int rc = check_geo(B, C, H, W, O, KH, KW, stride, pad, &g);
  if (rc) return rc;
  JX_REQUIRE(dw, "conv2d: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  const long long K = g.K(), NP = g.NP();
  if (B == 0) {
    JX_CUDA(cudaMemsetAsync(dw, 0, sizeof(float) * O * K, st));
    return JX_OK;
  }
  JX_REQUIRE(x && dy, "conv2d: NULL pointer");
  JX_REQUIRE(B * NP < (1LL << 31), "conv2d: weight gradient over 2^31 or more output pixels");
  if (implicit_fits(g, (K + 255) / 256 * 256, std::max(K, B * NP), C * H * W))
    return conv_bwd_filter_implicit(x, dy, dw, B, g, st);
  const long long Q = B * NP;  // contraction length: every image's every output pixel
  // slices: enough output tiles to fill the GPU twice over, each slice >= 1024 long
  const long long tiles = ((O + 127) / 128) * ((K + 255) / 256);
  long long S = (2LL * jx::num_sms() + tiles - 1) / tiles;
  S = std::max(1LL, std::min(S, std::min(64LL, Q / 1024)));
  const long long Ks = (Q + S - 1) / S, Ksp = jx::gemm_kpad(Ks);
  void* ws = nullptr;
  const size_t floats = (size_t)(2 * S * O * Ksp + 2 * S * K * Ksp + (S > 1 ? S * O * K : 0));
  if ((rc = jx::scratch_get(sizeof(float) * floats, &ws, st))) return rc;
  float* Ah = reinterpret_cast<float*>(ws);
  float* Al = Ah + S * O * Ksp;
  float* Bh = Al + S * O * Ksp;
  float* Bl = Bh + S * K * Ksp;
  float* part = S > 1 ? Bl + S * K * Ksp : dw;
  dy_rows_split<<<blocks_for(S * O, 16), 256, 0, st>>>(dy, Ah, Al, Q, Ks, (int)Ksp, (int)S, g);
  im2col_cols_split<<<blocks_for(S * K, 16), 256, 0, st>>>(x, Bh, Bl, Q, Ks, (int)Ksp, (int)S, g);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) rc = jx::check_cuda(e, "conv2d dW operand kernels");
  if (!rc)
    rc = jx::gemm_presplit_err(Ah, Al, Bh, Bl, part, (int)O, (int)K, (int)Ksp, K, O * K, (int)S, st,
                               jx::device_error_word(), false, false);
  if (!rc && S > 1) {
    slice_sum<<<blocks_for((O * K + 255) / 256, 8), 256, 0, st>>>(part, dw, O * K, (int)S);
    e = cudaGetLastError();
    if (e != cudaSuccess) rc = jx::check_cuda(e, "slice_sum");
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

}  // extern "C"
