// fft.cu -- batched complex FFTs, interleaved [re, im] f32.
//
// Replaces fft_recursive (src/ops/fft.rs:40-70, radix-2 recursion with a
// fresh Vec per level), ifft's 1/n scaling (:174-179), fft2/ifft2's row-then-
// column order (:261-396) and the reference's GPU FFT (gpu_fft_complex
// src/backend/ops.rs:1736-1910: one dispatch per radix-2 stage, no
// bit-reversal, wrong for every n).
//
// One transform (or a group of adjacent ones) per CTA, entirely in shared
// memory, Stockham autosort (no bit-reversal pass): a leading radix-2/4/8 pass
// when log2(n) is not a multiple of 4, then radix-16 passes.  Each thread
// keeps 16 points in registers through a pass; the first pass reads global
// memory and the last writes it, both coalesced, so an n = 4096 transform
// touches shared memory only twice.  Twiddles exp(-2 pi i t/n) come from a
// per-size table computed in double precision.  Columns of a 2-D transform
// run the same kernel with 8 adjacent columns per CTA, so every global
// access is a 64-byte row segment; 1024-row columns have their own kernel
// (32 x 32 in registers, tiles landed by TMA).
#include <math.h>

#include <mutex>
#include <vector>

#include <cudaTypedefs.h>

#include "jx_common.cuh"

namespace {

constexpr int MAX_LOGN = 13;  // shared-memory transforms up to 8192 points

// Offset, past the plain n-entry twiddle table, of radix-16 pass s's packed
// twiddles (pass s combines Ns = r0 16^s points; four entries per k < Ns).
__host__ __device__ constexpr int pass_twiddle_offset(int r0, int s) {
  return 4 * r0 * ((1 << (4 * s)) - 1) / 15;  // 4 (Ns_0 + ... + Ns_{s-1})
}

struct cf2 {
  float x, y;
};
__device__ __forceinline__ cf2 cadd(cf2 a, cf2 b) { return {a.x + b.x, a.y + b.y}; }
__device__ __forceinline__ cf2 csub(cf2 a, cf2 b) { return {a.x - b.x, a.y - b.y}; }
__device__ __forceinline__ cf2 cmul(cf2 a, cf2 b) { return {a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x}; }
// multiply by -i (forward) or +i (inverse)
template <bool INV>
__device__ __forceinline__ cf2 mul_mi(cf2 a) {
  return INV ? cf2{-a.y, a.x} : cf2{a.y, -a.x};
}

template <bool INV>
__device__ __forceinline__ void dft2(cf2* v) {
  cf2 a = v[0], b = v[1];
  v[0] = cadd(a, b);
  v[1] = csub(a, b);
}
template <bool INV>
__device__ __forceinline__ void dft4(cf2& a, cf2& b, cf2& c, cf2& d) {
  const cf2 t0 = cadd(a, c), t1 = csub(a, c), t2 = cadd(b, d), t3 = mul_mi<INV>(csub(b, d));
  a = cadd(t0, t2);
  c = csub(t0, t2);
  b = cadd(t1, t3);
  d = csub(t1, t3);
}
template <bool INV>
__device__ __forceinline__ void dft4v(cf2* v) {
  dft4<INV>(v[0], v[1], v[2], v[3]);
}
template <bool INV>
__device__ __forceinline__ void dft8(cf2* v) {
  cf2 e0 = v[0], e1 = v[2], e2 = v[4], e3 = v[6];
  cf2 o0 = v[1], o1 = v[3], o2 = v[5], o3 = v[7];
  dft4<INV>(e0, e1, e2, e3);
  dft4<INV>(o0, o1, o2, o3);
  const float r = 0.707106781186547524f;
  // W8^k, k = 1..3 (conjugated for the inverse)
  o1 = cmul(o1, cf2{r, INV ? r : -r});
  o2 = mul_mi<INV>(o2);
  o3 = cmul(o3, cf2{-r, INV ? r : -r});
  v[0] = cadd(e0, o0);
  v[4] = csub(e0, o0);
  v[1] = cadd(e1, o1);
  v[5] = csub(e1, o1);
  v[2] = cadd(e2, o2);
  v[6] = csub(e2, o2);
  v[3] = cadd(e3, o3);
  v[7] = csub(e3, o3);
}
// 16-point DFT as 4 x 4: inner radix-4 over x[4 n1 + n2], twiddles W16^(n2 k1),
// outer radix-4 over n2; output k = k1 + 4 k2.
template <bool INV>
__device__ __forceinline__ void dft16(cf2* v) {
#pragma unroll
  for (int n2 = 0; n2 < 4; ++n2) dft4<INV>(v[n2], v[4 + n2], v[8 + n2], v[12 + n2]);
  // after the inner pass, Y[n2][k1] sits at v[4 k1 + n2]
  const float c1 = 0.923879532511286756f, s1 = 0.382683432365089772f, r = 0.707106781186547524f;
  const float sg = INV ? 1.0f : -1.0f;
  // W16^m = (cos(2 pi m/16), sg*sin(2 pi m/16)) for m = n2*k1
  v[5] = cmul(v[5], cf2{c1, sg * s1});     // n2=1,k1=1: m=1
  v[9] = cmul(v[9], cf2{r, sg * r});       // n2=1,k1=2: m=2
  v[13] = cmul(v[13], cf2{s1, sg * c1});   // n2=1,k1=3: m=3
  v[6] = cmul(v[6], cf2{r, sg * r});       // n2=2,k1=1: m=2
  v[10] = mul_mi<INV>(v[10]);              // n2=2,k1=2: m=4
  v[14] = cmul(v[14], cf2{-r, sg * r});    // n2=2,k1=3: m=6
  v[7] = cmul(v[7], cf2{s1, sg * c1});     // n2=3,k1=1: m=3
  v[11] = cmul(v[11], cf2{-r, sg * r});    // n2=3,k1=2: m=6
  v[15] = cmul(v[15], cf2{-c1, -sg * s1}); // n2=3,k1=3: m=9
#pragma unroll
  for (int k1 = 0; k1 < 4; ++k1) dft4<INV>(v[4 * k1], v[4 * k1 + 1], v[4 * k1 + 2], v[4 * k1 + 3]);
  // X[k1 + 4 k2] is at v[4 k1 + k2]: transpose the 4x4 into natural order
  cf2 t[16];
#pragma unroll
  for (int k1 = 0; k1 < 4; ++k1)
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) t[k1 + 4 * k2] = v[4 * k1 + k2];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = t[i];
}

template <int R, bool INV>
__device__ __forceinline__ void dft_r(cf2* v) {
  if constexpr (R == 2) dft2<INV>(v);
  else if constexpr (R == 4) dft4v<INV>(v);
  else if constexpr (R == 8) dft8<INV>(v);
  else dft16<INV>(v);
}

// Shared-memory slot of point i of one transform.  Row transforms (a warp
// inside one transform) pad one slot per 16 points.  Column groups of 8 (a
// warp spans 8 columns x 4 consecutive points) give each column a region of
// N + 4 slots and XOR the low two bits of i with bits 2..3 and 4..5; with
// that, the stride-R0 writes of the leading pass and the stride-1, -2 and -16
// accesses of the radix-16 passes each touch all 16 eight-byte bank pairs
// exactly twice per warp (the two-wavefront minimum) for every N <= 1024.
template <bool SWZ>
__device__ __forceinline__ int sidx(int i) {
  if constexpr (SWZ) return (i & ~3) | ((i ^ (i >> 2) ^ (i >> 4)) & 3);
  else return i + (i >> 4);
}
template <int N, bool SWZ>
constexpr int region() {
  return SWZ ? N + 4 : N + N / 16;
}

template <bool COLS>
struct Addr {
  long long n, w, hw;  // COLS: image width w, image size hw; element i of transform t
  long long os;        // rows: distance between consecutive output transforms (0: n)
  __device__ __forceinline__ long long base(long long t) const {
    return COLS ? (t / w) * hw + (t % w) : t * n;
  }
  __device__ __forceinline__ long long obase(long long t) const {
    return COLS ? base(t) : t * (os ? os : n);
  }
  __device__ __forceinline__ long long estride() const { return COLS ? w : 1; }
};

// One CTA: TPC transforms of N = 2^LOGN points; T = N/16 threads each.  The
// launch bound keeps at least 1024 threads per SM resident (64 registers), so
// loads of one CTA overlap the butterflies of another.
template <int LOGN, int TPC, bool COLS, bool INV>
__global__ void __launch_bounds__(TPC*((1 << LOGN) / 16),
                                  (TPC * ((1 << LOGN) / 16)) >= 1024 ? 1 : 1024 / (TPC * ((1 << LOGN) / 16)))
    fft_kernel(const float2* __restrict__ in,
                                                                        float2* __restrict__ out,
                                                                        long long ntrans, Addr<COLS> ad,
                                                                        const float2* __restrict__ tw, float scale) {
  constexpr int N = 1 << LOGN;
  constexpr int T = N / 16;
  constexpr int R0 = 1 << (LOGN % 4);  // leading radix (1: none)
  constexpr bool SWZ = COLS && TPC == 8;
  constexpr int NPAD = region<N, SWZ>();
  extern __shared__ float2 sm_raw[];
  cf2* sm = reinterpret_cast<cf2*>(sm_raw);
  const int tid = threadIdx.x;
  const int tl = COLS ? tid % TPC : tid / T;  // transform within the CTA
  const int j = COLS ? tid / TPC : tid % T;   // thread within the transform
  const long long t = (long long)blockIdx.x * TPC + tl;
  const bool active = t < ntrans;
  const long long gbase = ad.base(active ? t : 0);
  const long long obase = ad.obase(active ? t : 0);
  const long long es = ad.estride();
  cf2* S = sm + tl * NPAD;
  cf2 v[16];
  constexpr int NSTAGE16 = LOGN / 4;
  int Ns = 1;
  // ---- leading radix-R0 pass (Ns = 1): each thread does 16/R0 butterflies ----
  if constexpr (R0 > 1) {
#pragma unroll
    for (int q = 0; q < 16 / R0; ++q) {
      const int b = j + q * T;  // butterfly index in [0, N/R0)
      cf2 u[R0];
#pragma unroll
      for (int i = 0; i < R0; ++i) {
        const float2 x = active ? __ldcs(in + gbase + (long long)(b + i * (N / R0)) * es) : make_float2(0.f, 0.f);
        u[i] = {x.x, x.y};
      }
      dft_r<R0, INV>(u);
#pragma unroll
      for (int i = 0; i < R0; ++i) S[sidx<SWZ>(b * R0 + i)] = u[i];
    }
    Ns = R0;
    __syncthreads();
  }
  // ---- radix-16 passes ----
#pragma unroll
  for (int s = 0; s < NSTAGE16; ++s) {
    const bool first = (R0 == 1 && s == 0);
    const bool last = (s == NSTAGE16 - 1);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      if (first) {
        const float2 x = active ? __ldcs(in + gbase + (long long)(j + r * T) * es) : make_float2(0.f, 0.f);
        v[r] = {x.x, x.y};
      } else {
        v[r] = S[sidx<SWZ>(j + r * T)];
      }
    }
    const int k = j % Ns;
    if (Ns > 1) {
      // v[r] *= w^r with w = exp(-+2 pi i k / (16 Ns)).  w, w^2, w^4, w^8
      // come from this pass's packed entries (two 16-byte loads); every
      // other power is a product of at most three of them (a few ulp).
      const float4* pk = reinterpret_cast<const float4*>(tw + N + pass_twiddle_offset(R0, s) + 4 * k);
      const float4 w12 = __ldg(pk), w48 = __ldg(pk + 1);
      const float sg = INV ? -1.f : 1.f;
      cf2 p[16];
      p[1] = cf2{w12.x, sg * w12.y};
      p[2] = cf2{w12.z, sg * w12.w};
      p[4] = cf2{w48.x, sg * w48.y};
      p[8] = cf2{w48.z, sg * w48.w};
      p[3] = cmul(p[1], p[2]);
      p[5] = cmul(p[1], p[4]);
      p[6] = cmul(p[2], p[4]);
      p[7] = cmul(p[3], p[4]);
#pragma unroll
      for (int r = 9; r < 16; ++r) p[r] = cmul(p[r - 8], p[8]);
#pragma unroll
      for (int r = 1; r < 16; ++r) v[r] = cmul(v[r], p[r]);
    }
    dft16<INV>(v);
    const int idxD = (j / Ns) * Ns * 16 + k;
    if (!first) __syncthreads();  // every thread has read its inputs
    if (last) {
      if (active) {
#pragma unroll
        for (int r = 0; r < 16; ++r)
          __stcs(out + obase + (long long)(idxD + r * Ns) * es, make_float2(v[r].x * scale, v[r].y * scale));
      }
    } else {
#pragma unroll
      for (int r = 0; r < 16; ++r) S[sidx<SWZ>(idxD + r * Ns)] = v[r];
      __syncthreads();
    }
    Ns *= 16;
  }
  if constexpr (NSTAGE16 == 0) {
    // N < 16 cannot happen here (handled by fft_tiny_kernel)
  }
}

// n in {1, 2, 4, 8}: one thread per transform, direct radix pass.
template <int R, bool INV>
__global__ void fft_tiny_kernel(const float2* __restrict__ in, float2* __restrict__ out, long long ntrans,
                                long long n_img_w, long long hw, int cols, float scale, long long os) {
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= ntrans) return;
  const long long base = cols ? (t / n_img_w) * hw + (t % n_img_w) : t * R;
  const long long ob = cols ? base : t * (os ? os : R);
  const long long es = cols ? n_img_w : 1;
  cf2 u[R > 1 ? R : 1];
  for (int i = 0; i < R; ++i) {
    const float2 x = in[base + i * es];
    u[i].x = x.x;
    u[i].y = x.y;
  }
  if constexpr (R > 1) dft_r<R, INV>(u);
  for (int i = 0; i < R; ++i) out[ob + i * es] = make_float2(u[i].x * scale, u[i].y * scale);
}

// ---- twiddle tables: exp(-2 pi i t / 2^logn), t < 2^logn, per device -------
// Entries [0, n) are the plain table.  After them, for fft_kernel, each
// radix-16 pass s (Ns = R0 16^s points already combined) has Ns packed
// entries of four values, w, w^2, w^4, w^8 with w = exp(-2 pi i k / (16 Ns)),
// at n + pass_twiddle_offset(R0, s) + 4 k: one thread reads its four
// twiddles as two 16-byte loads next to its neighbours' instead of four
// lookups that land on up to 32 different cache lines per warp.  The values
// are copies of plain-table entries, so both layouts give the same bits.
std::mutex g_tw_mu;
float2* g_tw[64][MAX_LOGN + 2];  // sizes up to 2^(MAX_LOGN+1): real transforms use size n for n/2 points

int twiddles(int logn, const float2** out) {
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_tw_mu);
  if (!g_tw[dev & 63][logn]) {
    const int n = 1 << logn;
    const int r0 = 1 << (logn % 4), nst = logn / 4;
    std::vector<float2> h(n + pass_twiddle_offset(r0, nst));
    for (int t = 0; t < n; ++t) {
      const double a = -2.0 * 3.14159265358979323846 * (double)t / (double)n;
      h[t] = make_float2((float)cos(a), (float)sin(a));
    }
    for (int s = 0, ns = r0; s < nst; ++s, ns *= 16) {
      const int step = n / (16 * ns);
      for (int k = 0; k < ns; ++k)
        for (int q = 0; q < 4; ++q)
          h[n + pass_twiddle_offset(r0, s) + 4 * k + q] = h[((1 << q) * k * step) & (n - 1)];
    }
    float2* d = nullptr;
    JX_CUDA(cudaMalloc(&d, sizeof(float2) * h.size()));
    JX_CUDA(cudaMemcpy(d, h.data(), sizeof(float2) * h.size(), cudaMemcpyHostToDevice));
    g_tw[dev & 63][logn] = d;
  }
  *out = g_tw[dev & 63][logn];
  return JX_OK;
}

// ---- 1024-point transforms as 32 x 32 in registers ------------------------
// n = n2 + 32 n1, k = k1 + 32 k2:
//   X[k1 + 32 k2] = sum_n2 W1024^(n2 k1) [sum_n1 x[n2 + 32 n1] W32^(n1 k1)] W32^(n2 k2).
// A thread owns one n2 (then one k1) of one transform: it loads 32 points,
// does the inner 32-point DFT in registers, applies W1024^(n2 k1) from the
// table, passes the values through shared memory once (a transpose), and
// does the outer 32-point DFT in registers.  Used for the column pass of 2-D
// transforms (rows measured faster on fft_kernel): C = 8 adjacent columns per
// CTA of 256 threads, a warp spanning the 8 columns x 4 consecutive points,
// so every global access is a 64-byte row segment (4 columns per CTA, 32-byte
// segments, measured slower).  With a row stride of 33 and a column region of
// 1060 eight-byte slots the transpose's writes and reads each touch every
// bank pair exactly twice per warp.
constexpr int F32_C = 8, F32_KS = 33, F32_RS = 1060;

// 32-point DFT, natural order in and out: two 16-point DFTs of the even and
// odd points, then X[k] = E[k] + W32^k O[k], X[k+16] = E[k] - W32^k O[k].
template <bool INV>
__device__ __forceinline__ void dft32(cf2* v) {
  cf2 e[16], o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    e[i] = v[2 * i];
    o[i] = v[2 * i + 1];
  }
  dft16<INV>(e);
  dft16<INV>(o);
  // cos(2 pi k / 32), k = 0..8
  constexpr float C32[9] = {1.0f, 0.98078528040323044913f, 0.92387953251128675613f, 0.83146961230254523708f,
                            0.70710678118654752440f, 0.55557023301960222474f, 0.38268343236508977173f,
                            0.19509032201612826785f, 0.0f};
  const float sg = INV ? 1.0f : -1.0f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    // W32^k = (cos(2 pi k/32), sg sin(2 pi k/32)); sin(2 pi k/32) = cos(2 pi (8-k)/32)
    const float c = k <= 8 ? C32[k] : -C32[16 - k];
    const float sn = k <= 8 ? C32[8 - k] : C32[k - 8];
    const cf2 t = k == 0 ? o[0] : cmul(o[k], cf2{c, sg * sn});
    v[k] = cadd(e[k], t);
    v[k + 16] = csub(e[k], t);
  }
}

template <bool COLS, bool INV>
__global__ void __launch_bounds__(32 * F32_C, 16 / F32_C)
    fft1024_kernel(const float2* __restrict__ in, float2* __restrict__ out, long long ntrans, Addr<COLS> ad,
                   const float2* __restrict__ tw, float scale) {
  extern __shared__ float2 f32_raw[];
  cf2* S = reinterpret_cast<cf2*>(f32_raw);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  static_assert(COLS, "rows use fft_kernel");
  const int c = lane % F32_C;                           // column within the CTA
  const int q = w * (32 / F32_C) + lane / F32_C;        // n2, then k1
  const long long t = (long long)blockIdx.x * F32_C + c;
  const bool active = t < ntrans;
  const long long gb = ad.base(active ? t : 0), ob = ad.obase(active ? t : 0), es = ad.estride();
  cf2 v[32];
#pragma unroll
  for (int n1 = 0; n1 < 32; ++n1) {
    const float2 x = active ? __ldcs(in + gb + (long long)(q + 32 * n1) * es) : make_float2(0.f, 0.f);
    v[n1] = {x.x, x.y};
  }
  dft32<INV>(v);  // v[k1] = Y[n2 = q][k1]
#pragma unroll
  for (int k1 = 1; k1 < 32; ++k1) {
    const float2 wv = __ldg(tw + ((q * k1) & 1023));
    v[k1] = cmul(v[k1], cf2{wv.x, INV ? -wv.y : wv.y});
  }
  cf2* Sc = S + c * F32_RS;
#pragma unroll
  for (int k1 = 0; k1 < 32; ++k1) Sc[k1 * F32_KS + q] = v[k1];
  __syncthreads();
#pragma unroll
  for (int n2 = 0; n2 < 32; ++n2) v[n2] = Sc[q * F32_KS + n2];  // now q = k1
  dft32<INV>(v);  // v[k2] = X[q + 32 k2]
  if (active) {
#pragma unroll
    for (int k2 = 0; k2 < 32; ++k2)
      __stcs(out + ob + (long long)(q + 32 * k2) * es, make_float2(v[k2].x * scale, v[k2].y * scale));
  }
}

// Column pass through TMA.  A tile is 8 adjacent columns of one 1024-row
// matrix (1024 rows x 64 bytes); one CTA transforms one tile.  Its first
// thread brings the tile into shared memory with four 256-row TMA boxes on
// one mbarrier; a thread then reads its 32 points from the buffer (row
// q + 32 n1 of column c), does the inner 32-point DFT and the twiddles (ten
// table entries, products of W^(q b) and W^(8 q a)), the 32 x 32 transpose
// goes through the same buffer in the padded layout of fft1024_kernel, and
// the outer DFT's results are written back into the buffer as a row-major
// tile that four TMA boxes store.  The copy engine takes the 64 global loads
// and stores a thread issued in fft1024_kernel, and two CTAs share an SM
// (66 KB of shared memory each), so one CTA's copies overlap the other's
// transforms.  The first thread also prefetches into L2 the tile of a CTA
// that starts later, so a CTA's own load mostly waits on L2, not DRAM.  The wait on the load is bounded (about 4 s of wall clock); on
// expiry the device error word gets JX_DEVERR_TIMEOUT and the CTA stops.
constexpr int FT_THREADS = 32 * F32_C;
constexpr int FT_ROWS_PER_BOX = 256;
constexpr unsigned FT_TILE_BYTES = 1024u * F32_C * 8u;                                  // 64 KB landed per tile
constexpr unsigned FT_BUF_BYTES = (unsigned)(F32_C * F32_RS * 8 + 127) / 128u * 128u;  // the padded transpose
constexpr size_t FT_SMEM = (size_t)FT_BUF_BYTES + 128 + 16;                             // + alignment + mbarrier

__device__ __forceinline__ uint64_t ft_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool ft_wait(uint64_t* bar, uint32_t parity) {
  if (jxd::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ft_ns();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (jxd::mbar_try_wait(bar, parity)) return true;
    if (ft_ns() - t0 > 4000000000ull) return false;
  }
}

// TMA store of a shared-memory box (no multicast), and the wait until the
// copy engine has read the box out of shared memory.
__device__ __forceinline__ void ft_store_3d(const void* tmap, const void* smem_src, int32_t x, int32_t y, int32_t z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tmap),
               "r"(jxd::smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
// L2 prefetch of a box (no shared-memory destination, no multicast).
__device__ __forceinline__ void ft_prefetch_3d(const void* tmap, int32_t x, int32_t y, int32_t z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(tmap), "r"(x), "r"(y),
               "r"(z)
               : "memory");
}
__device__ __forceinline__ void ft_store_commit_and_wait_read() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

template <bool INV>
__global__ void __launch_bounds__(FT_THREADS, 2)
    fft1024_tma_kernel(const __grid_constant__ CUtensorMap map, const __grid_constant__ CUtensorMap map_out,
                       long long tiles_per_mat, const float2* __restrict__ tw, float scale, unsigned* err,
                       unsigned ahead) {
  extern __shared__ uint8_t ft_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ft_raw) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + FT_BUF_BYTES);
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const int c = lane % F32_C;                     // column within the tile
  const int q = wp * (32 / F32_C) + lane / F32_C;  // n2, then k1
  const long long tile = blockIdx.x;
  const long long b = tile / tiles_per_mat, cb = tile % tiles_per_mat;
  if (tid == 0) {
    jxd::mbar_init(full, 1);
    jxd::fence_mbar_init();
    jxd::mbar_arrive_expect_tx(full, FT_TILE_BYTES);
#pragma unroll
    for (int k = 0; k < 1024 / FT_ROWS_PER_BOX; ++k)
      jxd::tma_load_3d(base + k * (FT_ROWS_PER_BOX * F32_C * 8), &map, full, (int32_t)(cb * 2 * F32_C),
                       k * FT_ROWS_PER_BOX, (int32_t)b);
    // The tile of the CTA `ahead` indices later (CTAs start in index order):
    // its DRAM reads overlap this CTA's transform, and that CTA's own load
    // then finds the tile in L2.
    const long long pt = tile + ahead;
    if (ahead && pt < (long long)gridDim.x) {
      const long long pb = pt / tiles_per_mat, pcb = pt % tiles_per_mat;
#pragma unroll
      for (int k = 0; k < 1024 / FT_ROWS_PER_BOX; ++k)
        ft_prefetch_3d(&map, (int32_t)(pcb * 2 * F32_C), k * FT_ROWS_PER_BOX, (int32_t)pb);
    }
  }
  __syncthreads();
  const bool ok = ft_wait(full, 0);
  if (!__syncthreads_and(ok)) {
    if (tid == 0) atomicOr(err, JX_DEVERR_TIMEOUT);
    return;
  }
  const cf2* T = reinterpret_cast<const cf2*>(base);
  cf2 v[32];
#pragma unroll
  for (int n1 = 0; n1 < 32; ++n1) v[n1] = T[(q + 32 * n1) * F32_C + c];
  dft32<INV>(v);  // v[k1] = Y[n2 = q][k1]
  {
    // W^(q k1) for k1 = 8a + b as W^(q b) W^(8 q a): ten table entries and at
    // most one complex product each, instead of 31 global loads
    cf2 lo[8], hi[4];
#pragma unroll
    for (int j = 1; j < 8; ++j) {
      const float2 t = __ldg(tw + ((q * j) & 1023));
      lo[j] = {t.x, INV ? -t.y : t.y};
    }
#pragma unroll
    for (int a = 1; a < 4; ++a) {
      const float2 t = __ldg(tw + ((q * 8 * a) & 1023));
      hi[a] = {t.x, INV ? -t.y : t.y};
    }
#pragma unroll
    for (int k1 = 1; k1 < 32; ++k1) {
      const int a = k1 >> 3, bb = k1 & 7;
      const cf2 wv = a == 0 ? lo[bb] : (bb == 0 ? hi[a] : cmul(lo[bb], hi[a]));
      v[k1] = cmul(v[k1], wv);
    }
  }
  __syncthreads();  // every thread has its points: the buffer takes the transpose
  cf2* Sc = reinterpret_cast<cf2*>(base) + c * F32_RS;
#pragma unroll
  for (int k1 = 0; k1 < 32; ++k1) Sc[k1 * F32_KS + q] = v[k1];
  __syncthreads();
#pragma unroll
  for (int n2 = 0; n2 < 32; ++n2) v[n2] = Sc[q * F32_KS + n2];  // now q = k1
  dft32<INV>(v);  // v[k2] = X[q + 32 k2]
  __syncthreads();  // the transpose is read: the buffer takes the output tile
  cf2* R = reinterpret_cast<cf2*>(base);
#pragma unroll
  for (int k2 = 0; k2 < 32; ++k2) R[(q + 32 * k2) * F32_C + c] = {v[k2].x * scale, v[k2].y * scale};
  jxd::fence_proxy_async_smem();  // this thread's writes, visible to the copy engine
  __syncthreads();
  if (tid == 0) {
#pragma unroll
    for (int k = 0; k < 1024 / FT_ROWS_PER_BOX; ++k)
      ft_store_3d(&map_out, base + k * (FT_ROWS_PER_BOX * F32_C * 8), (int32_t)(cb * 2 * F32_C), k * FT_ROWS_PER_BOX,
                  (int32_t)b);
    ft_store_commit_and_wait_read();  // the buffer must outlive the copy's reads
  }
}

// Eligible when the tensor map can describe the columns: 16-byte aligned
// input, whole 8-column tiles (w % 8 == 0), matrices 16-byte strided.
bool fft1024_tma_ok(const float2* in, const float2* out, long long w, long long hw, long long ntrans) {
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) || w % F32_C ||
      (hw * 8) % 16 || w <= 0)
    return false;
  const long long mats = ntrans / w;
  return ntrans % w == 0 && mats < (1LL << 31) && 2 * w < (1LL << 31);
}

int launch_fft1024_tma(const float2* in, float2* out, long long ntrans, long long w, long long hw, bool inv,
                       float scale, cudaStream_t st) {
  const float2* tw = nullptr;
  if (int rc = twiddles(10, &tw)) return rc;
  CUtensorMap map, map_out;
  const uint64_t dims[3] = {(uint64_t)(2 * w), 1024, (uint64_t)(ntrans / w)};
  const uint64_t strides[2] = {(uint64_t)w * 8, (uint64_t)hw * 8};
  const uint32_t box[3] = {2 * F32_C, FT_ROWS_PER_BOX, 1};
  if (int rc = jx::tensor_map_f32_3d(&map, in, dims, strides, box)) return rc;
  if (int rc = jx::tensor_map_f32_3d(&map_out, out, dims, strides, box)) return rc;
  const long long tiles_per_mat = w / F32_C, ntiles = ntrans / F32_C;
  if (ntiles == 0) return JX_OK;
  JX_REQUIRE(ntiles < (1LL << 31), "fft: batch too large");
  auto k = inv ? fft1024_tma_kernel<true> : fft1024_tma_kernel<false>;
  JX_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FT_SMEM));
  // Two CTAs per SM are resident; a CTA prefetches the tile one SM count of
  // CTAs later, about half a CTA lifetime ahead (measured at 1024^2 x 256:
  // column pass 0.867 ms without; 0.827 / 0.775 / 0.760 / 0.772 / 0.773 /
  // 0.821 ms at 1/4, 1/2, 1, 3/2, 2 and 3 tiles per SM ahead).
  const unsigned ahead = (unsigned)jx::num_sms();
  k<<<(unsigned)ntiles, FT_THREADS, FT_SMEM, st>>>(map, map_out, tiles_per_mat, tw, scale, jx::device_error_word(),
                                                   ahead);
  JX_LAUNCH_CHECK("fft1024_tma_kernel");
  return JX_OK;
}

template <bool COLS>
int launch_fft1024(const float2* in, float2* out, long long ntrans, Addr<COLS> ad, bool inv, float scale,
                   cudaStream_t st) {
  const size_t smem = sizeof(float2) * (size_t)F32_C * F32_RS;
  const float2* tw = nullptr;
  if (int rc = twiddles(10, &tw)) return rc;
  const long long blocks = (ntrans + F32_C - 1) / F32_C;
  JX_REQUIRE(blocks < (1LL << 31), "fft: batch too large");
  auto k = inv ? fft1024_kernel<COLS, true> : fft1024_kernel<COLS, false>;
  JX_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k<<<(unsigned)blocks, 32 * F32_C, smem, st>>>(in, out, ntrans, ad, tw, scale);
  JX_LAUNCH_CHECK("fft1024_kernel");
  return JX_OK;
}

template <int LOGN, int TPC, bool COLS>
int launch_fft(const float2* in, float2* out, long long ntrans, Addr<COLS> ad, bool inv, float scale,
               cudaStream_t st) {
  constexpr int N = 1 << LOGN;
  constexpr int THREADS = TPC * (N / 16);
  const size_t smem = sizeof(float2) * (size_t)TPC * region<N, COLS && TPC == 8>();
  const float2* tw = nullptr;
  int rc = twiddles(LOGN, &tw);
  if (rc) return rc;
  const long long blocks = (ntrans + TPC - 1) / TPC;
  JX_REQUIRE(blocks < (1LL << 31), "fft: batch too large");
  if (inv) {
    auto k = fft_kernel<LOGN, TPC, COLS, true>;
    JX_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<(unsigned)blocks, THREADS, smem, st>>>(in, out, ntrans, ad, tw, scale);
  } else {
    auto k = fft_kernel<LOGN, TPC, COLS, false>;
    JX_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<(unsigned)blocks, THREADS, smem, st>>>(in, out, ntrans, ad, tw, scale);
  }
  JX_LAUNCH_CHECK("fft_kernel");
  return JX_OK;
}

// Transforms per CTA: row transforms fill 256 threads; column transforms take
// 8 adjacent columns when the width allows.
template <int LOGN>
int dispatch_size(const float2* in, float2* out, long long ntrans, bool cols, long long w, long long hw, bool inv,
                  float scale, cudaStream_t st, long long os) {
  constexpr int N = 1 << LOGN;
  constexpr int T = N / 16;
  if (!cols) {
    Addr<false> ad{N, 0, 0, os};
    constexpr int TPC = T >= 256 ? 1 : 256 / T;
    return launch_fft<LOGN, TPC, false>(in, out, ntrans, ad, inv, scale, st);
  }
  Addr<true> ad{N, w, hw, 0};
  if constexpr (LOGN == 10) {
    if (fft1024_tma_ok(in, out, w, hw, ntrans)) return launch_fft1024_tma(in, out, ntrans, w, hw, inv, scale, st);
    if (w % F32_C == 0) return launch_fft1024<true>(in, out, ntrans, ad, inv, scale, st);
  }
  if constexpr (N <= 1024) {
    // 8 adjacent columns (64-byte row segments) per CTA: small enough that
    // several CTAs share an SM, so one CTA's loads overlap another's math.
    constexpr int TPC = T * 8 <= 512 ? 8 : 1;
    if (w % 8 == 0) return launch_fft<LOGN, TPC, true>(in, out, ntrans, ad, inv, scale, st);
  }
  return launch_fft<LOGN, 1, true>(in, out, ntrans, ad, inv, scale, st);
}

// os: rows only, the distance between consecutive output transforms (0: n).
int fft_batched(const float2* in, float2* out, int logn, long long ntrans, bool cols, long long w, long long hw,
                bool inv, cudaStream_t st, long long os = 0) {
  const float scale = inv ? 1.0f / (float)(1LL << logn) : 1.0f;  // ifft: 1.0 / (n as f32)
  if (logn <= 3) {
    const int threads = 256;
    const long long blocks = (ntrans + threads - 1) / threads;
    const int c = cols ? 1 : 0;
#define JX_TINY(R)                                                                                 \
  if (inv) fft_tiny_kernel<R, true><<<(unsigned)blocks, threads, 0, st>>>(in, out, ntrans, w, hw, c, scale, os); \
  else fft_tiny_kernel<R, false><<<(unsigned)blocks, threads, 0, st>>>(in, out, ntrans, w, hw, c, scale, os);
    switch (logn) {
      case 0: JX_TINY(1) break;
      case 1: JX_TINY(2) break;
      case 2: JX_TINY(4) break;
      default: JX_TINY(8) break;
    }
#undef JX_TINY
    JX_LAUNCH_CHECK("fft_tiny_kernel");
    return JX_OK;
  }
  switch (logn) {
    case 4: return dispatch_size<4>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    case 5: return dispatch_size<5>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    case 6: return dispatch_size<6>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    case 7: return dispatch_size<7>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    case 8: return dispatch_size<8>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    case 9: return dispatch_size<9>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    case 10: return dispatch_size<10>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    case 11: return dispatch_size<11>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    case 12: return dispatch_size<12>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
    default: return dispatch_size<13>(in, out, ntrans, cols, w, hw, inv, scale, st, os);
  }
}

// ---- real input / real output (fft, rfft, irfft, rfftn, irfftn) -----------
// An n-point real transform is an n/2-point complex transform of the real
// array read as interleaved complex, z[j] = x[2j] + i x[2j+1], followed by
// the split into even and odd spectra: with N2 = n/2 and W = e^{-2 pi i/n},
//   Fe[k] = (Z[k] + conj Z[N2-k]) / 2,   Fo[k] = -i (Z[k] - conj Z[N2-k]) / 2,
//   X[k] = Fe[k] + W^k Fo[k]   (k = 0..N2, indices of Z mod N2),
// and X[n-k] = conj X[k] for the full spectrum.  One thread handles the
// pair (k, N2-k): it reads exactly the two values it overwrites, so the split
// runs in place on the output.  rs: complex elements between output rows.
__device__ __forceinline__ cf2 r2c_bin(cf2 a, cf2 b_conj, cf2 w) {
  const cf2 fe{0.5f * (a.x + b_conj.x), 0.5f * (a.y + b_conj.y)};
  const cf2 d{a.x - b_conj.x, a.y - b_conj.y};
  const cf2 fo{0.5f * d.y, -0.5f * d.x};  // -i d / 2
  return cadd(fe, cmul(w, fo));
}

__global__ void r2c_split_kernel(float2* __restrict__ out, long long n, long long rs, long long rows, int full,
                                 const float2* __restrict__ tw) {
  const long long N2 = n / 2, pairs = N2 / 2 + 1;
  const long long total = rows * pairs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / pairs, k = i - r * pairs, k2 = N2 - k;
    float2* row = out + r * rs;
    const float2 zk = row[k % N2], zk2 = row[k2 % N2];
    const cf2 a{zk.x, zk.y}, b{zk2.x, zk2.y};
    const float2 wk = tw[k], wk2 = tw[k2];
    const cf2 xk = r2c_bin(a, cf2{b.x, -b.y}, cf2{wk.x, wk.y});
    const cf2 xk2 = r2c_bin(b, cf2{a.x, -a.y}, cf2{wk2.x, wk2.y});
    row[k] = make_float2(xk.x, xk.y);
    row[k2] = make_float2(xk2.x, xk2.y);
    if (full) {
      if (k > 0) row[n - k] = make_float2(xk.x, -xk.y);
      if (k2 > 0 && k2 < N2) row[n - k2] = make_float2(xk2.x, -xk2.y);
    }
  }
}

// irfft: from bins X[0..N2] (rows is = N2+1 complex apart; the imaginary parts
// of DC and Nyquist do not reach the real output, as in the reference's
// conjugate-symmetric extension), build
//   Z[k] = Xe[k] + i Xo[k],  Xe = (X[k] + conj X[N2-k]) / 2,
//   Xo = conj(W^k) (X[k] - conj X[N2-k]) / 2,
// whose N2-point inverse transform (scale 1/N2) is x[2j] + i x[2j+1].
__global__ void c2r_merge_kernel(const float2* __restrict__ in, long long is, float2* __restrict__ out, long long n,
                                 long long rows, const float2* __restrict__ tw) {
  const long long N2 = n / 2;
  const long long total = rows * N2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / N2, k = i - r * N2;
    const float2* row = in + r * is;
    float2 a = row[k], b = row[N2 - k];
    if (k == 0) {
      a.y = 0.f;
      b.y = 0.f;
    }
    const cf2 xe{0.5f * (a.x + b.x), 0.5f * (a.y - b.y)};  // (a + conj b) / 2
    const cf2 d{0.5f * (a.x - b.x), 0.5f * (a.y + b.y)};   // (a - conj b) / 2
    const float2 w = tw[k];
    const cf2 xo = cmul(cf2{w.x, -w.y}, d);
    out[r * N2 + k] = make_float2(xe.x - xo.y, xe.y + xo.x);  // xe + i xo
  }
}

int grid_for_elems(long long work) {
  long long b = (work + 255) / 256;
  const long long cap = (long long)jx::num_sms() * 8;
  if (b > cap) b = cap;
  return b < 1 ? 1 : (int)b;
}

int log2_exact(long long n) {
  int l = 0;
  while ((1LL << l) < n) ++l;
  return (1LL << l) == n ? l : -1;
}

}  // namespace

extern "C" {

int jx_fft_c2c_f32(const float* in, float* out, int64_t n, int64_t batch, int inverse, jx_stream_t stream) {
  JX_TRACE("jx_fft_c2c_f32");
  JX_REQUIRE(n >= 1 && batch >= 0, "fft: bad size");
  const int logn = log2_exact(n);
  JX_REQUIRE(logn >= 0, "FFT size must be a power of 2, got %lld", (long long)n);
  JX_REQUIRE(logn <= MAX_LOGN, "fft: n = %lld exceeds the largest supported size %d", (long long)n, 1 << MAX_LOGN);
  if (batch == 0) return JX_OK;
  JX_REQUIRE(in && out, "fft: NULL pointer");
  JX_REQUIRE((reinterpret_cast<uintptr_t>(in) & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0,
             "fft: complex buffers must be 8-byte aligned");
  return fft_batched(reinterpret_cast<const float2*>(in), reinterpret_cast<float2*>(out), logn, batch, false, 0, 0,
                     inverse != 0, jx::as_stream(stream));
}

int jx_fft2_c2c_f32(const float* in, float* out, int64_t h, int64_t w, int64_t batch, int inverse,
                    jx_stream_t stream) {
  JX_TRACE("jx_fft2_c2c_f32");
  JX_REQUIRE(h >= 1 && w >= 1 && batch >= 0, "fft2: bad size");
  const int lh = log2_exact(h), lw = log2_exact(w);
  JX_REQUIRE(lh >= 0 && lw >= 0, "FFT size must be a power of 2, got %lld x %lld", (long long)h, (long long)w);
  JX_REQUIRE(lh <= MAX_LOGN && lw <= MAX_LOGN, "fft2: sizes above %d are not supported", 1 << MAX_LOGN);
  if (batch == 0) return JX_OK;
  JX_REQUIRE(in && out, "fft2: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  // Rows of length w, then columns of length h (src/ops/fft.rs:261-313); the
  // column pass works in place on the output.
  int rc = fft_batched(reinterpret_cast<const float2*>(in), reinterpret_cast<float2*>(out), lw, h * batch, false, 0, 0,
                       inverse != 0, st);
  if (rc) return rc;
  return fft_batched(reinterpret_cast<const float2*>(out), reinterpret_cast<float2*>(out), lh, w * batch, true, w,
                     h * w, inverse != 0, st);
}

int jx_fft_r2c_f32(const float* in, float* out, int64_t n, int64_t batch, int full, jx_stream_t stream) {
  JX_TRACE("jx_fft_r2c_f32");
  JX_REQUIRE(n >= 2 && batch >= 0, "fft: bad size");
  const int logn = log2_exact(n);
  JX_REQUIRE(logn >= 0, "FFT size must be power of 2");
  JX_REQUIRE(logn - 1 <= MAX_LOGN, "fft: n = %lld exceeds the largest supported size %d", (long long)n,
             2 << MAX_LOGN);
  if (batch == 0) return JX_OK;
  JX_REQUIRE(in && out, "fft: NULL pointer");
  JX_REQUIRE((reinterpret_cast<uintptr_t>(in) & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0,
             "fft: buffers must be 8-byte aligned");
  cudaStream_t st = jx::as_stream(stream);
  const long long bins = full ? n : n / 2 + 1;
  const float2* tw = nullptr;
  int rc = twiddles(logn, &tw);
  if (!rc)
    rc = fft_batched(reinterpret_cast<const float2*>(in), reinterpret_cast<float2*>(out), logn - 1, batch, false, 0,
                     0, false, st, bins);
  if (rc) return rc;
  const long long work = batch * (n / 4 + 1);
  r2c_split_kernel<<<grid_for_elems(work), 256, 0, st>>>(reinterpret_cast<float2*>(out), n, bins, batch, full ? 1 : 0,
                                                         tw);
  JX_LAUNCH_CHECK("r2c_split_kernel");
  return JX_OK;
}

int jx_fft_c2r_f32(const float* in, float* out, int64_t n, int64_t batch, jx_stream_t stream) {
  JX_TRACE("jx_fft_c2r_f32");
  JX_REQUIRE(n >= 2 && batch >= 0, "irfft: bad size");
  const int logn = log2_exact(n);
  JX_REQUIRE(logn >= 0, "FFT size must be power of 2");
  JX_REQUIRE(logn - 1 <= MAX_LOGN, "irfft: n = %lld exceeds the largest supported size %d", (long long)n,
             2 << MAX_LOGN);
  if (batch == 0) return JX_OK;
  JX_REQUIRE(in && out, "irfft: NULL pointer");
  JX_REQUIRE((reinterpret_cast<uintptr_t>(in) & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0,
             "irfft: buffers must be 8-byte aligned");
  cudaStream_t st = jx::as_stream(stream);
  const float2* tw = nullptr;
  int rc = twiddles(logn, &tw);
  if (rc) return rc;
  c2r_merge_kernel<<<grid_for_elems(batch * (n / 2)), 256, 0, st>>>(reinterpret_cast<const float2*>(in), n / 2 + 1,
                                                                   reinterpret_cast<float2*>(out), n, batch, tw);
  JX_LAUNCH_CHECK("c2r_merge_kernel");
  return fft_batched(reinterpret_cast<const float2*>(out), reinterpret_cast<float2*>(out), logn - 1, batch, false, 0,
                     0, true, st);
}

int jx_rfft2_f32(const float* in, float* out, int64_t h, int64_t w, int64_t batch, jx_stream_t stream) {
  JX_TRACE("jx_rfft2_f32");
  JX_REQUIRE(h >= 1 && w >= 2 && batch >= 0, "rfftn: bad size");
  const int lh = log2_exact(h), lw = log2_exact(w);
  JX_REQUIRE(lh >= 0 && lw >= 0, "FFT size must be power of 2");
  JX_REQUIRE(lh <= MAX_LOGN && lw - 1 <= MAX_LOGN, "rfftn: size not supported");
  if (batch == 0) return JX_OK;
  // rows: w real -> w/2+1 bins (the reference keeps those of the full row
  // transform, src/ops/fft.rs:474-553); then the columns of the bins
  int rc = jx_fft_r2c_f32(in, out, w, h * batch, 0, stream);
  if (rc) return rc;
  const long long m = w / 2 + 1;
  return fft_batched(reinterpret_cast<const float2*>(out), reinterpret_cast<float2*>(out), lh, m * batch, true, m,
                     h * m, false, jx::as_stream(stream));
}

int jx_irfft2_f32(const float* in, float* out, int64_t h, int64_t w, int64_t batch, jx_stream_t stream) {
  JX_TRACE("jx_irfft2_f32");
  JX_REQUIRE(h >= 1 && w >= 2 && batch >= 0, "irfftn: bad size");
  const int lh = log2_exact(h), lw = log2_exact(w);
  JX_REQUIRE(lh >= 0 && lw >= 0, "FFT size must be power of 2");
  JX_REQUIRE(lh <= MAX_LOGN && lw - 1 <= MAX_LOGN, "irfftn: size not supported");
  if (batch == 0) return JX_OK;
  JX_REQUIRE(in && out, "irfftn: NULL pointer");
  // columns first (inverse, 1/h), then each row's real inverse (1/w), as
  // src/ops/fft.rs:554-628 orders them; the column result goes to scratch
  cudaStream_t st = jx::as_stream(stream);
  const long long m = w / 2 + 1;
  void* ws = nullptr;
  int rc = jx::scratch_get(sizeof(float2) * (size_t)(batch * h * m), &ws, st);
  if (rc) return rc;
  float2* cols = reinterpret_cast<float2*>(ws);
  rc = fft_batched(reinterpret_cast<const float2*>(in), cols, lh, m * batch, true, m, h * m, true, st);
  if (!rc) rc = jx_fft_c2r_f32(reinterpret_cast<const float*>(cols), out, w, h * batch, stream);
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

}  // extern "C"
