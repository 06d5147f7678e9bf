// random.cu -- the reference's PRNG streams generated on the device.
//
// PRNGKey (src/random.rs:15-97) is xorshift128+: state [s0, s1], next_u64
// shifts s0 into place and mixes it with (23, 17, 26) shifts, returns the sum.
// uniform_range (:161-181) maps next_f32 (the top 24 bits / 2^24) to
// min + (max - min) * u, randint (:189-210) takes next_u64 % range + min, and
// normal's CPU arm (:259-285) is Box-Muller over pairs of next_f32 (cos, then
// sin).  All of these are sequential on the host; the reference's GPU normal
// (src/backend/shaders.rs:814-905) is a Philox stream that does not match it.
//
// Here every thread reproduces a contiguous piece of the host stream.  The
// state update is linear over GF(2), s_{k+1} = M s_k, with a degree-128
// characteristic polynomial P (found once on the host by Berlekamp-Massey on
// one state bit).  Advancing j steps is M^j s = sum_i q_i M^i s for
// q(x) = x^j mod P(x): 128 generator steps with a conditional XOR each,
// whatever j is.  The host precomputes q for every chunk's start (a jump
// table cached per device); each thread jumps once, to the first of two
// consecutive chunks, draws both as one chain, and writes them through a
// per-warp shared-memory transpose so every store is a 128-byte row.  uniform and randint are bit-identical to the host stream; normal
// uses CUDA's logf/cosf/sinf (within a few ulp of glibc) with the
// reference's operation order otherwise.
#include <algorithm>
#include <mutex>
#include <vector>

#include "jx_common.cuh"

namespace {

constexpr int RNG_THREADS = 256;
constexpr int RNG_CHUNK = 1024;  // draws per chunk; each thread draws two consecutive chunks

struct P128 {
  uint64_t lo = 0, hi = 0;
};

// ---- the generator (host and device) ----------------------------------------
__host__ __device__ __forceinline__ uint64_t xs_next(uint64_t& a, uint64_t& b) {
  uint64_t s1 = a;
  const uint64_t s0 = b;
  a = s0;
  s1 ^= s1 << 23;
  s1 ^= s1 >> 17;
  s1 ^= s0;
  s1 ^= s0 >> 26;
  b = s1;
  return s1 + s0;
}

// state <- M^j state for q = x^j mod P (coefficients q_0..q_127)
__host__ __device__ __forceinline__ void xs_jump(uint64_t& a, uint64_t& b, uint64_t qlo, uint64_t qhi) {
  uint64_t ra = 0, rb = 0;
#pragma unroll 4
  for (int i = 0; i < 128; ++i) {
    const uint64_t bit = ((i < 64 ? qlo >> i : qhi >> (i - 64)) & 1ull);
    const uint64_t m = 0ull - bit;
    ra ^= a & m;
    rb ^= b & m;
    xs_next(a, b);
  }
  a = ra;
  b = rb;
}

// ---- host: characteristic polynomial and x^j mod P ---------------------------
struct Poly {
  bool ready = false;
  P128 p;  // P(x) = x^128 + sum p_k x^k
};
Poly g_poly;
std::mutex g_poly_mu;

// (a * x) mod P
P128 mulx(P128 a, const P128& p) {
  const uint64_t carry = a.hi >> 63;
  a.hi = (a.hi << 1) | (a.lo >> 63);
  a.lo <<= 1;
  if (carry) {
    a.lo ^= p.lo;
    a.hi ^= p.hi;
  }
  return a;
}
P128 mulmod(P128 a, const P128& b, const P128& p) {
  P128 r;
  for (int i = 0; i < 128; ++i) {
    const uint64_t bit = (i < 64 ? b.lo >> i : b.hi >> (i - 64)) & 1ull;
    if (bit) {
      r.lo ^= a.lo;
      r.hi ^= a.hi;
    }
    a = mulx(a, p);
  }
  return r;
}
P128 powx(uint64_t j, const P128& p) {
  P128 r;
  r.lo = 1;
  P128 base;
  base.lo = 2;  // x
  while (j) {
    if (j & 1) r = mulmod(r, base, p);
    base = mulmod(base, base, p);
    j >>= 1;
  }
  return r;
}

// Berlekamp-Massey over GF(2) on bit 0 of the first state word; the sequence
// of any nonzero linear functional of an irreducible recurrence has the full
// characteristic polynomial as its minimal polynomial.  Then a self-test:
// jumps by several distances must equal plain stepping.
int poly_init() {
  std::lock_guard<std::mutex> lk(g_poly_mu);
  if (g_poly.ready) return JX_OK;
  const int NS = 512;
  std::vector<int> s(NS);
  uint64_t a = 0x0123456789abcdefull, b = 0x0fedcba987654321ull;
  for (int i = 0; i < NS; ++i) {
    s[i] = (int)(a & 1);
    xs_next(a, b);
  }
  std::vector<int> C(NS + 1, 0), Bv(NS + 1, 0);
  C[0] = Bv[0] = 1;
  int L = 0, m = 1;
  for (int n = 0; n < NS; ++n) {
    int d = s[n];
    for (int i = 1; i <= L; ++i) d ^= C[i] & s[n - i];
    if (!d) {
      ++m;
      continue;
    }
    std::vector<int> T = C;
    for (int i = 0; i + m <= NS; ++i) C[i + m] ^= Bv[i];
    if (2 * L <= n) {
      L = n + 1 - L;
      Bv = T;
      m = 1;
    } else {
      ++m;
    }
  }
  if (L != 128) return jx::fail(JX_EINTERNAL, "random: recurrence of degree %d, expected 128", L);
  // P(x) = x^128 + sum_{i=1..128} C[i] x^(128-i)
  P128 p;
  for (int i = 1; i <= 128; ++i)
    if (C[i]) {
      const int k = 128 - i;
      if (k < 64) p.lo |= 1ull << k;
      else p.hi |= 1ull << (k - 64);
    }
  for (uint64_t j : {0ull, 1ull, 2ull, 3ull, 127ull, 128ull, 129ull, 1000ull, 4097ull}) {
    uint64_t x0 = 0x9e3779b97f4a7c15ull, x1 = 0x3c6ef372fe94f82aull, y0 = x0, y1 = x1;
    for (uint64_t k = 0; k < j; ++k) xs_next(x0, x1);
    const P128 q = powx(j, p);
    xs_jump(y0, y1, q.lo, q.hi);
    if (x0 != y0 || x1 != y1)
      return jx::fail(JX_EINTERNAL, "random: jump self-test failed at %llu steps", (unsigned long long)j);
  }
  g_poly.p = p;
  g_poly.ready = true;
  return JX_OK;
}

// Per device: the jump polynomial x^(c * RNG_CHUNK) mod P of every chunk c
// (grown on demand; 16 B per chunk).
struct Tables {
  ulonglong2* q = nullptr;
  long long threads = 0;
};
Tables g_tab[64];
std::mutex g_tab_mu;

int tables(long long chunks, const ulonglong2** q) {
  int rc = poly_init();
  if (rc) return rc;
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_tab_mu);
  Tables& t = g_tab[dev & 63];
  if (t.threads < chunks) {
    const P128& p = g_poly.p;
    const long long cap = std::max<long long>(chunks, 1LL << 18);
    std::vector<ulonglong2> h(cap);
    const P128 step = powx(RNG_CHUNK, p);
    P128 cur;
    cur.lo = 1;
    for (long long i = 0; i < cap; ++i) {
      h[i] = make_ulonglong2(cur.lo, cur.hi);
      cur = mulmod(cur, step, p);
    }
    ulonglong2* d = nullptr;
    JX_CUDA(cudaMalloc(&d, sizeof(ulonglong2) * cap));
    JX_CUDA(cudaMemcpy(d, h.data(), sizeof(ulonglong2) * cap, cudaMemcpyHostToDevice));
    if (t.q) JX_CUDA(cudaFree(t.q));
    t.q = d;
    t.threads = cap;
  }
  *q = t.q;
  return JX_OK;
}

// ---- device -----------------------------------------------------------------
__device__ __forceinline__ float u24(uint64_t u) {
  return __fmul_rn((float)(uint32_t)(u >> 40), 5.9604644775390625e-8f);  // top 24 bits / 2^24, exact
}

enum { RNG_UNIFORM = 0, RNG_RANDINT = 1, RNG_NORMAL = 2 };

template <int MODE>
__device__ __forceinline__ void emit2(float* row, int jj, uint64_t& a, uint64_t& b, float lo, float width,
                                      uint64_t range, int minval) {
  if constexpr (MODE == RNG_NORMAL) {
    float u1 = u24(xs_next(a, b));
    const float u2 = u24(xs_next(a, b));
    u1 = fmaxf(u1, 1e-10f);
    const float r = __fsqrt_rn(__fmul_rn(-2.0f, logf(u1)));
    const float theta = __fmul_rn(6.28318548202514648438f, u2);  // 2.0f * PI (exact doubling)
    row[jj] = __fmul_rn(r, cosf(theta));
    row[jj + 1] = __fmul_rn(r, sinf(theta));
  } else {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint64_t u = xs_next(a, b);
      if constexpr (MODE == RNG_UNIFORM) row[jj + k] = __fadd_rn(lo, __fmul_rn(width, u24(u)));
      else row[jj + k] = (float)((int)(u % range) + minval);
    }
  }
}

// Thread g draws chunks 2g and 2g+1 (2 * RNG_CHUNK consecutive values
// starting at 2g * RNG_CHUNK) as one chain from one jump, 32 per step into
// its row of the warp's tile; the warp then writes the tile row by row, each
// row one 128-byte segment of one thread's range.  (Two chains per thread,
// one jump each, with 64-byte row segments measured 3353 GB/s against 3498.)
template <int MODE>
__global__ void __launch_bounds__(RNG_THREADS) rng_kernel(uint64_t s0, uint64_t s1, const ulonglong2* __restrict__ tq,
                                                        float* __restrict__ out, long long n, float lo, float width,
                                                        uint64_t range, int minval) {
  constexpr int SPAN = 2 * RNG_CHUNK;
  __shared__ float tile[RNG_THREADS / 32][32][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long warp_first = (long long)blockIdx.x * RNG_THREADS + warp * 32;  // global thread of lane 0
  if (warp_first * SPAN >= n) return;  // whole warp past the end
  const long long g = warp_first + lane;
  uint64_t a = s0, b = s1;
  const ulonglong2 q = tq[2 * g];
  xs_jump(a, b, q.x, q.y);
  float (*T)[33] = tile[warp];
  for (int j0 = 0; j0 < SPAN; j0 += 32) {
#pragma unroll 4
    for (int jj = 0; jj < 32; jj += 2) emit2<MODE>(T[lane], jj, a, b, lo, width, range, minval);
    __syncwarp();
    // row r of the tile goes to (warp_first + r) * SPAN + j0 + lane
    const long long idx0 = warp_first * SPAN + j0 + lane;
    if ((warp_first + 31) * SPAN + j0 + 31 < n) {  // the whole tile is in range (warp-uniform)
      float* p = out + idx0;
#pragma unroll 8
      for (int r = 0; r < 32; ++r, p += SPAN) __stcs(p, T[r][lane]);
    } else {
#pragma unroll 4
      for (int r = 0; r < 32; ++r) {
        const long long idx = idx0 + (long long)r * SPAN;
        if (idx < n) __stcs(out + idx, T[r][lane]);
      }
    }
    __syncwarp();
  }
}

template <int MODE>
int launch_rng(uint64_t s0, uint64_t s1, float* out, long long n, float lo, float width, uint64_t range, int minval,
               cudaStream_t st) {
  const long long per_block = (long long)RNG_THREADS * 2 * RNG_CHUNK;
  const long long blocks = (n + per_block - 1) / per_block;
  JX_REQUIRE(blocks < (1LL << 31), "random: too many elements");
  const ulonglong2* tq = nullptr;
  int rc = tables(blocks * RNG_THREADS * 2, &tq);
  if (rc) return rc;
  rng_kernel<MODE><<<(unsigned)blocks, RNG_THREADS, 0, st>>>(s0, s1, tq, out, n, lo, width, range, minval);
  JX_LAUNCH_CHECK("rng_kernel");
  return JX_OK;
}

}  // namespace

extern "C" {

// PRNGKey::from_seed (src/random.rs:29-32): [seed, seed * 0x9e3779b97f4a7c15]
int jx_random_key_from_seed(uint64_t seed, uint64_t* s0, uint64_t* s1) {
  JX_TRACE("jx_random_key_from_seed");
  JX_REQUIRE(s0 && s1, "jx_random_key_from_seed: NULL");
  *s0 = seed;
  *s1 = seed * 0x9e3779b97f4a7c15ull;
  return JX_OK;
}

// PRNGKey::split (src/random.rs:35-48): the first key adds 0x9e3779b97f4a7c15
// to word 0 and rotates word 1 left by 27; the second adds 0x3c6ef372fe94f82a
// and rotates right by 17.
int jx_random_key_split(uint64_t s0, uint64_t s1, uint64_t* a0, uint64_t* a1, uint64_t* b0, uint64_t* b1) {
  JX_TRACE("jx_random_key_split");
  JX_REQUIRE(a0 && a1 && b0 && b1, "jx_random_key_split: NULL");
  *a0 = s0 + 0x9e3779b97f4a7c15ull;
  *a1 = (s1 << 27) | (s1 >> 37);
  *b0 = s0 + 0x3c6ef372fe94f82aull;
  *b1 = (s1 >> 17) | (s1 << 47);
  return JX_OK;
}

int jx_random_jump(uint64_t* s0, uint64_t* s1, uint64_t steps) {
  JX_TRACE("jx_random_jump");
  JX_REQUIRE(s0 && s1, "jx_random_jump: NULL");
  int rc = poly_init();
  if (rc) return rc;
  const P128 q = powx(steps, g_poly.p);
  xs_jump(*s0, *s1, q.lo, q.hi);
  return JX_OK;
}

int jx_random_uniform_f32(uint64_t s0, uint64_t s1, float* out, int64_t n, float minval, float maxval,
                          jx_stream_t stream) {
  JX_TRACE("jx_random_uniform_f32");
  JX_REQUIRE(n >= 0, "random: negative size");
  if (n == 0) return JX_OK;
  JX_REQUIRE(out, "random: NULL output");
  const float width = maxval - minval;  // f32, as the reference rounds (max - min) per draw
  return launch_rng<RNG_UNIFORM>(s0, s1, out, n, minval, width, 1, 0, jx::as_stream(stream));
}

int jx_random_randint_f32(uint64_t s0, uint64_t s1, float* out, int64_t n, int32_t minval, int32_t maxval,
                          jx_stream_t stream) {
  JX_TRACE("jx_random_randint_f32");
  JX_REQUIRE(n >= 0, "random: negative size");
  JX_REQUIRE(minval < maxval, "minval must be less than maxval");
  if (n == 0) return JX_OK;
  JX_REQUIRE(out, "random: NULL output");
  const uint64_t range = (uint64_t)(int64_t)(maxval - minval);
  return launch_rng<RNG_RANDINT>(s0, s1, out, n, 0.f, 0.f, range, minval, jx::as_stream(stream));
}

int jx_random_normal_f32(uint64_t s0, uint64_t s1, float* out, int64_t n, jx_stream_t stream) {
  JX_TRACE("jx_random_normal_f32");
  JX_REQUIRE(n >= 0, "random: negative size");
  if (n == 0) return JX_OK;
  JX_REQUIRE(out, "random: NULL output");
  return launch_rng<RNG_NORMAL>(s0, s1, out, n, 0.f, 0.f, 1, 0, jx::as_stream(stream));
}

}  // extern "C"
