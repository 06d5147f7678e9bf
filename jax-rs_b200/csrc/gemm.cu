// gemm.cu -- f32 GEMM for Array::matmul (src/ops/linalg.rs:154-237), the
// batched einsum "bij,bjk->bik" (src/ops/einsum.rs:488-523) and the matmul
// transposes used by transpose_matmul (src/trace/transpose_rules.rs:537-567).
//
// JX_PREC_3XTF32: f32 accuracy on the 5th-generation tensor cores.
//   1. split pass: every operand element x becomes hi = tf32_rn(x) and
//      lo = tf32_rn(x - hi), written K-major (rows of K contiguous floats,
//      K padded to the k-block) into library scratch; transposed operands are
//      transposed here, so the main kernel only ever sees K-major tiles.
//   2. main kernel (persistent, one CTA per SM, warp-specialised):
//        warp 0      TMA producer: Ahi, Alo, Bhi, Blo tiles -> smem ring
//        warp 1      TMEM allocator + single-thread tcgen05.mma issuer:
//                    D += Ah.Bh + Ah.Bl + Al.Bh  (kind::tf32, f32 accumulate in TMEM)
//        warps 2..9  epilogue: the tile's f32 accumulator lives in registers
//      K is consumed in spans of 128: the MMA warp sums one span into one of
//      two TMEM partial buffers (2 x 256 columns, ping-pong) while the
//      epilogue adds the previous span into registers with round-to-nearest.
//      The tensor core's internal accumulation truncates; short TMEM sums
//      keep that bias from growing with K, so the result holds f32 accuracy
//      at any K.  The epilogue stores C once per tile.
//   Row-major A and B (no transpose, 16-byte aligned rows) skip the split
//   pass: gemm_fused_split_kernel streams the raw f32 tiles by TMA (B as an
//   MN-major operand) and splits them in shared memory.
// JX_PREC_EXACT: one thread per output, sequential k, no FMA contraction: the
//   reference CPU loop's exact rounding sequence (bit-identical results).
#include <algorithm>
#include <mutex>

#include "tc_gemm.cuh"

namespace {

using namespace jxg;
constexpr size_t GEMM_SMEM = (size_t)STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                       const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                       float* __restrict__ C, int M, int N, int Kp, long long ldc, long long strideC,
                       int tiles_m, int tiles_n, int num_tiles, int a_bcast, int b_bcast, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = jxd::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;                     // [STAGES] TMA -> MMA
  uint64_t* empty = bars + STAGES;           // [STAGES] MMA -> TMA
  uint64_t* sfull = bars + 2 * STAGES;       // [2] span partial ready (MMA -> epilogue)
  uint64_t* sempty = bars + 2 * STAGES + 2;  // [2] span partial drained (epilogue -> MMA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = Kp / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      jxd::mbar_init(&full[s], 1);
      jxd::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      jxd::mbar_init(&sfull[a], 1);
      jxd::mbar_init(&sempty[a], EPI_WARPS);
    }
    *abort_flag = 0;
    jxd::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    jxd::tma_prefetch_desc(&tmAh);
    jxd::tma_prefetch_desc(&tmAl);
    jxd::tma_prefetch_desc(&tmBh);
    jxd::tma_prefetch_desc(&tmBl);
  }
  if (warp == 1) {
    jxd::tmem_alloc(tmem_slot, TMEM_COLS);
    jxd::tmem_relinquish();
  }
  jxd::tc_fence_before();
  __syncthreads();
  jxd::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (jxd::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        TileInfo ti = tile_coords(t, tiles_m, tiles_n);
        const int ya = ti.m_blk * BM, yb = ti.n_blk * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bounded(&empty[stage], phase ^ 1u, err)) { *abort_flag = 1; break; }
          uint8_t* st = smem + stage * STAGE_BYTES;
          jxd::mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          const int x = kb * BK;
          const int za = a_bcast ? 0 : ti.b, zb = b_bcast ? 0 : ti.b;  // a broadcast operand has one batch entry
          jxd::tma_load_3d(st, &tmAh, &full[stage], x, ya, za);
          jxd::tma_load_3d(st + A_TILE, &tmAl, &full[stage], x, ya, za);
          jxd::tma_load_3d(st + 2 * A_TILE, &tmBh, &full[stage], x, yb, zb);
          jxd::tma_load_3d(st + 2 * A_TILE + B_TILE, &tmBl, &full[stage], x, yb, zb);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: wait (bounded) until every load issued above has been consumed.
      for (int s = 0; s < STAGES; ++s) {
        if (!wait_bounded(&empty[stage], phase ^ 1u, err)) break;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (jxd::elect_one()) mma_issuer(smem, full, empty, sfull, sempty, tmem_base, num_tiles, num_kb, abort_flag, err);
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    // Thread: one output row (TMEM lane), EPI_COLS columns of the tile.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const bool vec_ok = ((ldc & 3) == 0) && ((strideC & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    uint32_t span_ctr = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      float acc[EPI_COLS];
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.0f;
      bool ok = true;
      for (int kb0 = 0; kb0 < num_kb; kb0 += SPAN_KB) {
        if (!drain_span(acc, tmem_base, span_ctr, sfull, sempty, warp, lane, abort_flag, err)) { ok = false; break; }
        ++span_ctr;
      }
      if (!ok) break;
      TileInfo ti = tile_coords(t, tiles_m, tiles_n);
      const int row = ti.m_blk * BM + q * 32 + lane;
      if (row < M) {
        float* crow = C + (long long)ti.b * strideC + (long long)row * ldc;
        const int col0 = ti.n_blk * BN + half * EPI_COLS;
        if (vec_ok && col0 + EPI_COLS <= N) {
          float4* dst = reinterpret_cast<float4*>(crow + col0);
#pragma unroll
          for (int v = 0; v < EPI_COLS / 4; ++v)
            dst[v] = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < EPI_COLS; ++j)
            if (col0 + j < N) crow[col0 + j] = acc[j];
        }
      }
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
// Fused split: C = A . B with A [batch][M][K] and B [batch][K][N] both
// row-major, straight from the caller's f32 buffers (no split pass, no
// workspace).  TMA streams the raw tiles -- A K-major with 128-byte swizzle,
// B MN-major as eight 32 x 32 boxes in the SWIZZLE_128B_ATOM_32B layout --
// into the hi slots of the stage, where they stay: the tf32 MMA reads a raw
// f32 value as hi = trunc(x) (its low 13 bits ignored), so the hi.hi products
// start as soon as the tiles land.  Meanwhile the eight epilogue warps write
// lo = tf32_rn(x - trunc(x)) into the lo slot (same offset, so the layout is
// kept) and publish it for the two cross products; as in the pre-split kernel
// they then drain the TMEM span partials and store C.  The operand error per
// element is at most 2^-21 relative (2^-22 for the pre-split kernel's
// round-to-nearest hi).  K beyond the matrix reads TMA's zero fill.  Warpgroup 0 (TMA, MMA, two idle warps) gives
// registers to the two epilogue warpgroups: 128 x 40 + 256 x 232 = 384 x 168.
// ---------------------------------------------------------------------------
constexpr int FS_THREADS = 384;
constexpr int FS_FIRST_EPI = 4;
constexpr int FS_LAUNCH_REGS = 168;
constexpr int FS_LOW_REGS = 40;
constexpr int FS_HIGH_REGS = 232;
static_assert(128 * FS_LOW_REGS + 256 * FS_HIGH_REGS <= FS_THREADS * FS_LAUNCH_REGS,
              "register split exceeds the launch allocation");
constexpr int B_BOX_BYTES = 32 * BK * 4;  // one 32 (N) x 32 (K) box of B
constexpr size_t FS_SMEM = (size_t)STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

__global__ void __launch_bounds__(FS_THREADS, 1)
    gemm_fused_split_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            float* __restrict__ C, int M, int N, int num_kb, long long ldc, long long strideC,
                            int tiles_m, int tiles_n, int num_tiles, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = jxd::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* raw_full = bars;                 // [STAGES] TMA landed the raw tiles
  uint64_t* full = bars + STAGES;            // [STAGES] hi/lo written (epilogue warps -> MMA)
  uint64_t* empty = bars + 2 * STAGES;       // [STAGES] MMA done with the stage
  uint64_t* sfull = bars + 3 * STAGES;       // [2] span partial ready
  uint64_t* sempty = bars + 3 * STAGES + 2;  // [2] span partial drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      jxd::mbar_init(&raw_full[s], 1);
      jxd::mbar_init(&full[s], EPI_WARPS);
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
    jxd::tma_prefetch_desc(&tmA);
    jxd::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    jxd::tmem_alloc(tmem_slot, TMEM_COLS);
    jxd::tmem_relinquish();
  }
  jxd::tc_fence_before();
  __syncthreads();
  jxd::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < FS_FIRST_EPI) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(FS_LOW_REGS));
    // ---------------- TMA: raw A and B tiles ----------------
    if (warp == 0 && jxd::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        const TileInfo ti = tile_coords(t, tiles_m, tiles_n);
        const int ya = ti.m_blk * BM, xb = ti.n_blk * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bounded(&empty[stage], phase ^ 1u, err)) { *abort_flag = 1; break; }
          uint8_t* st = smem + stage * STAGE_BYTES;
          jxd::mbar_arrive_expect_tx(&raw_full[stage], A_TILE + B_TILE);
          jxd::tma_load_3d(st, &tmA, &raw_full[stage], kb * BK, ya, ti.b);
#pragma unroll
          for (int i = 0; i < BN / 32; ++i)
            jxd::tma_load_3d(st + 2 * A_TILE + i * B_BOX_BYTES, &tmB, &raw_full[stage], xb + 32 * i, kb * BK, ti.b);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      for (int s = 0; s < STAGES; ++s) {
        if (!wait_bounded(&empty[stage], phase ^ 1u, err)) break;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
    // ---------------- MMA issuer ----------------
    if (warp == 1 && jxd::elect_one())
      mma_issuer<true>(smem, full, empty, sfull, sempty, tmem_base, num_tiles, num_kb, abort_flag, err, raw_full);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(FS_HIGH_REGS));
    // ---------------- split the stage in place, drain spans, store C ----------------
    const int gt = threadIdx.x - FS_FIRST_EPI * 32;  // 0..255
    const int q = warp & 3, half = (warp - FS_FIRST_EPI) >> 2;
    const bool vec_ok = ((ldc & 3) == 0) && ((strideC & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t span_ctr = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      float acc[EPI_COLS];
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.0f;
      bool ok = true;
      int spans_done = 0;
      const int nspan = (num_kb + SPAN_KB - 1) / SPAN_KB;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (*abort_flag || !wait_bounded(&raw_full[stage], phase, err)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        uint8_t* st = smem + stage * STAGE_BYTES;
        // 3072 float4 per stage (A: 1024, B: 2048), 12 per thread, consecutive
        // threads on consecutive 16-byte chunks
#pragma unroll
        for (int j = 0; j < (A_TILE + B_TILE) / 16 / 256; ++j) {
          const int f = gt + 256 * j;
          uint8_t* hp = f < A_TILE / 16 ? st + f * 16 : st + 2 * A_TILE + (f - A_TILE / 16) * 16;
          const int lo_off = f < A_TILE / 16 ? A_TILE : B_TILE;
          const float4 x = *reinterpret_cast<const float4*>(hp);
          float4 l;
          l.x = jxd::tf32_lo_of_trunc(x.x);
          l.y = jxd::tf32_lo_of_trunc(x.y);
          l.z = jxd::tf32_lo_of_trunc(x.z);
          l.w = jxd::tf32_lo_of_trunc(x.w);
          *reinterpret_cast<float4*>(hp + lo_off) = l;
        }
        jxd::fence_proxy_async_smem();  // generic-proxy writes -> tensor core reads
        __syncwarp();
        if (lane == 0) jxd::mbar_arrive(&full[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        // Once span i is fully split, drain span i-1.
        if ((kb % SPAN_KB == SPAN_KB - 1 || kb == num_kb - 1) && kb >= SPAN_KB) {
          if (!drain_span<32, FS_FIRST_EPI>(acc, tmem_base, span_ctr, sfull, sempty, warp, lane, abort_flag, err)) {
            ok = false;
            break;
          }
          ++span_ctr;
          ++spans_done;
        }
      }
      while (ok && spans_done < nspan) {
        if (!drain_span<32, FS_FIRST_EPI>(acc, tmem_base, span_ctr, sfull, sempty, warp, lane, abort_flag, err))
          ok = false;
        ++span_ctr;
        ++spans_done;
      }
      if (!ok) break;
      const TileInfo ti = tile_coords(t, tiles_m, tiles_n);
      const int row = ti.m_blk * BM + q * 32 + lane;
      if (row < M) {
        float* crow = C + (long long)ti.b * strideC + (long long)row * ldc;
        const int col0 = ti.n_blk * BN + half * EPI_COLS;
        if (vec_ok && col0 + EPI_COLS <= N) {
          float4* dst = reinterpret_cast<float4*>(crow + col0);
#pragma unroll
          for (int v = 0; v < EPI_COLS / 4; ++v)
            dst[v] = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < EPI_COLS; ++j)
            if (col0 + j < N) crow[col0 + j] = acc[j];
        }
      }
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
// Operand split: dst_hi/dst_lo [batch][rows][Kp] K-major, zero-padded K..Kp.
//   direct:     element (r, k) at src[b*sb + r*ld + k]
//   transposed: element (r, k) at src[b*sb + k*ld + r]
// ---------------------------------------------------------------------------
using jxd::split_tf32;

__global__ void split_direct_kernel(const float* __restrict__ src, float* __restrict__ hi,
                                    float* __restrict__ lo, int rows, int K, int Kp, long long ld,
                                    long long sb) {
  const int b = blockIdx.z;
  const long long total = (long long)rows * Kp;
  const float* s = src + (long long)b * sb;
  float* h = hi + (long long)b * total;
  float* l = lo + (long long)b * total;
  const bool vec = ((ld & 3) == 0) && ((sb & 3) == 0) && ((K & 3) == 0) &&
                   ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* sr = s + (long long)r * ld;
    float* hr = h + (long long)r * Kp;
    float* lr = l + (long long)r * Kp;
    if (vec) {
      for (int k = threadIdx.x * 4; k < Kp; k += blockDim.x * 4) {
        float4 x = k < K ? *reinterpret_cast<const float4*>(sr + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 xh, xl;
        split_tf32(x.x, xh.x, xl.x);
        split_tf32(x.y, xh.y, xl.y);
        split_tf32(x.z, xh.z, xl.z);
        split_tf32(x.w, xh.w, xl.w);
        *reinterpret_cast<float4*>(hr + k) = xh;
        *reinterpret_cast<float4*>(lr + k) = xl;
      }
    } else {
      for (int k = threadIdx.x; k < Kp; k += blockDim.x) {
        float x = k < K ? sr[k] : 0.0f;
        float xh, xl;
        split_tf32(x, xh, xl);
        hr[k] = xh;
        lr[k] = xl;
      }
    }
  }
}

__global__ void split_transpose_kernel(const float* __restrict__ src, float* __restrict__ hi,
                                       float* __restrict__ lo, int rows, int K, int Kp, long long ld,
                                       long long sb) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const float* s = src + (long long)b * sb;
  const long long total = (long long)rows * Kp;
  float* h = hi + (long long)b * total;
  float* l = lo + (long long)b * total;
  const int r0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  // read: element (r, k) lives at s[k*ld + r]; coalesced along r
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int k = k0 + j, r = r0 + threadIdx.x;
    tile[j][threadIdx.x] = (k < K && r < rows) ? s[(long long)k * ld + r] : 0.0f;
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int r = r0 + j, k = k0 + threadIdx.x;
    if (r < rows && k < Kp) {
      float xh, xl;
      split_tf32(tile[threadIdx.x][j], xh, xl);
      h[(long long)r * Kp + k] = xh;
      l[(long long)r * Kp + k] = xl;
    }
  }
}

// ---------------------------------------------------------------------------
// Exact path: the reference loop's rounding sequence (src/ops/linalg.rs:220-228):
// sum = 0; for p in 0..k { sum = sum + a*b } with each product and sum rounded.
// ---------------------------------------------------------------------------
// One thread per output of a 16 x 16 tile.  K streams through shared memory
// in chunks of EX_KC: the next chunk is loaded into registers while the
// current one is summed, so each chunk costs one barrier and its loads are in
// flight behind EX_KC dependent additions (K = 784 takes 7 round trips to L2,
// not 49).  Every output still sums its products in ascending k from 0.
constexpr int EX_T = 16, EX_KC = 128, EX_PER = EX_T * EX_KC / (EX_T * EX_T);  // 8 loads per operand

__global__ void __launch_bounds__(EX_T* EX_T)
    gemm_exact_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M, int N,
                      int K, int transA, int transB, long long lda, long long ldb, long long ldc, long long sA,
                      long long sB, long long sC) {
  __shared__ float As[2][EX_T][EX_KC + 1];  // [row][k]
  __shared__ float Bs[2][EX_KC][EX_T + 1];  // [k][col]
  const int b = blockIdx.z;
  const float* a = A + (long long)b * sA;
  const float* bb = B + (long long)b * sB;
  const int tid = threadIdx.y * EX_T + threadIdx.x;
  const int r0 = blockIdx.y * EX_T, c0 = blockIdx.x * EX_T;
  // Element e of this thread's share of a chunk: (tile row or column, k within
  // the chunk), arranged so that consecutive threads read consecutive
  // addresses of the operand as stored.
  auto a_at = [&](int e, int& r, int& k) {
    if (transA) { r = tid & (EX_T - 1); k = (tid >> 4) + 16 * e; }    // a[k][r]: r fastest
    else { k = tid & (EX_KC - 1); r = (tid >> 7) + 2 * e; }           // a[r][k]: k fastest
  };
  auto b_at = [&](int e, int& k, int& c) {
    if (transB) { k = tid & (EX_KC - 1); c = (tid >> 7) + 2 * e; }    // b[c][k]: k fastest
    else { c = tid & (EX_T - 1); k = (tid >> 4) + 16 * e; }           // b[k][c]: c fastest
  };
  float ra[EX_PER], rb[EX_PER];
  auto load = [&](int k0) {
#pragma unroll
    for (int e = 0; e < EX_PER; ++e) {
      int r, k, c, kb;
      a_at(e, r, k);
      const int gr = r0 + r, gk = k0 + k;
      ra[e] = (gr < M && gk < K) ? (transA ? a[(long long)gk * lda + gr] : a[(long long)gr * lda + gk]) : 0.0f;
      b_at(e, kb, c);
      const int gkb = k0 + kb, gc = c0 + c;
      rb[e] = (gkb < K && gc < N) ? (transB ? bb[(long long)gc * ldb + gkb] : bb[(long long)gkb * ldb + gc]) : 0.0f;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int e = 0; e < EX_PER; ++e) {
      int r, k, c, kb;
      a_at(e, r, k);
      As[buf][r][k] = ra[e];
      b_at(e, kb, c);
      Bs[buf][kb][c] = rb[e];
    }
  };
  const int nchunk = (K + EX_KC - 1) / EX_KC;
  load(0);
  store(0);
  __syncthreads();
  float sum = 0.0f;
  for (int ch = 0; ch < nchunk; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < nchunk) load((ch + 1) * EX_KC);
    const int kmax = min(EX_KC, K - ch * EX_KC);
    for (int kk = 0; kk < kmax; ++kk)
      sum = __fadd_rn(sum, __fmul_rn(As[buf][threadIdx.y][kk], Bs[buf][kk][threadIdx.x]));
    if (ch + 1 < nchunk) store(buf ^ 1);
    __syncthreads();
  }
  const int row = r0 + threadIdx.y, col = c0 + threadIdx.x;
  if (row < M && col < N) C[(long long)b * sC + (long long)row * ldc + col] = sum;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return jx::fail(JX_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  return JX_OK;
}

int make_kmajor_map(CUtensorMap* map, const float* base, int Kp, int rows, int batch, int box_rows) {
  cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)Kp * 4, (cuuint64_t)Kp * 4 * (cuuint64_t)rows};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return jx::fail(JX_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return JX_OK;
}

inline long long round_up(long long x, long long m) { return (x + m - 1) / m * m; }

// 3-D f32 tensor map: dims {d0 (contiguous), d1, d2}, byte strides s1, s2,
// box {b0, b1, 1}, the given swizzle.
int make_map_3d(CUtensorMap* map, const float* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
                uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return jx::fail(JX_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return JX_OK;
}

// The fused-split kernel reads A and B straight from the caller: both
// row-major (no transpose), rows and batch entries 16-byte aligned, one batch
// entry per product (no broadcast operand).
bool fused_split_ok(const float* A, const float* B, int transA, int transB, long long lda, long long ldb,
                    long long batch, long long sA, long long sB) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (transA || transB || !a16(A) || !a16(B) || (lda & 3) || (ldb & 3)) return false;
  if (batch > 1 && (sA <= 0 || sB <= 0 || (sA & 3) || (sB & 3))) return false;
  return true;
}

// Per device, once: the fused kernel's shared-memory limit and its register
// count at launch.
std::mutex g_prepare_mu;  // guards the per-device one-time attribute settings below

int fused_prepare(int* regs_out) {
  static int regs[64] = {0};
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_prepare_mu);
  if (!regs[dev & 63]) {
    cudaFuncAttributes fa;
    JX_CUDA(cudaFuncGetAttributes(&fa, gemm_fused_split_kernel));
    JX_CUDA(cudaFuncSetAttribute(gemm_fused_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FS_SMEM));
    regs[dev & 63] = fa.numRegs;
  }
  if (regs_out) *regs_out = regs[dev & 63];
  return JX_OK;
}

// Per device, once: the main kernel's shared-memory limit.  Two host threads
// making their first call on a device serialise on the mutex.
int main_prepare() {
  static bool attr_set[64] = {false};
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_prepare_mu);
  if (!attr_set[dev & 63]) {
    JX_CUDA(cudaFuncSetAttribute(gemm_3xtf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMM_SMEM));
    attr_set[dev & 63] = true;
  }
  return JX_OK;
}

int launch_fused_split(const float* A, const float* B, float* C, long long M, long long N, long long K, long long lda,
                       long long ldb, long long ldc, long long batch, long long sA, long long sB, long long sC,
                       cudaStream_t st) {
  int rc = get_encode();
  if (rc) return rc;
  // The register split inside the kernel assumes exactly FS_LAUNCH_REGS per
  // thread at launch; with any other allocation setmaxnreg.inc could wait for
  // registers that never come, so refuse to launch.
  int regs = 0;
  if ((rc = fused_prepare(&regs))) return rc;
  if (regs != FS_LAUNCH_REGS)
    return jx::fail(JX_EUNSUPPORTED, "gemm_fused_split_kernel built with %d registers per thread, expected %d",
                    regs, FS_LAUNCH_REGS);
  CUtensorMap mA, mB;
  const uint64_t sa = batch > 1 ? (uint64_t)sA * 4 : (uint64_t)lda * 4 * (uint64_t)M;
  const uint64_t sb = batch > 1 ? (uint64_t)sB * 4 : (uint64_t)ldb * 4 * (uint64_t)K;
  if ((rc = make_map_3d(&mA, A, K, M, batch, lda * 4, sa, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = make_map_3d(&mB, B, N, K, batch, ldb * 4, sb, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))) return rc;
  const int tiles_m = (int)((M + BM - 1) / BM), tiles_n = (int)((N + BN - 1) / BN);
  const long long nt = (long long)tiles_m * tiles_n * batch;
  if (nt > 0x7fffffffLL) return jx::fail(JX_EINVAL, "gemm: too many tiles");
  const int grid = (int)std::min<long long>(nt, jx::num_sms());
  const int num_kb = (int)((K + BK - 1) / BK);
  gemm_fused_split_kernel<<<grid, FS_THREADS, FS_SMEM, st>>>(mA, mB, C, (int)M, (int)N, num_kb, ldc, sC, tiles_m,
                                                             tiles_n, (int)nt, jx::device_error_word());
  JX_LAUNCH_CHECK("gemm_fused_split_kernel");
  return JX_OK;
}

// Split-K for products with too few output tiles to fill the GPU: the
// k-blocks are cut into S equal slices (S divides their number, so no slice
// reads past a padded row), each slice a batch entry of the same pre-split
// operands (a 3-D tensor map whose batch stride is the slice's offset along
// K), its partial product written to scratch; the partials are then added in
// slice order.
int splitk_slices(long long tiles, long long num_kb) {
  const long long want = std::min<long long>(16, jx::num_sms() / std::max<long long>(1, tiles));
  for (long long S = want; S >= 2; --S)
    if (num_kb % S == 0 && num_kb / S >= SPAN_KB) return (int)S;
  return 1;
}

__global__ void splitk_sum_kernel(const float* __restrict__ part, float* __restrict__ C, int M, int N, int S,
                                  long long ldc) {
  const long long total = (long long)M * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float acc = part[i];
    for (int sl = 1; sl < S; ++sl) acc += part[(long long)sl * total + i];
    const long long m = i / N, n = i - m * N;
    C[m * ldc + n] = acc;
  }
}

int launch_split(const float* src, float* hi, float* lo, int rows, int K, int Kp, long long ld, long long sb,
                 int batch, bool transposed, cudaStream_t st) {
  if (!transposed) {
    int blocks = (int)std::min<long long>(rows, (long long)jx::num_sms() * 16);
    split_direct_kernel<<<dim3(blocks, 1, batch), 256, 0, st>>>(src, hi, lo, rows, K, Kp, ld, sb);
  } else {
    dim3 grid((rows + 31) / 32, (Kp + 31) / 32, batch);
    split_transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(src, hi, lo, rows, K, Kp, ld, sb);
  }
  JX_LAUNCH_CHECK("gemm split kernel");
  return JX_OK;
}

}  // namespace

namespace jx {
// For the SM-pair kernel (gemm_pair.cu).
int get_encode_fn() { return get_encode(); }
int make_map_3d_fn(CUtensorMap* map, const float* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                   uint64_t s2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
  return make_map_3d(map, base, d0, d1, d2, s1, s2, b0, b1, sw);
}
bool pair_gemm_ok(const float* A, const float* B, long long M, long long N, long long lda, long long ldb,
                  long long batch, long long sA, long long sB);
int launch_pair_gemm(const float* A, const float* B, float* C, long long M, long long N, long long K, bool transA,
                     bool transB, long long lda, long long ldb, long long ldc, long long batch, long long sA,
                     long long sB, long long sC, cudaStream_t st);

// Shared by conv2d (implicit GEMM) and the dense layers: 3xTF32 GEMM on
// pre-split K-major operands.  Ah/Al: [batch][M][Kp]; Bh/Bl: [batch][N][Kp].
// Launches the main kernel; `err` is the device word it flags a timed-out wait in.
// a_bcast / b_bcast: that operand has a single batch entry shared by every
// batch entry of the other (conv2d's weights).
int gemm_presplit_err(const float* Ah, const float* Al, const float* Bh, const float* Bl, float* C, int M, int N,
                      int Kp, long long ldc, long long strideC, int batch, cudaStream_t st, unsigned int* err,
                      bool a_bcast, bool b_bcast) {
  int rc = get_encode();
  if (rc) return rc;
  CUtensorMap mAh, mAl, mBh, mBl;
  if ((rc = make_kmajor_map(&mAh, Ah, Kp, M, a_bcast ? 1 : batch, BM))) return rc;
  if ((rc = make_kmajor_map(&mAl, Al, Kp, M, a_bcast ? 1 : batch, BM))) return rc;
  if ((rc = make_kmajor_map(&mBh, Bh, Kp, N, b_bcast ? 1 : batch, BN))) return rc;
  if ((rc = make_kmajor_map(&mBl, Bl, Kp, N, b_bcast ? 1 : batch, BN))) return rc;
  if ((rc = main_prepare())) return rc;
  const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
  const long long nt = (long long)tiles_m * tiles_n * batch;
  if (nt > 0x7fffffffLL) return fail(JX_EINVAL, "gemm: too many tiles");
  const int grid = (int)std::min<long long>(nt, num_sms());
  gemm_3xtf32_kernel<<<grid, GEMM_THREADS, GEMM_SMEM, st>>>(mAh, mAl, mBh, mBl, C, M, N, Kp, ldc, strideC, tiles_m,
                                                          tiles_n, (int)nt, a_bcast ? 1 : 0, b_bcast ? 1 : 0, err);
  JX_LAUNCH_CHECK("gemm_3xtf32_kernel");
  return JX_OK;
}

int gemm_presplit(const float* Ah, const float* Al, const float* Bh, const float* Bl, float* C, int M, int N,
                  int Kp, long long ldc, long long strideC, int batch, cudaStream_t st) {
  return gemm_presplit_err(Ah, Al, Bh, Bl, C, M, N, Kp, ldc, strideC, batch, st, device_error_word(), false, false);
}

// One product (batch 1) on pre-split operands, cut into S k-slices.
int gemm_presplit_splitk(const float* Ah, const float* Al, const float* Bh, const float* Bl, float* C, int M, int N,
                         int Kp, long long ldc, int S, cudaStream_t st) {
  int rc = get_encode();
  if (rc) return rc;
  const int Ks = Kp / S;  // a multiple of BK
  CUtensorMap mAh, mAl, mBh, mBl;
  const uint64_t row = (uint64_t)Kp * 4, slice = (uint64_t)Ks * 4;
  if ((rc = make_map_3d(&mAh, Ah, Ks, M, S, row, slice, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = make_map_3d(&mAl, Al, Ks, M, S, row, slice, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = make_map_3d(&mBh, Bh, Ks, N, S, row, slice, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = make_map_3d(&mBl, Bl, Ks, N, S, row, slice, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = main_prepare())) return rc;
  void* part = nullptr;
  if ((rc = scratch_get(sizeof(float) * (size_t)S * M * N, &part, st))) return rc;
  const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
  const int nt = tiles_m * tiles_n * S;
  float* pp = static_cast<float*>(part);
  gemm_3xtf32_kernel<<<std::min(nt, num_sms()), GEMM_THREADS, GEMM_SMEM, st>>>(
      mAh, mAl, mBh, mBl, pp, M, N, Ks, N, (long long)M * N, tiles_m, tiles_n, nt, 0, 0, device_error_word());
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    const long long total = (long long)M * N;
    const int blocks = (int)std::min<long long>((total + 255) / 256, (long long)num_sms() * 8);
    splitk_sum_kernel<<<blocks, 256, 0, st>>>(pp, C, M, N, S, ldc);
    e = cudaGetLastError();
  }
  rc = e == cudaSuccess ? JX_OK : check_cuda(e, "split-K kernels");
  const int rc2 = scratch_release(part, st);
  return rc ? rc : rc2;
}

// Sets the main kernel's shared-memory limit on the current device once, up
// front (jx_init), so no later call -- e.g. one inside a stream capture -- has to.
int gemm_prepare() {
  int rc = get_encode();
  if (!rc) rc = main_prepare();
  return rc ? rc : fused_prepare(nullptr);
}

int gemm_split_operand(const float* src, float* hi, float* lo, int rows, int K, int Kp, long long ld, long long sb,
                       int batch, bool transposed, cudaStream_t st) {
  return launch_split(src, hi, lo, rows, K, Kp, ld, sb, batch, transposed, st);
}

long long gemm_kpad(long long K) { return round_up(K, BK); }

int gemm_make_kmajor_map(CUtensorMap* map, const float* base, int Kp, int rows, int batch, int box_rows) {
  int rc = get_encode();
  return rc ? rc : make_kmajor_map(map, base, Kp, rows, batch, box_rows);
}

int tensor_map_f32_3d(CUtensorMap_st* map, const void* base, const uint64_t* dims, const uint64_t* strides,
                      const uint32_t* box) {
  int rc = get_encode();
  return rc ? rc : make_map_3d(map, static_cast<const float*>(base), dims[0], dims[1], dims[2], strides[0],
                               strides[1], box[0], box[1], CU_TENSOR_MAP_SWIZZLE_NONE);
}
}  // namespace jx

extern "C" {

int jx_gemm_kpad(int64_t K, int64_t* Kp) {
  JX_TRACE("jx_gemm_kpad");
  JX_REQUIRE(Kp && K >= 0, "jx_gemm_kpad: bad argument");
  *Kp = round_up(K, BK);
  return JX_OK;
}

int jx_gemm_split_f32(const float* src, float* hi, float* lo, int64_t rows, int64_t K, int64_t ld, int trans,
                      int64_t batch, int64_t stride, jx_stream_t stream) {
  JX_TRACE("jx_gemm_split_f32");
  JX_REQUIRE(rows >= 0 && K >= 0 && batch >= 0, "gemm split: negative dimension");
  if (rows == 0 || batch == 0) return JX_OK;
  JX_REQUIRE(src && hi && lo, "gemm split: NULL pointer");
  JX_REQUIRE(rows < (1LL << 31) && K < (1LL << 31) && batch < 65536, "gemm split: dimension too large");
  JX_REQUIRE(ld >= (trans ? rows : K), "gemm split: leading dimension too small");
  const long long Kp = round_up(K, BK);
  return launch_split(src, hi, lo, (int)rows, (int)K, (int)Kp, ld, stride, (int)batch, trans != 0,
                      jx::as_stream(stream));
}

int jx_gemm_presplit_f32(const float* Ah, const float* Al, const float* Bh, const float* Bl, float* C, int64_t M,
                         int64_t N, int64_t Kp, int64_t ldc, int64_t batch, int64_t strideC, jx_stream_t stream) {
  JX_TRACE("jx_gemm_presplit_f32");
  JX_REQUIRE(M >= 0 && N >= 0 && Kp >= 0 && batch >= 0, "gemm presplit: negative dimension");
  if (M == 0 || N == 0 || batch == 0) return JX_OK;
  JX_REQUIRE(Ah && Al && Bh && Bl && C, "gemm presplit: NULL pointer");
  JX_REQUIRE(Kp > 0 && Kp % BK == 0, "gemm presplit: Kp must be a positive multiple of %d", BK);
  JX_REQUIRE(ldc >= N, "gemm presplit: ldc too small");
  JX_REQUIRE(M < (1LL << 31) && N < (1LL << 31) && Kp < (1LL << 31) && batch < 65536, "gemm presplit: too large");
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  JX_REQUIRE(a16(Ah) && a16(Al) && a16(Bh) && a16(Bl), "gemm presplit: operands must be 16-byte aligned");
  const long long tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int S = batch == 1 ? splitk_slices(tiles, Kp / BK) : 1;
  if (S > 1) return jx::gemm_presplit_splitk(Ah, Al, Bh, Bl, C, (int)M, (int)N, (int)Kp, ldc, S, jx::as_stream(stream));
  return jx::gemm_presplit(Ah, Al, Bh, Bl, C, (int)M, (int)N, (int)Kp, ldc, strideC, (int)batch,
                           jx::as_stream(stream));
}

int jx_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int64_t batch, size_t* bytes) {
  JX_TRACE("jx_gemm_workspace_size");
  JX_REQUIRE(bytes, "jx_gemm_workspace_size: NULL");
  long long Kp = round_up(K, BK);
  *bytes = (size_t)2 * (size_t)batch * (size_t)(M + N) * (size_t)Kp * sizeof(float);
  return JX_OK;
}

int jx_gemm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int transA, int transB,
                int64_t lda, int64_t ldb, int64_t ldc, int64_t batch, int64_t strideA, int64_t strideB,
                int64_t strideC, int precision, jx_stream_t stream) {
  JX_TRACE("jx_gemm_f32");
  JX_REQUIRE(M >= 0 && N >= 0 && K >= 0 && batch >= 0, "matmul: negative dimension");
  if (M == 0 || N == 0 || batch == 0) return JX_OK;
  JX_REQUIRE(A && B && C, "matmul: NULL operand");
  JX_REQUIRE(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31) && batch < 65536, "matmul: dimension too large");
  JX_REQUIRE(lda >= (transA ? M : K) && ldb >= (transB ? K : N) && ldc >= N, "matmul: leading dimension too small");
  cudaStream_t st = jx::as_stream(stream);
  if (K == 0) {
    for (int64_t b = 0; b < batch; ++b)
      JX_CUDA(cudaMemset2DAsync(C + b * strideC, ldc * 4, 0, N * 4, M, st));
    return JX_OK;
  }
  if (precision == JX_PREC_EXACT) {
    dim3 grid((unsigned)((N + 15) / 16), (unsigned)((M + 15) / 16), (unsigned)batch);
    JX_REQUIRE(grid.y < 65536, "matmul(exact): M too large");
    gemm_exact_kernel<<<grid, dim3(16, 16), 0, st>>>(A, B, C, (int)M, (int)N, (int)K, transA, transB, lda, ldb, ldc,
                                                     strideA, strideB, strideC);
    JX_LAUNCH_CHECK("gemm_exact_kernel");
    return JX_OK;
  }
  if (precision == JX_PREC_3XTF32_PAIR) {
    JX_REQUIRE(jx::pair_gemm_ok(A, B, M, N, lda, ldb, batch, strideA, strideB),
               "matmul: JX_PREC_3XTF32_PAIR needs 16-byte aligned operands with lda, ldb and batch strides "
               "multiples of 4 and at least one 256x256 tile per SM pair");
    return jx::launch_pair_gemm(A, B, C, M, N, K, transA != 0, transB != 0, lda, ldb, ldc, batch, strideA, strideB,
                                strideC, st);
  }
  if (precision == JX_PREC_3XTF32_FUSED) {
    JX_REQUIRE(fused_split_ok(A, B, transA, transB, lda, ldb, batch, strideA, strideB),
               "matmul: JX_PREC_3XTF32_FUSED needs untransposed, 16-byte aligned operands with lda, ldb and batch "
               "strides multiples of 4");
    return launch_fused_split(A, B, C, M, N, K, lda, ldb, ldc, batch, strideA, strideB, strideC, st);
  }
  JX_REQUIRE(precision == JX_PREC_3XTF32, "matmul: unknown precision %d", precision);
  // Enough 256x256 tiles for every SM pair: the pair kernel splits in shared
  // memory and needs no split pass (8192^3: 4.37 ms against 4.70 ms for the
  // split pass plus the main kernel).  Transposed products stay on it too:
  // it runs them at 4.90-5.00 ms, and the transposing split passes of the
  // wide MLP's tall backward operands cost more (taking the split path for
  // them slowed its step from 149.7k to 136.0k samples/s).
  if (jx::pair_gemm_ok(A, B, M, N, lda, ldb, batch, strideA, strideB))
    return jx::launch_pair_gemm(A, B, C, M, N, K, transA != 0, transB != 0, lda, ldb, ldc, batch, strideA, strideB,
                                strideC, st);
  // The split pass costs about 250 * (1/M + 1/N) of the main kernel's time
  // (12 bytes of HBM traffic per operand element against 2*M*N*K flop);
  // the fused kernel runs slower than the main kernel (its lo split sits on
  // the cross products' path with two stages), so it wins below that
  // crossover, given enough tiles to fill the GPU.  Products with fewer tiles
  // than SMs take the split pass and are cut along K (split-K).
  const long long tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * batch;
  if (fused_split_ok(A, B, transA, transB, lda, ldb, batch, strideA, strideB) &&
      250.0 * (1.0 / (double)M + 1.0 / (double)N) > 0.2 && tiles >= jx::num_sms())
    return launch_fused_split(A, B, C, M, N, K, lda, ldb, ldc, batch, strideA, strideB, strideC, st);
  const long long Kp = round_up(K, BK);
  size_t ws = 0;
  jx_gemm_workspace_size(M, N, K, batch, &ws);
  void* scratch = nullptr;
  int rc = jx::scratch_get(ws, &scratch, st);
  if (rc) return rc;
  float* Ah = reinterpret_cast<float*>(scratch);
  float* Al = Ah + (size_t)batch * M * Kp;
  float* Bh = Al + (size_t)batch * M * Kp;
  float* Bl = Bh + (size_t)batch * N * Kp;
  rc = launch_split(A, Ah, Al, (int)M, (int)K, (int)Kp, lda, strideA, (int)batch, transA != 0, st);
  if (!rc) rc = launch_split(B, Bh, Bl, (int)N, (int)K, (int)Kp, ldb, strideB, (int)batch, transB == 0, st);
  const int S = batch == 1 ? splitk_slices(tiles, Kp / BK) : 1;
  if (!rc && S > 1)
    rc = jx::gemm_presplit_splitk(Ah, Al, Bh, Bl, C, (int)M, (int)N, (int)Kp, ldc, S, st);
  else if (!rc)
    rc = jx::gemm_presplit(Ah, Al, Bh, Bl, C, (int)M, (int)N, (int)Kp, ldc, strideC, (int)batch, st);
  int rc2 = jx::scratch_release(scratch, st);
  return rc ? rc : rc2;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// jx_gemm_f32_noalloc: the 3xTF32 GEMM for callers that must not allocate.
//
// Some callers cannot let a library allocate device memory. A host process
// may have handed all of HBM to its own arena or caching allocator up front,
// so a library allocation either fails or fragments memory it does not own. A
// latency-critical loop may not afford an allocator call. A plugin host may
// forbid libraries from allocating behind its back. jx_gemm_f32 takes its
// operand-split workspace from the device memory pool on every call; this
// variant instead uses the fixed array below, so it performs no allocation of
// any kind. The caller still provides A, B and C.
//
// Limits and behaviour:
//   * The workspace holds NOALLOC_SCRATCH_FLOATS floats (64 MiB). A call needs
//     2 * batch * (M + N) * round_up(K, 32) floats; larger problems are
//     rejected with JX_EINVAL before anything is launched.
//   * Every GPU that loads this library keeps the 64 MiB array until the
//     process exits.
//   * The first call made on each device (with that device current) does
//     that device's one-time set-up under a mutex: it looks up the array's
//     device address with cudaGetSymbolAddress, resolves the tensor-map
//     encoder and sets the main kernel's shared-memory limit. That first call
//     should therefore come before any stream capture.
//   * All calls share the one array and it keeps the last call's contents:
//     the split pass rewrites every element a call reads (K padding included),
//     so nothing needs clearing. Calls that overlap on the GPU (for example
//     on two streams of one device) race on the array; the caller must
//     serialise them.
//   * A bounded wait that gives up inside one of these launches sets
//     JX_DEVERR_TIMEOUT in a second fixed device word, g_noalloc_err, which
//     jx_device_status reads, ORs into its result and clears, like the
//     context's own error word.
//   * K == 0 zero-fills C, as jx_gemm_f32 does (cudaMemset2DAsync, no
//     allocation).
// ---------------------------------------------------------------------------
namespace {
constexpr size_t NOALLOC_SCRATCH_FLOATS = (size_t)16 << 20;  // 64 MiB of f32
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];
static __device__ unsigned int g_noalloc_err;  // timed-out-wait flag of this entry point's launches

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64];
unsigned int* g_noalloc_err_ptr[64];

// Host code may not pass g_noalloc_scratch itself to a kernel: in host code
// that name is a host-side stand-in, not the device address.
int noalloc_setup(float** scratch, unsigned int** err) {
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return jx::fail(JX_EUNSUPPORTED, "gemm noalloc: device index %d >= 64", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    if (int rc = get_encode()) return rc;
    if (int rc = main_prepare()) return rc;
    void* p = nullptr;
    void* q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return jx::check_cuda(e, "gemm noalloc: cudaGetSymbolAddress(scratch)");
    e = cudaGetSymbolAddress(&q, g_noalloc_err);
    if (e != cudaSuccess) return jx::check_cuda(e, "gemm noalloc: cudaGetSymbolAddress(error word)");
    g_noalloc_err_ptr[dev] = reinterpret_cast<unsigned int*>(q);
    g_noalloc_ptr[dev] = reinterpret_cast<float*>(p);
  }
  *scratch = g_noalloc_ptr[dev];
  *err = g_noalloc_err_ptr[dev];
  return JX_OK;
}
}  // namespace

namespace jx {
// For jx_device_status: the current device's noalloc error word, read and
// cleared (0 when this entry point has not run on the device).  The caller
// has synchronised the device.
int noalloc_take_error(unsigned int* flags) {
  *flags = 0;
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return JX_OK;
  unsigned int* w = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    w = g_noalloc_err_ptr[dev];
  }
  if (!w) return JX_OK;
  JX_CUDA(cudaMemcpy(flags, w, sizeof(unsigned int), cudaMemcpyDeviceToHost));
  JX_CUDA(cudaMemset(w, 0, sizeof(unsigned int)));
  return JX_OK;
}
}  // namespace jx

// Test hook: ORs `flags` into the noalloc error word of the current device,
// so a test can check that the word reaches jx_device_status without making
// a kernel's wait run out.
extern "C" int jx_selftest_noalloc_flag(unsigned int flags) {
  JX_TRACE("jx_selftest_noalloc_flag");
  float* ws = nullptr;
  unsigned int* err = nullptr;
  int rc = noalloc_setup(&ws, &err);
  if (rc) return rc;
  unsigned int v = 0;
  JX_CUDA(cudaDeviceSynchronize());
  JX_CUDA(cudaMemcpy(&v, err, sizeof(v), cudaMemcpyDeviceToHost));
  v |= flags;
  JX_CUDA(cudaMemcpy(err, &v, sizeof(v), cudaMemcpyHostToDevice));
  return JX_OK;
}

extern "C" int jx_gemm_f32_noalloc(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                                   int transA, int transB, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch,
                                   int64_t strideA, int64_t strideB, int64_t strideC, jx_stream_t stream) {
  JX_TRACE("jx_gemm_f32_noalloc");
  JX_REQUIRE(M >= 0 && N >= 0 && K >= 0 && batch >= 0, "matmul: negative dimension");
  if (M == 0 || N == 0 || batch == 0) return JX_OK;
  JX_REQUIRE(A && B && C, "matmul: NULL operand");
  JX_REQUIRE(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31) && batch < 65536, "matmul: dimension too large");
  JX_REQUIRE(lda >= (transA ? M : K) && ldb >= (transB ? K : N) && ldc >= N, "matmul: leading dimension too small");
  cudaStream_t st = jx::as_stream(stream);
  if (K == 0) {
    for (int64_t b = 0; b < batch; ++b)
      JX_CUDA(cudaMemset2DAsync(C + b * strideC, ldc * 4, 0, N * 4, M, st));
    return JX_OK;
  }
  const long long Kp = round_up(K, BK);
  const double need = 2.0 * (double)batch * (double)(M + N) * (double)Kp;
  if (need > (double)NOALLOC_SCRATCH_FLOATS)
    return jx::fail(JX_EINVAL,
                    "gemm noalloc: needs %.0f workspace floats (2*batch*(M+N)*Kp), above the fixed maximum of %zu "
                    "(64 MiB); use jx_gemm_f32 for this size",
                    need, NOALLOC_SCRATCH_FLOATS);
  float* ws = nullptr;
  unsigned int* err = nullptr;
  int rc = noalloc_setup(&ws, &err);
  if (rc) return rc;
  float* Ah = ws;
  float* Al = Ah + (size_t)batch * M * Kp;
  float* Bh = Al + (size_t)batch * M * Kp;
  float* Bl = Bh + (size_t)batch * N * Kp;
  rc = launch_split(A, Ah, Al, (int)M, (int)K, (int)Kp, lda, strideA, (int)batch, transA != 0, st);
  if (!rc) rc = launch_split(B, Bh, Bl, (int)N, (int)K, (int)Kp, ldb, strideB, (int)batch, transB == 0, st);
  if (!rc)
    rc = jx::gemm_presplit_err(Ah, Al, Bh, Bl, C, (int)M, (int)N, (int)Kp, ldc, strideC, (int)batch, st, err, false,
                               false);
  return rc;
}
