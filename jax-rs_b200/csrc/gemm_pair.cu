// gemm_pair.cu -- 3xTF32 GEMM on SM pairs: C = op(A) . op(B) for Array::matmul
// (src/ops/linalg.rs:154-237), the batched einsum "bij,bjk->bik"
// (src/ops/einsum.rs:488-523) and the transposed products of
// transpose_matmul (src/trace/transpose_rules.rs:537-567), straight from the
// caller's f32 buffers: no split pass, no workspace.
//
// A cluster of two CTAs (an SM pair) owns a 256 x 256 output tile and issues
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 8): CTA r of the pair holds
// rows 128r..128r+127 of the A tile and columns 128r..128r+127 of the B tile,
// and its TMEM receives its 128 rows of the product.  Per k-block of 32, a
// CTA's shared memory therefore carries half of B instead of all of it: the
// operand bytes the tensor cores read from one SM's shared memory drop by a
// third against the one-CTA 128 x 256 tile, which is what leaves room for the
// hi/lo split to happen in shared memory.
//
//   warp 0 (each CTA)   TMA: this CTA's raw f32 A and B tiles into the stage
//   warp 1 (even CTA)   TMEM allocation (both CTAs) + the single-thread pair
//                       MMA issuer: Al.Bh + Ah.Bl + Ah.Bh per k-step, into
//                       one of two TMEM span buffers (256 columns each)
//   warps 4..7 (each)   split: lo = tf32_rn(x - trunc(x)) next to every raw
//                       value of the stage (the tf32 MMA reads the raw value
//                       as hi = trunc(x))
//   warps 8..15 (each)  drain the TMEM spans into the f32 accumulator
//                       registers and store C
// The split has a warpgroup of its own so that it never waits behind a span
// drain: with eight warps doing both, the MMA starved while they drained.
//
// Operand layouts by transposition: an operand whose K is contiguous in
// memory (A untransposed, B transposed) is a K-major tile with 128-byte
// swizzle; one whose M or N is contiguous (A transposed, B untransposed) is
// MN-major, streamed as 32 x 32 boxes in the SWIZZLE_128B_ATOM_32B layout.
// The split works on 16-byte chunks in place, whatever the layout.
//
// Handshakes (every wait bounded, about 4 s, then JX_DEVERR_TIMEOUT):
//   raw_full[s]  (each CTA)  its TMA landed stage s
//   full[s]      (even CTA)  both CTAs wrote lo of stage s (one arrival per CTA)
//   empty[s]     (each CTA)  the pair's MMAs on stage s retired (multicast commit)
//   sfull[p]     (each CTA)  span buffer p holds a finished partial sum (multicast commit)
//   sempty[p]    (even CTA)  both CTAs drained span buffer p (one arrival per CTA)
//   gfull[s], gempty[p] (each CTA)  local: the four split / eight drain warps are done
// Each warp of a group arrives on its CTA's local barrier (CTA-scope
// release); the group's first thread waits for all of them (bounded) and
// alone arrives, with release at cluster scope, on the even CTA's barrier:
// one cluster-scope release per stage per CTA instead of one per warp (the
// per-warp cluster-scope fences were the main stall, `membar`, of an earlier
// form).  Only the MMA issuer, whose barriers receive the other CTA's
// arrivals, waits with cluster-scope acquire.
// No TMA load uses cluster multicast: each CTA loads only its own tiles.
#include <algorithm>
#include <mutex>

#include "tc_gemm.cuh"

namespace {

using namespace jxg;

constexpr int PR_ROWS = PAIR_ROWS;                          // rows of A (and columns of B) per CTA
constexpr int PR_TILE = PAIR_TILE;                          // output tile edge per pair
constexpr int PR_STAGES = 3;
constexpr int PR_OP = PAIR_OP;                              // 16 KB: one operand's raw (or lo) tile per CTA
constexpr int PR_STAGE = 4 * PR_OP;                         // [A raw][A lo][B raw][B lo]
constexpr int PR_THREADS = 512;
constexpr int PR_FIRST_SPLIT = 4;                           // warps 4..7: the split warpgroup
constexpr int PR_SPLIT_WARPS = 4;
constexpr int PR_FIRST_EPI = 8;                             // warps 8..15: drain + store
constexpr int PR_LAUNCH_REGS = 128;
constexpr int PR_LOW_REGS = 40;                             // TMA / MMA warpgroup
constexpr int PR_SPLIT_REGS = 72;
constexpr int PR_HIGH_REGS = 200;
constexpr int PR_BOX = PAIR_BOX;                             // one 32 x 32 MN-major box: 4 KB
constexpr uint32_t PR_TMEM_COLS = 2 * PR_TILE;              // two span buffers of 256 columns
constexpr size_t PR_SMEM = (size_t)PR_STAGES * PR_STAGE + 1024 /*align*/ + 256 /*barriers*/;
static_assert(128 * PR_LOW_REGS + 128 * PR_SPLIT_REGS + 256 * PR_HIGH_REGS <= PR_THREADS * PR_LAUNCH_REGS,
              "register split exceeds the launch allocation");

// TMA of one CTA's 128-row slice of an operand for k-block kb: `row0` is the
// slice's first row (M for A, N for B).  K-major: one 32 x 128 box;
// MN-major: four 32 x 32 boxes along the rows.
template <bool MN>
__device__ __forceinline__ void load_op(uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, int kb, int row0,
                                        int b) {
  if constexpr (MN) {
#pragma unroll
    for (int i = 0; i < PR_ROWS / 32; ++i) jxd::tma_load_3d(dst + i * PR_BOX, tm, bar, row0 + 32 * i, kb * BK, b);
  } else {
    jxd::tma_load_3d(dst, tm, bar, kb * BK, row0, b);
  }
}

// A_MN: A is transposed (stored [K][M]); B_MN: B is not transposed (stored [K][N]).
template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(PR_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     float* __restrict__ C, int M, int N, int num_kb, long long ldc, long long strideC, int tiles_m,
                     int tiles_n, int num_tiles, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = jxd::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PR_STAGES * PR_STAGE);
  uint64_t* raw_full = bars;                       // [PR_STAGES]
  uint64_t* full = bars + PR_STAGES;               // [PR_STAGES] (even CTA)
  uint64_t* empty = bars + 2 * PR_STAGES;          // [PR_STAGES]
  uint64_t* sfull = bars + 3 * PR_STAGES;          // [2]
  uint64_t* sempty = bars + 3 * PR_STAGES + 2;     // [2] (even CTA)
  uint64_t* gfull = bars + 3 * PR_STAGES + 4;      // [PR_STAGES] local: split warps done
  uint64_t* gempty = bars + 4 * PR_STAGES + 4;     // [2] local: drain warps done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * PR_STAGES + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = jxd::cluster_ctarank();  // 0 or 1 within the pair
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PR_STAGES; ++s) {
      jxd::mbar_init(&raw_full[s], 1);
      jxd::mbar_init(&full[s], 2);
      jxd::mbar_init(&empty[s], 1);
      jxd::mbar_init(&gfull[s], PR_SPLIT_WARPS);
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
    jxd::tma_prefetch_desc(&tmA);
    jxd::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    jxd::tmem_alloc_pair(tmem_slot, PR_TMEM_COLS);
    jxd::tmem_relinquish_pair();
  }
  jxd::tc_fence_before();
  __syncthreads();
  jxd::cluster_sync_all();  // the peer's barriers are initialised before anyone signals them
  jxd::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full0 = jxd::mapa_shared(&full[0], 0), sempty0 = jxd::mapa_shared(&sempty[0], 0);

  auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    return warp_wait_bounded(bar, parity, abort_flag, err);
  };
  auto group_arrive = [&](uint64_t* gbar, uint32_t parity, uint32_t cluster_bar, bool first) -> bool {
    return group_arrive_cluster(gbar, parity, cluster_bar, first, lane, abort_flag, err);
  };

  if (warp < PR_FIRST_SPLIT) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PR_LOW_REGS));
    if (warp == 0 && jxd::elect_one()) {
      // ---------------- TMA: this CTA's raw A and B slices ----------------
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += npairs) {
        const TileInfo ti = pair_tile_coords(t, tiles_m, tiles_n);
        const int ya = ti.m_blk * PR_TILE + (int)rank * PR_ROWS, yb = ti.n_blk * PR_TILE + (int)rank * PR_ROWS;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bounded(&empty[stage], phase ^ 1u, err)) { *abort_flag = 1; break; }
          uint8_t* st = smem + stage * PR_STAGE;
          jxd::mbar_arrive_expect_tx(&raw_full[stage], 2 * PR_OP);
          load_op<A_MN>(st, &tmA, &raw_full[stage], kb, ya, ti.b);
          load_op<B_MN>(st + 2 * PR_OP, &tmB, &raw_full[stage], kb, yb, ti.b);
          if (++stage == PR_STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      for (int s = 0; s < PR_STAGES; ++s) {
        if (!wait_bounded(&empty[stage], phase ^ 1u, err)) break;
        if (++stage == PR_STAGES) { stage = 0; phase ^= 1u; }
      }
    }
    if (warp == 1 && rank == 0 && jxd::elect_one())
      // ---------------- pair MMA issuer (even CTA) ----------------
      pair_mma_issuer<A_MN, B_MN, PR_STAGES, PR_STAGE>(jxd::smem_u32(smem), full, empty, sfull, sempty, tmem_base,
                                                       pair, num_tiles, npairs, num_kb, abort_flag, err);
  } else if (warp < PR_FIRST_EPI) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PR_SPLIT_REGS));
    // ---------------- split (warps 4..7): lo next to every raw value ----------------
    const int sid = threadIdx.x - PR_FIRST_SPLIT * 32;  // 0..127
    constexpr int CHUNKS = 2 * PR_OP / 16 / (32 * PR_SPLIT_WARPS);  // 16-byte chunks per thread per stage
    constexpr int BATCH = 8;                                         // loads in flight before the arithmetic
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = pair; ok && t < num_tiles; t += npairs) {
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!warp_wait(&raw_full[stage], phase)) { ok = false; break; }
        uint8_t* st = smem + stage * PR_STAGE;
        // 2048 16-byte chunks of raw values per stage (A: 1024, then B: 1024),
        // consecutive threads on consecutive chunks; lo goes PR_OP bytes after
        // its raw chunk
#pragma unroll
        for (int j0 = 0; j0 < CHUNKS; j0 += BATCH) {
          float4 x[BATCH];
#pragma unroll
          for (int j = 0; j < BATCH; ++j) {
            const int f = sid + 32 * PR_SPLIT_WARPS * (j0 + j);
            x[j] = *reinterpret_cast<const float4*>(st + (f < PR_OP / 16 ? f * 16 : PR_OP + f * 16));
          }
#pragma unroll
          for (int j = 0; j < BATCH; ++j) {
            const int f = sid + 32 * PR_SPLIT_WARPS * (j0 + j);
            float4 l;
            l.x = jxd::tf32_lo_of_trunc(x[j].x);
            l.y = jxd::tf32_lo_of_trunc(x[j].y);
            l.z = jxd::tf32_lo_of_trunc(x[j].z);
            l.w = jxd::tf32_lo_of_trunc(x[j].w);
            *reinterpret_cast<float4*>(st + PR_OP + (f < PR_OP / 16 ? f * 16 : PR_OP + f * 16)) = l;
          }
        }
        jxd::fence_proxy_async_smem();  // this thread's generic-proxy writes -> the tensor cores
        if (!group_arrive(&gfull[stage], phase, full0 + stage * 8, sid == 0)) { ok = false; break; }
        if (++stage == PR_STAGES) { stage = 0; phase ^= 1u; }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(PR_HIGH_REGS));
    // ---------------- drain the spans, store C (warps 8..15) ----------------
    const int gt = threadIdx.x - PR_FIRST_EPI * 32;  // 0..255
    const int q = warp & 3, half = (warp - PR_FIRST_EPI) >> 2;
    const bool vec_ok = ((ldc & 3) == 0) && ((strideC & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    uint32_t span_ctr = 0;
    const int nspan = (num_kb + SPAN_KB - 1) / SPAN_KB;
    for (int t = pair; t < num_tiles; t += npairs) {
      float acc[EPI_COLS];
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.0f;
      bool ok = true;
      for (int sp = 0; sp < nspan; ++sp) {
        const uint32_t p = span_ctr & 1u, ph = (span_ctr >> 1) & 1u;
        if (!warp_wait(&sfull[p], ph)) { ok = false; break; }
        jxd::tc_fence_after();
        const uint32_t t_addr =
            tmem_base + ((uint32_t)(q * 32) << 16) + p * (uint32_t)PR_TILE + (uint32_t)(half * EPI_COLS);
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
        if (!group_arrive(&gempty[p], ph, sempty0 + p * 8, gt == 0)) { ok = false; break; }
      }
      if (!ok) break;
      const TileInfo ti = pair_tile_coords(t, tiles_m, tiles_n);
      const int row = ti.m_blk * PR_TILE + (int)rank * PR_ROWS + q * 32 + lane;
      if (row < M) {
        float* crow = C + (long long)ti.b * strideC + (long long)row * ldc;
        const int col0 = ti.n_blk * PR_TILE + half * EPI_COLS;
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
  jxd::cluster_sync_all();  // neither CTA leaves while its peer may still signal it
  jxd::tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    jxd::tmem_dealloc_pair(tmem_base, PR_TMEM_COLS);
  }
}

using PairKernel = void (*)(CUtensorMap, CUtensorMap, float*, int, int, int, long long, long long, int, int, int,
                            unsigned int*);

PairKernel pair_kernel(bool a_mn, bool b_mn) {
  if (a_mn) return b_mn ? gemm_pair_kernel<true, true> : gemm_pair_kernel<true, false>;
  return b_mn ? gemm_pair_kernel<false, true> : gemm_pair_kernel<false, false>;
}

std::mutex g_pair_mu;

// Per device and variant, once: the shared-memory limit, the register count
// the kernel was built with, and how many pairs can be resident at once.
int pair_prepare(PairKernel k, int variant, int* regs_out, int* max_pairs_out) {
  static int regs[64][4], max_pairs[64][4];
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_pair_mu);
  if (!regs[dev & 63][variant]) {
    cudaFuncAttributes fa;
    JX_CUDA(cudaFuncGetAttributes(&fa, k));
    JX_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PR_SMEM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)jx::num_sms());
    cfg.blockDim = dim3(PR_THREADS);
    cfg.dynamicSmemBytes = PR_SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int clusters = 0;
    JX_CUDA(cudaOccupancyMaxActiveClusters(&clusters, (void*)k, &cfg));
    regs[dev & 63][variant] = fa.numRegs;
    max_pairs[dev & 63][variant] = clusters;
  }
  *regs_out = regs[dev & 63][variant];
  *max_pairs_out = max_pairs[dev & 63][variant];
  return JX_OK;
}

}  // namespace

namespace jx {
int get_encode_fn();
int make_map_3d_fn(CUtensorMap* map, const float* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                   uint64_t s2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw);

// Products the pair kernel takes: 16-byte aligned operands whose leading
// dimensions and batch strides are multiples of 4 floats (TMA strides), and
// at least one 256 x 256 tile per SM pair.
bool pair_gemm_ok(const float* A, const float* B, long long M, long long N, long long lda, long long ldb,
                  long long batch, long long sA, long long sB) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!a16(A) || !a16(B) || (lda & 3) || (ldb & 3)) return false;
  if (batch > 1 && (sA <= 0 || sB <= 0 || (sA & 3) || (sB & 3))) return false;
  const long long tiles = ((M + PR_TILE - 1) / PR_TILE) * ((N + PR_TILE - 1) / PR_TILE) * batch;
  return tiles >= num_sms() / 2;
}

int launch_pair_gemm(const float* A, const float* B, float* C, long long M, long long N, long long K, bool transA,
                     bool transB, long long lda, long long ldb, long long ldc, long long batch, long long sA,
                     long long sB, long long sC, cudaStream_t st) {
  int rc = get_encode_fn();
  if (rc) return rc;
  const bool a_mn = transA, b_mn = !transB;
  PairKernel k = pair_kernel(a_mn, b_mn);
  int regs = 0, max_pairs = 0;
  if ((rc = pair_prepare(k, (a_mn ? 2 : 0) + (b_mn ? 1 : 0), &regs, &max_pairs))) return rc;
  // The register split inside the kernel assumes exactly PR_LAUNCH_REGS per
  // thread at launch; with any other allocation setmaxnreg.inc could wait for
  // registers that never come, so refuse to launch.
  if (regs != PR_LAUNCH_REGS)
    return fail(JX_EUNSUPPORTED, "gemm_pair_kernel built with %d registers per thread, expected %d", regs,
                PR_LAUNCH_REGS);
  if (max_pairs < 1) return fail(JX_EUNSUPPORTED, "gemm_pair_kernel: no SM pair can hold a cluster");
  CUtensorMap mA, mB;
  // a single batch entry: the batch stride only has to be a valid TMA stride
  const uint64_t sa = batch > 1 ? (uint64_t)sA * 4 : (uint64_t)lda * 4 * (uint64_t)(transA ? K : M);
  const uint64_t sb = batch > 1 ? (uint64_t)sB * 4 : (uint64_t)ldb * 4 * (uint64_t)(transB ? N : K);
  if (a_mn) rc = make_map_3d_fn(&mA, A, M, K, batch, lda * 4, sa, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  else rc = make_map_3d_fn(&mA, A, K, M, batch, lda * 4, sa, BK, PR_ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (b_mn) rc = make_map_3d_fn(&mB, B, N, K, batch, ldb * 4, sb, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  else rc = make_map_3d_fn(&mB, B, K, N, batch, ldb * 4, sb, BK, PR_ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int tiles_m = (int)((M + PR_TILE - 1) / PR_TILE), tiles_n = (int)((N + PR_TILE - 1) / PR_TILE);
  const long long nt = (long long)tiles_m * tiles_n * batch;
  if (nt > 0x7fffffffLL) return fail(JX_EINVAL, "gemm: too many tiles");
  const int pairs = (int)std::min<long long>(nt, max_pairs);
  const int num_kb = (int)((K + BK - 1) / BK);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(PR_THREADS);
  cfg.dynamicSmemBytes = PR_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  float* Cp = C;
  int Mi = (int)M, Ni = (int)N, tm = tiles_m, tn = tiles_n, nti = (int)nt;
  unsigned int* errw = device_error_word();
  JX_CUDA(cudaLaunchKernelEx(&cfg, k, mA, mB, Cp, Mi, Ni, num_kb, ldc, sC, tm, tn, nti, errw));
  return JX_OK;
}
}  // namespace jx
