// tc_gemm.cuh -- the pieces of the tcgen05 3xTF32 GEMM core shared by the
// plain GEMM (gemm.cu) and the implicit-GEMM convolutions (conv.cu): tile
// geometry, bounded mbarrier waits, the single-thread MMA issuer and the
// span drain that promotes TMEM partial sums into f32 registers.
//
// Shared-memory stage layout (1024-byte aligned), per k-block of BK = 32:
//   [Ah 128x32][Al 128x32][Bh 256x32][Bl 256x32], every tile K-major with
//   128-byte rows in the TMA SWIZZLE_128B pattern: 16-byte chunk c of row r
//   sits at r*128 + ((c ^ (r & 7)) * 16).
#pragma once
#include <cudaTypedefs.h>

#include "jx_common.cuh"

namespace jxg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 32;  // 32 f32 = 128 B rows -> 128-byte swizzle
constexpr int STAGES = 2;
constexpr int A_TILE = BM * BK * 4;  // 16 KB
constexpr int B_TILE = BN * BK * 4;  // 32 KB
constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;
constexpr int EPI_WARPS = 8;                       // epilogue warps (two per TMEM lane quarter)
constexpr int EPI_COLS = BN / 2;                   // columns of the tile each epilogue thread owns
constexpr int GEMM_THREADS = 64 + 32 * EPI_WARPS;  // producer warp + MMA warp + epilogue
constexpr int TMEM_COLS = 2 * BN;                  // two span partial buffers
constexpr int SPAN_KB = 4;                         // k-blocks per TMEM partial sum (128 K elements)
constexpr int GROUP_M = 16;

struct TileInfo {
  int m_blk, n_blk, b;
};

// Tile t of a [batch][tiles_m][tiles_n] grid, grouped GROUP_M M-blocks at a
// time so consecutive CTAs share B tiles in L2.
__device__ __forceinline__ TileInfo tile_coords(int t, int tiles_m, int tiles_n) {
  int per_batch = tiles_m * tiles_n;
  int b = t / per_batch;
  int r = t - b * per_batch;
  int in_group = GROUP_M * tiles_n;
  int g = r / in_group;
  int first_m = g * GROUP_M;
  int gsize = min(tiles_m - first_m, GROUP_M);
  int local = r - g * in_group;
  TileInfo ti;
  ti.m_blk = first_m + local % gsize;
  ti.n_blk = local / gsize;
  ti.b = b;
  return ti;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait on an mbarrier phase with a wall-clock limit (about 4 s); on expiry the
// device error word gets JX_DEVERR_TIMEOUT and the caller unwinds.
__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity, unsigned int* err) {
  if (jxd::mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (jxd::mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > 4000000000ull) {
      atomicOr(err, JX_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// Single elected thread: for every tile of this CTA, consume the k-blocks of
// the smem ring in spans of SPAN_KB.  Each span accumulates from zero into one
// of two TMEM partial buffers (ping-pong) that the epilogue drains; the
// tensor core's own accumulation truncates, so keeping each TMEM sum short
// bounds that bias (over a full K it would grow linearly with K).
// B_MN: the B tiles are MN-major (row-major B streamed as 32 x 32 boxes, 4 KB
// apart, in the SWIZZLE_128B_ATOM_32B layout) instead of K-major.
// raw_full (fused split only): the hi slots hold the raw f32 tiles as TMA
// landed them, which the tf32 MMA reads as trunc(x) (low 13 bits ignored);
// the hi.hi products are issued as soon as raw_full completes, overlapping
// the lo computation, and the two cross products once full completes.
template <bool B_MN = false>
__device__ __forceinline__ void mma_issuer(uint8_t* smem, uint64_t* full, uint64_t* empty, uint64_t* sfull,
                                           uint64_t* sempty, uint32_t tmem_base, int num_tiles, int num_kb,
                                           volatile int* abort_flag, unsigned int* err,
                                           uint64_t* raw_full = nullptr) {
  constexpr uint32_t idesc = jxd::idesc_tf32(BM, BN) | (B_MN ? (1u << 16) : 0u);
  int stage = 0;
  uint32_t phase = 0;
  uint32_t span_ctr = 0;
  const uint32_t smem_base = jxd::smem_u32(smem);
  for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
    for (int kb0 = 0; kb0 < num_kb && !*abort_flag; kb0 += SPAN_KB) {
      const uint32_t p = span_ctr & 1u, ph = (span_ctr >> 1) & 1u;
      if (!wait_bounded(&sempty[p], ph ^ 1u, err)) { *abort_flag = 1; break; }
      jxd::tc_fence_after();
      const uint32_t d_tmem = tmem_base + p * (uint32_t)BN;
      const int kb_end = min(kb0 + SPAN_KB, num_kb);
      for (int kb = kb0; kb < kb_end; ++kb) {
        const uint32_t sa_h = smem_base + stage * STAGE_BYTES;
        const uint32_t sa_l = sa_h + A_TILE;
        const uint32_t sb_h = sa_h + 2 * A_TILE;
        const uint32_t sb_l = sb_h + B_TILE;
        if (raw_full) {
          if (!wait_bounded(&raw_full[stage], phase, err)) { *abort_flag = 1; break; }
          jxd::tc_fence_after();
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t ah = jxd::smem_desc_k_sw128(sa_h + k * 32);
            const uint64_t bh = B_MN ? jxd::smem_desc_mn_sw128_32b(sb_h + k * 1024, 32 * BK * 4)
                                     : jxd::smem_desc_k_sw128(sb_h + k * 32);
            jxd::mma_tf32(d_tmem, ah, bh, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          if (!wait_bounded(&full[stage], phase, err)) { *abort_flag = 1; break; }
          jxd::tc_fence_after();
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t ah = jxd::smem_desc_k_sw128(sa_h + k * 32);
            const uint64_t al = jxd::smem_desc_k_sw128(sa_l + k * 32);
            uint64_t bh, bl;
            if constexpr (B_MN) {
              bh = jxd::smem_desc_mn_sw128_32b(sb_h + k * 1024, 32 * BK * 4);
              bl = jxd::smem_desc_mn_sw128_32b(sb_l + k * 1024, 32 * BK * 4);
            } else {
              bh = jxd::smem_desc_k_sw128(sb_h + k * 32);
              bl = jxd::smem_desc_k_sw128(sb_l + k * 32);
            }
            jxd::mma_tf32(d_tmem, al, bh, idesc, 1u);
            jxd::mma_tf32(d_tmem, ah, bl, idesc, 1u);
          }
          jxd::mma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          continue;
        }
        if (!wait_bounded(&full[stage], phase, err)) { *abort_flag = 1; break; }
        jxd::tc_fence_after();
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          const uint32_t off = k * 32;  // 8 tf32 = 32 bytes along the swizzled row
          const uint64_t ah = jxd::smem_desc_k_sw128(sa_h + off);
          const uint64_t al = jxd::smem_desc_k_sw128(sa_l + off);
          uint64_t bh, bl;
          if constexpr (B_MN) {
            // 8 k-rows of 128 B per MMA step
            bh = jxd::smem_desc_mn_sw128_32b(sb_h + k * 1024, 32 * BK * 4);
            bl = jxd::smem_desc_mn_sw128_32b(sb_l + k * 1024, 32 * BK * 4);
          } else {
            bh = jxd::smem_desc_k_sw128(sb_h + off);
            bl = jxd::smem_desc_k_sw128(sb_l + off);
          }
          jxd::mma_tf32(d_tmem, al, bh, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          jxd::mma_tf32(d_tmem, ah, bl, idesc, 1u);
          jxd::mma_tf32(d_tmem, ah, bh, idesc, 1u);
        }
        jxd::mma_commit(&empty[stage]);  // frees the smem slot once these MMAs retire
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      jxd::mma_commit(&sfull[p]);  // span partial complete
      ++span_ctr;
    }
  }
}

// Epilogue warp (warps FIRST..FIRST+7): wait for span partial `span_ctr`,
// add this thread's EPI_COLS columns of it into acc with round-to-nearest,
// release the buffer.  Warp w may access TMEM lanes 32*(w%4)..+31 (one output
// row per thread); the two warps sharing a lane quarter split the columns in
// halves.  CH: columns per tcgen05.ld (16 or 32).
template <int CH = 32, int FIRST = 2>
__device__ __forceinline__ bool drain_span(float (&acc)[EPI_COLS], uint32_t tmem_base, uint32_t span_ctr,
                                           uint64_t* sfull, uint64_t* sempty, int warp, int lane,
                                           volatile int* abort_flag, unsigned int* err) {
  const int q = warp & 3;
  const int half = (warp - FIRST) >> 2;
  const uint32_t p = span_ctr & 1u, ph = (span_ctr >> 1) & 1u;
  if (*abort_flag || !wait_bounded(&sfull[p], ph, err)) { *abort_flag = 1; return false; }
  jxd::tc_fence_after();
  const uint32_t t_addr = tmem_base + ((uint32_t)(q * 32) << 16) + p * (uint32_t)BN + (uint32_t)(half * EPI_COLS);
#pragma unroll
  for (int c = 0; c < EPI_COLS; c += CH) {
    uint32_t r[CH];
    if constexpr (CH == 32) jxd::tmem_ld32(t_addr + c, r);
    else jxd::tmem_ld16(t_addr + c, r);
    jxd::tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < CH; ++j) acc[c + j] = __fadd_rn(acc[c + j], __uint_as_float(r[j]));
  }
  jxd::tc_fence_before();
  __syncwarp();
  if (lane == 0) jxd::mbar_arrive(&sempty[p]);
  return true;
}

// ---- SM pairs (cta_group::2) -------------------------------------------------
// A cluster of two CTAs owns a PAIR_TILE x PAIR_TILE output tile; CTA r holds
// rows PAIR_ROWS*r.. of the A tile and of the B tile (K-major: the N rows of
// B^T) in the same stage layout [A hi][A lo][B hi][B lo], PAIR_OP bytes each,
// and its TMEM receives its PAIR_ROWS rows of the product.
constexpr int PAIR_TILE = 256;
constexpr int PAIR_ROWS = 128;
constexpr int PAIR_OP = PAIR_ROWS * BK * 4;  // 16 KB
constexpr int PAIR_BOX = 32 * BK * 4;        // one 32 x 32 MN-major box: 4 KB

// Tile t of a [batch][tiles_m][tiles_n] grid of pair tiles, grouped
// PAIR_GROUP_M row blocks at a time so the pairs of one wave share A and B
// tiles in L2.
constexpr int PAIR_GROUP_M = 8;
__device__ __forceinline__ TileInfo pair_tile_coords(int t, int tiles_m, int tiles_n) {
  const int per_batch = tiles_m * tiles_n;
  const int b = t / per_batch;
  const int r = t - b * per_batch;
  const int in_group = PAIR_GROUP_M * tiles_n;
  const int g = r / in_group;
  const int first_m = g * PAIR_GROUP_M;
  const int gsize = min(tiles_m - first_m, PAIR_GROUP_M);
  const int local = r - g * in_group;
  TileInfo ti;
  ti.m_blk = first_m + local % gsize;
  ti.n_blk = local / gsize;
  ti.b = b;
  return ti;
}

// wait_bounded with cluster-scope acquire: for barriers that receive the
// other CTA's arrivals.
__device__ __forceinline__ bool wait_bounded_cluster(uint64_t* bar, uint32_t parity, unsigned int* err) {
  if (jxd::mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (jxd::mbar_try_wait_cluster(bar, parity)) return true;
    if (global_ns() - t0 > 4000000000ull) {
      atomicOr(err, JX_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// A bounded wait whose outcome is the same in every lane of the warp (the
// warp is converged again on return, as tcgen05.ld needs).
__device__ __forceinline__ bool warp_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  unsigned int* err) {
  const bool got = !*abort_flag && wait_bounded(bar, parity, err);
  if (__all_sync(0xffffffffu, got)) return true;
  *abort_flag = 1;
  return false;
}

// Every warp of a group arrives on the local barrier `gbar`; the group's
// first thread (`first`) waits for its phase to complete (bounded), then
// alone arrives, with release at cluster scope, on the even CTA's barrier at
// shared::cluster address `cluster_bar`: one cluster-scope release per group
// instead of one per warp.  Warp-uniform outcome.
__device__ __forceinline__ bool group_arrive_cluster(uint64_t* gbar, uint32_t parity, uint32_t cluster_bar, bool first,
                                                     int lane, volatile int* abort_flag, unsigned int* err) {
  __syncwarp();
  if (lane == 0) jxd::mbar_arrive(gbar);
  int ok = 1;
  if (first) {
    ok = wait_bounded(gbar, parity, err) ? 1 : 0;
    if (ok) jxd::mbar_arrive_cluster(cluster_bar);
    else *abort_flag = 1;
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Shared-memory descriptor of k-step k (8 of the stage's 32 k) of a 128-row operand tile.
template <bool MN>
__device__ __forceinline__ uint64_t pair_op_desc(uint32_t base, int k) {
  if constexpr (MN) return jxd::smem_desc_mn_sw128_32b(base + k * 1024, PAIR_BOX);
  else return jxd::smem_desc_k_sw128(base + k * 32);
}

// The single-thread pair MMA issuer (even CTA): for every tile of this pair,
// Al.Bh + Ah.Bl + Ah.Bh per k-step into one of two TMEM span buffers of
// PAIR_TILE columns.  full[s] and sempty[p] live in the even CTA and collect
// one arrival per CTA; empty[s] and sfull[p] are committed to both CTAs.
// A_MN / B_MN: the operand tiles are MN-major (SWIZZLE_128B_ATOM_32B boxes).
template <bool A_MN, bool B_MN, int NSTAGE, int STAGE_BYTES_>
__device__ __forceinline__ void pair_mma_issuer(uint32_t smem_base, uint64_t* full, uint64_t* empty, uint64_t* sfull,
                                                uint64_t* sempty, uint32_t tmem_base, int first_tile, int num_tiles,
                                                int tile_step, int num_kb, volatile int* abort_flag,
                                                unsigned int* err) {
  constexpr uint32_t idesc =
      jxd::idesc_tf32(PAIR_TILE, PAIR_TILE) | (A_MN ? (1u << 15) : 0u) | (B_MN ? (1u << 16) : 0u);
  int stage = 0;
  uint32_t phase = 0, span_ctr = 0;
  for (int t = first_tile; t < num_tiles && !*abort_flag; t += tile_step) {
    for (int kb0 = 0; kb0 < num_kb && !*abort_flag; kb0 += SPAN_KB) {
      const uint32_t p = span_ctr & 1u, ph = (span_ctr >> 1) & 1u;
      if (!wait_bounded_cluster(&sempty[p], ph ^ 1u, err)) { *abort_flag = 1; break; }
      jxd::tc_fence_after();
      const uint32_t d_tmem = tmem_base + p * (uint32_t)PAIR_TILE;
      const int kb_end = min(kb0 + SPAN_KB, num_kb);
      for (int kb = kb0; kb < kb_end; ++kb) {
        if (!wait_bounded_cluster(&full[stage], phase, err)) { *abort_flag = 1; break; }
        jxd::tc_fence_after();
        const uint32_t sa = smem_base + stage * STAGE_BYTES_;
        const uint32_t sb = sa + 2 * PAIR_OP;
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          const uint64_t ah = pair_op_desc<A_MN>(sa, k), al = pair_op_desc<A_MN>(sa + PAIR_OP, k);
          const uint64_t bh = pair_op_desc<B_MN>(sb, k), bl = pair_op_desc<B_MN>(sb + PAIR_OP, k);
          jxd::mma_tf32_pair(d_tmem, al, bh, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          jxd::mma_tf32_pair(d_tmem, ah, bl, idesc, 1u);
          jxd::mma_tf32_pair(d_tmem, ah, bh, idesc, 1u);
        }
        jxd::mma_commit_pair(&empty[stage], 0x3);  // frees stage s in both CTAs
        if (++stage == NSTAGE) { stage = 0; phase ^= 1u; }
      }
      jxd::mma_commit_pair(&sfull[p], 0x3);  // span partial ready in both CTAs' TMEM
      ++span_ctr;
    }
  }
}

}  // namespace jxg

namespace jx {
// 3-D K-major tensor map [batch][rows][Kp] f32 with a BK x box_rows box and
// 128-byte swizzle (defined in gemm.cu).
int gemm_make_kmajor_map(CUtensorMap* map, const float* base, int Kp, int rows, int batch, int box_rows);
}  // namespace jx
