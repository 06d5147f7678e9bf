// jx_common.cuh -- shared helpers for the jax-rs CUDA backend (sm_100a only).
//
// Status/error plumbing for the C ABI, plus thin inline-PTX wrappers for the
// Blackwell features the kernels use: mbarriers, TMA tiled loads (no cluster
// multicast anywhere in this library), tcgen05 MMA/TMEM, and fences.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "../../include/jaxrs_cuda.h"

#include <nvtx3/nvToolsExt.h>

// ---------------------------------------------------------------------------
// Host-side error reporting
// ---------------------------------------------------------------------------
namespace jx {

void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

// Every C-ABI entry point that launches work goes through this so that a
// launch failure becomes a status code plus jx_last_error() text.
#define JX_CUDA(call)                                                       \
  do {                                                                      \
    cudaError_t _e = (call);                                                \
    if (_e != cudaSuccess) return ::jx::check_cuda(_e, #call);              \
  } while (0)

#define JX_LAUNCH_CHECK(name)                                               \
  do {                                                                      \
    cudaError_t _e = cudaGetLastError();                                    \
    if (_e != cudaSuccess) return ::jx::check_cuda(_e, name);               \
  } while (0)

#define JX_REQUIRE(cond, ...)                                               \
  do {                                                                      \
    if (!(cond)) return ::jx::fail(JX_EINVAL, __VA_ARGS__);                 \
  } while (0)

// NVTX range around a C-ABI entry point: an Nsight Systems / Nsight Compute
// timeline shows each call by its entry-point name, nested calls inside it.
// With no tool attached the push and pop return at once.
struct TraceRange {
  explicit TraceRange(const char* name) { nvtxRangePushA(name); }
  ~TraceRange() { nvtxRangePop(); }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};
#define JX_TRACE(name) ::jx::TraceRange jx_trace_range_(name)

int num_sms();                // SM count of the current device (cached)
cudaStream_t as_stream(jx_stream_t s);

// Stream-ordered scratch for one call (GEMM operand splitting, reduction
// partials): taken from the device's default memory pool with cudaMallocAsync
// on the call's stream and handed back with cudaFreeAsync after the call's
// last launch, so concurrent calls on different streams never share it.  The
// pool keeps freed memory cached (release threshold raised in jx_init).
int scratch_get(size_t bytes, void** out, cudaStream_t st);
int scratch_release(void* p, cudaStream_t st);

// Per-device error word written by kernels that detect bad input (NaN in an
// arg-reduction, a bounded wait that timed out).  Read with jx_device_status.
unsigned int* device_error_word();

}  // namespace jx

struct CUtensorMap_st;
namespace jx {
// 3-D f32 TMA descriptor without swizzle: dims {d0 (contiguous), d1, d2},
// byte strides {s1, s2}, box {b0, b1, 1}.
int tensor_map_f32_3d(CUtensorMap_st* map, const void* base, const uint64_t* dims, const uint64_t* strides,
                      const uint32_t* box);
}  // namespace jx

// Device error codes recorded in the device error word (bit flags).
#define JX_DEVERR_NAN 0x1u
#define JX_DEVERR_TIMEOUT 0x2u

// ---------------------------------------------------------------------------
// Device-side PTX helpers (sm_100a)
// ---------------------------------------------------------------------------
#if defined(__CUDACC__)
namespace jxd {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// --- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit` polls (each try_wait itself blocks for a
// hardware-defined time slice), records JX_DEVERR_TIMEOUT and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err,
                                          uint32_t limit = 2000000u) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, JX_DEVERR_TIMEOUT);
  return false;
}

// --- TMA (tiled, no multicast) ------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x,
                                            int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// --- tcgen05 ------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem], kind::tf32, single CTA.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: 8-row groups 1024 B apart (SBO), LBO unused (1),
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(1u) << 16;                 // LBO (ignored for swizzled K-major)
  d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;  // SBO
  d |= (uint64_t)1u << 46;                   // version
  d |= (uint64_t)2u << 61;                   // SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor for an MN-major 32-bit tile written by TMA
// with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B: rows of 32 MN-consecutive values
// (128 B) one per k, groups of 4 k-rows 512 B apart (SBO), 32-wide MN blocks
// `mn_block_bytes` apart (LBO), layout type 1 = SWIZZLE_128B_BASE32B (the only
// MN-major layout tf32 operands accept).
__device__ __forceinline__ uint64_t smem_desc_mn_sw128_32b(uint32_t smem_addr, uint32_t mn_block_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((mn_block_bytes >> 4) & 0x3FFFu) << 16;  // LBO
  d |= (uint64_t)((512u >> 4) & 0x3FFFu) << 32;            // SBO
  d |= (uint64_t)1u << 46;                                  // version
  d |= (uint64_t)1u << 61;                                  // SWIZZLE_128B_BASE32B
  return d;
}

// Instruction descriptor: kind::tf32, D=f32, A=B=tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4)                 // D format f32
         | (2u << 7)               // A format tf32
         | (2u << 10)              // B format tf32
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 3xTF32 operand split: hi = tf32_rn(x), lo = tf32_rn(x - hi).
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  hi = __uint_as_float(h);
  const float rem = __fsub_rn(x, hi);
  uint32_t l;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(rem));
  lo = __uint_as_float(l);
}

// lo part for a hi taken as the truncation of x to tf32 (what the tf32 MMA
// reads from a raw f32 value): x - trunc(x) is exact in f32, then rounded to
// the nearest tf32.
// The rounding is done on the bits (integer pipes): adding half of a tf32
// ulp (bit 12) to the magnitude and clearing the 13 low bits rounds to the
// nearest tf32 with ties away from zero, as cvt.rna.tf32.f32 does for any
// finite value.
__device__ __forceinline__ float tf32_lo_of_trunc(float x) {
  const float hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  const uint32_t r = __float_as_uint(__fsub_rn(x, hi));
  return __uint_as_float((r + 0x1000u) & 0xffffe000u);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// --- clusters and SM pairs (tcgen05 cta_group::2) ------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address in the shared::cluster window of the same offset in CTA `rank`'s shared memory.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Arrive on an mbarrier anywhere in the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// try_wait with cluster-scope acquire: for barriers that other CTAs arrive on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Every thread of both CTAs: arrive at and wait on the cluster barrier.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMEM allocation shared by an SM pair: one warp (same warp index) of each CTA issues it.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A * B over an SM pair, kind::tf32: issued by one
// thread of the pair's even CTA; each CTA supplies M/2 rows of A and N/2
// columns of B at the same shared-memory offsets.
__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at this offset in every CTA of cta_mask when all
// previously issued pair MMAs of this thread complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

}  // namespace jxd
#endif
