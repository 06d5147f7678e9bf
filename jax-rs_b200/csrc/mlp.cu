// mlp.cu -- native training step for a stack of Dense layers with softmax
// cross-entropy and Adam: the training loop the reference expresses as
// examples/mlp_training.rs:94-145 (matmul + broadcast bias + relu, finite
// differences and SGD there) with the reference's optim::adam_update
// (src/optim.rs:138-189) as the optimiser.
//
// Layout: parameters, gradients and the Adam moments each live in one flat
// device buffer ordered [W1, b1, W2, b2, ...] (W_l row-major [in, out]), so a
// layer's gradient is one contiguous bucket for the data-parallel all-reduce
// and Adam is one elementwise launch over everything.  On one GPU the whole
// step (forward, backward, Adam) is captured once into a CUDA graph and
// replayed; with a communicator attached, each layer's gradient bucket is
// all-reduced on a second stream as soon as backward produces it, overlapped
// with the backward of the layers below.
#include <math.h>

#include <new>
#include <vector>

#include "jx_common.cuh"
#include "nn_common.cuh"

namespace jx {
int col_sum(const float* dy, float* db, long long rows, int cols, cudaStream_t st);
int nccl_allreduce(void* comm, float* buf, long long count, cudaStream_t st);
int nccl_reduce_scatter(void* comm, float* buf, long long shard, cudaStream_t st);
int nccl_all_gather(void* comm, float* buf, long long shard, cudaStream_t st);
int nccl_rank(void* comm, int* rank, int* nranks);
}  // namespace jx

namespace {

constexpr long long ADAM_TABLE_STEPS = 1 << 20;

// Adam over the flat buffers.  The step number lives on the device (so a
// captured graph replays correctly) and indexes a host-computed table of
// (1/(1-b1^t), 1/(1-b2^t)) -- powf on the host as in optim::adam_update -- so
// the arithmetic is bit-identical to the reference's.
__global__ void adam_flat_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                 float* __restrict__ v, long long n, const int* __restrict__ step,
                                 const float2* __restrict__ tab, float lr, float b1, float b2, float eps, float omb1,
                                 float omb2) {
  const int t = *step;
  const float2 rr = tab[t - 1];
  const bool first = t == 1;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gi = g[i];
    const float mi = first ? __fmul_rn(gi, omb1) : __fadd_rn(__fmul_rn(m[i], b1), __fmul_rn(gi, omb1));
    const float g2 = __fmul_rn(gi, gi);
    const float vi = first ? __fmul_rn(g2, omb2) : __fadd_rn(__fmul_rn(v[i], b2), __fmul_rn(g2, omb2));
    const float mh = __fmul_rn(mi, rr.x);
    const float vh = __fmul_rn(vi, rr.y);
    p[i] = __fsub_rn(p[i], __fmul_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), eps)), lr));
    m[i] = mi;
    v[i] = vi;
  }
}

__global__ void step_inc_kernel(int* step) { *step += 1; }

// ---------------------------------------------------------------------------
// Fused step (JX_PREC_EXACT, one GPU): forward, softmax cross-entropy,
// backward and Adam in one cooperative launch instead of ~23 kernels.  Phases
// are separated by a grid barrier (2L of them; Adam runs inside the backward
// phases); inside a phase every block
// takes work items in a grid-stride loop.  The arithmetic is the separate
// kernels' own: the exact GEMM's ascending-k unfused sums (one thread per
// output of a 16 x 16 tile, K through a cp.async ring of 128-wide chunks),
// bias + activation, jxn::softmax_xent_row, the column sums' sequential row
// order, the activation derivative and Adam, so the results are bit-identical
// to the captured-graph path.  Data written inside the launch is read back
// through L2 (ld.global.cg): an SM's L1 may still hold the previous contents
// of a buffer that another SM rewrote.
// ---------------------------------------------------------------------------
constexpr int FS_MAXL = 8, FS_THREADS = 256, FS_T = 16, FS_KC = 128;

struct FusedStep {
  int L, B;
  int w[FS_MAXL + 1];
  int act[FS_MAXL];
  long long woff[FS_MAXL], boff[FS_MAXL];
  const float* x;
  const float* labels;
  float *params, *grads, *m, *v;
  float* h[FS_MAXL + 1];
  float* pre[FS_MAXL + 1];
  float *dzA, *dzB, *row_loss, *loss, *loss_out;
  int* step;
  const float2* tab;
  float lr, b1, b2, eps, omb1, omb2, count;
  long long nparams;
  unsigned* bar;   // two launch slots of barrier arrivals
  int slot;        // this launch's slot; it zeroes the other one for the next launch
  unsigned* err;
};

__device__ __forceinline__ unsigned long long fs_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid barrier number `index` (0-based) of this launch: every block adds one
// arrival and waits until all gridDim.x * (index + 1) have arrived.  The wait
// gives up after 2 s, records JX_DEVERR_TIMEOUT and returns false.
__device__ bool fs_grid_sync(unsigned* cnt, unsigned index, unsigned* err, int* ok_flag,
                             unsigned long long limit_ns = 2000000000ull, unsigned extra = 0) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned target = gridDim.x * (index + 1) + extra;
    __threadfence();
    atomicAdd(cnt, 1u);
    bool ok = true;
    const unsigned long long t0 = fs_ns();
    while (*reinterpret_cast<volatile unsigned*>(cnt) < target) {
      if (fs_ns() - t0 > limit_ns) {
        atomicOr(err, JX_DEVERR_TIMEOUT);
        ok = false;
        break;
      }
    }
    __threadfence();
    *ok_flag = ok;
  }
  __syncthreads();
  return *ok_flag;
}

constexpr int FS_NS = 4;  // cp.async stages of FS_KC k-values in flight per tile

// Shared-memory stage of one operand, kept in the orientation it has in
// global memory so that cp.async can move 16 bytes at a time: k-major rows
// [16][FS_KC + 4] when k is contiguous, else [FS_KC][16 + 4].
constexpr int FS_KP = FS_KC + 4, FS_MP = FS_T + 4;
constexpr int FS_OPF = FS_KC * FS_MP;  // floats per operand stage (the larger layout)
static_assert(FS_T * FS_KP <= FS_OPF, "stage size");
struct FsSmem {
  float A[FS_NS][FS_OPF];
  float B[FS_NS][FS_OPF];
  float red[32];
  int ok;
};

__device__ __forceinline__ void fs_cp4(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(jxd::smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void fs_cp16(float* dst, const float* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(jxd::smem_u32(dst)), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void fs_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void fs_cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copies one operand's chunk (FS_T rows/cols of the tile x FS_KC k-values
// starting at k0) into a stage.  KMAJ: k contiguous in global memory (the
// stage is [FS_T][FS_KP]); else the tile's 16 rows/cols are contiguous (the
// stage is [FS_KC][FS_MP]).  x0: the tile's first row/col, X: rows/cols in the
// matrix, ld: its row stride.  vec: 16-byte copies allowed (ld and the base
// 16-byte aligned); zero-filled outside the matrix either way.
template <bool KMAJ>
__device__ __forceinline__ void fs_load_op(float* stage, const float* __restrict__ g, int x0, int X, int k0, int K,
                                           int ld, bool vec) {
  const int tid = threadIdx.x;
  if (vec) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {  // 512 16-byte pieces per chunk
      const int idx = tid + 256 * e;
      if (KMAJ) {
        const int x = idx >> 5, kk = (idx & 31) * 4;
        const int gx = x0 + x, gk = k0 + kk;
        const int bytes = gx < X ? max(0, min(16, (K - gk) * 4)) : 0;
        fs_cp16(stage + x * FS_KP + kk, bytes ? g + (long long)gx * ld + gk : g, bytes);
      } else {
        const int kk = idx >> 2, x = (idx & 3) * 4;
        const int gx = x0 + x, gk = k0 + kk;
        const int bytes = gk < K ? max(0, min(16, (X - gx) * 4)) : 0;
        fs_cp16(stage + kk * FS_MP + x, bytes ? g + (long long)gk * ld + gx : g, bytes);
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {  // 2048 single floats, consecutive threads on consecutive addresses
      const int idx = tid + 256 * e;
      if (KMAJ) {
        const int x = idx >> 7, kk = idx & 127;
        const int gx = x0 + x, gk = k0 + kk;
        const bool v = gx < X && gk < K;
        fs_cp4(stage + x * FS_KP + kk, v ? g + (long long)gx * ld + gk : g, v);
      } else {
        const int kk = idx >> 4, x = idx & 15;
        const int gx = x0 + x, gk = k0 + kk;
        const bool v = gk < K && gx < X;
        fs_cp4(stage + kk * FS_MP + x, v ? g + (long long)gk * ld + gx : g, v);
      }
    }
  }
}

// Four consecutive k-values of row/col x of a stage.
template <bool KMAJ>
__device__ __forceinline__ float4 fs_get4(const float* stage, int x, int kk) {
  if (KMAJ) return *reinterpret_cast<const float4*>(stage + x * FS_KP + kk);
  return make_float4(stage[kk * FS_MP + x], stage[(kk + 1) * FS_MP + x], stage[(kk + 2) * FS_MP + x],
                     stage[(kk + 3) * FS_MP + x]);
}
template <bool KMAJ>
__device__ __forceinline__ float fs_get1(const float* stage, int x, int kk) {
  return KMAJ ? stage[x * FS_KP + kk] : stage[kk * FS_MP + x];
}

__device__ __forceinline__ bool fs_vec_ok(const float* p, int ld) {
  return (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// One 16 x 16 tile of C = op(A) . op(B) (M x N, K deep); epi(row, col, sum)
// for the in-range outputs.  TA / TB: A / B transposed in memory (A is then
// [K][M], B [N][K]).  K streams through a ring of FS_NS shared-memory stages
// filled by cp.async, FS_NS - 1 chunks ahead of the sums.  colsum (or null):
// the tile's first row of threads also sums B's columns over k in order --
// the column sums of the separate kernels (256-row chunk sums added in chunk
// order) -- for the tiles of the first row of C.
template <bool TA, bool TB, class Epi>
__device__ void fs_tile(FsSmem& sm, int tile, const float* __restrict__ a, const float* __restrict__ b, int M, int N,
                        int K, int lda, int ldb, Epi epi, float* colsum = nullptr) {
  constexpr bool AK = !TA, BK = TB;  // k contiguous in the stage
  const int tiles_n = (N + FS_T - 1) / FS_T;
  const int r0 = (tile / tiles_n) * FS_T, c0 = (tile % tiles_n) * FS_T;
  const int tid = threadIdx.x, tx = tid & (FS_T - 1), ty = tid >> 4;
  const bool va = fs_vec_ok(a, lda), vb = fs_vec_ok(b, ldb);
  auto issue = [&](int ch) {
    const int st = ch % FS_NS, k0 = ch * FS_KC;
    fs_load_op<AK>(sm.A[st], a, r0, M, k0, K, lda, va);
    fs_load_op<BK>(sm.B[st], b, c0, N, k0, K, ldb, vb);
  };
  const int nchunk = (K + FS_KC - 1) / FS_KC;
#pragma unroll
  for (int c = 0; c < FS_NS - 1; ++c) {
    if (c < nchunk) issue(c);
    fs_cp_commit();
  }
  const bool do_cs = colsum && r0 == 0 && ty == 0;
  float sum = 0.0f, cs_acc = 0.0f, cs_tot = 0.0f;
  for (int ch = 0; ch < nchunk; ++ch) {
    fs_cp_wait<FS_NS - 2>();  // this thread's copies of chunk ch have landed
    __syncthreads();          // everyone's; stage (ch - 1) % FS_NS is free again
    if (ch + FS_NS - 1 < nchunk) issue(ch + FS_NS - 1);
    fs_cp_commit();
    const float* As = sm.A[ch % FS_NS];
    const float* Bs = sm.B[ch % FS_NS];
    const int kmax = min(FS_KC, K - ch * FS_KC);
    const int k4 = kmax & ~3;
    // several 4-value reads in flight ahead of the dependent adds; the
    // products are still added one by one in ascending k
#pragma unroll 4
    for (int kk = 0; kk < k4; kk += 4) {
      const float4 av = fs_get4<AK>(As, ty, kk);
      const float4 bv = fs_get4<BK>(Bs, tx, kk);
      sum = __fadd_rn(sum, __fmul_rn(av.x, bv.x));
      sum = __fadd_rn(sum, __fmul_rn(av.y, bv.y));
      sum = __fadd_rn(sum, __fmul_rn(av.z, bv.z));
      sum = __fadd_rn(sum, __fmul_rn(av.w, bv.w));
    }
    for (int kk = k4; kk < kmax; ++kk) sum = __fadd_rn(sum, __fmul_rn(fs_get1<AK>(As, ty, kk), fs_get1<BK>(Bs, tx, kk)));
    if (do_cs) {
      if (ch > 0 && (ch * FS_KC) % 256 == 0) {
        cs_tot += cs_acc;
        cs_acc = 0.0f;
      }
      for (int kk = 0; kk < kmax; ++kk) cs_acc += fs_get1<BK>(Bs, tx, kk);
    }
  }
  fs_cp_wait<0>();
  __syncthreads();  // the ring is free for the next tile
  if (do_cs && c0 + tx < N) {
    cs_tot += cs_acc;
    colsum[c0 + tx] = cs_tot;
  }
  const int row = r0 + ty, col = c0 + tx;
  if (row < M && col < N) epi(row, col, sum);
}

__global__ void __launch_bounds__(FS_THREADS, 2) mlp_fused_step_kernel(FusedStep a) {
  extern __shared__ __align__(16) unsigned char fs_raw[];
  FsSmem& sm = *reinterpret_cast<FsSmem*>(fs_raw);
  const int t = *a.step;  // read before the first barrier; block 0 writes t + 1 at the end
  unsigned* cnt = a.bar + a.slot;
  if (blockIdx.x == 0 && threadIdx.x == 0) a.bar[a.slot ^ 1] = 0u;
  unsigned nbar = 0;
  const int lane = threadIdx.x & 31;
  const long long gtid = (long long)blockIdx.x * blockDim.x + threadIdx.x, gthreads = (long long)gridDim.x * blockDim.x;
  const int B = a.B;

  // ---- forward: h_l = act(h_{l-1} W_l + b_l) ----
  for (int l = 1; l <= a.L; ++l) {
    const int K = a.w[l - 1], N = a.w[l];
    const float* in = l == 1 ? a.x : a.h[l - 1];
    const float* W = a.params + a.woff[l - 1];
    const float* bias = a.params + a.boff[l - 1];
    float* out = a.h[l];
    float* pre = l < a.L ? a.pre[l] : nullptr;
    const int act = l < a.L ? a.act[l - 1] : 0;
    const int tiles = ((B + FS_T - 1) / FS_T) * ((N + FS_T - 1) / FS_T);
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x)
      fs_tile<false, false>(sm, tile, in, W, B, N, K, K, N, [&](int r, int c, float sum) {
        const float v = __fadd_rn(sum, __ldcg(bias + c));
        if (pre) pre[(long long)r * N + c] = v;
        out[(long long)r * N + c] = jxn::act_apply(act, v);
      });
    if (!fs_grid_sync(cnt, nbar++, a.err, &sm.ok)) return;
  }

  // ---- softmax cross-entropy: dz = dL/dlogits, per-row losses ----
  const int C = a.w[a.L];
  for (long long r = gtid >> 5; r < B; r += gthreads >> 5) {
    const float lr = jxn::softmax_xent_row(a.h[a.L] + r * C, __ldcg(a.labels + r), C, a.count, nullptr,
                                           a.dzA + r * C, lane);
    if (lane == 0) a.row_loss[r] = lr;
  }
  if (!fs_grid_sync(cnt, nbar++, a.err, &sm.ok)) return;

  // loss = sum of row losses / count, in the order of the 1024-thread
  // reduction the separate kernels use (block 0, overlapping the backward)
  if (blockIdx.x == 0) {
    const int wid = threadIdx.x >> 5;
    for (int w = wid; w < 32; w += FS_THREADS / 32) {
      float acc = 0.0f;
      for (long long i = w * 32 + lane; i < B; i += 1024) acc += __ldcg(a.row_loss + i);
      acc = jxn::warp_sum(acc);
      if (lane == 0) sm.red[w] = acc;
    }
    __syncthreads();
    if (wid == 0) {
      float acc = sm.red[lane];
      acc = jxn::warp_sum(acc);
      if (lane == 0) {
        const float loss = __fdiv_rn(acc, a.count);
        *a.loss = loss;
        if (a.loss_out) *a.loss_out = loss;
      }
    }
  }

  // Adam for parameter i with gradient gi (the separate kernel's formula).
  const float2 rr = a.tab[t - 1];
  const bool first = t == 1;
  auto adam = [&](long long i, float gi) {
    const float mi = first ? __fmul_rn(gi, a.omb1) : __fadd_rn(__fmul_rn(a.m[i], a.b1), __fmul_rn(gi, a.omb1));
    const float g2 = __fmul_rn(gi, gi);
    const float vi = first ? __fmul_rn(g2, a.omb2) : __fadd_rn(__fmul_rn(a.v[i], a.b2), __fmul_rn(g2, a.omb2));
    const float mh = __fmul_rn(mi, rr.x);
    const float vh = __fmul_rn(vi, rr.y);
    a.params[i] = __fsub_rn(a.params[i], __fmul_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), a.eps)), a.lr));
    a.m[i] = mi;
    a.v[i] = vi;
  };

  // ---- backward: dW_l = h_{l-1}^T dz, db_l = column sums of dz,
  //      dz_{l-1} = (dz W_l^T) * act'(pre_{l-1}) ----
  // Adam needs no phase of its own.  Layer l + 1's parameters are updated
  // during layer l's phase: W_{l+1} was last read by the previous phase,
  // whose barrier has passed, and nothing reads it again.  Layer 1's are
  // updated in the dW_1 tiles themselves (no later phase reads W_1), so the
  // last phase ends the kernel without a barrier.
  float* dz = a.dzA;
  float* dzn = a.dzB;
  for (int l = a.L; l >= 1; --l) {
    const int K = a.w[l - 1], N = a.w[l];
    const float* hin = l == 1 ? a.x : a.h[l - 1];
    const float* W = a.params + a.woff[l - 1];
    float* gW = a.grads + a.woff[l - 1];
    float* gb = a.grads + a.boff[l - 1];
    const int tiles_w = ((K + FS_T - 1) / FS_T) * ((N + FS_T - 1) / FS_T);
    const int tiles_h = l > 1 ? ((B + FS_T - 1) / FS_T) * ((K + FS_T - 1) / FS_T) : 0;
    for (int tile = blockIdx.x; tile < tiles_w + tiles_h; tile += gridDim.x) {
      if (tile < tiles_w) {
        const long long wo = a.woff[l - 1];
        fs_tile<true, false>(
            sm, tile, hin, dz, K, N, B, K, N,
            [&](int r, int c, float sum) {
              gW[(long long)r * N + c] = sum;
              if (l == 1) adam(wo + (long long)r * N + c, sum);
            },
            gb);
        if (l == 1) {
          // the bias gradient this thread's colsum wrote (first row of tiles, first row of threads)
          const int tiles_n = (N + FS_T - 1) / FS_T;
          const int c = (tile % tiles_n) * FS_T + (threadIdx.x & (FS_T - 1));
          if (tile / tiles_n == 0 && threadIdx.x < FS_T && c < N) adam(a.boff[0] + c, gb[c]);
        }
      } else {
        const float* pre = a.pre[l - 1];
        const int act = a.act[l - 2];
        fs_tile<false, true>(sm, tile - tiles_w, dz, W, B, K, N, N, N, [&](int r, int c, float sum) {
          dzn[(long long)r * K + c] = __fmul_rn(sum, jxn::act_grad_rt(act, __ldcg(pre + (long long)r * K + c)));
        });
      }
    }
    if (l < a.L) {
      // layer l + 1: its gradients are complete (previous phase)
      const int Kn = a.w[l], Nn = a.w[l + 1];
      const long long wo = a.woff[l], bo = a.boff[l], nw = (long long)Kn * Nn;
      for (long long i = gtid; i < nw + Nn; i += gthreads) {
        const long long p = i < nw ? wo + i : bo + (i - nw);
        adam(p, __ldcg(a.grads + p));
      }
    }
    if (l == 1) break;  // the last phase: no barrier, the kernel ends
    if (!fs_grid_sync(cnt, nbar++, a.err, &sm.ok)) return;
    float* tmp = dz;
    dz = dzn;
    dzn = tmp;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *a.step = t + 1;
}

}  // namespace

struct jx_mlp {
  int L = 0;
  std::vector<long long> w;  // widths, L + 1
  std::vector<int> act;      // activation of layer l at act[l-1]; the last layer has none
  long long B = 0;
  int prec = JX_PREC_3XTF32;
  long long nparams = 0;
  std::vector<long long> woff, boff;
  float *params = nullptr, *grads = nullptr, *m = nullptr, *v = nullptr;
  std::vector<float*> h;    // h[0] input copy, h[l] output of layer l (h[L] = logits)
  std::vector<float*> pre;  // pre-activations of hidden layers (index l)
  float *dz = nullptr, *dh = nullptr, *labels = nullptr, *loss = nullptr;
  int* step = nullptr;
  float2* tab = nullptr;
  float lr = 1e-3f, b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
  void* comm = nullptr;
  long long global_B = 0;
  cudaStream_t cstream = nullptr;
  std::vector<cudaEvent_t> ev;
  int dw1_chunks = 2;  // row chunks of layer 1's weight gradient under data parallelism
  int dp_rank = 0, dp_world = 1;
  bool dp_sharded = true;  // reduce-scatter + Adam on this rank's shard + all-gather
  // phase timing (jx_mlp_set_timing): events at step start, forward end,
  // backward end on the caller's stream, and step end
  bool timing = false;
  cudaEvent_t tev[4] = {nullptr, nullptr, nullptr, nullptr};
  bool tev_recorded = false;
  cudaGraphExec_t gexec = nullptr;
  long long steps = 0;
  // fused step (exact precision, one GPU)
  bool fused = true;
  unsigned* bar = nullptr;     // two slots of grid-barrier arrivals
  float* row_loss = nullptr;   // B per-row losses
  int fused_grid = 0;
  long long fused_launches = 0;  // alternates the barrier slot, whatever else runs between
};

namespace {

void free_all(jx_mlp* n) {
  if (n->gexec) cudaGraphExecDestroy(n->gexec);
  for (cudaEvent_t e : n->tev)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : n->ev) cudaEventDestroy(e);
  if (n->cstream) cudaStreamDestroy(n->cstream);
  for (float* p : n->h) cudaFree(p);
  for (float* p : n->pre) cudaFree(p);
  cudaFree(n->params);
  cudaFree(n->grads);
  cudaFree(n->m);
  cudaFree(n->v);
  cudaFree(n->dz);
  cudaFree(n->dh);
  cudaFree(n->labels);
  cudaFree(n->loss);
  cudaFree(n->step);
  cudaFree(n->tab);
  cudaFree(n->bar);
  cudaFree(n->row_loss);
}

int fill_adam_table(jx_mlp* n) {
  std::vector<float2> t(ADAM_TABLE_STEPS);
  for (long long s = 1; s <= ADAM_TABLE_STEPS; ++s) {
    const float tf = (float)s;
    const float bc1 = 1.0f - powf(n->b1, tf);
    const float bc2 = 1.0f - powf(n->b2, tf);
    t[s - 1] = make_float2(1.0f / bc1, 1.0f / bc2);
  }
  JX_CUDA(cudaMemcpy(n->tab, t.data(), sizeof(float2) * t.size(), cudaMemcpyHostToDevice));
  return JX_OK;
}

int grid_elems(long long n) {
  long long blocks = (n + 255) / 256;
  long long cap = (long long)jx::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

// Adam over params[off, off + count) (and the same range of the gradients and
// moments) on stream s.
void adam_range(jx_mlp* n, long long off, long long count, cudaStream_t s) {
  adam_flat_kernel<<<grid_elems(count), 256, 0, s>>>(n->params + off, n->grads + off, n->m + off, n->v + off, count,
                                                     n->step, n->tab, n->lr, n->b1, n->b2, n->eps, 1.0f - n->b1,
                                                     1.0f - n->b2);
}

// The exchange of one gradient bucket [off, off + count) under data
// parallelism, on the communication stream, in two halves: bucket_reduce as
// soon as backward has produced the gradient, bucket_update once nothing in
// the step reads the bucket's parameters any more.  Sharded (the default,
// when count divides by the rank count): reduce-scatter the gradient, Adam on
// this rank's 1/world of the bucket, all-gather the updated parameters; the
// same communication volume as an all-reduce, and each rank's Adam pass
// (28 bytes of HBM traffic per parameter) shrinks by the rank count.  Each
// rank keeps Adam moments only for its own shards.  Otherwise: all-reduce and
// Adam over the whole bucket on every rank.
bool bucket_sharded(const jx_mlp* n, long long count) {
  return n->dp_sharded && n->dp_world > 1 && count % n->dp_world == 0;
}

int bucket_reduce(jx_mlp* n, long long off, long long count) {
  if (bucket_sharded(n, count)) return jx::nccl_reduce_scatter(n->comm, n->grads + off, count / n->dp_world, n->cstream);
  return jx::nccl_allreduce(n->comm, n->grads + off, count, n->cstream);
}

int bucket_update(jx_mlp* n, long long off, long long count) {
  if (bucket_sharded(n, count)) {
    const long long shard = count / n->dp_world;
    adam_range(n, off + n->dp_rank * shard, shard, n->cstream);
    return jx::nccl_all_gather(n->comm, n->params + off, shard, n->cstream);
  }
  adam_range(n, off, count, n->cstream);
  return JX_OK;
}

// Layer 1's weight gradient under data parallelism, in n->dw1_chunks row
// chunks: each chunk's product is all-reduced and its Adam update applied on
// the communication stream while the next chunk's product runs.  This is the
// last gradient of the step, so without the chunks its whole all-reduce and
// update would sit behind the backward pass with nothing to overlap.  Rows
// r0.. of dW1 = h0^T dz are the product of columns r0.. of h0 (A transposed,
// lda = K) with dz.
int dw1_chunked(jx_mlp* n, cudaStream_t st, int& evi) {
  const long long B = n->B, K = n->w[0], N = n->w[1];
  const int S = n->dw1_chunks;
  const long long rows = K / S;
  float* gW = n->grads + n->woff[0];
  int rc = jx::col_sum(n->dz, n->grads + n->boff[0], B, (int)N, st);
  for (int c = 0; !rc && c < S; ++c) {
    const long long r0 = c * rows;
    rc = jx_gemm_f32(n->h[0] + r0, n->dz, gW + r0 * N, rows, N, B, 1, 0, K, N, N, 1, 0, 0, 0, n->prec, st);
    if (rc) break;
    cudaEvent_t e = n->ev[evi++];
    cudaError_t ce = cudaEventRecord(e, st);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(n->cstream, e, 0);
    if (ce != cudaSuccess) {
      rc = jx::check_cuda(ce, "mlp: layer-1 chunk hand-off");
      break;
    }
    // the last chunk carries the bias gradient, which follows W1 in the bucket
    const long long count = rows * N + (c == S - 1 ? N : 0);
    rc = bucket_reduce(n, n->woff[0] + r0 * N, count);
    if (!rc) rc = bucket_update(n, n->woff[0] + r0 * N, count);
  }
  return rc;
}

// One training step on stream st (forward, backward, optional all-reduce, Adam).
//
// With a communicator attached, layer l's gradient bucket (W_l then b_l) is
// reduced on the communication stream as soon as backward has produced it,
// and that bucket's Adam update (with the all-gather of the sharded form)
// follows on the same stream once the backward GEMM that reads W_l
// (dh = dz W_l^T) is done; both overlap the backward of the layers below.  The caller's stream waits for the
// communication stream before the step counter moves on.
int run_step(jx_mlp* n, cudaStream_t st) {
  int rc;
  const long long B = n->B;
  if (n->timing) JX_CUDA(cudaEventRecord(n->tev[0], st));
  for (int l = 1; l <= n->L; ++l) {
    const long long K = n->w[l - 1], N = n->w[l];
    if ((rc = jx_gemm_f32(n->h[l - 1], n->params + n->woff[l - 1], n->h[l], B, N, K, 0, 0, K, N, N, 1, 0, 0, 0,
                          n->prec, st)))
      return rc;
    if ((rc = jx_bias_act_f32(n->h[l], n->params + n->boff[l - 1], l < n->L ? n->pre[l] : nullptr, B, N,
                              l < n->L ? n->act[l - 1] : 0, st)))
      return rc;
  }
  const long long C = n->w[n->L];
  if ((rc = jx_softmax_xent_f32(n->h[n->L], n->labels, nullptr, n->dz, n->loss, B, C, n->global_B * C, st)))
    return rc;
  if (n->timing) JX_CUDA(cudaEventRecord(n->tev[1], st));
  int evi = 0;
  // the communication stream waits for everything enqueued on st so far
  auto hand_off = [&]() -> int {
    cudaEvent_t e = n->ev[evi++];
    JX_CUDA(cudaEventRecord(e, st));
    JX_CUDA(cudaStreamWaitEvent(n->cstream, e, 0));
    return JX_OK;
  };
  for (int l = n->L; l >= 1; --l) {
    const long long K = n->w[l - 1], N = n->w[l];
    float* gW = n->grads + n->woff[l - 1];
    const long long bucket = K * N + N;  // W_l then b_l, contiguous
    const bool chunked = n->comm && l == 1 && n->prec == JX_PREC_3XTF32 && n->dw1_chunks > 1 &&
                         K % (n->dw1_chunks * 128LL) == 0;
    if (chunked) {
      if ((rc = dw1_chunked(n, st, evi))) return rc;
    } else {
      // dW_l = h_{l-1}^T dz (transpose_matmul's dB = A^T dC, src/trace/transpose_rules.rs:537-567)
      if ((rc = jx_gemm_f32(n->h[l - 1], n->dz, gW, K, N, B, 1, 0, K, N, N, 1, 0, 0, 0, n->prec, st))) return rc;
      if ((rc = jx::col_sum(n->dz, n->grads + n->boff[l - 1], B, (int)N, st))) return rc;
      if (n->comm) {
        if ((rc = hand_off())) return rc;
        if ((rc = bucket_reduce(n, n->woff[l - 1], bucket))) return rc;
      }
    }
    if (l > 1) {
      // dh = dz W_l^T (transpose_matmul's dA = dC B^T), then dz = dh * act'(pre)
      if ((rc = jx_gemm_f32(n->dz, n->params + n->woff[l - 1], n->dh, B, K, N, 0, 1, N, N, K, 1, 0, 0, 0, n->prec,
                            st)))
        return rc;
      if ((rc = jx_act_bwd_f32(n->dh, n->pre[l - 1], n->dz, nullptr, B, K, n->act[l - 2], st))) return rc;
    }
    if (n->comm && !chunked) {
      if ((rc = hand_off())) return rc;  // W_l is no longer read by this step
      if ((rc = bucket_update(n, n->woff[l - 1], bucket))) return rc;
    }
  }
  if (n->timing) JX_CUDA(cudaEventRecord(n->tev[2], st));
  if (n->comm) {
    cudaEvent_t e = n->ev[evi++];
    JX_CUDA(cudaEventRecord(e, n->cstream));
    JX_CUDA(cudaStreamWaitEvent(st, e, 0));
  } else {
    adam_range(n, 0, n->nparams, st);
  }
  step_inc_kernel<<<1, 1, 0, st>>>(n->step);
  JX_LAUNCH_CHECK("adam_flat_kernel");
  if (n->timing) {
    JX_CUDA(cudaEventRecord(n->tev[3], st));
    n->tev_recorded = true;
  }
  return JX_OK;
}

// A grid barrier that waits for one arrival more than the grid has: every
// block's bounded wait runs out after limit_ns, records JX_DEVERR_TIMEOUT and
// returns; status[0] = 1 if the block saw the timeout.
__global__ void fs_barrier_selftest_kernel(unsigned* cnt, unsigned* err, unsigned long long limit_ns, int* status) {
  __shared__ int ok;
  const bool passed = fs_grid_sync(cnt, 0, err, &ok, limit_ns, 1u);
  if (threadIdx.x == 0 && !passed) atomicOr(status, 1);
}

bool fused_eligible(const jx_mlp* n) {
  if (!n->fused || n->comm || n->timing || n->prec != JX_PREC_EXACT || n->L > FS_MAXL || n->B > (1 << 24)) return false;
  for (long long x : n->w)
    if (x > (1 << 24)) return false;
  return true;
}

int run_fused_step(jx_mlp* n, const float* x, const float* labels, float* loss_out, cudaStream_t st) {
  if (!n->bar) {
    JX_CUDA(cudaMalloc(&n->bar, 2 * sizeof(unsigned)));
    JX_CUDA(cudaMemset(n->bar, 0, 2 * sizeof(unsigned)));
    JX_CUDA(cudaMalloc(&n->row_loss, sizeof(float) * n->B));
  }
  if (!n->fused_grid) {
    int per_sm = 0;
    JX_CUDA(cudaFuncSetAttribute(mlp_fused_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(FsSmem)));
    JX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mlp_fused_step_kernel, FS_THREADS,
                                                          sizeof(FsSmem)));
    JX_REQUIRE(per_sm >= 1, "jx_mlp_train_step: fused step does not fit on an SM");
    // two CTAs per SM: enough for the largest phase, few arrivals per barrier
    n->fused_grid = jx::num_sms() * (per_sm < 2 ? per_sm : 2);
  }
  FusedStep a;
  a.L = n->L;
  a.B = (int)n->B;
  for (int l = 0; l <= n->L; ++l) a.w[l] = (int)n->w[l];
  for (int l = 0; l < n->L; ++l) {
    a.act[l] = n->act[l];
    a.woff[l] = n->woff[l];
    a.boff[l] = n->boff[l];
    a.h[l + 1] = n->h[l + 1];
    a.pre[l + 1] = n->pre[l + 1];
  }
  a.h[0] = nullptr;
  a.pre[0] = nullptr;
  a.x = x;
  a.labels = labels;
  a.params = n->params;
  a.grads = n->grads;
  a.m = n->m;
  a.v = n->v;
  a.dzA = n->dz;
  a.dzB = n->dh;
  a.row_loss = n->row_loss;
  a.loss = n->loss;
  a.loss_out = loss_out;
  a.step = n->step;
  a.tab = n->tab;
  a.lr = n->lr;
  a.b1 = n->b1;
  a.b2 = n->b2;
  a.eps = n->eps;
  a.omb1 = 1.0f - n->b1;
  a.omb2 = 1.0f - n->b2;
  a.count = (float)(n->global_B * n->w[n->L]);
  a.nparams = n->nparams;
  a.bar = n->bar;
  a.slot = (int)(n->fused_launches & 1);
  a.err = jx::device_error_word();
  void* args[] = {&a};
  JX_CUDA(cudaLaunchCooperativeKernel((const void*)mlp_fused_step_kernel, dim3(n->fused_grid), dim3(FS_THREADS), args,
                                      sizeof(FsSmem), st));
  ++n->fused_launches;
  return JX_OK;
}

}  // namespace

extern "C" {

int jx_mlp_create(const int64_t* widths, int n_layers, const int* acts, int64_t batch, int precision, jx_mlp** out) {
  JX_TRACE("jx_mlp_create");
  JX_REQUIRE(out && widths, "jx_mlp_create: NULL argument");
  *out = nullptr;
  JX_REQUIRE(n_layers >= 1 && n_layers <= 64, "jx_mlp_create: 1..64 layers");
  JX_REQUIRE(batch >= 1, "jx_mlp_create: batch must be positive");
  JX_REQUIRE(precision == JX_PREC_3XTF32 || precision == JX_PREC_EXACT, "jx_mlp_create: unknown precision");
  for (int l = 0; l <= n_layers; ++l) JX_REQUIRE(widths[l] >= 1 && widths[l] < (1LL << 31), "jx_mlp_create: bad width");
  for (int l = 0; l + 1 < n_layers; ++l)
    JX_REQUIRE(acts && acts[l] >= 0 && acts[l] <= 2, "jx_mlp_create: hidden activation must be 0, 1 or 2");
  jx_mlp* n = new (std::nothrow) jx_mlp();
  if (!n) return jx::fail(JX_ENOMEM, "jx_mlp_create: out of host memory");
  n->L = n_layers;
  n->B = batch;
  n->global_B = batch;
  n->prec = precision;
  for (int l = 0; l <= n_layers; ++l) n->w.push_back(widths[l]);
  for (int l = 0; l < n_layers; ++l) n->act.push_back(l + 1 < n_layers ? acts[l] : 0);
  long long off = 0, maxw = 0;
  for (int l = 1; l <= n_layers; ++l) {
    n->woff.push_back(off);
    off += n->w[l - 1] * n->w[l];
    n->boff.push_back(off);
    off += n->w[l];
    off = (off + 3) & ~3LL;  // keep every W/b 16-byte aligned
  }
  for (long long x : n->w) maxw = x > maxw ? x : maxw;
  n->nparams = off;
  auto alloc = [&](float** p, long long count) -> bool {
    return cudaMalloc(p, sizeof(float) * (size_t)(count > 0 ? count : 1)) == cudaSuccess;
  };
  bool ok = alloc(&n->params, off) && alloc(&n->grads, off) && alloc(&n->m, off) && alloc(&n->v, off) &&
            alloc(&n->dz, batch * maxw) && alloc(&n->dh, batch * maxw) && alloc(&n->labels, batch) &&
            alloc(&n->loss, 1);
  n->h.assign(n_layers + 1, nullptr);
  n->pre.assign(n_layers + 1, nullptr);
  for (int l = 0; ok && l <= n_layers; ++l) ok = alloc(&n->h[l], batch * n->w[l]);
  for (int l = 1; ok && l < n_layers; ++l) ok = alloc(&n->pre[l], batch * n->w[l]);
  ok = ok && cudaMalloc(&n->step, sizeof(int)) == cudaSuccess &&
       cudaMalloc(&n->tab, sizeof(float2) * ADAM_TABLE_STEPS) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    free_all(n);
    delete n;
    return jx::fail(JX_ENOMEM, "jx_mlp_create: device allocation failed");
  }
  cudaMemset(n->params, 0, sizeof(float) * off);
  cudaMemset(n->grads, 0, sizeof(float) * off);
  cudaMemset(n->m, 0, sizeof(float) * off);
  cudaMemset(n->v, 0, sizeof(float) * off);
  const int one = 1;
  cudaMemcpy(n->step, &one, sizeof(int), cudaMemcpyHostToDevice);
  int rc = fill_adam_table(n);
  if (rc) {
    free_all(n);
    delete n;
    return rc;
  }
  *out = n;
  return JX_OK;
}

int jx_mlp_param_count(const jx_mlp* n, int64_t* count) {
  JX_TRACE("jx_mlp_param_count");
  JX_REQUIRE(n && count, "jx_mlp_param_count: NULL argument");
  *count = n->nparams;
  return JX_OK;
}

int jx_mlp_param_offsets(const jx_mlp* n, int64_t* w_off, int64_t* b_off) {
  JX_TRACE("jx_mlp_param_offsets");
  JX_REQUIRE(n && w_off && b_off, "jx_mlp_param_offsets: NULL argument");
  for (int l = 0; l < n->L; ++l) {
    w_off[l] = n->woff[l];
    b_off[l] = n->boff[l];
  }
  return JX_OK;
}

int jx_mlp_set_params(jx_mlp* n, const float* host, int64_t count) {
  JX_TRACE("jx_mlp_set_params");
  JX_REQUIRE(n && host, "jx_mlp_set_params: NULL argument");
  JX_REQUIRE(count == n->nparams, "jx_mlp_set_params: expected %lld floats, got %lld", (long long)n->nparams,
             (long long)count);
  JX_CUDA(cudaMemcpy(n->params, host, sizeof(float) * count, cudaMemcpyHostToDevice));
  return JX_OK;
}

int jx_mlp_get_params(const jx_mlp* n, float* host, int64_t count) {
  JX_TRACE("jx_mlp_get_params");
  JX_REQUIRE(n && host, "jx_mlp_get_params: NULL argument");
  JX_REQUIRE(count == n->nparams, "jx_mlp_get_params: expected %lld floats", (long long)n->nparams);
  JX_CUDA(cudaDeviceSynchronize());
  JX_CUDA(cudaMemcpy(host, n->params, sizeof(float) * count, cudaMemcpyDeviceToHost));
  return JX_OK;
}

int jx_mlp_set_adam(jx_mlp* n, float lr, float beta1, float beta2, float eps) {
  JX_TRACE("jx_mlp_set_adam");
  JX_REQUIRE(n, "jx_mlp_set_adam: NULL");
  n->lr = lr;
  n->b1 = beta1;
  n->b2 = beta2;
  n->eps = eps;
  // a fresh optimiser state: m = v = None, step 0 (src/optim.rs:116-124 adam_init)
  JX_CUDA(cudaMemset(n->m, 0, sizeof(float) * n->nparams));
  JX_CUDA(cudaMemset(n->v, 0, sizeof(float) * n->nparams));
  const int one = 1;
  JX_CUDA(cudaMemcpy(n->step, &one, sizeof(int), cudaMemcpyHostToDevice));
  n->steps = 0;
  if (n->gexec) {  // the captured graph bakes the Adam scalars in
    cudaGraphExecDestroy(n->gexec);
    n->gexec = nullptr;
  }
  return fill_adam_table(n);
}

int jx_mlp_attach_comm(jx_mlp* n, void* comm, int world, int64_t global_batch) {
  JX_TRACE("jx_mlp_attach_comm");
  JX_REQUIRE(n && comm, "jx_mlp_attach_comm: NULL argument");
  JX_REQUIRE(world >= 1 && global_batch == n->B * world, "jx_mlp_attach_comm: global batch must be batch * world");
  int rank = 0, nranks = 0;
  if (int rc = jx::nccl_rank(comm, &rank, &nranks)) return rc;
  JX_REQUIRE(nranks == world, "jx_mlp_attach_comm: the communicator has %d ranks, world is %d", nranks, world);
  n->comm = comm;
  n->dp_rank = rank;
  n->dp_world = world;
  n->global_B = global_batch;
  if (!n->cstream) JX_CUDA(cudaStreamCreateWithFlags(&n->cstream, cudaStreamNonBlocking));
  if (n->ev.empty()) {
    // hand-offs per step: two per layer above the first, up to dw1_chunks
    // (or two) for the first, one at the end
    n->ev.resize(2 * n->L + 8);
    for (auto& e : n->ev) JX_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  if (n->gexec) {
    cudaGraphExecDestroy(n->gexec);
    n->gexec = nullptr;
  }
  return JX_OK;
}

int jx_mlp_train_step(jx_mlp* n, const float* x, const float* labels, float* loss_out, jx_stream_t stream) {
  JX_TRACE("jx_mlp_train_step");
  JX_REQUIRE(n && x && labels, "jx_mlp_train_step: NULL argument");
  JX_REQUIRE(n->steps < ADAM_TABLE_STEPS, "jx_mlp_train_step: more than %lld steps", ADAM_TABLE_STEPS);
  cudaStream_t st = jx::as_stream(stream);
  if (fused_eligible(n)) {
    if (int rc = run_fused_step(n, x, labels, loss_out, st)) return rc;
    ++n->steps;
    return JX_OK;
  }
  JX_CUDA(cudaMemcpyAsync(n->h[0], x, sizeof(float) * n->B * n->w[0], cudaMemcpyDeviceToDevice, st));
  JX_CUDA(cudaMemcpyAsync(n->labels, labels, sizeof(float) * n->B, cudaMemcpyDeviceToDevice, st));
  int rc;
  if (n->comm || n->timing) {
    rc = run_step(n, st);  // collectives and phase-timing events stay outside graphs
  } else {
    if (!n->gexec) {
      // capture on a private stream, then replay on the caller's stream
      cudaStream_t cap;
      JX_CUDA(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
      rc = e == cudaSuccess ? run_step(n, cap) : jx::check_cuda(e, "cudaStreamBeginCapture");
      cudaError_t e2 = cudaStreamEndCapture(cap, &g);
      if (!rc && e2 != cudaSuccess) rc = jx::check_cuda(e2, "cudaStreamEndCapture");
      if (!rc) {
        e = cudaGraphInstantiate(&n->gexec, g, 0);
        if (e != cudaSuccess) rc = jx::check_cuda(e, "cudaGraphInstantiate");
      }
      if (g) cudaGraphDestroy(g);
      cudaStreamDestroy(cap);
      if (rc) {
        n->gexec = nullptr;
        return rc;
      }
    }
    JX_CUDA(cudaGraphLaunch(n->gexec, st));
    rc = JX_OK;
  }
  if (rc) return rc;
  if (loss_out) JX_CUDA(cudaMemcpyAsync(loss_out, n->loss, sizeof(float), cudaMemcpyDeviceToDevice, st));
  ++n->steps;
  return JX_OK;
}

int jx_selftest_barrier_timeout(int timeout_ms, int* timed_out) {
  JX_TRACE("jx_selftest_barrier_timeout");
  JX_REQUIRE(timed_out && timeout_ms >= 1 && timeout_ms <= 5000, "jx_selftest_barrier_timeout: 1..5000 ms");
  void* buf = nullptr;
  JX_CUDA(cudaMalloc(&buf, 64));
  JX_CUDA(cudaMemset(buf, 0, 64));
  unsigned* cnt = static_cast<unsigned*>(buf);
  int* status = reinterpret_cast<int*>(static_cast<char*>(buf) + 32);
  unsigned* err = jx::device_error_word();
  unsigned long long limit = (unsigned long long)timeout_ms * 1000000ull;
  void* args[] = {&cnt, &err, &limit, &status};
  cudaError_t e = cudaLaunchCooperativeKernel((const void*)fs_barrier_selftest_kernel, dim3(2), dim3(64), args, 0,
                                              nullptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  int h = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&h, status, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(buf);
  if (e != cudaSuccess) return jx::check_cuda(e, "barrier self-test");
  *timed_out = h;
  return JX_OK;
}

int jx_mlp_set_dp_sharded(jx_mlp* n, int enable) {
  JX_TRACE("jx_mlp_set_dp_sharded");
  JX_REQUIRE(n, "jx_mlp_set_dp_sharded: NULL");
  JX_REQUIRE(n->steps == 0, "jx_mlp_set_dp_sharded: set before the first step (Adam moments live with their shard)");
  n->dp_sharded = enable != 0;
  return JX_OK;
}

int jx_mlp_set_timing(jx_mlp* n, int enable) {
  JX_TRACE("jx_mlp_set_timing");
  JX_REQUIRE(n, "jx_mlp_set_timing: NULL");
  if (enable)
    for (cudaEvent_t& e : n->tev)
      if (!e) JX_CUDA(cudaEventCreate(&e));
  n->timing = enable != 0;
  n->tev_recorded = false;
  return JX_OK;
}

int jx_mlp_step_times(jx_mlp* n, float* ms) {
  JX_TRACE("jx_mlp_step_times");
  JX_REQUIRE(n && ms, "jx_mlp_step_times: NULL argument");
  JX_REQUIRE(n->timing && n->tev_recorded, "jx_mlp_step_times: no timed step yet (call jx_mlp_set_timing first)");
  JX_CUDA(cudaEventSynchronize(n->tev[3]));
  for (int i = 0; i < 3; ++i) JX_CUDA(cudaEventElapsedTime(&ms[i], n->tev[i], n->tev[i + 1]));
  return JX_OK;
}

int jx_mlp_set_fused(jx_mlp* n, int enable) {
  JX_TRACE("jx_mlp_set_fused");
  JX_REQUIRE(n, "jx_mlp_set_fused: NULL");
  n->fused = enable != 0;
  return JX_OK;
}

int jx_mlp_destroy(jx_mlp* n) {
  JX_TRACE("jx_mlp_destroy");
  if (!n) return JX_OK;
  cudaDeviceSynchronize();
  free_all(n);
  delete n;
  return JX_OK;
}

}  // extern "C"
