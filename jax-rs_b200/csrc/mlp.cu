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

namespace jx {
int col_sum(const float* dy, float* db, long long rows, int cols, cudaStream_t st);
int nccl_allreduce(void* comm, float* buf, long long count, cudaStream_t st);
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
  cudaGraphExec_t gexec = nullptr;
  long long steps = 0;
};

namespace {

void free_all(jx_mlp* n) {
  if (n->gexec) cudaGraphExecDestroy(n->gexec);
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

// One training step on stream st (forward, backward, optional all-reduce, Adam).
int run_step(jx_mlp* n, cudaStream_t st) {
  int rc;
  const long long B = n->B;
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
  for (int l = n->L; l >= 1; --l) {
    const long long K = n->w[l - 1], N = n->w[l];
    float* gW = n->grads + n->woff[l - 1];
    // dW_l = h_{l-1}^T dz (transpose_matmul's dB = A^T dC, src/trace/transpose_rules.rs:537-567)
    if ((rc = jx_gemm_f32(n->h[l - 1], n->dz, gW, K, N, B, 1, 0, K, N, N, 1, 0, 0, 0, n->prec, st))) return rc;
    if ((rc = jx::col_sum(n->dz, n->grads + n->boff[l - 1], B, (int)N, st))) return rc;
    if (n->comm) {
      JX_CUDA(cudaEventRecord(n->ev[l - 1], st));
      JX_CUDA(cudaStreamWaitEvent(n->cstream, n->ev[l - 1], 0));
      if ((rc = jx::nccl_allreduce(n->comm, gW, K * N + N, n->cstream))) return rc;
    }
    if (l > 1) {
      // dh = dz W_l^T (transpose_matmul's dA = dC B^T), then dz = dh * act'(pre)
      if ((rc = jx_gemm_f32(n->dz, n->params + n->woff[l - 1], n->dh, B, K, N, 0, 1, N, N, K, 1, 0, 0, 0, n->prec,
                            st)))
        return rc;
      if ((rc = jx_act_bwd_f32(n->dh, n->pre[l - 1], n->dz, nullptr, B, K, n->act[l - 2], st))) return rc;
    }
  }
  if (n->comm) {
    JX_CUDA(cudaEventRecord(n->ev[n->L], n->cstream));
    JX_CUDA(cudaStreamWaitEvent(st, n->ev[n->L], 0));
  }
  adam_flat_kernel<<<grid_elems(n->nparams), 256, 0, st>>>(n->params, n->grads, n->m, n->v, n->nparams, n->step,
                                                           n->tab, n->lr, n->b1, n->b2, n->eps, 1.0f - n->b1,
                                                           1.0f - n->b2);
  step_inc_kernel<<<1, 1, 0, st>>>(n->step);
  JX_LAUNCH_CHECK("adam_flat_kernel");
  return JX_OK;
}

}  // namespace

extern "C" {

int jx_mlp_create(const int64_t* widths, int n_layers, const int* acts, int64_t batch, int precision, jx_mlp** out) {
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
  JX_REQUIRE(n && count, "jx_mlp_param_count: NULL argument");
  *count = n->nparams;
  return JX_OK;
}

int jx_mlp_param_offsets(const jx_mlp* n, int64_t* w_off, int64_t* b_off) {
  JX_REQUIRE(n && w_off && b_off, "jx_mlp_param_offsets: NULL argument");
  for (int l = 0; l < n->L; ++l) {
    w_off[l] = n->woff[l];
    b_off[l] = n->boff[l];
  }
  return JX_OK;
}

int jx_mlp_set_params(jx_mlp* n, const float* host, int64_t count) {
  JX_REQUIRE(n && host, "jx_mlp_set_params: NULL argument");
  JX_REQUIRE(count == n->nparams, "jx_mlp_set_params: expected %lld floats, got %lld", (long long)n->nparams,
             (long long)count);
  JX_CUDA(cudaMemcpy(n->params, host, sizeof(float) * count, cudaMemcpyHostToDevice));
  return JX_OK;
}

int jx_mlp_get_params(const jx_mlp* n, float* host, int64_t count) {
  JX_REQUIRE(n && host, "jx_mlp_get_params: NULL argument");
  JX_REQUIRE(count == n->nparams, "jx_mlp_get_params: expected %lld floats", (long long)n->nparams);
  JX_CUDA(cudaDeviceSynchronize());
  JX_CUDA(cudaMemcpy(host, n->params, sizeof(float) * count, cudaMemcpyDeviceToHost));
  return JX_OK;
}

int jx_mlp_set_adam(jx_mlp* n, float lr, float beta1, float beta2, float eps) {
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
  JX_REQUIRE(n && comm, "jx_mlp_attach_comm: NULL argument");
  JX_REQUIRE(world >= 1 && global_batch == n->B * world, "jx_mlp_attach_comm: global batch must be batch * world");
  n->comm = comm;
  n->global_B = global_batch;
  if (!n->cstream) JX_CUDA(cudaStreamCreateWithFlags(&n->cstream, cudaStreamNonBlocking));
  if (n->ev.empty()) {
    n->ev.resize(n->L + 1);
    for (auto& e : n->ev) JX_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  if (n->gexec) {
    cudaGraphExecDestroy(n->gexec);
    n->gexec = nullptr;
  }
  return JX_OK;
}

int jx_mlp_train_step(jx_mlp* n, const float* x, const float* labels, float* loss_out, jx_stream_t stream) {
  JX_REQUIRE(n && x && labels, "jx_mlp_train_step: NULL argument");
  JX_REQUIRE(n->steps < ADAM_TABLE_STEPS, "jx_mlp_train_step: more than %lld steps", ADAM_TABLE_STEPS);
  cudaStream_t st = jx::as_stream(stream);
  JX_CUDA(cudaMemcpyAsync(n->h[0], x, sizeof(float) * n->B * n->w[0], cudaMemcpyDeviceToDevice, st));
  JX_CUDA(cudaMemcpyAsync(n->labels, labels, sizeof(float) * n->B, cudaMemcpyDeviceToDevice, st));
  int rc;
  if (n->comm) {
    rc = run_step(n, st);  // collectives stay outside graphs
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

int jx_mlp_destroy(jx_mlp* n) {
  if (!n) return JX_OK;
  cudaDeviceSynchronize();
  free_all(n);
  delete n;
  return JX_OK;
}

}  // extern "C"
