// host_pipeline.cu -- operations on host buffers, with the transfers pipelined
// against the math.
//
// The reference keeps every Buffer on one device and reads results back with
// a blocking copy (src/buffer.rs:581-590, 711-749), so a host-to-host
// operation is upload, compute, download, one after another.  These entry
// points take host pointers and overlap the three: a copy-in stream uploads
// block i+1 while the compute stream works on block i and a copy-out stream
// downloads block i-1, so the host link's two directions and the GPU all run
// at once.  Ring buffers of NBUF device blocks and events keep each block's
// buffer alive until its download finishes.  The caller's stream waits for
// the last download, so synchronising (or timing) the caller's stream covers
// the whole operation.  Host memory should be pinned (cudaHostAlloc or
// cudaHostRegister); pageable memory still works but its copies serialise.
#include <algorithm>
#include <mutex>

#include "jx_common.cuh"

namespace jx {
int gemm_presplit(const float* Ah, const float* Al, const float* Bh, const float* Bl, float* C, int M, int N, int Kp,
                  long long ldc, long long strideC, int batch, cudaStream_t st);
int gemm_split_operand(const float* src, float* hi, float* lo, int rows, int K, int Kp, long long ld, long long sb,
                       int batch, bool transposed, cudaStream_t st);
long long gemm_kpad(long long K);
}  // namespace jx

namespace {

constexpr int NBUF = 3;

struct Streams {
  cudaStream_t in = nullptr, comp = nullptr, out = nullptr;
};
Streams g_streams[64];
std::mutex g_streams_mu;

int streams(Streams** s) {
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_streams_mu);
  Streams& t = g_streams[dev & 63];
  if (!t.in) {
    JX_CUDA(cudaStreamCreateWithFlags(&t.in, cudaStreamNonBlocking));
    JX_CUDA(cudaStreamCreateWithFlags(&t.comp, cudaStreamNonBlocking));
    JX_CUDA(cudaStreamCreateWithFlags(&t.out, cudaStreamNonBlocking));
  }
  *s = &t;
  return JX_OK;
}

// Events for one pipelined call: per ring slot "input landed", "math done",
// "output read back", plus one for operands shared by every block.
struct Events {
  cudaEvent_t landed[NBUF] = {}, done[NBUF] = {}, drained[NBUF] = {}, shared = nullptr, start = nullptr;
  ~Events() {
    for (int i = 0; i < NBUF; ++i) {
      if (landed[i]) cudaEventDestroy(landed[i]);
      if (done[i]) cudaEventDestroy(done[i]);
      if (drained[i]) cudaEventDestroy(drained[i]);
    }
    if (shared) cudaEventDestroy(shared);
    if (start) cudaEventDestroy(start);
  }
  int create() {
    for (int i = 0; i < NBUF; ++i) {
      JX_CUDA(cudaEventCreateWithFlags(&landed[i], cudaEventDisableTiming));
      JX_CUDA(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
      JX_CUDA(cudaEventCreateWithFlags(&drained[i], cudaEventDisableTiming));
    }
    JX_CUDA(cudaEventCreateWithFlags(&shared, cudaEventDisableTiming));
    JX_CUDA(cudaEventCreateWithFlags(&start, cudaEventDisableTiming));
    return JX_OK;
  }
};

// Streams nblk blocks through NBUF device slots: up(i, slot, stream) issues
// block i's uploads, math(i, slot, stream) its computation, down(i, slot,
// stream) its downloads.  Slot reuse waits for the block NBUF earlier: its
// math before the next upload, its download before the next math.  `ready`
// (may be null) gates the first math (operands shared by every block).
template <class Up, class Math, class Down>
int pipeline(long long nblk, Streams* s, Events& ev, cudaStream_t caller, cudaEvent_t ready, Up up, Math math,
             Down down) {
  int rc = JX_OK;
  JX_CUDA(cudaEventRecord(ev.start, caller));
  for (cudaStream_t x : {s->in, s->comp, s->out}) JX_CUDA(cudaStreamWaitEvent(x, ev.start, 0));
  if (ready) JX_CUDA(cudaStreamWaitEvent(s->comp, ready, 0));
  for (long long i = 0; i < nblk && !rc; ++i) {
    const int b = (int)(i % NBUF);
    if (i >= NBUF) JX_CUDA(cudaStreamWaitEvent(s->in, ev.done[b], 0));
    if ((rc = up(i, b, s->in))) break;
    JX_CUDA(cudaEventRecord(ev.landed[b], s->in));
    JX_CUDA(cudaStreamWaitEvent(s->comp, ev.landed[b], 0));
    if (i >= NBUF) JX_CUDA(cudaStreamWaitEvent(s->comp, ev.drained[b], 0));
    if ((rc = math(i, b, s->comp))) break;
    JX_CUDA(cudaEventRecord(ev.done[b], s->comp));
    JX_CUDA(cudaStreamWaitEvent(s->out, ev.done[b], 0));
    if ((rc = down(i, b, s->out))) break;
    JX_CUDA(cudaEventRecord(ev.drained[b], s->out));
  }
  // the caller's stream waits for all three
  for (cudaStream_t x : {s->in, s->comp, s->out}) {
    JX_CUDA(cudaEventRecord(ev.shared, x));
    JX_CUDA(cudaStreamWaitEvent(caller, ev.shared, 0));
  }
  return rc;
}

int copy_up(void* dst, const void* src, size_t bytes, cudaStream_t st) {
  JX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st));
  return JX_OK;
}
int copy_down(void* dst, const void* src, size_t bytes, cudaStream_t st) {
  JX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st));
  return JX_OK;
}

}  // namespace

extern "C" {

int jx_gemm_f32_host(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                     int64_t ldb, int64_t ldc, int64_t block_rows, jx_stream_t stream) {
  JX_TRACE("jx_gemm_f32_host");
  JX_REQUIRE(M >= 0 && N >= 0 && K >= 0, "matmul: negative dimension");
  if (M == 0 || N == 0) return JX_OK;
  JX_REQUIRE(K > 0, "gemm host: K must be positive");
  JX_REQUIRE(A && B && C, "matmul: NULL operand");
  JX_REQUIRE(lda >= K && ldb >= N && ldc >= N, "matmul: leading dimension too small");
  JX_REQUIRE(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), "matmul: dimension too large");
  cudaStream_t caller = jx::as_stream(stream);
  Streams* s = nullptr;
  int rc = streams(&s);
  if (rc) return rc;
  Events ev;
  if ((rc = ev.create())) return rc;
  const long long Kp = jx::gemm_kpad(K);
  long long rb = block_rows > 0 ? block_rows : std::max<long long>(128, (M / 8 + 127) / 128 * 128);
  rb = std::min<long long>(rb, M);
  const long long nblk = (M + rb - 1) / rb;
  // device: B [K][N] and its hi/lo split, NBUF blocks of A [rb][K] (+ hi/lo) and C [rb][N]
  const size_t fB = (size_t)K * N, fBs = 2 * (size_t)N * Kp, fA = (size_t)rb * K, fAs = 2 * (size_t)rb * Kp,
               fC = (size_t)rb * N;
  void* ws = nullptr;
  // the caller's stream orders the workspace's life: taken here, returned after the last download
  if ((rc = jx::scratch_get(sizeof(float) * (fB + fBs + NBUF * (fA + fAs + fC)), &ws, caller))) return rc;
  JX_CUDA(cudaEventRecord(ev.start, caller));
  float* dB = reinterpret_cast<float*>(ws);
  float* dBh = dB + fB;
  float* dBl = dBh + (size_t)N * Kp;
  float* slot0 = dBh + fBs;
  auto dA = [&](int i) { return slot0 + (size_t)i * (fA + fAs + fC); };
  auto dAh = [&](int i) { return dA(i) + fA; };
  auto dAl = [&](int i) { return dAh(i) + (size_t)rb * Kp; };
  auto dC = [&](int i) { return dA(i) + fA + fAs; };
  for (cudaStream_t x : {s->in, s->comp, s->out}) JX_CUDA(cudaStreamWaitEvent(x, ev.start, 0));
  // B once: upload, split (K-major, transposed)
  JX_CUDA(cudaMemcpy2DAsync(dB, N * sizeof(float), B, ldb * sizeof(float), N * sizeof(float), K,
                            cudaMemcpyHostToDevice, s->in));
  JX_CUDA(cudaEventRecord(ev.shared, s->in));
  JX_CUDA(cudaStreamWaitEvent(s->comp, ev.shared, 0));
  rc = jx::gemm_split_operand(dB, dBh, dBl, (int)N, (int)K, (int)Kp, N, 0, 1, true, s->comp);
  for (long long i = 0; i < nblk && !rc; ++i) {
    const int b = (int)(i % NBUF);
    const long long r0 = i * rb, rows = std::min(rb, M - r0);
    // upload A block i once the math of block i-NBUF has released the slot
    if (i >= NBUF) JX_CUDA(cudaStreamWaitEvent(s->in, ev.done[b], 0));
    JX_CUDA(cudaMemcpy2DAsync(dA(b), K * sizeof(float), A + r0 * lda, lda * sizeof(float), K * sizeof(float), rows,
                              cudaMemcpyHostToDevice, s->in));
    JX_CUDA(cudaEventRecord(ev.landed[b], s->in));
    // math once the block landed and block i-NBUF's result has been read back
    JX_CUDA(cudaStreamWaitEvent(s->comp, ev.landed[b], 0));
    if (i >= NBUF) JX_CUDA(cudaStreamWaitEvent(s->comp, ev.drained[b], 0));
    rc = jx::gemm_split_operand(dA(b), dAh(b), dAl(b), (int)rows, (int)K, (int)Kp, K, 0, 1, false, s->comp);
    if (!rc) rc = jx::gemm_presplit(dAh(b), dAl(b), dBh, dBl, dC(b), (int)rows, (int)N, (int)Kp, N, 0, 1, s->comp);
    if (rc) break;
    JX_CUDA(cudaEventRecord(ev.done[b], s->comp));
    // download
    JX_CUDA(cudaStreamWaitEvent(s->out, ev.done[b], 0));
    JX_CUDA(cudaMemcpy2DAsync(C + r0 * ldc, ldc * sizeof(float), dC(b), N * sizeof(float), N * sizeof(float), rows,
                              cudaMemcpyDeviceToHost, s->out));
    JX_CUDA(cudaEventRecord(ev.drained[b], s->out));
  }
  // the caller's stream waits for everything, then returns the workspace
  for (cudaStream_t x : {s->in, s->comp, s->out}) {
    JX_CUDA(cudaEventRecord(ev.shared, x));
    JX_CUDA(cudaStreamWaitEvent(caller, ev.shared, 0));
  }
  const int rc2 = jx::scratch_release(ws, caller);
  return rc ? rc : rc2;
}

int jx_tape_run_host(const jx_tape* tape, const float* const* ins, float* const* outs, int64_t n,
                     int64_t block_elems, jx_stream_t stream) {
  JX_TRACE("jx_tape_run_host");
  JX_REQUIRE(tape && n >= 0, "jx_tape_run_host: bad arguments");
  if (n == 0) return JX_OK;
  int n_in = 0, n_out = 0;
  int rc = jx_tape_info(tape, &n_in, &n_out, nullptr);
  if (rc) return rc;
  for (int i = 0; i < n_in; ++i) JX_REQUIRE(ins && ins[i], "jx_tape_run_host: input %d is NULL", i);
  for (int i = 0; i < n_out; ++i) JX_REQUIRE(outs && outs[i], "jx_tape_run_host: output %d is NULL", i);
  cudaStream_t caller = jx::as_stream(stream);
  Streams* s = nullptr;
  if ((rc = streams(&s))) return rc;
  Events ev;
  if ((rc = ev.create())) return rc;
  long long blk = block_elems > 0 ? block_elems : (8LL << 20);  // 32 MiB per operand by default
  blk = std::min<long long>((blk + 3) / 4 * 4, n);
  const long long nblk = (n + blk - 1) / blk;
  const int nio = n_in + n_out;
  void* ws = nullptr;
  if ((rc = jx::scratch_get(sizeof(float) * (size_t)blk * nio * NBUF, &ws, caller))) return rc;
  auto buf = [&](int slot, int k) { return reinterpret_cast<float*>(ws) + ((size_t)slot * nio + k) * blk; };
  auto count = [&](long long i) { return std::min(blk, (long long)n - i * blk); };
  rc = pipeline(
      nblk, s, ev, caller, nullptr,
      [&](long long i, int b, cudaStream_t st) {
        for (int k = 0; k < n_in; ++k) {
          const int r = copy_up(buf(b, k), ins[k] + i * blk, sizeof(float) * count(i), st);
          if (r) return r;
        }
        return (int)JX_OK;
      },
      [&](long long i, int b, cudaStream_t st) {
        const float* tin[JX_TAPE_MAX_IO];
        float* tout[JX_TAPE_MAX_IO];
        for (int k = 0; k < n_in; ++k) tin[k] = buf(b, k);
        for (int k = 0; k < n_out; ++k) tout[k] = buf(b, n_in + k);
        return jx_tape_run(tape, tin, tout, count(i), st);
      },
      [&](long long i, int b, cudaStream_t st) {
        for (int k = 0; k < n_out; ++k) {
          const int r = copy_down(outs[k] + i * blk, buf(b, n_in + k), sizeof(float) * count(i), st);
          if (r) return r;
        }
        return (int)JX_OK;
      });
  const int rc2 = jx::scratch_release(ws, caller);
  return rc ? rc : rc2;
}

// Batched FFTs over host buffers: blocks of whole transforms (1-D rows of n
// points, or 2-D images of h x w) stream through the device.
int fft_host(const float* in, float* out, long long elems_per_item, long long items, long long block_items,
             bool two_d, long long n_or_h, long long w, int inverse, jx_stream_t stream) {
  cudaStream_t caller = jx::as_stream(stream);
  Streams* s = nullptr;
  int rc = streams(&s);
  if (rc) return rc;
  Events ev;
  if ((rc = ev.create())) return rc;
  const long long per = 2 * elems_per_item;  // floats per item (complex)
  long long blk = block_items > 0 ? block_items : std::max(1LL, (32LL << 20) / (long long)(per * 4));
  blk = std::min(blk, items);
  const long long nblk = (items + blk - 1) / blk;
  void* ws = nullptr;
  if ((rc = jx::scratch_get(sizeof(float) * (size_t)(2 * NBUF * blk * per), &ws, caller))) return rc;
  auto dbuf = [&](int slot, int k) { return reinterpret_cast<float*>(ws) + ((size_t)slot * 2 + k) * blk * per; };
  auto count = [&](long long i) { return std::min(blk, items - i * blk); };
  rc = pipeline(
      nblk, s, ev, caller, nullptr,
      [&](long long i, int b, cudaStream_t st) {
        return copy_up(dbuf(b, 0), in + i * blk * per, sizeof(float) * count(i) * per, st);
      },
      [&](long long i, int b, cudaStream_t st) {
        return two_d ? jx_fft2_c2c_f32(dbuf(b, 0), dbuf(b, 1), n_or_h, w, count(i), inverse, st)
                     : jx_fft_c2c_f32(dbuf(b, 0), dbuf(b, 1), n_or_h, count(i), inverse, st);
      },
      [&](long long i, int b, cudaStream_t st) {
        return copy_down(out + i * blk * per, dbuf(b, 1), sizeof(float) * count(i) * per, st);
      });
  const int rc2 = jx::scratch_release(ws, caller);
  return rc ? rc : rc2;
}

int jx_fft_c2c_f32_host(const float* in, float* out, int64_t n, int64_t batch, int inverse, int64_t block_items,
                        jx_stream_t stream) {
  JX_TRACE("jx_fft_c2c_f32_host");
  JX_REQUIRE(n >= 1 && batch >= 0, "fft: bad size");
  if (batch == 0) return JX_OK;
  JX_REQUIRE(in && out, "fft: NULL pointer");
  return fft_host(in, out, n, batch, block_items, false, n, 0, inverse, stream);
}

int jx_fft2_c2c_f32_host(const float* in, float* out, int64_t h, int64_t w, int64_t batch, int inverse,
                         int64_t block_items, jx_stream_t stream) {
  JX_TRACE("jx_fft2_c2c_f32_host");
  JX_REQUIRE(h >= 1 && w >= 1 && batch >= 0, "fft2: bad size");
  if (batch == 0) return JX_OK;
  JX_REQUIRE(in && out, "fft2: NULL pointer");
  return fft_host(in, out, h * w, batch, block_items, true, h, w, inverse, stream);
}

int jx_gemm_batched_f32_host(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                             int64_t batch, int64_t block_items, jx_stream_t stream) {
  JX_TRACE("jx_gemm_batched_f32_host");
  JX_REQUIRE(M >= 0 && N >= 0 && K >= 0 && batch >= 0, "matmul: negative dimension");
  if (M == 0 || N == 0 || batch == 0) return JX_OK;
  JX_REQUIRE(K > 0, "gemm host: K must be positive");
  JX_REQUIRE(A && B && C, "matmul: NULL operand");
  cudaStream_t caller = jx::as_stream(stream);
  Streams* s = nullptr;
  int rc = streams(&s);
  if (rc) return rc;
  Events ev;
  if ((rc = ev.create())) return rc;
  const long long fa = M * K, fb = K * N, fc = M * N, per = fa + fb + fc;  // floats per batch entry
  long long blk = block_items > 0 ? block_items : std::max(1LL, (96LL << 20) / (per * 4));
  blk = std::min(blk, (long long)batch);
  const long long nblk = (batch + blk - 1) / blk;
  void* ws = nullptr;
  if ((rc = jx::scratch_get(sizeof(float) * (size_t)(NBUF * blk * per), &ws, caller))) return rc;
  auto slot = [&](int b) { return reinterpret_cast<float*>(ws) + (size_t)b * blk * per; };
  auto count = [&](long long i) { return std::min(blk, (long long)batch - i * blk); };
  rc = pipeline(
      nblk, s, ev, caller, nullptr,
      [&](long long i, int b, cudaStream_t st) {
        int r = copy_up(slot(b), A + i * blk * fa, sizeof(float) * count(i) * fa, st);
        if (!r) r = copy_up(slot(b) + blk * fa, B + i * blk * fb, sizeof(float) * count(i) * fb, st);
        return r;
      },
      [&](long long i, int b, cudaStream_t st) {
        float* a = slot(b);
        float* bb = a + blk * fa;
        float* c = bb + blk * fb;
        return jx_gemm_f32(a, bb, c, M, N, K, 0, 0, K, N, N, count(i), fa, fb, fc, JX_PREC_3XTF32, st);
      },
      [&](long long i, int b, cudaStream_t st) {
        return copy_down(C + i * blk * fc, slot(b) + blk * (fa + fb), sizeof(float) * count(i) * fc, st);
      });
  const int rc2 = jx::scratch_release(ws, caller);
  return rc ? rc : rc2;
}

int jx_pool2d_f32_host(const float* x, float* y, int64_t batch, int64_t channels, int64_t input_h, int64_t input_w,
                       int64_t pool_h, int64_t pool_w, int64_t stride_h, int64_t stride_w, int64_t pad_h,
                       int64_t pad_w, int op, int64_t block_items, jx_stream_t stream) {
  JX_TRACE("jx_pool2d_f32_host");
  // geometry checks (and their messages) are jx_pool2d_f32's: run them once on an empty batch
  if (int rc = jx_pool2d_f32(nullptr, nullptr, 0, channels, input_h, input_w, pool_h, pool_w, stride_h, stride_w,
                             pad_h, pad_w, op, stream))
    return rc;
  JX_REQUIRE(batch >= 0, "jx_pool2d_f32_host: negative batch");
  if (batch == 0 || channels == 0) return JX_OK;
  JX_REQUIRE(x && y, "jx_pool2d_f32_host: NULL buffer");
  cudaStream_t caller = jx::as_stream(stream);
  Streams* s = nullptr;
  int rc = streams(&s);
  if (rc) return rc;
  Events ev;
  if ((rc = ev.create())) return rc;
  const long long oh = (input_h + 2 * pad_h - pool_h) / stride_h + 1, ow = (input_w + 2 * pad_w - pool_w) / stride_w + 1;
  const long long fi = channels * input_h * input_w, fo = channels * oh * ow;  // floats per image
  long long blk = block_items > 0 ? block_items : std::max(1LL, (32LL << 20) / (fi * 4));
  blk = std::min(blk, (long long)batch);
  const long long nblk = (batch + blk - 1) / blk;
  void* ws = nullptr;
  if ((rc = jx::scratch_get(sizeof(float) * (size_t)(NBUF * blk * (fi + fo)), &ws, caller))) return rc;
  auto slot = [&](int b) { return reinterpret_cast<float*>(ws) + (size_t)b * blk * (fi + fo); };
  auto count = [&](long long i) { return std::min(blk, (long long)batch - i * blk); };
  rc = pipeline(
      nblk, s, ev, caller, nullptr,
      [&](long long i, int b, cudaStream_t st) {
        return copy_up(slot(b), x + i * blk * fi, sizeof(float) * count(i) * fi, st);
      },
      [&](long long i, int b, cudaStream_t st) {
        return jx_pool2d_f32(slot(b), slot(b) + blk * fi, count(i), channels, input_h, input_w, pool_h, pool_w,
                             stride_h, stride_w, pad_h, pad_w, op, st);
      },
      [&](long long i, int b, cudaStream_t st) {
        return copy_down(y + i * blk * fo, slot(b) + blk * fi, sizeof(float) * count(i) * fo, st);
      });
  const int rc2 = jx::scratch_release(ws, caller);
  return rc ? rc : rc2;
}

}  // extern "C"
