// runtime.cu -- context, error reporting, storage and streams of the C ABI.
//
// Replaces the reference's WebGPU context (src/backend/webgpu.rs:6-75: a global
// OnceLock device + queue) with one CUDA context per device, and its Buffer
// storage (src/buffer.rs:12-122, 581-749) with stream-ordered allocations.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "jx_common.cuh"

namespace jx {

int gemm_prepare();
int noalloc_take_error(unsigned int* flags);
static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return JX_OK;
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return e == cudaErrorMemoryAllocation ? JX_ENOMEM : JX_ECUDA;
}

cudaStream_t as_stream(jx_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

static const int kMaxDev = 64;
static std::mutex g_mu;
static std::atomic<int> g_sms[kMaxDev];  // SM count per device, 0 until first asked
static unsigned int* g_err_word[kMaxDev];

static int cur_dev() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int num_sms() {
  int d = cur_dev();
  if (d < 0 || d >= kMaxDev) return 148;
  int n = g_sms[d].load(std::memory_order_relaxed);
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    if (n <= 0) n = 148;
    g_sms[d].store(n, std::memory_order_relaxed);  // every thread that races here stores the same value
  }
  return n;
}

// Allocation-failure injection (jx_selftest_fail_alloc): the next N device
// allocations of jx_malloc and of the library's scratch fail with JX_ENOMEM.
static std::atomic<int> g_fail_allocs{0};

static bool injected_alloc_failure() {
  int n = g_fail_allocs.load();
  while (n > 0)
    if (g_fail_allocs.compare_exchange_weak(n, n - 1)) return true;
  return false;
}

int scratch_get(size_t bytes, void** out, cudaStream_t st) {
  *out = nullptr;
  if (injected_alloc_failure()) return fail(JX_ENOMEM, "scratch allocation of %zu bytes failed (injected)", bytes);
  cudaError_t e = cudaMallocAsync(out, bytes ? bytes : 16, st);
  if (e != cudaSuccess) {
    *out = nullptr;
    return check_cuda(e, "scratch cudaMallocAsync");
  }
  return JX_OK;
}

int scratch_release(void* p, cudaStream_t st) {
  if (!p) return JX_OK;
  cudaError_t e = cudaFreeAsync(p, st);
  return e == cudaSuccess ? JX_OK : check_cuda(e, "scratch cudaFreeAsync");
}

unsigned int* device_error_word() {
  int d = cur_dev();
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_word[d]) {
    if (cudaMalloc(&g_err_word[d], sizeof(unsigned int)) != cudaSuccess) return nullptr;
    cudaMemset(g_err_word[d], 0, sizeof(unsigned int));
    cudaDeviceSynchronize();
  }
  return g_err_word[d];
}

// JAXRS_CHECK=1 (read at each jx_malloc): every buffer gets GUARD_BYTES of
// canary bytes after its end, checked when it is freed and by
// jx_check_guards, so a kernel that writes past the end of a buffer is caught
// (the guard is real allocated memory, so the stray write itself is harmless).
static constexpr size_t GUARD_BYTES = 256;
static constexpr unsigned char CANARY = 0xA5;
static std::mutex g_guard_mu;
static std::unordered_map<void*, size_t> g_guarded;  // device pointer -> the caller's byte count

static bool check_mode() {
  const char* e = getenv("JAXRS_CHECK");
  return e && *e && strcmp(e, "0") != 0;
}

// Reads the canary tail of a guarded buffer; *intact = false if any byte changed.
static int guard_intact(void* p, size_t nbytes, cudaStream_t st, bool* intact) {
  unsigned char tail[GUARD_BYTES];
  JX_CUDA(cudaMemcpyAsync(tail, static_cast<char*>(p) + nbytes, GUARD_BYTES, cudaMemcpyDeviceToHost, st));
  JX_CUDA(cudaStreamSynchronize(st));
  *intact = true;
  for (size_t i = 0; i < GUARD_BYTES; ++i)
    if (tail[i] != CANARY) *intact = false;
  return JX_OK;
}

}  // namespace jx

using namespace jx;

extern "C" {

const char* jx_last_error(void) { return g_last_error.c_str(); }

int jx_version(void) { return 1; }

int jx_device_count(int* count) {
  JX_TRACE("jx_device_count");
  JX_REQUIRE(count, "jx_device_count: count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *count = 0;
    return check_cuda(e, "cudaGetDeviceCount");
  }
  *count = n;
  return JX_OK;
}

int jx_init(int device) {
  JX_TRACE("jx_init");
  int n = 0;
  JX_CUDA(cudaGetDeviceCount(&n));
  if (device < 0) {  // the process default: JAXRS_DEVICE, else device 0
    const char* e = getenv("JAXRS_DEVICE");
    device = e && *e ? atoi(e) : 0;
  }
  JX_REQUIRE(device >= 0 && device < n, "jx_init: device %d out of range (%d devices)", device, n);
  JX_CUDA(cudaSetDevice(device));
  cudaDeviceProp p;
  JX_CUDA(cudaGetDeviceProperties(&p, device));
  if (p.major != 10)
    return fail(JX_EUNSUPPORTED, "jx_init: device %d is sm_%d%d; this library is built for sm_100a only",
                device, p.major, p.minor);
  JX_CUDA(cudaFree(0));  // create the primary context
  {
    // Keep stream-ordered scratch cached in the pool between calls.
    cudaMemPool_t pool;
    JX_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
    uint64_t thr = UINT64_MAX;
    JX_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
  }
  (void)num_sms();
  if (!device_error_word()) return fail(JX_ENOMEM, "jx_init: cannot allocate the device error word");
  if (int rc = gemm_prepare()) return rc;
  return JX_OK;
}

int jx_set_device(int device) {
  JX_TRACE("jx_set_device");
  JX_CUDA(cudaSetDevice(device));
  return JX_OK;
}

int jx_get_device(int* device) {
  JX_TRACE("jx_get_device");
  JX_REQUIRE(device, "jx_get_device: NULL");
  JX_CUDA(cudaGetDevice(device));
  return JX_OK;
}

int jx_device_status(unsigned int* flags) {
  JX_TRACE("jx_device_status");
  JX_REQUIRE(flags, "jx_device_status: NULL");
  unsigned int* w = device_error_word();
  if (!w) return fail(JX_ENOMEM, "device error word unavailable");
  JX_CUDA(cudaDeviceSynchronize());
  unsigned int v = 0;
  JX_CUDA(cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost));
  JX_CUDA(cudaMemset(w, 0, sizeof(v)));
  // jx_gemm_f32_noalloc's launches flag into their own fixed word
  unsigned int na = 0;
  if (int rc = noalloc_take_error(&na)) return rc;
  *flags = v | na;
  return JX_OK;
}

int jx_malloc(void** ptr, size_t nbytes, int zero, jx_stream_t stream) {
  JX_TRACE("jx_malloc");
  JX_REQUIRE(ptr, "jx_malloc: ptr is NULL");
  *ptr = nullptr;
  if (nbytes == 0) nbytes = 16;
  if (injected_alloc_failure()) return fail(JX_ENOMEM, "jx_malloc: allocation of %zu bytes failed (injected)", nbytes);
  const bool guarded = check_mode();
  cudaError_t e = cudaMallocAsync(ptr, nbytes + (guarded ? GUARD_BYTES : 0), as_stream(stream));
  if (e != cudaSuccess) {
    *ptr = nullptr;
    return check_cuda(e, "jx_malloc: cudaMallocAsync");
  }
  if (zero) JX_CUDA(cudaMemsetAsync(*ptr, 0, nbytes, as_stream(stream)));
  if (guarded) {
    JX_CUDA(cudaMemsetAsync(static_cast<char*>(*ptr) + nbytes, CANARY, GUARD_BYTES, as_stream(stream)));
    std::lock_guard<std::mutex> lk(g_guard_mu);
    g_guarded[*ptr] = nbytes;
  }
  return JX_OK;
}

int jx_free(void* ptr, jx_stream_t stream) {
  JX_TRACE("jx_free");
  if (!ptr) return JX_OK;
  size_t nbytes = 0;
  bool guarded = false;
  {
    std::lock_guard<std::mutex> lk(g_guard_mu);
    auto it = g_guarded.find(ptr);
    if (it != g_guarded.end()) {
      guarded = true;
      nbytes = it->second;
      g_guarded.erase(it);
    }
  }
  bool intact = true;
  if (guarded)
    if (int rc = guard_intact(ptr, nbytes, as_stream(stream), &intact)) return rc;
  JX_CUDA(cudaFreeAsync(ptr, as_stream(stream)));
  if (!intact)
    return fail(JX_EDEVICE, "jx_free: bytes written past the end of a %zu-byte buffer (JAXRS_CHECK canary)",
                nbytes);
  return JX_OK;
}

int jx_check_guards(int* corrupted) {
  JX_TRACE("jx_check_guards");
  JX_REQUIRE(corrupted, "jx_check_guards: NULL");
  *corrupted = 0;
  JX_CUDA(cudaDeviceSynchronize());
  std::lock_guard<std::mutex> lk(g_guard_mu);
  for (const auto& kv : g_guarded) {
    bool intact = true;
    if (int rc = guard_intact(kv.first, kv.second, nullptr, &intact)) return rc;
    if (!intact) ++*corrupted;
  }
  return JX_OK;
}

int jx_selftest_fail_alloc(int count) {
  JX_TRACE("jx_selftest_fail_alloc");
  JX_REQUIRE(count >= 0, "jx_selftest_fail_alloc: negative count");
  g_fail_allocs.store(count);
  return JX_OK;
}

int jx_memcpy_h2d(void* dst, const void* src, size_t nbytes, jx_stream_t stream) {
  JX_TRACE("jx_memcpy_h2d");
  if (nbytes == 0) return JX_OK;
  JX_REQUIRE(dst && src, "jx_memcpy_h2d: NULL pointer");
  JX_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice, as_stream(stream)));
  return JX_OK;
}

int jx_memcpy_d2h(void* dst, const void* src, size_t nbytes, jx_stream_t stream) {
  JX_TRACE("jx_memcpy_d2h");
  if (nbytes == 0) return JX_OK;
  JX_REQUIRE(dst && src, "jx_memcpy_d2h: NULL pointer");
  JX_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost, as_stream(stream)));
  JX_CUDA(cudaStreamSynchronize(as_stream(stream)));
  return JX_OK;
}

int jx_memcpy_d2d(void* dst, const void* src, size_t nbytes, jx_stream_t stream) {
  JX_TRACE("jx_memcpy_d2d");
  if (nbytes == 0) return JX_OK;
  JX_REQUIRE(dst && src, "jx_memcpy_d2d: NULL pointer");
  JX_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToDevice, as_stream(stream)));
  return JX_OK;
}

int jx_stream_create(jx_stream_t* stream) {
  JX_TRACE("jx_stream_create");
  JX_REQUIRE(stream, "jx_stream_create: NULL");
  cudaStream_t s;
  JX_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = reinterpret_cast<jx_stream_t>(s);
  return JX_OK;
}

int jx_stream_destroy(jx_stream_t stream) {
  JX_TRACE("jx_stream_destroy");
  if (stream) JX_CUDA(cudaStreamDestroy(as_stream(stream)));
  return JX_OK;
}

int jx_stream_sync(jx_stream_t stream) {
  JX_TRACE("jx_stream_sync");
  JX_CUDA(cudaStreamSynchronize(as_stream(stream)));
  return JX_OK;
}

int jx_host_register(void* ptr, size_t nbytes) {
  JX_TRACE("jx_host_register");
  JX_REQUIRE(ptr && nbytes, "jx_host_register: NULL or empty range");
  JX_CUDA(cudaHostRegister(ptr, nbytes, cudaHostRegisterDefault));
  return JX_OK;
}

int jx_host_unregister(void* ptr) {
  JX_TRACE("jx_host_unregister");
  JX_REQUIRE(ptr, "jx_host_unregister: NULL");
  JX_CUDA(cudaHostUnregister(ptr));
  return JX_OK;
}

}  // extern "C"
