// dp.cu -- NCCL plumbing for data-parallel training (no reference counterpart:
// jax-rs has one global device, src/backend/webgpu.rs:6).
//
// Communicators are created non-blocking and every wait is bounded: init and
// collectives poll ncclCommGetAsyncError, and when the host watchdog's limit
// passes the communicator is aborted and the call returns JX_ETIMEOUT, so a
// rank that never joins ends the others' calls with an error, not a hang.
//
// NCCL is resolved at first use with dlopen/dlsym, preferring a libnccl.so.2
// the process has already loaded (e.g. the one torch ships), so loading this
// library never pins a different NCCL than the rest of the process uses.
#include <dlfcn.h>
#include <stdlib.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "jx_common.cuh"

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommFinalize)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*ReduceScatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
  bool ok;
};
NcclApi g_nccl;
std::once_flag g_nccl_once;

const NcclApi* nccl() {
  std::call_once(g_nccl_once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    bool ok = true;
    auto sym = [&](const char* name) {
      void* f = dlsym(h, name);
      ok = ok && f != nullptr;
      return f;
    };
    g_nccl.GetUniqueId = reinterpret_cast<decltype(g_nccl.GetUniqueId)>(sym("ncclGetUniqueId"));
    g_nccl.CommInitRankConfig = reinterpret_cast<decltype(g_nccl.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
    g_nccl.CommGetAsyncError = reinterpret_cast<decltype(g_nccl.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
    g_nccl.CommAbort = reinterpret_cast<decltype(g_nccl.CommAbort)>(sym("ncclCommAbort"));
    g_nccl.CommFinalize = reinterpret_cast<decltype(g_nccl.CommFinalize)>(sym("ncclCommFinalize"));
    g_nccl.CommDestroy = reinterpret_cast<decltype(g_nccl.CommDestroy)>(sym("ncclCommDestroy"));
    g_nccl.AllReduce = reinterpret_cast<decltype(g_nccl.AllReduce)>(sym("ncclAllReduce"));
    g_nccl.ReduceScatter = reinterpret_cast<decltype(g_nccl.ReduceScatter)>(sym("ncclReduceScatter"));
    g_nccl.AllGather = reinterpret_cast<decltype(g_nccl.AllGather)>(sym("ncclAllGather"));
    g_nccl.GetErrorString = reinterpret_cast<decltype(g_nccl.GetErrorString)>(sym("ncclGetErrorString"));
    g_nccl.ok = ok;
  });
  return g_nccl.ok ? &g_nccl : nullptr;
}

#define JX_NCCL_API(api)                                                              \
  const NcclApi* api = nccl();                                                        \
  if (!api) return jx::fail(JX_ENCCL, "NCCL (libnccl.so.2) could not be loaded");

int nccl_fail(ncclResult_t r, const char* what) {
  const NcclApi* api = nccl();
  return jx::fail(JX_ENCCL, "%s: %s", what, api ? api->GetErrorString(r) : "NCCL unavailable");
}

struct Comm {
  ncclComm_t comm;
  int timeout_ms;
  int rank, nranks;
};

// Polls the communicator until its pending operation leaves ncclInProgress.
int wait_comm(Comm* c, int timeout_ms, const char* what) {
  JX_NCCL_API(api);
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st;
    ncclResult_t r = api->CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) return nccl_fail(r, what);
    if (st == ncclSuccess) return JX_OK;
    if (st != ncclInProgress) return nccl_fail(st, what);
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > timeout_ms) {
      api->CommAbort(c->comm);
      c->comm = nullptr;
      return jx::fail(JX_ETIMEOUT, "%s: no progress within %d ms; communicator aborted", what, timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

}  // namespace

namespace jx {
// Used by the trainer: enqueue an in-place sum all-reduce on `st`.
int nccl_allreduce(void* comm, float* buf, long long count, cudaStream_t st) {
  JX_NCCL_API(api);
  Comm* c = reinterpret_cast<Comm*>(comm);
  JX_REQUIRE(c && c->comm, "allreduce: communicator is NULL or was aborted");
  ncclResult_t r = api->AllReduce(buf, buf, (size_t)count, ncclFloat, ncclSum, c->comm, st);
  if (r == ncclInProgress) return wait_comm(c, c->timeout_ms, "ncclAllReduce");
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
  return JX_OK;
}

// In place: rank r receives the sum of every rank's [r*shard, (r+1)*shard)
// of buf at that same offset.
int nccl_reduce_scatter(void* comm, float* buf, long long shard, cudaStream_t st) {
  JX_NCCL_API(api);
  Comm* c = reinterpret_cast<Comm*>(comm);
  JX_REQUIRE(c && c->comm, "reduce-scatter: communicator is NULL or was aborted");
  ncclResult_t r = api->ReduceScatter(buf, buf + (long long)c->rank * shard, (size_t)shard, ncclFloat, ncclSum,
                                      c->comm, st);
  if (r == ncclInProgress) return wait_comm(c, c->timeout_ms, "ncclReduceScatter");
  if (r != ncclSuccess) return nccl_fail(r, "ncclReduceScatter");
  return JX_OK;
}

// In place: every rank's [r*shard, (r+1)*shard) of buf goes to all ranks.
int nccl_all_gather(void* comm, float* buf, long long shard, cudaStream_t st) {
  JX_NCCL_API(api);
  Comm* c = reinterpret_cast<Comm*>(comm);
  JX_REQUIRE(c && c->comm, "all-gather: communicator is NULL or was aborted");
  ncclResult_t r = api->AllGather(buf + (long long)c->rank * shard, buf, (size_t)shard, ncclFloat, c->comm, st);
  if (r == ncclInProgress) return wait_comm(c, c->timeout_ms, "ncclAllGather");
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
  return JX_OK;
}

int nccl_rank(void* comm, int* rank, int* nranks) {
  Comm* c = reinterpret_cast<Comm*>(comm);
  JX_REQUIRE(c, "communicator is NULL");
  *rank = c->rank;
  *nranks = c->nranks;
  return JX_OK;
}
}  // namespace jx

extern "C" {

int jx_nccl_unique_id_size(void) { return (int)sizeof(ncclUniqueId); }

int jx_nccl_get_unique_id(void* id_out) {
  JX_TRACE("jx_nccl_get_unique_id");
  JX_REQUIRE(id_out, "jx_nccl_get_unique_id: NULL");
  JX_NCCL_API(api);
  ncclUniqueId id;
  ncclResult_t r = api->GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(id_out, &id, sizeof(id));
  return JX_OK;
}

int jx_nccl_init(const void* id, int nranks, int rank, int timeout_ms, void** comm_out) {
  JX_TRACE("jx_nccl_init");
  JX_REQUIRE(id && comm_out, "jx_nccl_init: NULL argument");
  JX_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "jx_nccl_init: rank %d of %d", rank, nranks);
  if (timeout_ms <= 0) {  // the process default: JAXRS_NCCL_TIMEOUT_MS, else 120 s
    const char* e = getenv("JAXRS_NCCL_TIMEOUT_MS");
    timeout_ms = e && *e ? atoi(e) : 0;
    if (timeout_ms <= 0) timeout_ms = 120000;
  }
  *comm_out = nullptr;
  JX_NCCL_API(api);
  Comm* c = new Comm();
  c->timeout_ms = timeout_ms;
  c->rank = rank;
  c->nranks = nranks;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = api->CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  int rc = wait_comm(c, timeout_ms, "ncclCommInitRankConfig");
  if (rc) {
    if (c->comm) api->CommAbort(c->comm);
    delete c;
    return rc;
  }
  *comm_out = c;
  return JX_OK;
}

int jx_nccl_allreduce_sum_f32(void* comm, float* buf, int64_t count, jx_stream_t stream) {
  JX_TRACE("jx_nccl_allreduce_sum_f32");
  JX_REQUIRE(count >= 0, "allreduce: negative count");
  if (count == 0) return JX_OK;
  JX_REQUIRE(buf, "allreduce: NULL buffer");
  return jx::nccl_allreduce(comm, buf, count, jx::as_stream(stream));
}

int jx_nccl_wait(void* comm, jx_stream_t stream, int timeout_ms) {
  JX_TRACE("jx_nccl_wait");
  JX_NCCL_API(api);
  Comm* c = reinterpret_cast<Comm*>(comm);
  JX_REQUIRE(c && c->comm, "jx_nccl_wait: communicator is NULL or was aborted");
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaStreamQuery(jx::as_stream(stream));
    if (q == cudaSuccess) return JX_OK;
    if (q != cudaErrorNotReady) return jx::check_cuda(q, "jx_nccl_wait: cudaStreamQuery");
    ncclResult_t st;
    api->CommGetAsyncError(c->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) return nccl_fail(st, "jx_nccl_wait");
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > timeout_ms) {
      api->CommAbort(c->comm);
      c->comm = nullptr;
      return jx::fail(JX_ETIMEOUT, "jx_nccl_wait: stream not done within %d ms; communicator aborted", timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

int jx_nccl_destroy(void* comm) {
  JX_TRACE("jx_nccl_destroy");
  Comm* c = reinterpret_cast<Comm*>(comm);
  if (!c) return JX_OK;
  JX_NCCL_API(api);
  int rc = JX_OK;
  if (c->comm) {
    ncclResult_t r = api->CommFinalize(c->comm);
    if (r == ncclInProgress) rc = wait_comm(c, c->timeout_ms, "ncclCommFinalize");
    else if (r != ncclSuccess) rc = nccl_fail(r, "ncclCommFinalize");
    if (c->comm) api->CommDestroy(c->comm);
  }
  delete c;
  return rc;
}

}  // extern "C"
