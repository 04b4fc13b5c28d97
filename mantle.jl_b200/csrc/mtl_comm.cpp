// NCCL communicators for the final all-gather over NVLink. NCCL is opened with
// dlopen so that the library loads (and everything else works) on a machine
// without it; the first communicator call reports its absence as an error.
//
// Communicators are created non-blocking (ncclConfig_t.blocking = 0) and every
// wait on them is bounded on the host, so a rank that never arrives ends in
// MTL_ERR_TIMEOUT and mtl_comm_abort, never in a hang.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "mtl_internal.hpp"

using namespace mtl;


namespace {
struct Nccl {
  void* h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};
Nccl g_nccl;
std::mutex g_nccl_mu;
// How long a communicator's set-up and each collective may take, in seconds.
std::atomic<double> g_timeout_s{60.0};

mtl_status load_nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.h) return MTL_OK;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return fail(MTL_ERR_NCCL, "NCCL is not available: %s", dlerror());
#define SYM(f, name)                                           \
  *(void**)(&g_nccl.f) = dlsym(h, name);                       \
  if (!g_nccl.f) return fail(MTL_ERR_NCCL, "NCCL lacks %s", name);
  SYM(GetUniqueId, "ncclGetUniqueId");
  SYM(CommInitRankConfig, "ncclCommInitRankConfig");
  SYM(AllGather, "ncclAllGather");
  SYM(CommDestroy, "ncclCommDestroy");
  SYM(CommAbort, "ncclCommAbort");
  SYM(CommGetAsyncError, "ncclCommGetAsyncError");
  SYM(GetErrorString, "ncclGetErrorString");
#undef SYM
  g_nccl.h = h;
  return MTL_OK;
}
}  // namespace

struct mtl_comm {
  ncclComm_t comm = nullptr;
  mtl_device* dev = nullptr;
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  int nranks = 0, rank = 0;
};

// Bounded wait for a non-blocking communicator to leave ncclInProgress. An
// enqueued collective is ready within microseconds, so the first few
// milliseconds spin (yielding the core); only a longer wait (communicator
// setup, a peer that is late) sleeps between polls.
static mtl_status wait_ready(mtl_comm* c, double seconds) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    g_nccl.CommGetAsyncError(c->comm, &st);
    if (st == ncclSuccess) return MTL_OK;
    if (st != ncclInProgress) return fail(MTL_ERR_NCCL, "NCCL: %s", g_nccl.GetErrorString(st));
    double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (dt > seconds) return fail(MTL_ERR_TIMEOUT, "NCCL: communicator not ready after %.1f s", seconds);
    if (dt < 0.005)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

extern "C" {

mtl_status mtl_device_stream(mtl_device* dev, void** stream);

mtl_status mtl_comm_unique_id(void* id) {
  if (!id) return fail(MTL_ERR_ARGUMENT, "mtl_comm_unique_id: NULL argument");
  if (mtl_status s = load_nccl()) return s;
  ncclUniqueId u;
  ncclResult_t r = g_nccl.GetUniqueId(&u);
  if (r != ncclSuccess) return fail(MTL_ERR_NCCL, "ncclGetUniqueId: %s", g_nccl.GetErrorString(r));
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
  memcpy(id, &u, 128);
  return MTL_OK;
}

mtl_status mtl_comm_init(mtl_device* dev, int32_t nranks, int32_t rank, const void* id, mtl_comm** out) {
  if (!dev || !id || !out) return fail(MTL_ERR_ARGUMENT, "mtl_comm_init: NULL argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(MTL_ERR_ARGUMENT, "mtl_comm_init: rank %d of %d", rank, nranks);
  if (mtl_status s = injected("mtl_comm_init")) return s;
  if (mtl_status s = load_nccl()) return s;
  auto* c = new mtl_comm();
  c->dev = dev;
  retain_device(dev);
  c->nranks = nranks;
  c->rank = rank;
  void* st = nullptr;
  mtl_device_stream(dev, &st);
  c->stream = (cudaStream_t)st;
  ncclUniqueId u;
  memcpy(&u, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = g_nccl.CommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    release_device(c->dev);
    delete c;
    return fail(MTL_ERR_NCCL, "ncclCommInitRankConfig: %s", g_nccl.GetErrorString(r));
  }
  if (mtl_status s = wait_ready(c, g_timeout_s.load())) {
    std::string msg = mtl_last_error();
    g_nccl.CommAbort(c->comm);
    release_device(c->dev);
    delete c;
    return fail(s, "%s", msg.c_str());
  }
  *out = c;
  return MTL_OK;
}

mtl_status mtl_comm_release(mtl_comm* c) {
  if (!c) return MTL_OK;
  if (c->comm) g_nccl.CommDestroy(c->comm);
  release_device(c->dev);
  delete c;
  return MTL_OK;
}

mtl_status mtl_comm_abort(mtl_comm* c) {
  if (!c) return MTL_OK;
  if (c->comm) g_nccl.CommAbort(c->comm);
  release_device(c->dev);
  delete c;
  return MTL_OK;
}

mtl_status mtl_allgather(mtl_comm* c, const void* send, void* recv, uint64_t bytes) {
  if (!c || !send || !recv) return fail(MTL_ERR_ARGUMENT, "mtl_allgather: NULL argument");
  if (mtl_status s = injected("mtl_allgather")) return s;
  ncclResult_t r = g_nccl.AllGather(send, recv, bytes, ncclUint8, c->comm, c->stream);
  if (r != ncclSuccess && r != ncclInProgress) return fail(MTL_ERR_NCCL, "ncclAllGather: %s", g_nccl.GetErrorString(r));
  return wait_ready(c, g_timeout_s.load());
}

mtl_status mtl_comm_set_timeout(double seconds) {
  if (!(seconds > 0.0)) return fail(MTL_ERR_ARGUMENT, "mtl_comm_set_timeout: %g s is not positive", seconds);
  g_timeout_s.store(seconds);
  return MTL_OK;
}

}  // extern "C"
