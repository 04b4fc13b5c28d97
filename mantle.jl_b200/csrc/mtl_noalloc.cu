// Scatter-add / histogram for callers that cannot allocate GPU memory.
//
// Some callers of this library must not call cudaMalloc (or any allocating
// routine) on the path where they scatter: code running inside another
// runtime's memory budget, a pool-managed process whose allocator owns every
// byte, or a real-time loop where an allocation could stall or fail at an
// arbitrary frame. The regular entry point asks the caller for scratch; this
// one takes it from a fixed array compiled into the library instead.
//
// The array is a file-scope __device__ array, so every GPU that loads the
// library holds it until the process exits, and every call on a device uses
// the same bytes. Two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) therefore race on the scratch: order them
// on one stream, or with events. Each call writes every scratch byte it later
// reads before reading it, so nothing has to be cleared between calls and the
// leftovers of the previous call never reach a result.
//
// Host code must not pass the array's name to a kernel: on the host that name
// is only a stand-in for the device symbol, not a device address. The first
// call on each device looks the real address up with cudaGetSymbolAddress,
// with that device current, and keeps it together with the CUDA context it
// belongs to; later calls in the same context reuse it. A call that finds a
// different current context (after cudaDeviceReset, or under a context the
// caller made current itself) looks the address up again, because the module
// may then sit at another address. Make the first call on a device, and the
// first after a reset, outside any stream capture (the lookup may load the
// module).

#include <cuda_runtime.h>

#include <mutex>

#include "mtl_internal.hpp"

namespace mtl {
uint64_t scatter_workspace_min(const LaunchArgs& la);
}

using namespace mtl;

// The scratch: MTL_NOALLOC_SCRATCH_BYTES on every device that loads the library.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MTL_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};
void* g_ctx[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};

// The driver's current context (CUcontext), through the runtime's entry-point
// lookup so that nothing links libcuda directly; null where unavailable.
void* current_context() {
  using Fn = int (*)(void**);
  static Fn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<Fn>(p);
    return static_cast<Fn>(nullptr);
  }();
  void* ctx = nullptr;
  if (fn && fn(&ctx) != 0) ctx = nullptr;
  return ctx;
}

// With the device current: the device address of the array, looked up once
// per device and context.
mtl_status scratch_for(int dev, void** ptr, int* sms) {
  if (dev < 0 || dev >= kMaxDevices) return fail(MTL_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  void* ctx = current_context();
  if (!g_scratch[dev] || ctx != g_ctx[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(MTL_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev, cudaGetErrorString(e));
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "device %d: %s", dev, cudaGetErrorString(e));
    g_scratch[dev] = p;
    g_sms[dev] = n;
    // looked up under the context current now (cudaGetSymbolAddress makes the
    // primary context current when none was)
    g_ctx[dev] = current_context();
  }
  *ptr = g_scratch[dev];
  *sms = g_sms[dev];
  return MTL_OK;
}

}  // namespace

extern "C" mtl_status mtl_scatter_add_noalloc(float* acc, uint32_t* hist, const float* values,
                                              const int32_t* idx, int64_t n, int32_t nbins,
                                              int32_t accumulate, void* stream) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "scatter_add_noalloc: %s", cudaGetErrorString(e));
  if (n < 0) return fail(MTL_ERR_ARGUMENT, "scatter_add_noalloc: negative element count");
  if (n > 0 && !idx) return fail(MTL_ERR_ARGUMENT, "scatter_add_noalloc: indices are NULL");
  void* scratch = nullptr;
  int sms = 0;
  if (mtl_status s = scratch_for(dev, &scratch, &sms)) return s;

  LaunchArgs la;
  la.ndim = 1;
  la.nd[0] = n;
  la.sm_count = sms;
  la.device = dev;
  auto ptr_arg = [](const void* p) {
    Arg a;
    a.kind = p ? MTL_ARG_PTR : MTL_ARG_NULL;
    a.ptr = (uint64_t)p;
    return a;
  };
  la.a.push_back(ptr_arg(acc));
  la.a.push_back(ptr_arg(hist));
  la.a.push_back(ptr_arg(values));
  // With n == 0 the indices are never read; any valid address will do.
  la.a.push_back(ptr_arg(idx ? (const void*)idx : scratch));
  Arg nb;
  nb.kind = MTL_ARG_I32;
  nb.i32 = nbins;
  la.a.push_back(nb);
  Arg accu;
  accu.kind = MTL_ARG_I32;
  accu.i32 = accumulate;
  la.a.push_back(accu);
  if (nbins <= 0) return fail(MTL_ERR_ARGUMENT, "scatter_add_noalloc: nbins must be positive");

  // the smallest scratch the scatter can run with (its one-launch form)
  const uint64_t need = scatter_workspace_min(la);
  if (need > MTL_NOALLOC_SCRATCH_BYTES)
    return fail(MTL_ERR_ARGUMENT,
                "scatter_add_noalloc: %d bins need %llu bytes of scratch; this entry point has a fixed "
                "%llu-byte array (use mtl_launch with caller-provided scratch instead)",
                nbins, (unsigned long long)need, (unsigned long long)MTL_NOALLOC_SCRATCH_BYTES);
  static int kernel = kernel_find("scatter_add");
  if (kernel < 0) return fail(MTL_ERR_STATE, "scatter_add kernel missing from the registry");
  return launch_kernel(kernel, la, scratch, MTL_NOALLOC_SCRATCH_BYTES, stream);
}
