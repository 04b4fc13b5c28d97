// Scatter-add and histogram into bins.
//
//   for i in 0..n-1:  b = idx[i];  if 0 <= b < nbins:  acc[b] += v[i];  hist[b] += 1
//
// Either output may be absent. Indices outside [0, nbins) are skipped, never
// written. `accumulate` = 0 overwrites the outputs with the sums of this call,
// 1 adds them to what is there.
//
// Layout of the work on B200: a thread-block cluster of c CTAs (c <= 8, one
// portable cluster) privatises the whole bin range in distributed shared
// memory — CTA r owns bins [r*per, (r+1)*per) of every table — so each element
// costs one `red.shared::cluster` into the owning CTA instead of a global atomic
// that would serialise in L2. The input is streamed once with 128-bit loads.
// Each cluster then writes its private bins to scratch, and a second kernel
// sums the clusters' partials per bin in a fixed order, so the float sums do
// not depend on which cluster finished first and the integer counts are exact.
//
// Bins larger than the cluster's shared memory fall back to global atomics
// (L2-resident tables), which needs no scratch.

#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "../mtl_internal.hpp"

namespace cg = cooperative_groups;

namespace mtl {

// Shared-memory bytes of bins per CTA that still leave room for two CTAs per SM.
static constexpr uint32_t kBinsSmemPerCta = 96 * 1024;
static constexpr int kThreads = 512;
static constexpr int kCtasPerSm = 2;

struct ScatterShape {
  bool cluster;     // false: global-atomic fallback
  int c;            // cluster size
  int shift;        // per = 1 << shift bins per CTA
  int tables;       // 1 or 2
  int nclusters;    // grid = nclusters * c
  uint32_t smem;    // dynamic shared bytes per CTA
};

static int ceil_log2(uint64_t x) {
  int s = 0;
  while ((uint64_t(1) << s) < x) ++s;
  return s;
}

static ScatterShape scatter_shape(int nbins, int tables, int sm_count) {
  ScatterShape sh{};
  sh.tables = tables;
  int lg = ceil_log2((uint64_t)std::max(nbins, 1));
  for (int c = 1; c <= 8; c *= 2) {
    int shift = std::max(lg - ceil_log2((uint64_t)c), 0);
    uint64_t smem = (uint64_t)tables * (uint64_t(1) << shift) * 4;
    if (smem <= kBinsSmemPerCta) {
      sh.cluster = true;
      sh.c = c;
      sh.shift = shift;
      sh.smem = (uint32_t)smem;
      sh.nclusters = std::max(1, sm_count * kCtasPerSm / c);
      return sh;
    }
  }
  sh.cluster = false;
  return sh;
}

__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void red_cluster_f32(uint32_t addr, float v) {
  asm volatile("red.shared::cluster.add.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void red_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("red.shared::cluster.add.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int4 ld_nc_v4(const int* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ float4 ld_nc_v4f(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

template <bool ACC, bool HIST>
__device__ __forceinline__ void scatter_one(int b, float v, uint32_t nbins, int shift,
                                            uint32_t acc_base, uint32_t hist_base) {
  if ((uint32_t)b >= nbins) return;
  const uint32_t owner = (uint32_t)b >> shift;
  const uint32_t local = (uint32_t)b & ((1u << shift) - 1);
  if (ACC) red_cluster_f32(mapa_shared(acc_base + local * 4, owner), v);
  if (HIST) red_cluster_u32(mapa_shared(hist_base + local * 4, owner), 1u);
}

// One cluster privatises all bins; partials go to ws[cluster][table][nbins].
template <bool ACC, bool HIST>
__global__ void __launch_bounds__(kThreads) scatter_cluster_kernel(
    const float* __restrict__ v, const int* __restrict__ idx, int64_t n, uint32_t nbins, int shift,
    float* __restrict__ ws_acc, uint32_t* __restrict__ ws_hist) {
  extern __shared__ __align__(16) uint32_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t per = 1u << shift;
  const uint32_t tables = (ACC ? 1 : 0) + (HIST ? 1 : 0);
  for (uint32_t i = threadIdx.x; i < tables * per; i += blockDim.x) smem[i] = 0;
  // Every CTA's bins are zero before any CTA of the cluster adds into them.
  cluster.sync();

  const uint32_t base = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t acc_base = base;
  const uint32_t hist_base = base + (ACC ? per * 4 : 0);
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(idx) | (ACC ? reinterpret_cast<uintptr_t>(v) : 0)) & 15) == 0;
  int64_t done = 0;
  if (vec) {
    const int64_t n4 = n / 4;
    int64_t q = tid;
    // Two groups of four per iteration keep 64 bytes per thread in flight.
    for (; q + nthreads < n4; q += 2 * nthreads) {
      int4 b0 = ld_nc_v4(idx + 4 * q);
      int4 b1 = ld_nc_v4(idx + 4 * (q + nthreads));
      float4 v0 = make_float4(0, 0, 0, 0), v1 = v0;
      if (ACC) {
        v0 = ld_nc_v4f(v + 4 * q);
        v1 = ld_nc_v4f(v + 4 * (q + nthreads));
      }
      scatter_one<ACC, HIST>(b0.x, v0.x, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.y, v0.y, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.z, v0.z, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.w, v0.w, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b1.x, v1.x, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b1.y, v1.y, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b1.z, v1.z, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b1.w, v1.w, nbins, shift, acc_base, hist_base);
    }
    for (; q < n4; q += nthreads) {
      int4 b0 = ld_nc_v4(idx + 4 * q);
      float4 v0 = make_float4(0, 0, 0, 0);
      if (ACC) v0 = ld_nc_v4f(v + 4 * q);
      scatter_one<ACC, HIST>(b0.x, v0.x, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.y, v0.y, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.z, v0.z, nbins, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.w, v0.w, nbins, shift, acc_base, hist_base);
    }
    done = n4 * 4;
  }
  for (int64_t i = done + tid; i < n; i += nthreads)
    scatter_one<ACC, HIST>(idx[i], ACC ? v[i] : 0.f, nbins, shift, acc_base, hist_base);

  // All adds into this CTA's bins have landed before it reads them.
  cluster.sync();
  const uint32_t rank = cluster.block_rank();
  const int64_t cl = blockIdx.x / cluster.num_blocks();
  const uint32_t lo = rank * per;
  for (uint32_t i = threadIdx.x; i < per && lo + i < nbins; i += blockDim.x) {
    if (ACC) ws_acc[cl * nbins + lo + i] = __uint_as_float(smem[i]);
    if (HIST) ws_hist[cl * nbins + lo + i] = smem[(ACC ? per : 0) + i];
  }
}

// out[b] = (accumulate ? out[b] : 0) + sum over clusters of the partials, in
// cluster order.
__global__ void scatter_reduce_kernel(const float* __restrict__ ws_acc,
                                      const uint32_t* __restrict__ ws_hist, int nclusters,
                                      uint32_t nbins, float* __restrict__ acc,
                                      uint32_t* __restrict__ hist, int accumulate) {
  const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nbins) return;
  if (acc) {
    float s = accumulate ? acc[b] : 0.f;
    for (int c = 0; c < nclusters; ++c) s += ws_acc[(int64_t)c * nbins + b];
    acc[b] = s;
  }
  if (hist) {
    uint32_t s = accumulate ? hist[b] : 0u;
    for (int c = 0; c < nclusters; ++c) s += ws_hist[(int64_t)c * nbins + b];
    hist[b] = s;
  }
}

// Fallback for bin ranges no cluster can hold: atomics on the L2-resident table.
__global__ void scatter_global_kernel(const float* __restrict__ v, const int* __restrict__ idx,
                                      int64_t n, uint32_t nbins, float* __restrict__ acc,
                                      uint32_t* __restrict__ hist) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int b = idx[i];
    if ((uint32_t)b >= nbins) continue;
    if (acc) atomicAdd(acc + b, v[i]);
    if (hist) atomicAdd(hist + b, 1u);
  }
}

// Arguments: acc (b), hist (b), values (b), idx (B), nbins (i), accumulate (i).
static void scatter_unpack(const LaunchArgs& la, float*& acc, uint32_t*& hist, const float*& v,
                           const int*& idx, int& nbins, int& accumulate, int64_t& n) {
  acc = reinterpret_cast<float*>(la.a[0].kind == MTL_ARG_PTR ? la.a[0].ptr : 0);
  hist = reinterpret_cast<uint32_t*>(la.a[1].kind == MTL_ARG_PTR ? la.a[1].ptr : 0);
  v = reinterpret_cast<const float*>(la.a[2].kind == MTL_ARG_PTR ? la.a[2].ptr : 0);
  idx = reinterpret_cast<const int*>(la.a[3].ptr);
  nbins = la.a[4].i32;
  accumulate = la.a[5].i32;
  n = la.nd[0];
}

mtl_status scatter_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.ndim != 1) return fail(MTL_ERR_ARGUMENT, "scatter_add: ndrange must be one-dimensional (the element count)");
  const int64_t n = la.nd[0];
  const int nbins = la.a[4].i32;
  if (nbins <= 0) return fail(MTL_ERR_ARGUMENT, "scatter_add: nbins must be positive");
  bool has_acc = la.a[0].kind != MTL_ARG_NULL, has_hist = la.a[1].kind != MTL_ARG_NULL;
  if (!has_acc && !has_hist) return fail(MTL_ERR_ARGUMENT, "scatter_add: needs an accumulator, a histogram or both");
  if (has_acc && la.a[2].kind == MTL_ARG_NULL) return fail(MTL_ERR_ARGUMENT, "scatter_add: an accumulator needs values");
  auto need = [&](int i, uint64_t b, const char* what) -> mtl_status {
    if (bytes[i] && bytes[i] < b)
      return fail(MTL_ERR_ARGUMENT, "scatter_add: %s has %llu bytes, the launch touches %llu", what,
                  (unsigned long long)bytes[i], (unsigned long long)b);
    return MTL_OK;
  };
  if (has_acc)
    if (mtl_status s = need(0, (uint64_t)nbins * 4, "the accumulator")) return s;
  if (has_hist)
    if (mtl_status s = need(1, (uint64_t)nbins * 4, "the histogram")) return s;
  if (has_acc)
    if (mtl_status s = need(2, (uint64_t)n * 4, "values")) return s;
  return need(3, (uint64_t)n * 4, "indices");
}

uint64_t scatter_workspace(const LaunchArgs& la) {
  int tables = (la.a[0].kind != MTL_ARG_NULL) + (la.a[1].kind != MTL_ARG_NULL);
  ScatterShape sh = scatter_shape(la.a[4].i32, tables, la.sm_count);
  if (!sh.cluster) return 0;
  return (uint64_t)sh.nclusters * tables * (uint64_t)la.a[4].i32 * 4;
}

template <bool ACC, bool HIST>
static cudaError_t launch_cluster(const ScatterShape& sh, cudaStream_t s, const float* v,
                                  const int* idx, int64_t n, uint32_t nbins, float* ws_acc,
                                  uint32_t* ws_hist) {
  auto k = scatter_cluster_kernel<ACC, HIST>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(sh.nclusters * sh.c));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sh.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = sh.c;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, v, idx, n, nbins, sh.shift, ws_acc, ws_hist);
}

// Shared by the graph path and the direct and no-scratch entry points.
mtl_status scatter_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream) {
  float* acc;
  uint32_t* hist;
  const float* v;
  const int* idx;
  int nbins, accumulate;
  int64_t n;
  scatter_unpack(la, acc, hist, v, idx, nbins, accumulate, n);
  cudaStream_t s = (cudaStream_t)stream;
  const int tables = (acc != nullptr) + (hist != nullptr);
  ScatterShape sh = scatter_shape(nbins, tables, la.sm_count);
  cudaError_t e = cudaSuccess;
  if (sh.cluster) {
    uint64_t need = (uint64_t)sh.nclusters * tables * (uint64_t)nbins * 4;
    if (!ws || ws_bytes < need)
      return fail(MTL_ERR_ARGUMENT, "scatter_add: needs %llu bytes of scratch, got %llu",
                  (unsigned long long)need, (unsigned long long)ws_bytes);
    float* ws_acc = acc ? reinterpret_cast<float*>(ws) : nullptr;
    uint32_t* ws_hist = hist ? reinterpret_cast<uint32_t*>(ws) + (acc ? (uint64_t)sh.nclusters * nbins : 0) : nullptr;
    int ncl = sh.nclusters;
    if (n > 0) {
      if (acc && hist)
        e = launch_cluster<true, true>(sh, s, v, idx, n, nbins, ws_acc, ws_hist);
      else if (acc)
        e = launch_cluster<true, false>(sh, s, v, idx, n, nbins, ws_acc, ws_hist);
      else
        e = launch_cluster<false, true>(sh, s, v, idx, n, nbins, ws_acc, ws_hist);
    } else {
      ncl = 0;
    }
    if (e == cudaSuccess) {
      unsigned blocks = (unsigned)((nbins + 255) / 256);
      scatter_reduce_kernel<<<blocks, 256, 0, s>>>(ws_acc, ws_hist, ncl, nbins, acc, hist, accumulate);
      e = cudaGetLastError();
    }
  } else {
    if (!accumulate) {
      if (acc) e = cudaMemsetAsync(acc, 0, (size_t)nbins * 4, s);
      if (e == cudaSuccess && hist) e = cudaMemsetAsync(hist, 0, (size_t)nbins * 4, s);
    }
    if (e == cudaSuccess && n > 0) {
      int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)la.sm_count * 8);
      scatter_global_kernel<<<(unsigned)blocks, 256, 0, s>>>(v, idx, n, nbins, acc, hist);
      e = cudaGetLastError();
    }
  }
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "scatter_add: %s", cudaGetErrorString(e));
  return MTL_OK;
}

}  // namespace mtl
