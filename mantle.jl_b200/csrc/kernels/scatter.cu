// Scatter-add and histogram into bins.
//
//   for i in 0..n-1:  b = idx[i];  if 0 <= b < nbins:  acc[b] += v[i];  hist[b] += 1
//
// Either output may be absent. Indices outside [0, nbins) are skipped, never
// written. `accumulate` = 0 overwrites the outputs with the sums of this call,
// 1 adds them to what is there.
//
// Layout of the work on B200 (measured there: shared-memory atomics run at
// 8.5 u32 / 2.5 f32 per clock per SM, remote distributed-shared-memory atomics
// 10-40x slower, L2 atomics ~190 G/s for the whole GPU): a thread-block
// cluster of c co-scheduled CTAs splits the bin range, CTA r keeping bins
// [r*per, (r+1)*per) of every table in its own shared memory. All c CTAs
// stream the cluster's contiguous chunk of the input — one of the c reads comes
// from HBM, the others hit L2 — and each applies only the elements whose bin it
// owns, with local shared-memory atomics. No atomic leaves the SM.
// Each CTA then writes its private bins to scratch, and a second kernel sums the
// clusters' partials per bin in a fixed order, so the float sums do not depend
// on which cluster finished first and the integer counts are exact.
//
// Inputs whose bins pile up (most elements of a warp on one or a few bins) make
// plain shared-memory atomics serialise. The scatter_add_dense family runs the
// same kernel with a warp-aggregated form besides the plain one: each warp
// that finds its first elements piling up sums its lanes' values per bin first
// and issues one atomic per bin (scatter_agg, chosen by piles_up). Measured on
// B200 (2^24 elements, values + histogram): all in one bin 5.6 ms plain, 0.46 ms
// dense; 90 % in 64 of 2^16 bins 0.21 ms plain, 0.22 ms dense (the warps take
// the plain form); uniform over 2^16 bins 77 us plain, 100 us dense.
//
// Bins larger than a cluster's shared memory fall back to global atomics
// (L2-resident tables), which needs no scratch.

#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "../mtl_internal.hpp"

namespace cg = cooperative_groups;

namespace mtl {

// Shared-memory bytes of bins per CTA (one CTA per SM) and threads per CTA.
#ifndef MTL_SCATTER_SMEM_KB
#define MTL_SCATTER_SMEM_KB 128
#endif
#ifndef MTL_SCATTER_THREADS
#define MTL_SCATTER_THREADS 1024
#endif
#ifndef MTL_SCATTER_CTAS_PER_SM
#define MTL_SCATTER_CTAS_PER_SM 1
#endif
static constexpr uint32_t kBinsSmemPerCta = MTL_SCATTER_SMEM_KB * 1024;
static constexpr int kThreads = MTL_SCATTER_THREADS;
static constexpr int kCtasPerSm = MTL_SCATTER_CTAS_PER_SM;

struct ScatterShape {
  bool cluster;     // false: global-atomic fallback
  int c;            // cluster size: CTAs sharing one chunk, each owning 1/c of the bins
  int shift;        // per = 1 << shift bins per CTA
  int tables;       // 1 or 2
  int nclusters;    // grid = nclusters * c, one CTA per SM
  uint32_t smem;    // dynamic shared bytes per CTA
};

static int ceil_log2(uint64_t x) {
  int s = 0;
  while ((uint64_t(1) << s) < x) ++s;
  return s;
}

template <bool ACC, bool HIST, bool DENSE>
__global__ void scatter_cluster_kernel(const float* __restrict__, const int* __restrict__, int64_t,
                                       uint32_t, int, float* __restrict__, uint32_t* __restrict__);

// How many clusters of this shape the device runs at once: a grid larger than
// that would run in a second, mostly idle wave (clusters must fit inside one
// GPC, so the answer is not simply SMs / c). Cached per device and shape.
static int max_active_clusters(int device, int tables, int c, uint32_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, uint32_t>, int> cache;
  auto key = std::make_tuple(device, tables, c, smem);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
  const void* k = tables == 2 ? (const void*)scatter_cluster_kernel<true, true, false>
                              : (const void*)scatter_cluster_kernel<true, false, false>;
  int n = 0;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = c;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = n;
  return n;
}

static ScatterShape scatter_shape(int nbins, int tables, int sm_count, int device) {
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
      sh.smem = (uint32_t)std::max<uint64_t>(smem, 16);
      sh.nclusters = std::max(1, sm_count * kCtasPerSm / c);
      if (device >= 0) {
        int fit = max_active_clusters(device, tables, c, sh.smem);
        if (fit > 0) sh.nclusters = std::min(sh.nclusters, fit);
      }
      return sh;
    }
  }
  sh.cluster = false;
  return sh;
}

__device__ __forceinline__ int4 ld_nc_v4(const int* p) {
  int4 r;
  asm volatile("ld.global.nc.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ float4 ld_nc_v4f(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

// One element: applied by the CTA that owns its bin, skipped by the others.
// Branch-free: the owner test is a predicate on the shared-memory reductions.
// Bins outside [0, nbins) have an owner >= c (negative indices wrap to a huge
// unsigned value), so no CTA applies them.
template <bool ACC, bool HIST>
__device__ __forceinline__ void scatter_one(int b, float v, uint32_t rank, int shift, uint32_t acc_base,
                                            uint32_t hist_base) {
  const uint32_t owner = (uint32_t)b >> shift;
  const uint32_t off = ((uint32_t)b & ((1u << shift) - 1)) * 4;
  if (ACC)
    asm volatile("{ .reg .pred p; setp.eq.u32 p, %0, %1; @p red.shared.add.f32 [%2], %3; }" ::"r"(owner),
                 "r"(rank), "r"(acc_base + off), "f"(v)
                 : "memory");
  if (HIST)
    asm volatile("{ .reg .pred p; setp.eq.u32 p, %0, %1; @p red.shared.add.u32 [%2], 1; }" ::"r"(owner),
                 "r"(rank), "r"(hist_base + off)
                 : "memory");
}

// The warp-aggregated form of scatter_one, for inputs whose bins repeat (a
// splat that lands many points on the same pixels, a skewed histogram): the
// lanes whose elements fall in the same bin of this CTA's range find each
// other with __match_any_sync, sum their values inside the warp (a pairwise
// tree over the group's lanes in rank order), and the group's first lane
// issues one shared-memory atomic per table, adding the group's size to the
// histogram. Lanes whose element this CTA does not own, or that carry no
// element (bin -1), get a key of their own and do nothing. The whole warp
// must be converged here.
template <bool ACC, bool HIST>
__device__ __forceinline__ void scatter_agg(int b, float v, uint32_t rank, int shift, uint32_t acc_base,
                                            uint32_t hist_base) {
  const unsigned lane = threadIdx.x & 31;
  const bool mine = ((uint32_t)b >> shift) == rank;
  const unsigned peers = __match_any_sync(0xffffffffu, mine ? (uint32_t)b : (0x80000000u | lane));
  const int r = __popc(peers & ((1u << lane) - 1u));  // this lane's rank in its group
  const int gsz = __popc(peers);
  float sum = v;
  if (ACC) {
    for (int d = 1; __any_sync(0xffffffffu, d < gsz); d <<= 1) {
      const bool has = r + d < gsz;
      const int src = has ? (int)__fns(peers, 0, r + d + 1) : (int)lane;
      const float t = __shfl_sync(0xffffffffu, sum, src);
      if (has && (r & (2 * d - 1)) == 0) sum += t;
    }
  }
  if (mine && r == 0) {
    const uint32_t off = ((uint32_t)b & ((1u << shift) - 1)) * 4;
    if (ACC) asm volatile("red.shared.add.f32 [%0], %1;" ::"r"(acc_base + off), "f"(sum) : "memory");
    if (HIST) asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(hist_base + off), "r"(gsz) : "memory");
  }
}

// Whether a warp's elements pile onto so few bins that the aggregated form
// pays: shared-memory atomics that hit one address from several lanes are
// serialised, so plain atomics cost about as many passes as the largest group
// of lanes sharing a bin, while the aggregated form costs a fixed ~6-7 times a
// conflict-free pass (measured on B200: 2^24 elements, uniform over 2^16 bins
// 77 us plain, 531 us aggregated; 90 % in 64 bins 210 us plain, 515 us
// aggregated; all in one bin 5581 us plain, 468 us aggregated). So the warp
// aggregates when, over the eight elements a lane holds, the largest group
// sharing a bin averages eight lanes or more. Warp-uniform.
__device__ __forceinline__ bool piles_up(const int4& b0, const int4& b1, uint32_t rank, int shift) {
  const unsigned lane = threadIdx.x & 31;
  const int bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  unsigned total = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const bool mine = ((uint32_t)bb[k] >> shift) == rank;
    const unsigned peers = __match_any_sync(0xffffffffu, mine ? (uint32_t)bb[k] : (0x80000000u | lane));
    total += __reduce_max_sync(0xffffffffu, mine ? (unsigned)__popc(peers) : 0u);
  }
  return total >= 8 * 8;
}

// The chunk loop of the vectorised path (see scatter_cluster_kernel), plain or
// aggregated.
template <bool ACC, bool HIST, bool AGG>
__device__ __forceinline__ void scatter_chunk(const float* __restrict__ v, const int* __restrict__ idx, int64_t q,
                                              int64_t g1, int4 nb0, int4 nb1, float4 nv0, float4 nv1, uint32_t rank,
                                              int shift, uint32_t acc_base, uint32_t hist_base) {
  const int64_t stride = blockDim.x;
  const int4 none = make_int4(-1, -1, -1, -1);
  for (int64_t w = q - (threadIdx.x & 31); w < g1; w += 2 * stride, q += 2 * stride) {
    const int4 b0 = nb0, b1 = nb1;
    const float4 v0 = nv0, v1 = nv1;
    const int64_t qn = q + 2 * stride;
    nb0 = none;
    nb1 = none;
    if (qn < g1) {
      nb0 = ld_nc_v4(idx + 4 * qn);
      if (ACC) nv0 = ld_nc_v4f(v + 4 * qn);
    }
    if (qn + stride < g1) {
      nb1 = ld_nc_v4(idx + 4 * (qn + stride));
      if (ACC) nv1 = ld_nc_v4f(v + 4 * (qn + stride));
    }
    if (AGG) {
      scatter_agg<ACC, HIST>(b0.x, v0.x, rank, shift, acc_base, hist_base);
      scatter_agg<ACC, HIST>(b0.y, v0.y, rank, shift, acc_base, hist_base);
      scatter_agg<ACC, HIST>(b0.z, v0.z, rank, shift, acc_base, hist_base);
      scatter_agg<ACC, HIST>(b0.w, v0.w, rank, shift, acc_base, hist_base);
      scatter_agg<ACC, HIST>(b1.x, v1.x, rank, shift, acc_base, hist_base);
      scatter_agg<ACC, HIST>(b1.y, v1.y, rank, shift, acc_base, hist_base);
      scatter_agg<ACC, HIST>(b1.z, v1.z, rank, shift, acc_base, hist_base);
      scatter_agg<ACC, HIST>(b1.w, v1.w, rank, shift, acc_base, hist_base);
    } else {
      scatter_one<ACC, HIST>(b0.x, v0.x, rank, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.y, v0.y, rank, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.z, v0.z, rank, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b0.w, v0.w, rank, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b1.x, v1.x, rank, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b1.y, v1.y, rank, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b1.z, v1.z, rank, shift, acc_base, hist_base);
      scatter_one<ACC, HIST>(b1.w, v1.w, rank, shift, acc_base, hist_base);
    }
  }
}

template <bool ACC, bool HIST>
__device__ __noinline__ void scatter_chunk_agg(const float* __restrict__ v, const int* __restrict__ idx, int64_t q,
                                               int64_t g1, int4 nb0, int4 nb1, float4 nv0, float4 nv1, uint32_t rank,
                                               int shift, uint32_t acc_base, uint32_t hist_base) {
  scatter_chunk<ACC, HIST, true>(v, idx, q, g1, nb0, nb1, nv0, nv1, rank, shift, acc_base, hist_base);
}

// CTA `rank` of cluster `cl` applies the elements of chunk `cl` that fall in its
// bin range; partials go to ws[cl][nbins] per table. DENSE: the kernel of the
// scatter_add_dense family, whose warps each measure their first elements and
// take the aggregated form when their bins pile up. Only that kernel carries
// the aggregated code: measured on B200, merely having it in the kernel (even
// out of line, never taken) slows the plain loop by a quarter (2^24 elements
// over 2^16 bins, values + histogram: 77 us without, 99-100 us with).
template <bool ACC, bool HIST, bool DENSE>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) scatter_cluster_kernel(
    const float* __restrict__ v, const int* __restrict__ idx, int64_t n, uint32_t nbins, int shift,
    float* __restrict__ ws_acc, uint32_t* __restrict__ ws_hist) {
  extern __shared__ __align__(16) uint32_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t per = 1u << shift;
  const uint32_t tables = (ACC ? 1 : 0) + (HIST ? 1 : 0);
  for (uint32_t i = threadIdx.x; i < tables * per; i += blockDim.x) smem[i] = 0;
  __syncthreads();
  float* sacc = reinterpret_cast<float*>(smem);
  uint32_t* shist = smem + (ACC ? per : 0);
  const uint32_t acc_base = (uint32_t)__cvta_generic_to_shared(sacc);
  const uint32_t hist_base = (uint32_t)__cvta_generic_to_shared(shist);

  const uint32_t rank = cluster.block_rank();
  const uint32_t c = cluster.num_blocks();
  const int64_t cl = blockIdx.x / c;
  const int64_t ncl = gridDim.x / c;
  // This cluster's chunk, in groups of four elements.
  const int64_t n4 = n / 4;
  const int64_t per_cl = (n4 + ncl - 1) / ncl;
  const int64_t g0 = cl * per_cl;
  const int64_t g1 = min(n4, g0 + per_cl);
  const bool vec = ((reinterpret_cast<uintptr_t>(idx) | (ACC ? reinterpret_cast<uintptr_t>(v) : 0)) & 15) == 0;
  if (vec) {
    const int64_t stride = blockDim.x;
    int64_t q = g0 + threadIdx.x;
    // Two groups of four per iteration (q and q + stride), and the next
    // iteration's two groups are loaded before this one's atomics are issued
    // (the loads are volatile asm, so they stay in this order): 64 bytes per
    // thread stay in flight while the thread works through its shared-memory
    // atomics. Every lane of a warp makes the same number of iterations (while
    // the warp's first group is in the chunk); a lane past the chunk's end
    // carries bin -1, which no CTA owns. So warps stay converged, which the
    // aggregated form needs.
    const int4 none = make_int4(-1, -1, -1, -1);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    int4 nb0 = none, nb1 = none;
    float4 nv0 = zero, nv1 = zero;
    if (q < g1) {
      nb0 = ld_nc_v4(idx + 4 * q);
      if (ACC) nv0 = ld_nc_v4f(v + 4 * q);
    }
    if (q + stride < g1) {
      nb1 = ld_nc_v4(idx + 4 * (q + stride));
      if (ACC) nv1 = ld_nc_v4f(v + 4 * (q + stride));
    }
    // dense kernel: each warp measures its first 256 elements once and takes
    // one form for the rest of the chunk
    if (DENSE && piles_up(nb0, nb1, rank, shift)) {
      scatter_chunk_agg<ACC, HIST>(v, idx, q, g1, nb0, nb1, nv0, nv1, rank, shift, acc_base, hist_base);
    } else {
      for (int64_t w = q - (threadIdx.x & 31); w < g1; w += 2 * stride, q += 2 * stride) {
        const int4 b0 = nb0, b1 = nb1;
        const float4 v0 = nv0, v1 = nv1;
        const int64_t qn = q + 2 * stride;
        nb0 = none;
        nb1 = none;
        if (qn < g1) {
          nb0 = ld_nc_v4(idx + 4 * qn);
          if (ACC) nv0 = ld_nc_v4f(v + 4 * qn);
        }
        if (qn + stride < g1) {
          nb1 = ld_nc_v4(idx + 4 * (qn + stride));
          if (ACC) nv1 = ld_nc_v4f(v + 4 * (qn + stride));
        }
        const int bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) scatter_one<ACC, HIST>(bb[k], vv[k], rank, shift, acc_base, hist_base);
      }
    }
    // The ragged tail (n not a multiple of four) belongs to the last cluster.
    if (cl == ncl - 1)
      for (int64_t i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x)
        scatter_one<ACC, HIST>(idx[i], ACC ? v[i] : 0.f, rank, shift, acc_base, hist_base);
  } else {
    // Unaligned inputs: plain loads over an element range of the cluster's
    // own, chunked by elements (not groups), so every element of [0, n) lies
    // in exactly one cluster's range whatever n and ncl are.
    const int64_t per_e = (n + ncl - 1) / ncl;
    const int64_t e0 = min(n, cl * per_e), e1 = min(n, e0 + per_e);
    for (int64_t i = e0 + threadIdx.x; i < e1; i += blockDim.x)
      scatter_one<ACC, HIST>(idx[i], ACC ? v[i] : 0.f, rank, shift, acc_base, hist_base);
  }
  __syncthreads();
  const uint32_t lo = rank * per;
  for (uint32_t i = threadIdx.x; i < per && lo + i < nbins; i += blockDim.x) {
    if (ACC) ws_acc[cl * nbins + lo + i] = sacc[i];
    if (HIST) ws_hist[cl * nbins + lo + i] = shist[i];
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
#pragma unroll 8
    for (int c = 0; c < nclusters; ++c) s += ws_acc[(int64_t)c * nbins + b];
    acc[b] = s;
  }
  if (hist) {
    uint32_t s = accumulate ? hist[b] : 0u;
#pragma unroll 8
    for (int c = 0; c < nclusters; ++c) s += ws_hist[(int64_t)c * nbins + b];
    hist[b] = s;
  }
}

// The same sums with 16-byte loads and many more of them in flight (the
// one-bin-a-thread form waits on L2 latency): a block takes 128 bins as 32
// groups of four and splits the clusters eight ways, thread row g summing
// clusters g, g + 8, ... in order; the eight row sums are then added in row
// order. The order is fixed, so the result does not depend on scheduling.
constexpr int kRedSplit = 8, kRedQuads = 32;
template <bool ACC, bool HIST>
__global__ void __launch_bounds__(kRedSplit* kRedQuads)
    scatter_reduce4_kernel(const float4* __restrict__ ws_acc, const uint4* __restrict__ ws_hist, int nclusters,
                           uint32_t nquads, float4* __restrict__ acc, uint4* __restrict__ hist, int accumulate) {
  __shared__ float4 ra[kRedSplit][kRedQuads];
  __shared__ uint4 rh[kRedSplit][kRedQuads];
  const int q = threadIdx.x % kRedQuads, g = threadIdx.x / kRedQuads;
  const uint32_t b = blockIdx.x * kRedQuads + q;
  const bool in = b < nquads;
  float4 sa = make_float4(0.f, 0.f, 0.f, 0.f);
  uint4 sh = make_uint4(0u, 0u, 0u, 0u);
  if (in) {
#pragma unroll 4
    for (int c = g; c < nclusters; c += kRedSplit) {
      const int64_t o = (int64_t)c * nquads + b;
      if (ACC) {
        const float4 x = ws_acc[o];
        sa.x += x.x, sa.y += x.y, sa.z += x.z, sa.w += x.w;
      }
      if (HIST) {
        const uint4 y = ws_hist[o];
        sh.x += y.x, sh.y += y.y, sh.z += y.z, sh.w += y.w;
      }
    }
  }
  if (ACC) ra[g][q] = sa;
  if (HIST) rh[g][q] = sh;
  __syncthreads();
  if (g != 0 || !in) return;
  if (ACC) {
    float4 t = accumulate ? acc[b] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < kRedSplit; ++j) {
      const float4 x = ra[j][q];
      t.x += x.x, t.y += x.y, t.z += x.z, t.w += x.w;
    }
    acc[b] = t;
  }
  if (HIST) {
    uint4 t = accumulate ? hist[b] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < kRedSplit; ++j) {
      const uint4 y = rh[j][q];
      t.x += y.x, t.y += y.y, t.z += y.z, t.w += y.w;
    }
    hist[b] = t;
  }
}

// The fixed-order sum of the clusters' partial tables into acc / hist: four
// bins a thread when every table allows 16-byte loads, else one.
static cudaError_t launch_reduce(cudaStream_t s, const float* ws_acc, const uint32_t* ws_hist, int ncl,
                                 uint32_t nbins, float* acc, uint32_t* hist, int accumulate) {
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (nbins % 4 == 0 && a16(ws_acc) && a16(ws_hist) && a16(acc) && a16(hist)) {
    const uint32_t nq = nbins / 4;
    const unsigned blocks = (nq + kRedQuads - 1) / kRedQuads;
    const auto* wa = reinterpret_cast<const float4*>(ws_acc);
    const auto* wh = reinterpret_cast<const uint4*>(ws_hist);
    auto* oa = reinterpret_cast<float4*>(acc);
    auto* oh = reinterpret_cast<uint4*>(hist);
    if (acc && hist)
      scatter_reduce4_kernel<true, true><<<blocks, kRedSplit * kRedQuads, 0, s>>>(wa, wh, ncl, nq, oa, oh, accumulate);
    else if (acc)
      scatter_reduce4_kernel<true, false><<<blocks, kRedSplit * kRedQuads, 0, s>>>(wa, wh, ncl, nq, oa, oh, accumulate);
    else
      scatter_reduce4_kernel<false, true><<<blocks, kRedSplit * kRedQuads, 0, s>>>(wa, wh, ncl, nq, oa, oh, accumulate);
  } else {
    const unsigned blocks = (nbins + 255) / 256;
    scatter_reduce_kernel<<<blocks, 256, 0, s>>>(ws_acc, ws_hist, ncl, nbins, acc, hist, accumulate);
  }
  return cudaGetLastError();
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

// Scratch for the clusters' partial bins. With both an accumulator and a
// histogram the two tables are best applied by two launches of one table each
// (2-CTA clusters on every SM instead of 4-CTA clusters, which fit 132 of 148
// SMs): that takes scatter_workspace bytes. scatter_workspace_min is what the
// one-launch form needs; scatter_run picks the form the scratch it gets allows.
static uint64_t combined_bytes(const LaunchArgs& la, int tables) {
  ScatterShape sh = scatter_shape(la.a[4].i32, tables, la.sm_count, la.device);
  return sh.cluster ? (uint64_t)sh.nclusters * tables * (uint64_t)la.a[4].i32 * 4 : 0;
}
static uint64_t split_bytes(const LaunchArgs& la) {
  ScatterShape sh = scatter_shape(la.a[4].i32, 1, la.sm_count, la.device);
  return sh.cluster ? 2 * (uint64_t)sh.nclusters * (uint64_t)la.a[4].i32 * 4 : 0;
}
uint64_t scatter_workspace_min(const LaunchArgs& la) {
  int tables = (la.a[0].kind != MTL_ARG_NULL) + (la.a[1].kind != MTL_ARG_NULL);
  return combined_bytes(la, tables);
}
uint64_t scatter_workspace(const LaunchArgs& la) {
  int tables = (la.a[0].kind != MTL_ARG_NULL) + (la.a[1].kind != MTL_ARG_NULL);
  const uint64_t one = combined_bytes(la, tables);
  return tables == 2 && one ? std::max(one, split_bytes(la)) : one;
}

template <bool ACC, bool HIST>
static cudaError_t launch_cluster(const ScatterShape& sh, cudaStream_t s, const float* v,
                                  const int* idx, int64_t n, uint32_t nbins, float* ws_acc,
                                  uint32_t* ws_hist, bool dense) {
  auto k = dense ? scatter_cluster_kernel<ACC, HIST, true> : scatter_cluster_kernel<ACC, HIST, false>;
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

// Shared by the graph path and the direct and no-scratch entry points; `dense`
// for the scatter_add_dense family.
static mtl_status scatter_launch(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream, bool dense) {
  float* acc;
  uint32_t* hist;
  const float* v;
  const int* idx;
  int nbins, accumulate;
  int64_t n;
  scatter_unpack(la, acc, hist, v, idx, nbins, accumulate, n);
  cudaStream_t s = (cudaStream_t)stream;
  const int tables = (acc != nullptr) + (hist != nullptr);
  ScatterShape sh = scatter_shape(nbins, tables, la.sm_count, la.device);
  cudaError_t e = cudaSuccess;
  if (sh.cluster && tables == 2 && ws && ws_bytes >= split_bytes(la)) {
    // Two launches of one table each, then one reduction of both.
    ScatterShape s1 = scatter_shape(nbins, 1, la.sm_count, la.device);
    float* ws_acc = reinterpret_cast<float*>(ws);
    uint32_t* ws_hist = reinterpret_cast<uint32_t*>(ws) + (uint64_t)s1.nclusters * nbins;
    int ncl = s1.nclusters;
    if (n > 0) {
      e = launch_cluster<true, false>(s1, s, v, idx, n, nbins, ws_acc, nullptr, dense);
      if (e == cudaSuccess) e = launch_cluster<false, true>(s1, s, v, idx, n, nbins, nullptr, ws_hist, dense);
    } else {
      ncl = 0;
    }
    if (e == cudaSuccess) {
      e = launch_reduce(s, ws_acc, ws_hist, ncl, (uint32_t)nbins, acc, hist, accumulate);
    }
  } else if (sh.cluster) {
    uint64_t need = (uint64_t)sh.nclusters * tables * (uint64_t)nbins * 4;
    if (!ws || ws_bytes < need)
      return fail(MTL_ERR_ARGUMENT, "scatter_add: needs %llu bytes of scratch, got %llu",
                  (unsigned long long)need, (unsigned long long)ws_bytes);
    float* ws_acc = acc ? reinterpret_cast<float*>(ws) : nullptr;
    uint32_t* ws_hist = hist ? reinterpret_cast<uint32_t*>(ws) + (acc ? (uint64_t)sh.nclusters * nbins : 0) : nullptr;
    int ncl = sh.nclusters;
    if (n > 0) {
      if (acc && hist)
        e = launch_cluster<true, true>(sh, s, v, idx, n, nbins, ws_acc, ws_hist, dense);
      else if (acc)
        e = launch_cluster<true, false>(sh, s, v, idx, n, nbins, ws_acc, ws_hist, dense);
      else
        e = launch_cluster<false, true>(sh, s, v, idx, n, nbins, ws_acc, ws_hist, dense);
    } else {
      ncl = 0;
    }
    if (e == cudaSuccess) {
      e = launch_reduce(s, ws_acc, ws_hist, ncl, (uint32_t)nbins, acc, hist, accumulate);
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

mtl_status scatter_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream) {
  return scatter_launch(la, ws, ws_bytes, stream, false);
}
mtl_status scatter_dense_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream) {
  return scatter_launch(la, ws, ws_bytes, stream, true);
}

}  // namespace mtl
