// Batched dense GEMM on the 5th-generation tensor cores:
//
//   C[b] = A[b] · B[b]     A: M×K bf16 row-major, B: K×N bf16 row-major,
//                          C: M×N fp32 row-major, fp32 accumulation.
//
// One persistent CTA per SM walks output tiles of 128×256 (grouped so that the
// CTAs running at the same time share A row-panels and B column-panels in L2).
// Warp roles inside the 192-thread CTA:
//   warp 0      TMA producer: one thread streams 128×64 A tiles (K-major) and
//               four 64×64 B tiles (N-major) per k-block into a 4-stage ring
//               of 48 KiB stages, 128-byte swizzled, completion counted on a
//               per-stage mbarrier;
//   warp 1      owns the tensor memory (512 columns: two 128×256 fp32
//               accumulators) and one thread issues tcgen05.mma (M=128, N=256,
//               K=16, both operands from shared memory through matrix
//               descriptors), four per k-block; tcgen05.commit frees a stage
//               when its MMAs have read it and publishes a finished
//               accumulator;
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp reads its
//               32 TMEM lanes = 32 rows), fp32 stores to C, then hand the
//               accumulator back. With two accumulators the epilogue of tile
//               i overlaps the main loop of tile i+1.
// TMA loads use no cluster multicast: every CTA fetches its own tiles, and the
// reuse between CTAs comes from L2.
//
// Shapes: any M; N and K multiples of 8 (TMA needs 16-byte row strides); edges
// read as zeros (TMA out-of-bounds fill) and are masked on store. Buffers 16-byte
// aligned.
//
// Every wait on an mbarrier is bounded by a wall-clock limit (%globaltimer);
// a wait that runs out sets an abort flag that the other roles see, so the CTA
// winds down, releases its tensor memory and returns, and the host reads the
// count of such CTAs from g_gemm_timeouts. `stall_cta` (-1 normally) is the
// test hook for that path: the producer of that CTA issues no load at all, so
// its MMA issuer waits on a stage that never fills until the limit runs out
// (mtl_inject_stall; nothing is in flight when the CTA winds down).

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "../mtl_internal.hpp"
#include "tc_common.cuh"

namespace mtl {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr uint32_t kAStage = kBM * kBK * 2;  // 16 KiB: one 128-row run of A
constexpr uint32_t kBStage = kBK * kBN * 2;  // 32 KiB
constexpr int kGemmThreads = 192;
constexpr int kGroupM = 16;  // tile rows per raster group (MTL_GEMM_GROUP_M overrides it, for tuning)
constexpr uint32_t kTmemCols = 512;

// RUNS 128-row runs of A per tile, sharing each k-block's B. One run: 4
// stages of 48 KiB and two accumulators, so a tile's epilogue overlaps the
// next tile's main loop. Two runs (256 x 256 tiles): 3 stages of 64 KiB, the
// two runs' accumulators filling the 512 TMEM columns, so the epilogue runs
// between tiles, but each k-block moves 64 KiB for eight MMAs instead of 48
// KiB for four: a third fewer operand bytes per MAC from L2 and shared
// memory.
template <int RUNS>
struct GemmCfg {
  static constexpr int kStages = RUNS == 1 ? 4 : 3;
  static constexpr uint32_t kStageBytes = RUNS * kAStage + kBStage;
  static constexpr int kAcc = RUNS == 1 ? 2 : 1;  // accumulator sets of RUNS x 256 columns
  static constexpr int kTileM = kBM * RUNS;
  // ring + barriers + alignment slack
  static constexpr int kSmem = kStages * (int)kStageBytes + 1024 + 1024;
};

__device__ int g_gemm_timeouts;

// Instruction descriptor, kind::f16: fp32 accumulator (bit 4), bf16 A and B
// (bits 7, 10), A K-major, B N-major (bit 16), N>>3 at bit 17, M>>4 at bit 24.
constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, kBN, false, true);

struct TileCoord {
  int b, m0, n0;
};
template <int RUNS>
__device__ __forceinline__ TileCoord tile_coord(int64_t t, int tiles_m, int tiles_n, int group_m) {
  const int64_t per = (int64_t)tiles_m * tiles_n;
  TileCoord c;
  c.b = (int)(t / per);
  int r = (int)(t % per);
  const int group = r / (group_m * tiles_n);
  const int first_m = group * group_m;
  const int gsize = min(group_m, tiles_m - first_m);
  const int in_group = r % (group_m * tiles_n);
  c.m0 = (first_m + in_group % gsize) * GemmCfg<RUNS>::kTileM;
  c.n0 = (in_group / gsize) * kBN;
  return c;
}

template <int RUNS>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     float* __restrict__ C, int M, int N, int K, int batch, int stall_cta, int group_m) {
  using Cfg = GemmCfg<RUNS>;
  constexpr int kStages = Cfg::kStages, kAcc = Cfg::kAcc;
  constexpr uint32_t kStageBytes = Cfg::kStageBytes;
  extern __shared__ unsigned char gsm_raw[];
  // 1024-byte alignment: the 128-byte swizzle repeats every 8 rows of 128 B.
  unsigned char* gsm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* ring = gsm;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gsm + kStages * kStageBytes);
  uint64_t* full = bars;                   // [kStages]
  uint64_t* empty = bars + kStages;        // [kStages]
  uint64_t* tfull = bars + 2 * kStages;    // [kAcc]
  uint64_t* tempty = bars + 2 * kStages + 2;  // [kAcc]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tiles_m = (M + Cfg::kTileM - 1) / Cfg::kTileM, tiles_n = (N + kBN - 1) / kBN;
  const int64_t ntiles = (int64_t)tiles_m * tiles_n * batch;
  const int kblocks = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 4);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ── TMA producer ──
    if (lane == 0 && (int)blockIdx.x != stall_cta) {
      int s = 0;
      uint32_t ph = 0;
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const TileCoord tc = tile_coord<RUNS>(t, tiles_m, tiles_n, group_m);
        // runs and B chunks that start past M or N feed only outputs that are
        // never stored: they are not loaded (a box wholly outside the tensor)
        const int runs = min(RUNS, (M - tc.m0 + kBM - 1) / kBM);
        const int nchunks = min(kBN / 64, (N - tc.n0 + 63) / 64);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_gemm_timeouts)) goto producer_done;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, (uint32_t)runs * kAStage + (uint32_t)nchunks * (kBK * 128));
          const uint32_t a_dst = smem_u32(ring + s * kStageBytes);
          const uint32_t b_dst = a_dst + RUNS * kAStage;
          for (int r = 0; r < runs; ++r) tma_load_3d(a_dst + r * kAStage, &tmA, kb * kBK, tc.m0 + r * kBM, tc.b, fb);
          for (int c = 0; c < nchunks; ++c) tma_load_3d(b_dst + c * (kBK * 128), &tmB, tc.n0 + c * 64, kb * kBK, tc.b, fb);
          if (++s == kStages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ── MMA issuer ──
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int i = 0;
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
        const int a = i % kAcc;
        if (!wait_phase(smem_u32(&tempty[a]), ((i / kAcc) & 1) ^ 1, abort, &g_gemm_timeouts)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(a * kBN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_phase(smem_u32(&full[s]), ph, abort, &g_gemm_timeouts)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + s * kStageBytes);
          const uint32_t b_addr = a_addr + RUNS * kAStage;
          // A: K-major, rows of 128 B, 8-row groups 1024 B apart (SBO); a K=16
          // slice is 32 B further along the swizzled row.
          // B: N-major, 64-column chunks kBK*128 B apart (LBO), 8-row K groups
          // 1024 B apart (SBO); a K=16 slice is 16 rows = 2048 B further.
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t bd = smem_desc(b_addr + kk * 2048, kBK * 128, 1024);
#pragma unroll
            for (int r = 0; r < RUNS; ++r) {
              // run r's accumulator: the second 256 columns (two runs)
              const uint64_t ad = smem_desc(a_addr + r * kAStage + kk * 32, 16, 1024);
              if (kk == 0)
                tc_mma(d + (uint32_t)(r * kBN), ad, bd, kIdesc, kb != 0);
              else
                tc_mma_acc(d + (uint32_t)(r * kBN), ad, bd, kIdesc);
            }
          }
          tc_commit(smem_u32(&empty[s]));
          if (++s == kStages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&tfull[a]));
      }
    }
  } else {
    // ── epilogue: warps 2..5 read TMEM lanes 32*(warp%4) .. +32 ──
    const int q = warp & 3;
    int i = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      const int a = i % kAcc;
      if (!wait_phase(smem_u32(&tfull[a]), (i / kAcc) & 1, abort, &g_gemm_timeouts)) break;
      tc_fence_after();
      const TileCoord tc = tile_coord<RUNS>(t, tiles_m, tiles_n, group_m);
#pragma unroll 1
      for (int run = 0; run < RUNS; ++run) {
        const int row = tc.m0 + run * kBM + q * 32 + lane;
        float* crow = C + ((int64_t)tc.b * M + row) * (int64_t)N;
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((a + run) * kBN);
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          const int col = tc.n0 + c * 32;
          if (row < M) {
            if (col + 32 <= N) {
              float4* dst = reinterpret_cast<float4*>(crow + col);
#pragma unroll
              for (int v = 0; v < 8; ++v)
                dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                     __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
            } else {
#pragma unroll
              for (int v = 0; v < 32; ++v)
                if (col + v < N) crow[col + v] = __uint_as_float(r[v]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[a]));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// ── host side ────────────────────────────────────────────────────────────────
EncodeTiledFn encode_tiled_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  });
  return fn;
}

// A 3-D bf16 tensor map: dims {inner, outer, batch}, box {64, box_outer, 1},
// 128-byte swizzle, zeros outside the tensor.
mtl_status make_bf16_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t batch,
                         uint32_t box_outer) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(MTL_ERR_CUDA, "gemm: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {inner * 2, inner * outer * 2};
  cuuint32_t box[3] = {64, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTL_ERR_ARGUMENT, "gemm: tensor map rejected (CUresult %d)", (int)r);
  return MTL_OK;
}

// Launches left whose CTA 0 stalls (mtl_inject_stall("gemm_bf16", n)).
static std::atomic<int> g_gemm_stalls{0};
void gemm_inject_stall(int launches) { g_gemm_stalls.store(launches > 0 ? launches : 0); }

// Tile rows per raster group: kGroupM, or MTL_GEMM_GROUP_M (1..1024) read once.
static int group_m() {
  static const int g = [] {
    const char* e = std::getenv("MTL_GEMM_GROUP_M");
    const int v = e ? std::atoi(e) : 0;
    return v >= 1 && v <= 1024 ? v : kGroupM;
  }();
  return g;
}

// 128-row runs of A per tile: two (256 x 256 tiles) where M has more than
// one run, unless MTL_GEMM_RUNS=1 (read once).
static int gemm_runs(int M) {
  static const bool one = [] {
    const char* e = std::getenv("MTL_GEMM_RUNS");
    return e && e[0] == '1';
  }();
  return one || M <= kBM ? 1 : 2;
}

// Host: the bounded waits' limit of this file's kernels on the current device.
cudaError_t gemm_set_wait_limit(unsigned long long ns) { return set_wait_limit_this_file(ns); }

// Arguments: C (B, f32), A (B, bf16), B (B, bf16), M, N, K (i); ndrange = batch.
mtl_status gemm_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.ndim != 1) return fail(MTL_ERR_ARGUMENT, "gemm: ndrange must be one-dimensional (the batch count)");
  const int64_t M = la.a[3].i32, N = la.a[4].i32, K = la.a[5].i32, batch = la.nd[0];
  if (M < 0 || N < 0 || K < 0) return fail(MTL_ERR_ARGUMENT, "gemm: negative dimension");
  if (N % 8 || K % 8)
    return fail(MTL_ERR_UNSUPPORTED, "gemm: N and K must be multiples of 8 (16-byte rows), got N=%lld K=%lld",
                (long long)N, (long long)K);
  const uint64_t need[3] = {(uint64_t)(batch * M * N * 4), (uint64_t)(batch * M * K * 2), (uint64_t)(batch * K * N * 2)};
  const char* what[3] = {"C", "A", "B"};
  for (int i = 0; i < 3; ++i) {
    if (bytes[i] && bytes[i] < need[i])
      return fail(MTL_ERR_ARGUMENT, "gemm: %s has %llu bytes, the launch touches %llu", what[i],
                  (unsigned long long)bytes[i], (unsigned long long)need[i]);
    if (la.a[i].ptr & 15) return fail(MTL_ERR_ARGUMENT, "gemm: %s must be 16-byte aligned", what[i]);
  }
  return MTL_OK;
}

mtl_status gemm_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  float* C = reinterpret_cast<float*>(la.a[0].ptr);
  const void* A = reinterpret_cast<const void*>(la.a[1].ptr);
  const void* B = reinterpret_cast<const void*>(la.a[2].ptr);
  const int M = la.a[3].i32, N = la.a[4].i32, K = la.a[5].i32;
  const int64_t batch = la.nd[0];
  cudaStream_t s = (cudaStream_t)stream;
  if (batch == 0 || M == 0 || N == 0) return MTL_OK;
  if (batch > 65535) return fail(MTL_ERR_UNSUPPORTED, "gemm: batch above 65535");
  if (K == 0) {
    cudaError_t e = cudaMemsetAsync(C, 0, (size_t)batch * M * N * 4, s);
    return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "gemm: %s", cudaGetErrorString(e));
  }
  CUtensorMap ta, tb;
  if (mtl_status st = make_bf16_map(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)batch, kBM)) return st;
  if (mtl_status st = make_bf16_map(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)batch, kBK)) return st;
  const int runs = gemm_runs(M);
  const int tile_m = kBM * runs;
  const int64_t tiles = (int64_t)((M + tile_m - 1) / tile_m) * ((N + kBN - 1) / kBN) * batch;
  const int grid = (int)std::min<int64_t>(tiles, la.sm_count);
  int stall = -1;
  for (int left = g_gemm_stalls.load(); left > 0;)
    if (g_gemm_stalls.compare_exchange_weak(left, left - 1)) {
      stall = 0;
      break;
    }
  cudaError_t e;
  if (runs == 2) {
    e = cudaFuncSetAttribute(gemm_bf16_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<2>::kSmem);
    if (e == cudaSuccess)
      gemm_bf16_kernel<2><<<grid, kGemmThreads, GemmCfg<2>::kSmem, s>>>(ta, tb, C, M, N, K, (int)batch, stall,
                                                                        group_m());
  } else {
    e = cudaFuncSetAttribute(gemm_bf16_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<1>::kSmem);
    if (e == cudaSuccess)
      gemm_bf16_kernel<1><<<grid, kGemmThreads, GemmCfg<1>::kSmem, s>>>(ta, tb, C, M, N, K, (int)batch, stall,
                                                                        group_m());
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "gemm: %s", cudaGetErrorString(e));
  return MTL_OK;
}

// Host: read (and with reset, clear) this file's count of bounded waits that
// ran out on the current device.
int gemm_timeouts(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_timeouts, sizeof v) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_timeouts, &zero, sizeof zero);
  }
  return v;
}

}  // namespace mtl

