// Device-side building blocks shared by the tensor-core kernels (GEMM and
// implicit-GEMM convolution): mbarriers with bounded waits, TMA tile loads,
// tcgen05 MMA / commit / TMEM loads, and the shared-memory matrix descriptor.
// Inline PTX for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <utility>

#include "../mtl_internal.hpp"

namespace mtl {

// The wall-clock limit of every bounded wait in this translation unit, in ns:
// 2 s unless the host shortened it (mtl_set_wait_limit, for the tests that
// make a wait run out). One copy per .cu file that includes this header.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
static __device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;
static inline cudaError_t set_wait_limit_this_file(unsigned long long ns) {
  return cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof ns);
}

// ── PTX wrappers ─────────────────────────────────────────────────────────────
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// try_wait with a suspend-time hint: the thread sleeps in the barrier until the
// phase completes or the hint (ns) runs out, instead of re-polling shared
// memory. Polling warps take shared-memory cycles from the tensor core's
// operand reads (an M=128, N=64 MMA reads 6 KiB of operands in 48 cycles, the
// whole shared-memory bandwidth).
constexpr uint32_t kSuspendHintNs = 1000000;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// A wait ran out: the CTA aborts, and the thread that raises its abort flag
// (the first of its threads whose wait ran out) counts one timeout, so the
// counter counts CTAs that gave up, however many of their threads were waiting.
__device__ __forceinline__ void abort_cta(volatile int* abort, int* timeouts) {
  if (atomicExch(const_cast<int*>(abort), 1) == 0) atomicAdd(timeouts, 1);
}

// Bounded wait for the phase of `bar` with the given parity. Returns false when
// the CTA is aborting (this wait ran out, or another role's did).
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort, int* timeouts) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer(), limit = g_wait_limit_ns;
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > limit) {
      abort_cta(abort, timeouts);
      return false;
    }
  }
}
// Wait, bounded, for an operation this CTA started itself (a load landing, its
// MMAs finishing) before leaving; used on exit paths, so it ignores `abort`.
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return;
  const unsigned long long t0 = globaltimer(), limit = g_wait_limit_ns;
  while (!mbar_try_wait_sleep(bar, parity))
    if (globaltimer() - t0 > limit) return;
}
// Bounded wait until another role's progress counter (in shared memory)
// reaches `target`.
__device__ __forceinline__ bool wait_progress(volatile int* counter, int target, volatile int* abort, int* timeouts) {
  if (*counter >= target) return true;
  const unsigned long long t0 = globaltimer(), limit = g_wait_limit_ns;
  for (;;) {
    __nanosleep(64);
    if (*counter >= target) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > limit) {
      abort_cta(abort, timeouts);
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
// Programmatic dependent launch. A kernel launched by launch_pdl may become
// resident while the previous kernel in its stream is still finishing:
// pdl_wait() returns once that kernel has completed and its writes are
// visible (at once for an ordinary launch), so every global access that can
// touch another kernel's data must follow it; pdl_trigger() lets the next
// launch in the stream be scheduled as this one's CTAs leave their SMs.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  // MTL_NO_PDL=1 launches in plain stream order (for comparison and debugging)
  static const bool off = [] {
    const char* v = std::getenv("MTL_NO_PDL");
    return v && v[0] == '1';
  }();
  cfg.numAttrs = off ? 0 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same, always accumulating. With N = 64 an MMA takes about 48 cycles of
// tensor work; the single issuing thread keeps up only when little else runs
// between MMAs (measured: a runtime accumulate flag and loop control per MMA
// cost 71 cycles per MMA, fully unrolled issue with this form 51).
__device__ __forceinline__ void tc_mma_acc(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, 1, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d), "l"(a),
      "l"(b), "r"(idesc)
      : "memory");
}
// 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// The same without the wait: issue several, then tmem_wait_ld() once.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05): start address, leading and stride
// byte offsets (all >> 4), version 1 at bit 46, layout at bit 61 (2 = 128-byte
// swizzle, 4 = 64-byte swizzle, 0 = none).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint64_t layout = 2) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (layout << 61);
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// Plain bulk copy global -> shared (both 16-byte aligned, size a multiple of
// 16), completing on the mbarrier's transaction count.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// TMA store of a 3-D box from shared memory (bulk-group completion): the
// caller fences the async proxy first and waits with bulk_wait_read before
// overwriting the shared-memory source.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most N committed bulk groups may still be reading their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Every committed bulk group complete (writes visible).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Shared-memory matrix descriptor without swizzling (K-major): 8-row x 16-byte
// core matrices, `lbo` bytes between the 16-byte K chunks, `sbo` bytes between
// 8-row groups.
__device__ __forceinline__ uint64_t smem_desc_noswizzle(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// TMA load in im2col mode from a 4-D NHWC tensor map: the pixel run starting
// at base coordinates (w, h, n), channels from c, shifted by the filter tap
// (off_w, off_h).
__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const CUtensorMap* map, int c, int w, int h, int n,
                                                   uint16_t off_w, uint16_t off_h, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(n), "r"(bar), "h"(off_w), "h"(off_h)
      : "memory");
}

// A tcgen05 instruction descriptor for kind::f16 with bf16 A and B, fp32
// accumulation: bit 4 = F32 accumulator, bits 7/10 = BF16 A/B, bit 15/16 =
// A/B MN-major, N>>3 at bit 17, M>>4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Host: the driver's cuTensorMapEncodeTiled (through the runtime's entry-point
// lookup, so nothing links libcuda directly).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// Host: a 3-D bf16 tensor map {inner, outer, batch} with box {64, box_outer, 1},
// 128-byte swizzle, zeros outside the tensor (defined in gemm.cu).
mtl_status make_bf16_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t batch,
                         uint32_t box_outer);

}  // namespace mtl
