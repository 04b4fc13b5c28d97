// Batched 1-D complex FFT, interleaved ComplexF32, lengths 16, 256 and 4096
// (16^P for P = 1..3), forward or inverse:
//
//   forward  X[k] = sum_n x[n] exp(-2 pi i n k / N)
//   inverse  x[n] = (1/N) sum_k X[k] exp(+2 pi i n k / N)
//
// One transform is N/16 threads; a 256-thread CTA runs 256/(N/16) transforms
// (one at N = 4096). Each of the P passes is a radix-16 Stockham step: every
// thread holds 16 points in registers, multiplies them by the pass twiddles,
// runs a 16-point DFT (two radix-4 stages) and writes them back; passes trade
// points through shared memory, padded by one element every 16 so that the
// stride-16 writes of the first pass do not pile onto one bank. The first pass
// reads global memory and the last one writes it, both at stride N/16 points
// per register, i.e. 256 contiguous bytes per warp per register: every byte is
// read once and written once (16 B per point per direction, the roofline).
//
// The inverse runs the forward transform on conj(x) and stores conj(.)/N.
// Twiddles exp(-2 pi i m / 4096) come from a table computed on the host in
// double precision and rounded once to float, uploaded on the first launch on
// each device.

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "../mtl_internal.hpp"

namespace mtl {

constexpr int kFftMaxN = 4096;
constexpr int kFftThreads = 256;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
// a * (-i)
__device__ __forceinline__ float2 mul_mi(float2 a) { return make_float2(a.y, -a.x); }

// 4-point forward DFT in place on a[0], a[s], a[2s], a[3s] of v.
template <int S>
__device__ __forceinline__ void dft4(float2* v, int o) {
  float2 a0 = v[o], a1 = v[o + S], a2 = v[o + 2 * S], a3 = v[o + 3 * S];
  float2 s02 = cadd(a0, a2), d02 = csub(a0, a2);
  float2 s13 = cadd(a1, a3), d13 = mul_mi(csub(a1, a3));
  v[o] = cadd(s02, s13);
  v[o + S] = cadd(d02, d13);
  v[o + 2 * S] = csub(s02, s13);
  v[o + 3 * S] = csub(d02, d13);
}

// 16-point forward DFT of v[0..15], result in natural order.
// n = n1 + 4 n2, k = 4 k1 + k2:
//   Y[n1][k2] = DFT4_n2(v[n1 + 4 n2]) * W16^(n1 k2),  X[4 k1 + k2] = DFT4_n1(Y[n1][k2]).
__device__ __forceinline__ void dft16(float2* v) {
  // Stage A: for each n1, a DFT4 over v[n1], v[n1+4], v[n1+8], v[n1+12];
  // the result for k2 lands in v[n1 + 4 k2].
  dft4<4>(v, 0);
  dft4<4>(v, 1);
  dft4<4>(v, 2);
  dft4<4>(v, 3);
  // Twiddles W16^(n1 k2) on v[n1 + 4 k2].
  const float c1 = 0.92387953251128674f, s1 = 0.38268343236508979f, r2 = 0.70710678118654752f;
  v[5] = cmul(v[5], make_float2(c1, -s1));     // n1=1,k2=1: W^1
  v[9] = cmul(v[9], make_float2(r2, -r2));     // n1=1,k2=2: W^2
  v[13] = cmul(v[13], make_float2(s1, -c1));   // n1=1,k2=3: W^3
  v[6] = cmul(v[6], make_float2(r2, -r2));     // n1=2,k2=1: W^2
  v[10] = mul_mi(v[10]);                       // n1=2,k2=2: W^4 = -i
  v[14] = cmul(v[14], make_float2(-r2, -r2));  // n1=2,k2=3: W^6
  v[7] = cmul(v[7], make_float2(s1, -c1));     // n1=3,k2=1: W^3
  v[11] = cmul(v[11], make_float2(-r2, -r2));  // n1=3,k2=2: W^6
  v[15] = cmul(v[15], make_float2(-c1, s1));   // n1=3,k2=3: W^9
  // Stage B: for each k2, a DFT4 over n1 (v[4 k2 + n1]); result k1 in v[4 k2 + k1].
  dft4<1>(v, 0);
  dft4<1>(v, 4);
  dft4<1>(v, 8);
  dft4<1>(v, 12);
  // X[4 k1 + k2] sits in v[4 k2 + k1]: transpose the 4x4.
  float2 t;
#define SWAP(a, b) t = v[a], v[a] = v[b], v[b] = t;
  SWAP(1, 4) SWAP(2, 8) SWAP(3, 12) SWAP(6, 9) SWAP(7, 13) SWAP(11, 14)
#undef SWAP
}

__device__ __forceinline__ int pad(int i) { return i + (i >> 4); }

// Twiddles of pass p >= 1 (Ns = 16^p points already combined): point r of
// thread j is multiplied by W_(16 Ns)^((j mod Ns) r). They depend on Ns only,
// not on N, so two tables cover every length: row r-1 holds q = 0..Ns-1, and a
// warp reads 16 or 32 consecutive entries — one or two sectors per load.
__device__ float2 g_fft_tw16[15 * 16];    // W_256^(q r)
__device__ float2 g_fft_tw256[15 * 256];  // W_4096^(q r)

template <int Ns>
__device__ __forceinline__ float2 twiddle(int r, int q) {
  return Ns == 16 ? __ldg(&g_fft_tw16[(r - 1) * 16 + q]) : __ldg(&g_fft_tw256[(r - 1) * 256 + q]);
}

// Pass p >= 1 of a transform held in the exchange buffer `s`: read, twiddle,
// 16-point DFT. Leaves the 16 results in v; the caller stores them.
template <int P, int p>
__device__ __forceinline__ void middle_pass(float2* v, const float2* s, int j) {
  constexpr int N = 1 << (4 * P);
  constexpr int T = N / 16;
  constexpr int Ns = 1 << (4 * p);
#pragma unroll
  for (int r = 0; r < 16; ++r) v[r] = s[pad(j + r * T)];
  __syncthreads();
  const int q = j & (Ns - 1);
#pragma unroll
  for (int r = 1; r < 16; ++r) v[r] = cmul(v[r], twiddle<Ns>(r, q));
  dft16(v);
}

// Stores of pass p into the exchange buffer (p < P-1).
template <int p>
__device__ __forceinline__ void exchange_store(const float2* v, float2* s, int j) {
  constexpr int Ns = 1 << (4 * p);
  const int base = (j / Ns) * Ns * 16 + (j & (Ns - 1));
#pragma unroll
  for (int r = 0; r < 16; ++r) s[pad(base + r * Ns)] = v[r];
}

// Passes 1..P-1 on the points of pass 0 (already in v, after its DFT), ending
// with the coalesced store of the last pass to y (point j + r*T).
template <int P>
__device__ __forceinline__ void finish_transform(float2* v, float2* s, int j, bool active, float2* y,
                                                 float sign, float scale) {
  constexpr int T = (1 << (4 * P)) / 16;
  if constexpr (P >= 2) {
    exchange_store<0>(v, s, j);
    __syncthreads();
    middle_pass<P, 1>(v, s, j);
  }
  if constexpr (P >= 3) {
    exchange_store<1>(v, s, j);
    __syncthreads();
    middle_pass<P, 2>(v, s, j);
  }
  if (active) {
#pragma unroll
    for (int r = 0; r < 16; ++r) __stcs(y + j + r * T, make_float2(v[r].x * scale, sign * v[r].y * scale));
  }
}

// Plain kernel: one tile (256 threads, PER transforms) per CTA, inputs loaded
// straight into registers. Used when a pointer is not 16-byte aligned.
template <int P>
__global__ void __launch_bounds__(kFftThreads, 3)
    fft_kernel(const float2* in, float2* out, int64_t batch, int inverse) {
  constexpr int N = 1 << (4 * P);
  constexpr int T = N / 16;
  constexpr int PER = kFftThreads / T;
  constexpr int PADN = N + N / 16;
  extern __shared__ float2 fft_smem[];
  const int j = threadIdx.x % T;
  const int local = threadIdx.x / T;
  const int64_t tr = (int64_t)blockIdx.x * PER + local;
  const bool active = tr < batch;
  const float sign = inverse ? -1.f : 1.f;
  float2 v[16];
  if (active) {
    const float2* x = in + tr * N;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float2 a = __ldcs(x + j + r * T);
      v[r] = make_float2(a.x, sign * a.y);
    }
  }
  dft16(v);
  finish_transform<P>(v, fft_smem + local * PADN, j, active, out + tr * N, sign, inverse ? 1.f / N : 1.f);
}

// ── pipelined kernel ─────────────────────────────────────────────────────────
// A tile is PER consecutive transforms = 4096 points = 32 KiB of contiguous
// input at every length. Persistent CTAs walk the tiles with a stride of the
// grid; one thread streams each CTA's next tiles into two shared buffers with
// bulk asynchronous copies (cp.async.bulk, completion counted on an mbarrier),
// so the loads of tile k+1 and k+2 are in flight while tile k is transformed.
// Stores go straight from registers, 256 contiguous bytes per warp.
constexpr uint32_t kTileBytes = 4096 * sizeof(float2);
constexpr int kPipeSmem = 2 * (int)kTileBytes + (4096 + 256) * (int)sizeof(float2) + 16;
constexpr uint32_t kSpinLimit = 1u << 26;  // bounded wait on a tile's copy

__device__ int g_fft_timeouts;  // tiles whose copy never completed (never expected)

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
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
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

template <int P>
__global__ void __launch_bounds__(kFftThreads, 2)
    fft_pipe_kernel(const float2* in, float2* out, int64_t batch, int inverse) {
  constexpr int N = 1 << (4 * P);
  constexpr int T = N / 16;
  constexpr int PER = kFftThreads / T;
  constexpr int PADN = N + N / 16;
  extern __shared__ __align__(128) unsigned char pipe_smem[];
  float2* buf = reinterpret_cast<float2*>(pipe_smem);                     // 2 tiles of input
  float2* xch = reinterpret_cast<float2*>(pipe_smem + 2 * kTileBytes);    // exchange, padded
  uint64_t* bars = reinterpret_cast<uint64_t*>(pipe_smem + 2 * kTileBytes + (4096 + 256) * sizeof(float2));
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&bars[0]);
  const uint32_t buf0 = (uint32_t)__cvta_generic_to_shared(buf);

  const int j = threadIdx.x % T;
  const int local = threadIdx.x / T;
  const int64_t ntiles = (batch + PER - 1) / PER;
  const float sign = inverse ? -1.f : 1.f;
  const float scale = inverse ? 1.f / N : 1.f;

  auto issue = [&](int64_t tile, int b) {
    const int64_t first = tile * PER;
    const uint32_t bytes = (uint32_t)(min((int64_t)PER, batch - first) * N * sizeof(float2));
    mbar_expect_tx(bar0 + 8 * b, bytes);
    bulk_load(buf0 + b * kTileBytes, in + first * N, bytes, bar0 + 8 * b);
  };
  if (threadIdx.x == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar0 + 8, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (blockIdx.x < ntiles) issue(blockIdx.x, 0);
    if (blockIdx.x + gridDim.x < ntiles) issue(blockIdx.x + gridDim.x, 1);
  }
  int k = 0;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++k) {
    const int b = k & 1;
    bool ok = false;
    for (uint32_t it = 0; it < kSpinLimit && !ok; ++it) ok = mbar_try_wait(bar0 + 8 * b, (k >> 1) & 1);
    if (__syncthreads_or(!ok)) {
      // A copy that never lands: record it and stop this CTA (nothing more is
      // issued, and no thread touches the buffers again).
      if (threadIdx.x == 0) atomicAdd(&g_fft_timeouts, 1);
      return;
    }
    const int64_t tr = tile * PER + local;
    const bool active = tr < batch;
    const float2* x = buf + b * 4096 + local * N;
    float2 v[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float2 a = x[j + r * T];
      v[r] = make_float2(a.x, sign * a.y);
    }
    // Every thread has its points of tile k (buffer b is free again) and has
    // finished reading the exchange buffer for tile k-1.
    __syncthreads();
    if (threadIdx.x == 0 && tile + 2 * gridDim.x < ntiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(tile + 2 * gridDim.x, b);
    }
    dft16(v);
    finish_transform<P>(v, xch + local * PADN, j, active, out + tr * N, sign, scale);
  }
}

// ── twiddle tables: once per device, outside any stream capture ─────────────
static std::mutex g_tw_mu;
static bool g_tw_ready[64] = {};

static mtl_status ensure_twiddles() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(MTL_ERR_CUDA, "fft: no device");
  std::lock_guard<std::mutex> lk(g_tw_mu);
  if (g_tw_ready[dev]) return MTL_OK;
  static float2 t16[15 * 16], t256[15 * 256];
  const double two_pi = 6.283185307179586476925286766559;
  auto w = [&](int m, int n) {
    double a = two_pi * (double)m / (double)n;
    return make_float2((float)std::cos(a), (float)-std::sin(a));
  };
  for (int r = 1; r < 16; ++r) {
    for (int q = 0; q < 16; ++q) t16[(r - 1) * 16 + q] = w(q * r, 256);
    for (int q = 0; q < 256; ++q) t256[(r - 1) * 256 + q] = w(q * r, 4096);
  }
  // A private stream: the caller's stream may be capturing a graph, and the
  // tables must be in place before the first kernel runs, not as graph nodes.
  cudaStream_t st = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_fft_tw16, t16, sizeof t16, 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_fft_tw256, t256, sizeof t256, 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (st) cudaStreamDestroy(st);
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "fft twiddle table: %s", cudaGetErrorString(e));
  g_tw_ready[dev] = true;
  return MTL_OK;
}

static int fft_passes(int n) {
  switch (n) {
    case 16: return 1;
    case 256: return 2;
    case 4096: return 3;
    default: return 0;
  }
}

// Arguments: out (B), in (B), n (i), inverse (i); ndrange = number of transforms.
mtl_status fft_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.ndim != 1) return fail(MTL_ERR_ARGUMENT, "fft: ndrange must be one-dimensional (the number of transforms)");
  const int n = la.a[2].i32;
  if (!fft_passes(n)) return fail(MTL_ERR_UNSUPPORTED, "fft: length %d is not supported (16, 256 or 4096)", n);
  const uint64_t need = (uint64_t)la.nd[0] * (uint64_t)n * 8;
  for (int i = 0; i < 2; ++i)
    if (bytes[i] && bytes[i] < need)
      return fail(MTL_ERR_ARGUMENT, "fft: %s has %llu bytes, %lld transforms of %d ComplexF32 need %llu",
                  i ? "the input" : "the output", (unsigned long long)bytes[i], (long long)la.nd[0], n,
                  (unsigned long long)need);
  const uint64_t o = la.a[0].ptr, x = la.a[1].ptr;
  if (o != x && o < x + need && x < o + need)
    return fail(MTL_ERR_ARGUMENT, "fft: input and output overlap without being the same buffer");
  if ((o | x) & 7) return fail(MTL_ERR_ARGUMENT, "fft: buffers must be 8-byte aligned (ComplexF32)");
  return MTL_OK;
}

template <int P>
static cudaError_t launch_fft(const float2* in, float2* out, int64_t batch, int inverse, int sm_count,
                              cudaStream_t s) {
  constexpr int N = 1 << (4 * P);
  constexpr int PER = kFftThreads / (N / 16);
  const int64_t tiles = (batch + PER - 1) / PER;
  if ((reinterpret_cast<uintptr_t>(in) & 15) == 0) {
    cudaError_t e = cudaFuncSetAttribute(fft_pipe_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPipeSmem);
    if (e != cudaSuccess) return e;
    // Two persistent CTAs per SM (two input tiles + the exchange each).
    const int64_t grid = std::min<int64_t>(tiles, 2 * (int64_t)sm_count);
    fft_pipe_kernel<P><<<(unsigned)grid, kFftThreads, kPipeSmem, s>>>(in, out, batch, inverse);
    return cudaGetLastError();
  }
  const size_t smem = (size_t)PER * (N + N / 16) * sizeof(float2);
  cudaError_t e = cudaFuncSetAttribute(fft_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  fft_kernel<P><<<(unsigned)tiles, kFftThreads, smem, s>>>(in, out, batch, inverse);
  return cudaGetLastError();
}

mtl_status fft_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t batch = la.nd[0];
  const int n = la.a[2].i32;
  if (batch <= 0) return MTL_OK;
  if (batch > (int64_t)0x7fffffff) return fail(MTL_ERR_UNSUPPORTED, "fft: too many transforms in one launch");
  if (mtl_status st = ensure_twiddles()) return st;
  auto* out = reinterpret_cast<float2*>(la.a[0].ptr);
  auto* in = reinterpret_cast<const float2*>(la.a[1].ptr);
  const int inv = la.a[3].i32 != 0;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  switch (fft_passes(n)) {
    case 1: e = launch_fft<1>(in, out, batch, inv, la.sm_count, s); break;
    case 2: e = launch_fft<2>(in, out, batch, inv, la.sm_count, s); break;
    default: e = launch_fft<3>(in, out, batch, inv, la.sm_count, s); break;
  }
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "fft: %s", cudaGetErrorString(e));
  return MTL_OK;
}

// Host: read (and with reset, clear) this file's count of bounded waits that
// ran out on the current device.
int fft_timeouts(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fft_timeouts, sizeof v) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_fft_timeouts, &zero, sizeof zero);
  }
  return v;
}

}  // namespace mtl

