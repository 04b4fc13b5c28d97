// Convolution as an implicit GEMM on the tcgen05 tensor cores, plus the two
// small kernels around it in a CNN forward pass.
//
// conv2d_bf16: out = relu?(conv(in, w)), NHWC bf16 activations, fp32
// accumulation, no bias.
//   GEMM view: M = images × Ho × Wo output pixels, N = Cout, K = kh × kw × Cin,
//   A[m][k] = in[n][ho*s - p + r][wo*s - p + c][ci] with k = (r*kw + c)*Cin + ci
//   (zero outside the image), B[k][co] = w[r][c][ci][co] (HWIO, i.e. K×Cout
//   row-major), C[m][co] = the NHWC output row of pixel m.
//   A is never materialised: four gather warps copy, for each of the 128
//   output pixels of a tile, the eight 16-byte channel chunks of the current
//   64-wide K block straight from the NHWC input into the 128-byte-swizzled
//   shared-memory layout the MMA reads (cp.async with zero fill for padding),
//   then fence the async proxy and arrive on the stage's mbarrier. B (weights)
//   comes in by TMA as in the GEMM. One thread issues tcgen05.mma (M=128, N=BN)
//   into double-buffered TMEM accumulators; four epilogue warps read them back,
//   apply ReLU, round to bf16 and store NHWC rows. Requires Cin a multiple of 8
//   (16-byte chunks) and Cout a multiple of BN (64, 128 or 256).
//
// nchw_to_nhwc_bf16: the network input (NCHW) to NHWC with channels padded
//   with zeros to a multiple of 8.
// gap_fc: global average pool over H×W per channel (fp32), then a fully
//   connected layer (fp32 weights [classes][C]) to fp32 logits.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "../mtl_internal.hpp"
#include "tc_common.cuh"

namespace mtl {

__device__ int g_conv_timeouts;

struct ConvShape {
  int n, h, w, cin, cout, k, stride, pad, ho, wo;
  int taps, cpt;  // kh*kw; 16-byte chunks per pixel (cin / 8)
  int kblocks;    // ceil(taps * cin / 64)
  int64_t mtot;   // n * ho * wo
};

constexpr int kConvStages = 4;
constexpr int kConvThreads = 320;  // warp 0 TMA, 1 MMA, 2-5 epilogue, 6-9 gather
constexpr int kConvGroupM = 16;
constexpr uint32_t kConvA = 128 * 64 * 2;  // 16 KiB

template <int BN>
struct ConvCfg {
  static constexpr uint32_t kB = 64 * BN * 2;
  static constexpr uint32_t kStage = kConvA + kB;
  static constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kSmem = kConvStages * (int)kStage + 2048;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, BN, false, true);
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

template <int BN>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_bf16_kernel(const __grid_constant__ CUtensorMap tmW, const __nv_bfloat16* __restrict__ in,
                     __nv_bfloat16* __restrict__ out, const ConvShape sh, int relu) {
  using Cfg = ConvCfg<BN>;
  extern __shared__ unsigned char csm_raw[];
  unsigned char* ring =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(csm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kConvStages * Cfg::kStage);
  uint64_t* full = bars;
  uint64_t* empty = bars + kConvStages;
  uint64_t* tfull = bars + 2 * kConvStages;
  uint64_t* tempty = bars + 2 * kConvStages + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * kConvStages + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tiles_m = (int)((sh.mtot + 127) / 128), tiles_n = sh.cout / BN;
  const int64_t ntiles = (int64_t)tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kConvStages; ++s) {
      mbar_init(smem_u32(&full[s]), 128 + 1);  // 128 gather threads + the weight producer
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 4);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(Cfg::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  auto coord = [&](int64_t t, int& m0, int& n0) {
    const int r = (int)t;
    const int group = r / (kConvGroupM * tiles_n);
    const int first_m = group * kConvGroupM;
    const int gsize = min(kConvGroupM, tiles_m - first_m);
    const int in_group = r % (kConvGroupM * tiles_n);
    m0 = (first_m + in_group % gsize) * 128;
    n0 = (in_group / gsize) * BN;
  };

  if (warp == 0) {
    // ── weights by TMA ──
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        int m0, n0;
        coord(t, m0, n0);
        for (int kb = 0; kb < sh.kblocks; ++kb) {
          if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) goto w_done;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, Cfg::kB);
          const uint32_t b_dst = smem_u32(ring + s * Cfg::kStage) + kConvA;
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) tma_load_3d(b_dst + c * 8192, &tmW, n0 + c * 64, kb * 64, 0, fb);
          if (++s == kConvStages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    w_done:;
    }
  } else if (warp == 1) {
    // ── MMA ──
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int i = 0;
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
        const int a = i & 1;
        if (!wait_phase(smem_u32(&tempty[a]), ((i >> 1) & 1) ^ 1, abort, &g_conv_timeouts)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(a * BN);
        bool ok = true;
        for (int kb = 0; kb < sh.kblocks; ++kb) {
          if (!wait_phase(smem_u32(&full[s]), ph, abort, &g_conv_timeouts)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + s * Cfg::kStage);
          const uint32_t b_addr = a_addr + kConvA;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma(d, smem_desc(a_addr + kk * 32, 16, 1024), smem_desc(b_addr + kk * 2048, 64 * 128, 1024),
                   Cfg::kIdesc, (kb | kk) != 0);
          tc_commit(smem_u32(&empty[s]));
          if (++s == kConvStages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&tfull[a]));
      }
    }
  } else if (warp < 6) {
    // ── epilogue: ReLU, bf16, NHWC rows ──
    const int q = warp & 3;
    int i = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      const int a = i & 1;
      if (!wait_phase(smem_u32(&tfull[a]), (i >> 1) & 1, abort, &g_conv_timeouts)) break;
      tc_fence_after();
      int m0, n0;
      coord(t, m0, n0);
      const int64_t m = (int64_t)m0 + q * 32 + lane;
      __nv_bfloat16* orow = out + m * sh.cout + n0;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + c * 32, r);
        if (m < sh.mtot) {
          uint32_t pk[16];
#pragma unroll
          for (int v = 0; v < 16; ++v) {
            float x0 = __uint_as_float(r[2 * v]), x1 = __uint_as_float(r[2 * v + 1]);
            if (relu) {
              x0 = fmaxf(x0, 0.f);
              x1 = fmaxf(x1, 0.f);
            }
            __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
            pk[v] = *reinterpret_cast<uint32_t*>(&h);
          }
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[a]));
    }
  } else {
    // ── A gather: thread g owns row g (one output pixel) of every tile ──
    const int g = threadIdx.x - 192;
    constexpr int kLag = 2;  // stages in flight per thread before it signals
    int s = 0, it = 0;
    uint32_t ph = 0;
    int s_sig = 0;  // next stage to signal
    bool alive = true;
    for (int64_t t = blockIdx.x; t < ntiles && alive; t += gridDim.x) {
      int m0, n0;
      coord(t, m0, n0);
      const int64_t m = (int64_t)m0 + g;
      const bool mvalid = m < sh.mtot;
      int n = 0, oh = 0, ow = 0;
      if (mvalid) {
        n = (int)(m / ((int64_t)sh.ho * sh.wo));
        const int rem = (int)(m - (int64_t)n * sh.ho * sh.wo);
        oh = rem / sh.wo;
        ow = rem - oh * sh.wo;
      }
      const int ih0 = oh * sh.stride - sh.pad, iw0 = ow * sh.stride - sh.pad;
      const __nv_bfloat16* img = in + (int64_t)n * sh.h * sh.w * sh.cin;
      for (int kb = 0; kb < sh.kblocks; ++kb) {
        if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) {
          alive = false;
          break;
        }
        const uint32_t a_row = smem_u32(ring + s * Cfg::kStage) + g * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int qk = kb * 8 + j;  // 16-byte chunk index along K
          const int tap = qk / sh.cpt;
          const int ci0 = (qk - tap * sh.cpt) * 8;
          const int r = tap / sh.k, c = tap - r * sh.k;
          const int ih = ih0 + r, iw = iw0 + c;
          const bool ok = mvalid && tap < sh.taps && (unsigned)ih < (unsigned)sh.h && (unsigned)iw < (unsigned)sh.w;
          const __nv_bfloat16* src = ok ? img + ((int64_t)ih * sh.w + iw) * sh.cin + ci0 : in;
          cp_async16(a_row + ((j ^ (g & 7)) << 4), src, ok ? 16u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (++it > kLag) {
          // The copies of the stage issued kLag iterations ago are done: make
          // them visible to the tensor core (async proxy) and signal it.
          asm volatile("cp.async.wait_group %0;" ::"n"(kLag) : "memory");
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(smem_u32(&full[s_sig]));
          if (++s_sig == kConvStages) s_sig = 0;
        }
        if (++s == kConvStages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (alive)
      for (int k = 0; k < min(it, kLag); ++k) {
        mbar_arrive(smem_u32(&full[s_sig]));
        if (++s_sig == kConvStages) s_sig = 0;
      }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmemCols) : "memory");
}

// ── NCHW -> NHWC, channels zero-padded to cpad ──
__global__ void nchw_to_nhwc_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int c,
                                    int cpad, int64_t hw, int64_t n_pixels) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n_pixels; p += stride) {
    const int64_t img = p / hw, off = p - img * hw;
    const __nv_bfloat16* src = in + img * c * hw + off;
    __nv_bfloat16* dst = out + p * cpad;
    if (cpad == 8) {
      __align__(16) __nv_bfloat16 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = k < c ? src[k * hw] : __float2bfloat16_rn(0.f);
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
    } else {
      for (int k = 0; k < cpad; ++k) dst[k] = k < c ? src[k * hw] : __float2bfloat16_rn(0.f);
    }
  }
}

// ── global average pool + fully connected ──
// One CTA per image: the channel means (fp32, summed in pixel order) go to
// shared memory, then each thread computes logits j = tid, tid + blockDim, ...
// as a dot product in channel order.
__global__ void gap_fc_kernel(const __nv_bfloat16* __restrict__ act, const float* __restrict__ w,
                              float* __restrict__ logits, int hw, int c, int classes) {
  extern __shared__ float mean[];
  const int img = blockIdx.x;
  const __nv_bfloat16* a = act + (int64_t)img * hw * c;
  for (int ch = threadIdx.x; ch < c; ch += blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < hw; ++p) s += __bfloat162float(a[(int64_t)p * c + ch]);
    mean[ch] = s / (float)hw;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < classes; j += blockDim.x) {
    const float* wr = w + (int64_t)j * c;
    float s = 0.f;
    for (int ch = 0; ch < c; ++ch) s = fmaf(mean[ch], wr[ch], s);
    logits[(int64_t)img * classes + j] = s;
  }
}

// ── host side ────────────────────────────────────────────────────────────────
// conv2d_bf16 arguments: out (B), in (B), w (B), H, W, Cin, Cout, k, stride,
// pad, relu (i); ndrange = number of images.
static ConvShape conv_shape(const LaunchArgs& la) {
  ConvShape sh{};
  sh.n = (int)la.nd[0];
  sh.h = la.a[3].i32;
  sh.w = la.a[4].i32;
  sh.cin = la.a[5].i32;
  sh.cout = la.a[6].i32;
  sh.k = la.a[7].i32;
  sh.stride = la.a[8].i32;
  sh.pad = la.a[9].i32;
  if (sh.stride > 0) {
    sh.ho = (sh.h + 2 * sh.pad - sh.k) / sh.stride + 1;
    sh.wo = (sh.w + 2 * sh.pad - sh.k) / sh.stride + 1;
  }
  sh.taps = sh.k * sh.k;
  sh.cpt = sh.cin / 8;
  sh.kblocks = (sh.taps * sh.cin + 63) / 64;
  sh.mtot = (int64_t)sh.n * sh.ho * sh.wo;
  return sh;
}

mtl_status conv_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.ndim != 1) return fail(MTL_ERR_ARGUMENT, "conv2d: ndrange must be one-dimensional (the image count)");
  ConvShape sh = conv_shape(la);
  if (sh.n < 0 || sh.h <= 0 || sh.w <= 0 || sh.k <= 0 || sh.stride <= 0 || sh.pad < 0 || sh.cin <= 0 || sh.cout <= 0)
    return fail(MTL_ERR_ARGUMENT, "conv2d: sizes must be positive (padding non-negative)");
  if (sh.ho <= 0 || sh.wo <= 0) return fail(MTL_ERR_ARGUMENT, "conv2d: the filter does not fit the padded input");
  if (sh.cin % 8) return fail(MTL_ERR_UNSUPPORTED, "conv2d: Cin must be a multiple of 8 (pad the channels), got %d", sh.cin);
  if (sh.cout % 64) return fail(MTL_ERR_UNSUPPORTED, "conv2d: Cout must be a multiple of 64, got %d", sh.cout);
  const uint64_t need[3] = {(uint64_t)sh.mtot * sh.cout * 2, (uint64_t)sh.n * sh.h * sh.w * sh.cin * 2,
                            (uint64_t)sh.taps * sh.cin * sh.cout * 2};
  const char* what[3] = {"the output", "the input", "the weights"};
  for (int i = 0; i < 3; ++i) {
    if (bytes[i] && bytes[i] < need[i])
      return fail(MTL_ERR_ARGUMENT, "conv2d: %s has %llu bytes, the launch touches %llu", what[i],
                  (unsigned long long)bytes[i], (unsigned long long)need[i]);
    if (la.a[i].ptr & 15) return fail(MTL_ERR_ARGUMENT, "conv2d: %s must be 16-byte aligned", what[i]);
  }
  return MTL_OK;
}

template <int BN>
static cudaError_t launch_conv(const CUtensorMap& tw, const void* in, void* out, const ConvShape& sh, int relu,
                               int sm_count, cudaStream_t s) {
  using Cfg = ConvCfg<BN>;
  cudaError_t e = cudaFuncSetAttribute(conv_bf16_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((sh.mtot + 127) / 128) * (sh.cout / BN);
  const int grid = (int)std::min<int64_t>(tiles, sm_count);
  conv_bf16_kernel<BN><<<grid, kConvThreads, Cfg::kSmem, s>>>(tw, reinterpret_cast<const __nv_bfloat16*>(in),
                                                              reinterpret_cast<__nv_bfloat16*>(out), sh, relu);
  return cudaGetLastError();
}

mtl_status conv_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  ConvShape sh = conv_shape(la);
  if (sh.mtot == 0) return MTL_OK;
  if (sh.mtot > (int64_t)1 << 31) return fail(MTL_ERR_UNSUPPORTED, "conv2d: more than 2^31 output pixels");
  const int relu = la.a[10].i32 != 0;
  CUtensorMap tw;
  const int BN = sh.cout % 256 == 0 ? 256 : sh.cout % 128 == 0 ? 128 : 64;
  if (mtl_status st = make_bf16_map(&tw, reinterpret_cast<const void*>(la.a[2].ptr), (uint64_t)sh.cout,
                                    (uint64_t)sh.taps * sh.cin, 1, 64))
    return st;
  cudaStream_t s = (cudaStream_t)stream;
  const void* in = reinterpret_cast<const void*>(la.a[1].ptr);
  void* out = reinterpret_cast<void*>(la.a[0].ptr);
  cudaError_t e = BN == 256   ? launch_conv<256>(tw, in, out, sh, relu, la.sm_count, s)
                  : BN == 128 ? launch_conv<128>(tw, in, out, sh, relu, la.sm_count, s)
                              : launch_conv<64>(tw, in, out, sh, relu, la.sm_count, s);
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
  return MTL_OK;
}

// nchw_to_nhwc arguments: out (B), in (B), C, H, W, Cpad (i); ndrange = images.
mtl_status nhwc_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int64_t n = la.nd[0], c = la.a[2].i32, h = la.a[3].i32, w = la.a[4].i32, cp = la.a[5].i32;
  if (la.ndim != 1 || n < 0 || c <= 0 || h <= 0 || w <= 0 || cp < c)
    return fail(MTL_ERR_ARGUMENT, "nchw_to_nhwc: bad sizes (Cpad must be at least C)");
  if (bytes[0] && bytes[0] < (uint64_t)(n * h * w * cp * 2)) return fail(MTL_ERR_ARGUMENT, "nchw_to_nhwc: output too small");
  if (bytes[1] && bytes[1] < (uint64_t)(n * c * h * w * 2)) return fail(MTL_ERR_ARGUMENT, "nchw_to_nhwc: input too small");
  if (cp == 8 && (la.a[0].ptr & 15)) return fail(MTL_ERR_ARGUMENT, "nchw_to_nhwc: output must be 16-byte aligned");
  return MTL_OK;
}

mtl_status nhwc_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = la.nd[0], hw = (int64_t)la.a[3].i32 * la.a[4].i32;
  const int64_t pixels = n * hw;
  if (pixels == 0) return MTL_OK;
  const int64_t blocks = std::min<int64_t>((pixels + 255) / 256, (int64_t)la.sm_count * 16);
  nchw_to_nhwc_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(la.a[1].ptr), reinterpret_cast<__nv_bfloat16*>(la.a[0].ptr),
      la.a[2].i32, la.a[5].i32, hw, pixels);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "nchw_to_nhwc: %s", cudaGetErrorString(e));
}

// gap_fc arguments: logits (B, f32), act (B, bf16 NHWC), w (B, f32), HW, C,
// classes (i); ndrange = images.
mtl_status gapfc_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int64_t n = la.nd[0], hw = la.a[3].i32, c = la.a[4].i32, k = la.a[5].i32;
  if (la.ndim != 1 || n < 0 || hw <= 0 || c <= 0 || k <= 0) return fail(MTL_ERR_ARGUMENT, "gap_fc: bad sizes");
  if (c > 12288) return fail(MTL_ERR_UNSUPPORTED, "gap_fc: more than 12288 channels");
  if (bytes[0] && bytes[0] < (uint64_t)(n * k * 4)) return fail(MTL_ERR_ARGUMENT, "gap_fc: logits too small");
  if (bytes[1] && bytes[1] < (uint64_t)(n * hw * c * 2)) return fail(MTL_ERR_ARGUMENT, "gap_fc: activations too small");
  if (bytes[2] && bytes[2] < (uint64_t)(k * c * 4)) return fail(MTL_ERR_ARGUMENT, "gap_fc: weights too small");
  return MTL_OK;
}

mtl_status gapfc_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = la.nd[0];
  if (n == 0) return MTL_OK;
  const int c = la.a[4].i32;
  gap_fc_kernel<<<(unsigned)n, 256, (size_t)c * 4, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(la.a[1].ptr), reinterpret_cast<const float*>(la.a[2].ptr),
      reinterpret_cast<float*>(la.a[0].ptr), la.a[3].i32, c, la.a[5].i32);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "gap_fc: %s", cudaGetErrorString(e));
}

}  // namespace mtl
