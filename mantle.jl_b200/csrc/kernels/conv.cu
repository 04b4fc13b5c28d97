// Convolution as an implicit GEMM on the tcgen05 tensor cores, plus the two
// small kernels around it in a CNN forward pass.
//
// conv2d_bf16: out = relu?(conv(in, w)), NHWC bf16 activations, fp32
// accumulation, no bias.
//   GEMM view: M = images × Ho × Wo output pixels, N = Cout, K = kh × kw × Cin,
//   A[m][k] = in[n][ho*s - p + r][wo*s - p + c][ci] with k = (r*kw + c)*Cin + ci
//   (zero outside the image), B[k][co] = w[r][c][ci][co] (HWIO, i.e. K×Cout
//   row-major), C[m][co] = the NHWC output row of pixel m.
//   A is never materialised. For Cin a multiple of 64 one TMA load in im2col
//   mode brings a K block's A tile (128 output pixels x 64 channels of one
//   filter tap, padding as zero fill, 128-byte swizzled); for the 8-channel
//   stem input eight such loads (one tap each, 16 B per pixel) fill an
//   unswizzled K-major tile; otherwise four gather warps copy 16-byte channel
//   chunks with cp.async into the swizzled layout, fence the async proxy and
//   arrive on the stage's mbarrier (see AMode). B (weights) comes in by TMA as
//   in the GEMM. One thread issues tcgen05.mma (M=128, N=BN)
//   into double-buffered TMEM accumulators; four epilogue warps read them back,
//   apply ReLU, round to bf16 and store NHWC rows. Requires Cin a multiple of 8
//   (16-byte chunks) and Cout a multiple of BN (64, 128 or 256).
//
// nchw_to_nhwc_bf16: the network input (NCHW) to NHWC with channels padded
//   with zeros to a multiple of 8.
// gap_fc: global average pool over H×W per channel (fp32, into scratch), then
//   a fully connected layer (fp32 weights [C][classes]) to fp32 logits.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "../mtl_internal.hpp"
#include "tc_common.cuh"

namespace mtl {

__device__ int g_conv_timeouts;

struct ConvShape {
  int n, h, w, cin, cout, k, stride, pad, ho, wo;
  int wpad, ws;   // zero columns stored on each side of every input row; stored width w + 2*wpad
  int taps, cpt;  // kh*kw; 16-byte chunks per pixel (cin / 8)
  int kblocks;    // ceil(taps * cin / 64)
  int64_t mtot;   // n * ho * wo
};

constexpr int kConvStages = 4;
constexpr int kConvGroupM = 16;
constexpr uint32_t kConvA = 128 * 64 * 2;  // 16 KiB

// How the A (activation) tile of a K block reaches shared memory.
enum AMode {
  // Four gather warps, one output pixel each, copy 16-byte channel chunks with
  // cp.async into the 128-byte-swizzled layout (any Cin multiple of 8).
  A_GATHER = 0,
  // One TMA load in im2col mode: 128 output pixels x 64 channels of one filter
  // tap, 128-byte swizzled (Cin a multiple of 64).
  A_IM2COL = 1,
  // Eight TMA im2col loads of 128 pixels x 8 channels (16 B per pixel), one per
  // filter tap, each filling a 2 KiB region: the K-major layout without swizzle
  // whose 16-byte K chunks are 2 KiB apart (Cin = 8, the padded stem input).
  A_IM2COL_CHUNK = 2,
  // Cin = 8 with the input stored with `pad` zero columns on each side: a K
  // block is one filter row, and its A tile is ONE im2col load through a view
  // whose "pixels" are 8 consecutive stored pixels (128 B, overlapping by
  // 16*(8 - stride) bytes) stepping `stride` pixels per output column. The
  // filter row is widened to 8 taps; the weights come through a 4-D map whose
  // out-of-range 8th column reads as zero (the stem: 7x7, stride 2).
  A_WINDOW = 3
};

template <int BN, int AM>
struct ConvCfg {
  static constexpr uint32_t kB = 64 * BN * 2;
  static constexpr uint32_t kStage = kConvA + kB;
  static constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kThreads = AM == A_GATHER ? 320 : 192;  // + 4 gather warps
  // 64-wide tiles: two CTAs per SM (96 KiB of stages and 128 TMEM columns
  // each), so one CTA's epilogue and loads overlap the other's MMAs.
  static constexpr int kCtasPerSm = BN == 64 && AM != A_GATHER ? 2 : 1;
  static constexpr int kSmem = kConvStages * (int)kStage + 2048;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, BN, false, true);
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

template <int BN, int AM>
__global__ void __launch_bounds__(ConvCfg<BN, AM>::kThreads, ConvCfg<BN, AM>::kCtasPerSm)
    conv_bf16_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                     const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, const ConvShape sh,
                     int relu) {
  using Cfg = ConvCfg<BN, AM>;
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
      // gather mode: 128 gather threads + the weight producer arrive
      mbar_init(smem_u32(&full[s]), AM == A_GATHER ? 128 + 1 : 1);
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
    // ── TMA: weights, and the activations in the im2col modes ──
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      const int cblocks = sh.cin / 64;
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        int m0, n0;
        coord(t, m0, n0);
        const int img = m0 / (sh.ho * sh.wo);
        const int rem = m0 - img * sh.ho * sh.wo;
        const int oh = rem / sh.wo, ow = rem - (rem / sh.wo) * sh.wo;
        const int bw = ow * sh.stride - sh.pad + sh.wpad, bh = oh * sh.stride - sh.pad;
        int tap = 0, cb = 0;
        for (int kb = 0; kb < sh.kblocks; ++kb) {
          if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) goto w_done;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, Cfg::kB + (AM == A_GATHER ? 0u : kConvA));
          const uint32_t a_dst = smem_u32(ring + s * Cfg::kStage);
          const uint32_t b_dst = a_dst + kConvA;
          if (AM == A_IM2COL) {
            const int r = tap / sh.k, c = tap - (tap / sh.k) * sh.k;
            tma_load_im2col_4d(a_dst, &tmA, cb * 64, bw, bh, img, (uint16_t)c, (uint16_t)r, fb);
            if (++cb == cblocks) {
              cb = 0;
              ++tap;
            }
          } else if (AM == A_WINDOW) {
            // K block kb = filter row kb; the view's pixel index is the output column
            tma_load_im2col_4d(a_dst, &tmA, 0, ow, bh, img, 0, (uint16_t)kb, fb);
          } else if (AM == A_IM2COL_CHUNK) {
            for (int j = 0; j < 8; ++j) {
              // taps past the filter multiply zero weight rows: load any real tap
              const int tj = min(kb * 8 + j, sh.taps - 1);
              const int r = tj / sh.k, c = tj - (tj / sh.k) * sh.k;
              tma_load_im2col_4d(a_dst + j * 2048, &tmA, 0, bw, bh, img, (uint16_t)c, (uint16_t)r, fb);
            }
          }
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) {
            if (AM == A_WINDOW)  // {co, ci, filter column 0..7, filter row kb}
              tma_load_4d(b_dst + c * 8192, &tmW, n0 + c * 64, 0, 0, kb, fb);
            else
              tma_load_3d(b_dst + c * 8192, &tmW, n0 + c * 64, kb * 64, 0, fb);
          }
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
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = AM == A_IM2COL_CHUNK ? smem_desc_noswizzle(a_addr + kk * 4096, 2048, 128)
                                                     : smem_desc(a_addr + kk * 32, 16, 1024);
            tc_mma(d, ad, smem_desc(b_addr + kk * 2048, 64 * 128, 1024), Cfg::kIdesc, (kb | kk) != 0);
          }
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
  } else if (AM == A_GATHER) {
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
      const __nv_bfloat16* img = in + (int64_t)n * sh.h * sh.ws * sh.cin;
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
          const int xs = iw + sh.wpad;  // stored column
          const bool ok = mvalid && tap < sh.taps && (unsigned)ih < (unsigned)sh.h && (unsigned)xs < (unsigned)sh.ws;
          const __nv_bfloat16* src = ok ? img + ((int64_t)ih * sh.ws + xs) * sh.cin + ci0 : in;
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

// ── NCHW -> NHWC, channels zero-padded to cpad, wpad zero columns each side ──
__global__ void nchw_to_nhwc_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int c,
                                    int cpad, int h, int w, int wpad, int64_t n_stored) {
  const int ws = w + 2 * wpad;
  const int64_t hw = (int64_t)h * w;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n_stored; p += stride) {
    const int64_t row = p / ws;  // image * h + y
    const int x = (int)(p - row * ws) - wpad;
    const int64_t img = row / h, y = row - img * h;
    const bool inside = x >= 0 && x < w;
    const __nv_bfloat16* src = in + img * c * hw + y * w + x;
    __nv_bfloat16* dst = out + p * cpad;
    if (cpad == 8) {
      __align__(16) __nv_bfloat16 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = (inside && k < c) ? src[k * hw] : __float2bfloat16_rn(0.f);
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
    } else {
      for (int k = 0; k < cpad; ++k) dst[k] = (inside && k < c) ? src[k * hw] : __float2bfloat16_rn(0.f);
    }
  }
}

// Vector form for W a multiple of 8, C <= 8 and Cpad = 8: a thread converts 8
// consecutive pixels of one row (one 16-byte load per channel plane, eight
// 16-byte stores); thread group w/8 of each row writes the 2*wpad margin pixels.
__global__ void nchw_to_nhwc8_vec_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int c,
                                         int h, int w, int wpad, int64_t rows) {
  const int groups = w / 8 + 1;
  const int ws = w + 2 * wpad;
  const int64_t hw = (int64_t)h * w;
  const int64_t total = rows * groups;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    const int64_t row = t / groups;
    const int g = (int)(t - row * groups);
    uint4* orow = reinterpret_cast<uint4*>(out + row * ws * 8);
    if (g == w / 8) {
      for (int x = 0; x < wpad; ++x) {
        orow[x] = make_uint4(0, 0, 0, 0);
        orow[wpad + w + x] = make_uint4(0, 0, 0, 0);
      }
      continue;
    }
    const int64_t img = row / h, y = row - img * h;
    const __nv_bfloat16* src = in + img * c * hw + y * w + g * 8;
    __align__(16) __nv_bfloat16 plane[8][8];  // [channel][pixel]
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < c)
        *reinterpret_cast<uint4*>(plane[k]) = __ldcs(reinterpret_cast<const uint4*>(src + k * hw));
      else
        *reinterpret_cast<uint4*>(plane[k]) = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int px = 0; px < 8; ++px) {
      __align__(16) __nv_bfloat16 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = plane[k][px];
      orow[wpad + g * 8 + px] = *reinterpret_cast<const uint4*>(v);
    }
  }
}

// ── global average pool + fully connected ──
// Two kernels. gap_kernel: one thread per (image, channel pair), summing the
// H×W pixels in order (fp32, 4-byte coalesced loads), means into scratch.
// fc_kernel: logits = means · W with W stored [C][classes]; a CTA computes a
// 32-image × 64-class tile, staging 32-channel slices of both operands in
// shared memory, each thread 2 images × 4 classes, channels summed in order.
__global__ void gap_kernel(const __nv_bfloat16* __restrict__ act, float* __restrict__ mean, int nimg, int hw,
                           int c) {
  const int pairs = c / 2;
  const int64_t items = (int64_t)nimg * pairs;
  const float inv = 1.f / (float)hw;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < items; t += stride) {
    const int64_t img = t / pairs;
    const int cp = (int)(t - img * pairs);
    const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(act + img * hw * c) + cp;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 7
    for (int p = 0; p < hw; ++p) {
      const float2 v = __bfloat1622float2(a[(int64_t)p * pairs]);
      s0 += v.x;
      s1 += v.y;
    }
    reinterpret_cast<float2*>(mean + img * c)[cp] = make_float2(s0 * inv, s1 * inv);
  }
}

constexpr int kFcTI = 32, kFcTJ = 64, kFcTK = 32;

__global__ void __launch_bounds__(256) fc_kernel(const float* __restrict__ mean, const float* __restrict__ w,
                                                 float* __restrict__ logits, int nimg, int c, int classes) {
  __shared__ float sm[kFcTK][kFcTI + 1];
  __shared__ float sw[kFcTK][kFcTJ];
  const int i0 = blockIdx.x * kFcTI, j0 = blockIdx.y * kFcTJ;
  const int tj = threadIdx.x % 16, ti = threadIdx.x / 16;  // 16 x 16 threads: 4 classes x 2 images each
  float acc[2][4] = {};
  for (int k0 = 0; k0 < c; k0 += kFcTK) {
    for (int e = threadIdx.x; e < kFcTI * kFcTK; e += 256) {
      const int ii = e / kFcTK, kk = e % kFcTK;
      sm[kk][ii] = (i0 + ii < nimg && k0 + kk < c) ? mean[(int64_t)(i0 + ii) * c + k0 + kk] : 0.f;
    }
    for (int e = threadIdx.x; e < kFcTK * kFcTJ; e += 256) {
      const int kk = e / kFcTJ, jj = e % kFcTJ;
      sw[kk][jj] = (k0 + kk < c && j0 + jj < classes) ? w[(int64_t)(k0 + kk) * classes + j0 + jj] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kFcTK; ++kk) {
      const float a0 = sm[kk][2 * ti], a1 = sm[kk][2 * ti + 1];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float b = sw[kk][tj + 16 * q];
        acc[0][q] = fmaf(a0, b, acc[0][q]);
        acc[1][q] = fmaf(a1, b, acc[1][q]);
      }
    }
    __syncthreads();
  }
  for (int r = 0; r < 2; ++r) {
    const int i = i0 + 2 * ti + r;
    if (i >= nimg) continue;
    for (int q = 0; q < 4; ++q) {
      const int j = j0 + tj + 16 * q;
      if (j < classes) logits[(int64_t)i * classes + j] = acc[r][q];
    }
  }
}

// ── host side ────────────────────────────────────────────────────────────────
// conv2d_bf16 arguments: out (B), in (B), w (B), H, W, Cin, Cout, k, stride,
// pad, relu, in_wpad (i); ndrange = number of images. in_wpad: zero columns
// the input buffer stores on each side of every row (its rows are W + 2*in_wpad
// pixels long); the convolution's own padding is still `pad`.
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
  sh.wpad = la.a.size() > 11 ? la.a[11].i32 : 0;
  sh.ws = sh.w + 2 * sh.wpad;
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
  if (sh.n < 0 || sh.h <= 0 || sh.w <= 0 || sh.k <= 0 || sh.stride <= 0 || sh.pad < 0 || sh.cin <= 0 || sh.cout <= 0 ||
      sh.wpad < 0)
    return fail(MTL_ERR_ARGUMENT, "conv2d: sizes must be positive (paddings non-negative)");
  if (sh.ho <= 0 || sh.wo <= 0) return fail(MTL_ERR_ARGUMENT, "conv2d: the filter does not fit the padded input");
  if (sh.cin % 8) return fail(MTL_ERR_UNSUPPORTED, "conv2d: Cin must be a multiple of 8 (pad the channels), got %d", sh.cin);
  if (sh.cout % 64) return fail(MTL_ERR_UNSUPPORTED, "conv2d: Cout must be a multiple of 64, got %d", sh.cout);
  const uint64_t need[3] = {(uint64_t)sh.mtot * sh.cout * 2, (uint64_t)sh.n * sh.h * sh.ws * sh.cin * 2,
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

typedef CUresult (*EncodeIm2colFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const int*, const int*, cuuint32_t, cuuint32_t,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeIm2colFn im2col_fn() {
  static std::once_flag once;
  static EncodeIm2colFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeIm2colFn>(p);
    cudaGetLastError();
  });
  return fn;
}

// The im2col tensor map of an NHWC input: dims {C, W, H, N}; a pixel run walks
// output positions, i.e. base coordinates from -pad in steps of `stride` while
// the filter still fits (lower corner -pad, upper corner pad - (k - 1)); each
// pixel brings `cpp` channels; 128 pixels per load.
static mtl_status make_im2col_map(CUtensorMap* map, const void* in, const ConvShape& sh, uint32_t cpp, bool swizzle,
                                  bool window = false) {
  EncodeIm2colFn enc = im2col_fn();
  if (!enc) return fail(MTL_ERR_CUDA, "conv2d: cuTensorMapEncodeIm2col is not available from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)sh.cin, (cuuint64_t)sh.ws, (cuuint64_t)sh.h, (cuuint64_t)sh.n};
  cuuint64_t strides[3] = {(cuuint64_t)sh.cin * 2, (cuuint64_t)sh.ws * sh.cin * 2, (cuuint64_t)sh.h * sh.ws * sh.cin * 2};
  // Stored margin columns shift the first window start right by wpad and the
  // last one left by wpad.
  int lower[2] = {sh.wpad - sh.pad, -sh.pad};
  int upper[2] = {sh.pad - (sh.k - 1) - sh.wpad, sh.pad - (sh.k - 1)};
  cuuint32_t estr[4] = {1, (cuuint32_t)sh.stride, (cuuint32_t)sh.stride, 1};
  if (window) {
    // "Pixels" of 8 stored pixels (128 B) starting every `stride` stored
    // pixels: pixel u covers stored columns stride*u .. stride*u + 7, the
    // widened filter row of output column u.
    dims[0] = 64;
    dims[1] = (cuuint64_t)sh.wo;
    strides[0] = (cuuint64_t)sh.stride * sh.cin * 2;
    lower[0] = 0;
    upper[0] = 0;
    estr[1] = 1;
  }
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(in), dims, strides, lower, upper, cpp, 128,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTL_ERR_ARGUMENT, "conv2d: im2col tensor map rejected (CUresult %d)", (int)r);
  return MTL_OK;
}

// Weights [k][k][8][cout] read as {cout, ci, filter column, filter row} with
// box {64, 8, 8, 1}: one filter row widened to 8 columns, the 8th (past k)
// out of range and so zero.
static mtl_status make_window_weight_map(CUtensorMap* map, const void* w, const ConvShape& sh) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(MTL_ERR_CUDA, "conv2d: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)sh.cout, 8, (cuuint64_t)sh.k, (cuuint64_t)sh.k};
  cuuint64_t strides[3] = {(cuuint64_t)sh.cout * 2, (cuuint64_t)sh.cout * 8 * 2, (cuuint64_t)sh.cout * 8 * sh.k * 2};
  cuuint32_t box[4] = {64, 8, 8, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTL_ERR_ARGUMENT, "conv2d: weight tensor map rejected (CUresult %d)", (int)r);
  return MTL_OK;
}

template <int BN, int AM>
static cudaError_t launch_conv(const CUtensorMap& tw, const CUtensorMap& ta, const void* in, void* out,
                               const ConvShape& sh, int relu, int sm_count, cudaStream_t s) {
  using Cfg = ConvCfg<BN, AM>;
  cudaError_t e =
      cudaFuncSetAttribute(conv_bf16_kernel<BN, AM>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((sh.mtot + 127) / 128) * (sh.cout / BN);
  const int grid = (int)std::min<int64_t>(tiles, (int64_t)sm_count * Cfg::kCtasPerSm);
  conv_bf16_kernel<BN, AM><<<grid, Cfg::kThreads, Cfg::kSmem, s>>>(
      tw, ta, reinterpret_cast<const __nv_bfloat16*>(in), reinterpret_cast<__nv_bfloat16*>(out), sh, relu);
  return cudaGetLastError();
}

template <int AM>
static cudaError_t launch_conv_bn(int bn, const CUtensorMap& tw, const CUtensorMap& ta, const void* in, void* out,
                                  const ConvShape& sh, int relu, int sm_count, cudaStream_t s) {
  return bn == 256   ? launch_conv<256, AM>(tw, ta, in, out, sh, relu, sm_count, s)
         : bn == 128 ? launch_conv<128, AM>(tw, ta, in, out, sh, relu, sm_count, s)
                     : launch_conv<64, AM>(tw, ta, in, out, sh, relu, sm_count, s);
}

// Which A path a convolution takes. The im2col paths need the im2col corners
// to fit the 4-D encoding ([-128, 127]) and, as a precaution, an input of at
// least 128 KiB (CUTLASS patches im2col descriptors of smaller tensors on
// drivers up to 13.1; those small inputs take the gather path instead).
static int conv_amode(const ConvShape& sh) {
  const uint64_t in_bytes = (uint64_t)sh.n * sh.h * sh.ws * sh.cin * 2;
  const bool corners_ok = sh.pad + sh.wpad <= 127 && sh.pad - (sh.k - 1) - sh.wpad >= -128;
  if (!corners_ok || in_bytes < (128u << 10) || sh.stride > 8) return A_GATHER;
  if (sh.cin % 64 == 0) return A_IM2COL;
  if (sh.cin == 8 && sh.k <= 8 && sh.wpad == sh.pad && sh.stride * (sh.wo - 1) + 8 <= sh.ws) return A_WINDOW;
  if (sh.cin == 8) return A_IM2COL_CHUNK;
  return A_GATHER;
}

mtl_status conv_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  ConvShape sh = conv_shape(la);
  if (sh.mtot == 0) return MTL_OK;
  if (sh.mtot > (int64_t)1 << 31) return fail(MTL_ERR_UNSUPPORTED, "conv2d: more than 2^31 output pixels");
  const int relu = la.a[10].i32 != 0;
  CUtensorMap tw, ta;
  memset(&ta, 0, sizeof ta);
  // The widest tile N that divides Cout (measured: 256-wide tiles beat 128-wide
  // ones even where they leave the last wave of SMs partly idle).
  const int BN = sh.cout % 256 == 0 ? 256 : sh.cout % 128 == 0 ? 128 : 64;
  if (mtl_status st = make_bf16_map(&tw, reinterpret_cast<const void*>(la.a[2].ptr), (uint64_t)sh.cout,
                                    (uint64_t)sh.taps * sh.cin, 1, 64))
    return st;
  const void* in = reinterpret_cast<const void*>(la.a[1].ptr);
  void* out = reinterpret_cast<void*>(la.a[0].ptr);
  const int am = conv_amode(sh);
  if (am == A_IM2COL)
    if (mtl_status st = make_im2col_map(&ta, in, sh, 64, true)) return st;
  if (am == A_IM2COL_CHUNK)
    if (mtl_status st = make_im2col_map(&ta, in, sh, 8, false)) return st;
  if (am == A_WINDOW) {
    if (mtl_status st = make_im2col_map(&ta, in, sh, 64, true, true)) return st;
    if (mtl_status st = make_window_weight_map(&tw, reinterpret_cast<const void*>(la.a[2].ptr), sh)) return st;
    sh.kblocks = sh.k;  // one K block per filter row
  }
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = am == A_IM2COL         ? launch_conv_bn<A_IM2COL>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                  : am == A_IM2COL_CHUNK ? launch_conv_bn<A_IM2COL_CHUNK>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                  : am == A_WINDOW       ? launch_conv_bn<A_WINDOW>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                                         : launch_conv_bn<A_GATHER>(BN, tw, ta, in, out, sh, relu, la.sm_count, s);
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
  return MTL_OK;
}

// nchw_to_nhwc arguments: out (B), in (B), C, H, W, Cpad, Wpad (i); ndrange =
// images. The output rows are W + 2*Wpad pixels of Cpad channels.
mtl_status nhwc_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int64_t n = la.nd[0], c = la.a[2].i32, h = la.a[3].i32, w = la.a[4].i32, cp = la.a[5].i32, wp = la.a[6].i32;
  if (la.ndim != 1 || n < 0 || c <= 0 || h <= 0 || w <= 0 || cp < c || wp < 0)
    return fail(MTL_ERR_ARGUMENT, "nchw_to_nhwc: bad sizes (Cpad must be at least C, Wpad non-negative)");
  if (bytes[0] && bytes[0] < (uint64_t)(n * h * (w + 2 * wp) * cp * 2))
    return fail(MTL_ERR_ARGUMENT, "nchw_to_nhwc: output too small");
  if (bytes[1] && bytes[1] < (uint64_t)(n * c * h * w * 2)) return fail(MTL_ERR_ARGUMENT, "nchw_to_nhwc: input too small");
  if (cp == 8 && (la.a[0].ptr & 15)) return fail(MTL_ERR_ARGUMENT, "nchw_to_nhwc: output must be 16-byte aligned");
  return MTL_OK;
}

mtl_status nhwc_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int h = la.a[3].i32, w = la.a[4].i32, wp = la.a[6].i32;
  const int64_t stored = la.nd[0] * h * (int64_t)(w + 2 * wp);
  if (stored == 0) return MTL_OK;
  const int c = la.a[2].i32;
  if (w % 8 == 0 && c <= 8 && la.a[5].i32 == 8 && (la.a[1].ptr & 15) == 0) {
    const int64_t rows = la.nd[0] * h, work = rows * (w / 8 + 1);
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)la.sm_count * 16);
    nchw_to_nhwc8_vec_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(la.a[1].ptr), reinterpret_cast<__nv_bfloat16*>(la.a[0].ptr), c, h, w,
        wp, rows);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "nchw_to_nhwc: %s", cudaGetErrorString(e));
  }
  const int64_t blocks = std::min<int64_t>((stored + 255) / 256, (int64_t)la.sm_count * 16);
  nchw_to_nhwc_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(la.a[1].ptr), reinterpret_cast<__nv_bfloat16*>(la.a[0].ptr),
      la.a[2].i32, la.a[5].i32, h, w, wp, stored);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "nchw_to_nhwc: %s", cudaGetErrorString(e));
}

// gap_fc arguments: logits (B, f32), act (B, bf16 NHWC), w (B, f32,
// [C][classes]), HW, C, classes (i); ndrange = images.
mtl_status gapfc_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int64_t n = la.nd[0], hw = la.a[3].i32, c = la.a[4].i32, k = la.a[5].i32;
  if (la.ndim != 1 || n < 0 || hw <= 0 || c <= 0 || k <= 0) return fail(MTL_ERR_ARGUMENT, "gap_fc: bad sizes");
  if (c > 1536 || c % 2) return fail(MTL_ERR_UNSUPPORTED, "gap_fc: C must be even and at most 1536");
  if (bytes[0] && bytes[0] < (uint64_t)(n * k * 4)) return fail(MTL_ERR_ARGUMENT, "gap_fc: logits too small");
  if (bytes[1] && bytes[1] < (uint64_t)(n * hw * c * 2)) return fail(MTL_ERR_ARGUMENT, "gap_fc: activations too small");
  if (bytes[2] && bytes[2] < (uint64_t)(k * c * 4)) return fail(MTL_ERR_ARGUMENT, "gap_fc: weights too small");
  return MTL_OK;
}

uint64_t gapfc_workspace(const LaunchArgs& la) { return (uint64_t)la.nd[0] * la.a[4].i32 * 4; }

mtl_status gapfc_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream) {
  const int64_t n = la.nd[0];
  if (n == 0) return MTL_OK;
  const int hw = la.a[3].i32, c = la.a[4].i32, classes = la.a[5].i32;
  if (!ws || ws_bytes < gapfc_workspace(la))
    return fail(MTL_ERR_ARGUMENT, "gap_fc: needs %llu bytes of scratch, got %llu",
                (unsigned long long)gapfc_workspace(la), (unsigned long long)ws_bytes);
  if (n > (int64_t)1 << 24) return fail(MTL_ERR_UNSUPPORTED, "gap_fc: too many images");
  float* mean = reinterpret_cast<float*>(ws);
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t items = n * (c / 2);
  const int64_t blocks = std::min<int64_t>((items + 255) / 256, (int64_t)la.sm_count * 32);
  gap_kernel<<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(la.a[1].ptr), mean, (int)n, hw, c);
  dim3 grid((unsigned)((n + kFcTI - 1) / kFcTI), (unsigned)((classes + kFcTJ - 1) / kFcTJ));
  fc_kernel<<<grid, 256, 0, s>>>(mean, reinterpret_cast<const float*>(la.a[2].ptr), reinterpret_cast<float*>(la.a[0].ptr),
                                 (int)n, c, classes);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "gap_fc: %s", cudaGetErrorString(e));
}

// Host: read (and with reset, clear) this file's count of bounded waits that
// ran out on the current device.
int conv_timeouts(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_conv_timeouts, sizeof v) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_conv_timeouts, &zero, sizeof zero);
  }
  return v;
}

}  // namespace mtl

