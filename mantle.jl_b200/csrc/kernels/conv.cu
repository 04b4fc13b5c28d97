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

#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "../mtl_internal.hpp"
#include "tc_common.cuh"

namespace mtl {

__device__ int g_conv_timeouts;

struct ConvShape {
  int n, h, w, cin, cout, k, stride, pad, ho, wo;
  // Rectangular M tiles (the *_RECT paths): th x tw output pixels of one image,
  // tiles_x x tiles_y of them per image. 0 for flat tiles of 128 pixels.
  int tw, th, tiles_x, tiles_y;
  int wpad, ws;   // zero columns stored on each side of every input row; stored width w + 2*wpad
  int owp, wso;   // the same for the output rows (written as zeros); stored output width wo + 2*owp
  // Stride-2 halo (A_HALO at stride 2): positions per frame row pq = Wo + 1,
  // output rows per tile ph_rows, bytes of one plane frame ph_box_bytes
  int pq, ph_rows, ph_box_bytes;
  // A_HALO: halo rows per channel block, tiles per image, A stages and their
  // bytes, column blocks (Cout / BN)
  int halo_rows, halo_tiles, halo_stages, halo_stage_bytes, nblk;
  int halo_stg;  // the halo epilogue stages its stores (2 KiB per epilogue warp after the barriers)
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
  A_WINDOW = 3,
  // The same with Cin = 4: a window is 8 pixels x 4 channels = 64 B, so a
  // 64-wide K block holds two filter rows, each loaded by one im2col load into
  // its own 8 KiB half of the A stage with the 64-byte swizzle (K-major,
  // 64-byte rows). Half the bytes and half the K of the 8-channel form.
  A_WINDOW4 = 4,
  // Rectangular tiles: a tile is th x tw output pixels of one image, and the
  // A tile of a K block is ONE tiled TMA box — {64 channels, tw, th} with
  // traversal stride `stride` — instead of 128 pixel requests: the im2col
  // request rate, not bytes, bounds the narrow-N layers (Cin % 64 == 0).
  A_RECT = 5,
  // The 4-channel window as rectangles: per filter row one box {8 stored
  // pixels x 4 channels, tw windows, th rows} of the overlapping window view.
  A_WINDOW4_RECT = 6,
  // Stride 1 over a flat halo with resident weights: conv_halo_kernel.
  A_HALO = 7,
  // stride * Cin * 2 == 16 over raw input rows: conv_rows_kernel.
  A_ROWS = 8
};
__host__ __device__ constexpr bool is_rect(int am) { return am == A_RECT || am == A_WINDOW4_RECT; }

// One 32-channel chunk of a warp's 32 output rows: lane l's 64 bytes (pk)
// go to dst (null: this row is not stored) through the warp's 2 KiB of
// staging (16-byte unit v of row l at v ^ ((l >> 1) & 3): no bank conflicts),
// then four lanes per row store whole 64-byte runs, eight rows an instruction,
// instead of every lane writing its own row (32 lines per instruction).
__device__ __forceinline__ void stage_store_chunk(unsigned char* stg, int lane, uint4* dst, const uint32_t (&pk)[16]) {
#pragma unroll
  for (int v = 0; v < 4; ++v)
    *reinterpret_cast<uint4*>(stg + lane * 64 + ((v ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int p = it * 8 + (lane >> 2), u = lane & 3;
    uint4* d = reinterpret_cast<uint4*>(__shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst), p));
    const uint4 val = *reinterpret_cast<const uint4*>(stg + p * 64 + ((u ^ ((p >> 1) & 3)) << 4));
    if (d) d[u] = val;
  }
  __syncwarp();
}

// ReLU and bf16 of 32 fp32 accumulator columns, as 16 packed pairs.
__device__ __forceinline__ void pack_bf16x32(const uint32_t (&r)[32], int relu, uint32_t (&pk)[16]) {
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
}

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
                     int relu, float* __restrict__ part, int ks) {
  using Cfg = ConvCfg<BN, AM>;
  extern __shared__ unsigned char csm_raw[];
  unsigned char* ring =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(csm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kConvStages * Cfg::kStage);
  uint64_t* full = bars;
  uint64_t* empty = bars + kConvStages;
  uint64_t* tfull = bars + 2 * kConvStages;
  uint64_t* tempty = bars + 2 * kConvStages + 2;
  uint64_t* idle = bars + 2 * kConvStages + 4;  // the issuer's MMAs all done (drain before exit)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * kConvStages + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tiles_m = is_rect(AM) ? sh.n * sh.tiles_x * sh.tiles_y : (int)((sh.mtot + 127) / 128);
  const int tiles_n = sh.cout / BN;
  // Work item w: K part w % ks of tile w / ks, K blocks [kb0, kb1) (ks = 1:
  // the whole tile; the gather mode always runs whole tiles).
  const int64_t nitems = (int64_t)tiles_m * tiles_n * ks;
  auto item = [&](int64_t w, int64_t& t, int& kb0, int& kb1) {
    t = w / ks;
    const int r = (int)(w - t * ks);
    kb0 = (int)((int64_t)sh.kblocks * r / ks);
    kb1 = (int)((int64_t)sh.kblocks * (r + 1) / ks);
  };

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
    mbar_init(smem_u32(idle), 1);
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
  pdl_wait();  // the input (and the output's previous readers) are the last kernel's
  pdl_trigger();

  // Tile t -> M tile and column offset, grouped 16 M tiles at a time. Flat
  // tiles start at pixel m0 = mt * 128; rectangles at (img, oh0, ow0).
  auto coord = [&](int64_t t, int& m0, int& n0) {
    const int r = (int)t;
    const int group = r / (kConvGroupM * tiles_n);
    const int first_m = group * kConvGroupM;
    const int gsize = min(kConvGroupM, tiles_m - first_m);
    const int in_group = r % (kConvGroupM * tiles_n);
    m0 = (first_m + in_group % gsize) * (is_rect(AM) ? 1 : 128);  // rect: the M tile's index
    n0 = (in_group / gsize) * BN;
  };
  auto rect_of = [&](int mt, int& img, int& oh0, int& ow0) {
    const int per = sh.tiles_x * sh.tiles_y;
    img = mt / per;
    const int r = mt - img * per;
    oh0 = (r / sh.tiles_x) * sh.th;
    ow0 = (r - (r / sh.tiles_x) * sh.tiles_x) * sh.tw;
  };

  if (warp == 0) {
    // ── TMA: weights, and the activations in the im2col modes ──
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int64_t loads = 0;
      const int cblocks = sh.cin / 64;
      for (int64_t w = blockIdx.x; w < nitems; w += gridDim.x) {
        int64_t t;
        int m0, n0, img, oh, ow, kb0, kb1;
        item(w, t, kb0, kb1);
        coord(t, m0, n0);
        if (is_rect(AM)) {
          rect_of(m0, img, oh, ow);
        } else {
          img = m0 / (sh.ho * sh.wo);
          const int rem = m0 - img * sh.ho * sh.wo;
          oh = rem / sh.wo;
          ow = rem - (rem / sh.wo) * sh.wo;
        }
        const int bw = ow * sh.stride - sh.pad + sh.wpad, bh = oh * sh.stride - sh.pad;
        int tap = kb0 / cblocks, cb = kb0 - (kb0 / cblocks) * cblocks;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) goto w_done;
          const uint32_t fb = smem_u32(&full[s]);
          // rectangles land th*tw rows (the rest of the 128-row tile is unused)
          const uint32_t a_bytes = AM == A_GATHER ? 0u : is_rect(AM) ? (uint32_t)(sh.th * sh.tw * 128) : kConvA;
          mbar_expect_tx(fb, Cfg::kB + a_bytes);
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
          } else if (AM == A_WINDOW4) {
            // K block kb = filter rows 2kb, 2kb+1; a row past the filter meets
            // zero weight rows: load a real one
            for (int half = 0; half < 2; ++half)
              tma_load_im2col_4d(a_dst + half * 8192, &tmA, 0, ow, bh, img, 0, (uint16_t)min(2 * kb + half, sh.k - 1),
                                 fb);
          } else if (AM == A_RECT) {
            const int r = tap / sh.k, c = tap - (tap / sh.k) * sh.k;
            tma_load_4d(a_dst, &tmA, cb * 64, bw + c, bh + r, img, fb);
            if (++cb == cblocks) {
              cb = 0;
              ++tap;
            }
          } else if (AM == A_WINDOW4_RECT) {
            for (int half = 0; half < 2; ++half)
              tma_load_4d(a_dst + half * 8192, &tmA, 0, ow, bh + min(2 * kb + half, sh.k - 1), img, fb);
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
            else if (AM == A_WINDOW4 || AM == A_WINDOW4_RECT)  // {co, ci, column 0..7, rows 2kb, 2kb+1}
              tma_load_4d(b_dst + c * 8192, &tmW, n0 + c * 64, 0, 0, 2 * kb, fb);
            else
              tma_load_3d(b_dst + c * 8192, &tmW, n0 + c * 64, kb * 64, 0, fb);
          }
          ++loads;
          if (++s == kConvStages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    w_done:
      // no load may still be landing when the CTA leaves (an aborted run):
      // wait for the last phase armed on each stage used (the gather mode's
      // stages also count the gather threads' arrivals: not waited for here)
      if (AM != A_GATHER)
        for (int u = 0; u < kConvStages && u < loads; ++u) {
          const int64_t g = loads - 1 - u;
          drain_phase(smem_u32(&full[g % kConvStages]), (uint32_t)((g / kConvStages) & 1));
        }
    }
  } else if (warp == 1) {
    // ── MMA ──
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int i = 0;
      // Descriptors of stage 0; a stage or K step moves only the start address
      // field (address >> 4 in the low bits, which never carries: shared memory
      // is below 256 KiB), so each MMA costs two adds. One thread issues every
      // MMA: with N = 64 an MMA is 32 tensor cycles of work, and the issue loop
      // must stay shorter than that.
      const uint32_t ring0 = smem_u32(ring);
      const uint64_t a0 = AM == A_IM2COL_CHUNK ? smem_desc_noswizzle(ring0, 2048, 128)
                          : (AM == A_WINDOW4 || AM == A_WINDOW4_RECT) ? smem_desc(ring0, 16, 512, 4)
                                                                       : smem_desc(ring0, 16, 1024);
      const uint64_t b0 = smem_desc(ring0 + kConvA, 64 * 128, 1024);
      for (int64_t w = blockIdx.x; w < nitems; w += gridDim.x, ++i) {
        int64_t t;
        int kb0, kb1;
        item(w, t, kb0, kb1);
        const int a = i & 1;
        if (!wait_phase(smem_u32(&tempty[a]), ((i >> 1) & 1) ^ 1, abort, &g_conv_timeouts)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(a * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_phase(smem_u32(&full[s]), ph, abort, &g_conv_timeouts)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t so = (uint64_t)((s * Cfg::kStage) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t ao = AM == A_IM2COL_CHUNK                        ? kk * 256
                                : (AM == A_WINDOW4 || AM == A_WINDOW4_RECT) ? (kk >> 1) * 512 + (kk & 1) * 2
                                                                             : kk * 2;
            if (kk == 0)
              tc_mma(d, a0 + so + ao, b0 + so, Cfg::kIdesc, kb != kb0);
            else
              tc_mma_acc(d, a0 + so + ao, b0 + so + kk * 128, Cfg::kIdesc);
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
      // every MMA issued has finished before TMEM is freed
      tc_commit(smem_u32(idle));
      drain_phase(smem_u32(idle), 0);
    }
  } else if (warp < 6) {
    // ── epilogue: ReLU, bf16, NHWC rows ──
    const int q = warp & 3;
    int i = 0;
    for (int64_t w = blockIdx.x; w < nitems; w += gridDim.x, ++i) {
      int64_t t;
      int kb0, kb1;
      item(w, t, kb0, kb1);
      const int a = i & 1;
      if (!wait_phase(smem_u32(&tfull[a]), (i >> 1) & 1, abort, &g_conv_timeouts)) break;
      tc_fence_after();
      int m0, n0;
      coord(t, m0, n0);
      int64_t m = (int64_t)m0 + q * 32 + lane;  // output pixel of this thread's row
      bool mok;
      int img = 0, y = 0, x = 0;
      if (is_rect(AM)) {
        int oh0, ow0;
        rect_of(m0, img, oh0, ow0);
        const int ml = q * 32 + lane;
        y = oh0 + ml / sh.tw;
        x = ow0 + ml - (ml / sh.tw) * sh.tw;
        mok = ml < sh.th * sh.tw && y < sh.ho && x < sh.wo;
      } else {
        mok = m < sh.mtot;
        if (sh.owp && mok) {
          img = (int)(m / ((int64_t)sh.ho * sh.wo));
          const int rem = (int)(m - (int64_t)img * sh.ho * sh.wo);
          y = rem / sh.wo;
          x = rem - y * sh.wo;
        }
      }
      if (ks > 1) {
        // this K part's fp32 sums, unrounded, into its plane (row = output
        // pixel, in image order); the reduction kernel stores the layer
        float* prow = part + (w - t * ks) * sh.mtot * sh.cout +
                      (is_rect(AM) ? ((int64_t)img * sh.ho + y) * sh.wo + x : m) * sh.cout + n0;
        const uint32_t pbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(pbase + c * 32, r);
          if (mok) {
            float4* dst = reinterpret_cast<float4*>(prow + c * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                   __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tempty[a]));
        continue;
      }
      if (is_rect(AM) || sh.owp) m = ((int64_t)img * sh.ho + y) * sh.wso + sh.owp + x;  // stored output pixel
      // the first and last pixel of an output row also zero the row's margins
      const int margin = sh.owp && mok && (x == 0 || x == sh.wo - 1) ? (x == 0 ? -1 : 1) : 0;
      __nv_bfloat16* orow = out + m * sh.cout + n0;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + c * 32, r);
        if (mok) {
          uint32_t pk[16];
          pack_bf16x32(r, relu, pk);
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          for (int e = 1; margin && e <= sh.owp; ++e) {
            uint4* z = reinterpret_cast<uint4*>(orow + (int64_t)margin * e * sh.cout + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) z[v] = make_uint4(0, 0, 0, 0);
          }
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
    for (int64_t t = blockIdx.x; t < nitems && alive; t += gridDim.x) {  // ks = 1: items are tiles
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

// The second kernel of a layer split over K: output pixel m, channels
// c8..c8+7 = the sum of the ks parts' fp32 planes, added in part order, then
// ReLU and bf16 rounding as in the epilogues; stored at the pixel's stored
// position (rows with owp zero margin columns get them written at their ends).
__global__ void __launch_bounds__(256) conv_splitk_reduce_kernel(const float* __restrict__ part,
                                                                 __nv_bfloat16* __restrict__ out, const ConvShape sh,
                                                                 int relu, int ks) {
  const int g8 = sh.cout / 8;
  const int64_t groups = sh.mtot * g8, plane = sh.mtot * sh.cout;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = g / g8;
    const int c8 = (int)(g - m * g8) * 8;
    const float4* p = reinterpret_cast<const float4*>(part + m * sh.cout + c8);
    float4 a = __ldcs(p), b = __ldcs(p + 1);
    for (int r = 1; r < ks; ++r) {
      const float4* q = reinterpret_cast<const float4*>(part + r * plane + m * sh.cout + c8);
      const float4 u = __ldcs(q), v = __ldcs(q + 1);
      a.x += u.x, a.y += u.y, a.z += u.z, a.w += u.w;
      b.x += v.x, b.y += v.y, b.z += v.z, b.w += v.w;
    }
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t pk[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float x0 = f[2 * e], x1 = f[2 * e + 1];
      if (relu) {
        x0 = fmaxf(x0, 0.f);
        x1 = fmaxf(x1, 0.f);
      }
      __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
      pk[e] = *reinterpret_cast<uint32_t*>(&h);
    }
    int64_t ms = m;
    int lmargin = 0, rmargin = 0;
    if (sh.owp) {
      const int img = (int)(m / ((int64_t)sh.ho * sh.wo));
      const int rem = (int)(m - (int64_t)img * sh.ho * sh.wo);
      const int y = rem / sh.wo, x = rem - (rem / sh.wo) * sh.wo;
      ms = ((int64_t)img * sh.ho + y) * sh.wso + sh.owp + x;
      lmargin = x == 0;
      rmargin = x == sh.wo - 1;
    }
    __nv_bfloat16* o = out + ms * sh.cout + c8;
    *reinterpret_cast<uint4*>(o) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    for (int e = 1; e <= sh.owp; ++e) {
      if (lmargin) *reinterpret_cast<uint4*>(o - (int64_t)e * sh.cout) = make_uint4(0, 0, 0, 0);
      if (rmargin) *reinterpret_cast<uint4*>(o + (int64_t)e * sh.cout) = make_uint4(0, 0, 0, 0);
    }
  }
}

// ── two M tiles per CTA over flat im2col runs (A_IM2COL, Cout % 256 == 0) ──
// These layers wait on their loads, not on the tensor core: with four 48 KiB
// stages in flight a K block took about 950 cycles against 512 of MMAs (the
// loads' latency under load, about 2 us, over the bytes in flight). A CTA
// here computes 256 pixels x 256 channels: per K block it loads two 128-pixel
// A runs and ONE 256-channel weight block (64 KiB, three stages) and issues
// eight N = 256 MMAs, so the same bytes in flight carry half again as many
// MACs. The two accumulators (pixels 0-127 and 128-255 of the tile) fill the
// 512 TMEM columns, so a tile's epilogue does not overlap the next tile.
constexpr int kM2Stages = 3;
constexpr uint32_t kM2B = 64 * 256 * 2;               // one K block of 256 output channels
constexpr uint32_t kM2Stage = 2 * kConvA + kM2B;      // 64 KiB
constexpr int kM2Smem = kM2Stages * (int)kM2Stage + 2048;
constexpr uint32_t kM2Idesc = idesc_bf16_f32(128, 256, false, true);

__global__ void __launch_bounds__(192, 1)
    conv_m2_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                   __nv_bfloat16* __restrict__ out, const ConvShape sh, int relu) {
  constexpr int S = kM2Stages;
  extern __shared__ unsigned char msm_raw[];
  unsigned char* ring =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(msm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + S * kM2Stage);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 1;
  uint64_t* idle = bars + 2 * S + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * S + 3);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tiles_m = (int)((sh.mtot + 255) / 256);
  const int tiles_n = sh.cout / 256;
  const int64_t ntiles = (int64_t)tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), 1);
    }
    mbar_init(smem_u32(tfull), 1);
    mbar_init(smem_u32(tempty), 4);
    mbar_init(smem_u32(idle), 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // the input (and the output's previous readers) are the last kernel's
  pdl_trigger();

  // tile t -> first pixel m0 (256 a tile) and column offset n0, grouped 16 M
  // tiles at a time (the weight blocks of one column range stay in L2)
  auto coord = [&](int64_t t, int64_t& m0, int& n0) {
    const int r = (int)t;
    const int group = r / (kConvGroupM * tiles_n);
    const int first_m = group * kConvGroupM;
    const int gsize = min(kConvGroupM, tiles_m - first_m);
    const int in_group = r % (kConvGroupM * tiles_n);
    m0 = (int64_t)(first_m + in_group % gsize) * 256;
    n0 = (in_group / gsize) * 256;
  };

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int64_t loads = 0;
      const int cblocks = sh.cin / 64;
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        int64_t m0;
        int n0;
        coord(t, m0, n0);
        // the two 128-pixel runs: im2col base corners (a run past the last
        // pixel is not loaded; its rows are never stored)
        int bw[2], bh[2], img[2];
        bool has[2];
        for (int hf = 0; hf < 2; ++hf) {
          const int64_t mr = m0 + hf * 128;
          has[hf] = mr < sh.mtot;
          img[hf] = 0;
          int oh = 0, ow = 0;
          if (has[hf]) {
            img[hf] = (int)(mr / ((int64_t)sh.ho * sh.wo));
            const int rem = (int)(mr - (int64_t)img[hf] * sh.ho * sh.wo);
            oh = rem / sh.wo;
            ow = rem - oh * sh.wo;
          }
          bw[hf] = ow * sh.stride - sh.pad + sh.wpad;
          bh[hf] = oh * sh.stride - sh.pad;
        }
        int tap = 0, cb = 0;
        for (int kb = 0; kb < sh.kblocks; ++kb) {
          if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) goto w_done;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, kM2B + (has[0] ? kConvA : 0u) + (has[1] ? kConvA : 0u));
          const uint32_t a_dst = smem_u32(ring + s * kM2Stage);
          const int r = tap / sh.k, c = tap - (tap / sh.k) * sh.k;
          for (int hf = 0; hf < 2; ++hf)
            if (has[hf])
              tma_load_im2col_4d(a_dst + hf * kConvA, &tmA, cb * 64, bw[hf], bh[hf], img[hf], (uint16_t)c,
                                 (uint16_t)r, fb);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            tma_load_3d(a_dst + 2 * kConvA + q * 8192, &tmW, n0 + q * 64, kb * 64, 0, fb);
          if (++cb == cblocks) {
            cb = 0;
            ++tap;
          }
          ++loads;
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    w_done:
      for (int u = 0; u < S && u < loads; ++u) {
        const int64_t g = loads - 1 - u;
        drain_phase(smem_u32(&full[g % S]), (uint32_t)((g / S) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int i = 0;
      const uint32_t ring0 = smem_u32(ring);
      const uint64_t a0 = smem_desc(ring0, 16, 1024);
      const uint64_t b0 = smem_desc(ring0 + 2 * kConvA, 64 * 128, 1024);
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
        if (!wait_phase(smem_u32(tempty), (i & 1) ^ 1, abort, &g_conv_timeouts)) break;
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < sh.kblocks; ++kb) {
          if (!wait_phase(smem_u32(&full[s]), ph, abort, &g_conv_timeouts)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t so = (uint64_t)((s * kM2Stage) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t b = b0 + so + kk * 128;
            if (kk == 0) {
              tc_mma(tmem, a0 + so, b, kM2Idesc, kb != 0);
              tc_mma(tmem + 256, a0 + so + (kConvA >> 4), b, kM2Idesc, kb != 0);
            } else {
              tc_mma_acc(tmem, a0 + so + kk * 2, b, kM2Idesc);
              tc_mma_acc(tmem + 256, a0 + so + (kConvA >> 4) + kk * 2, b, kM2Idesc);
            }
          }
          tc_commit(smem_u32(&empty[s]));
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(tfull));
      }
      tc_commit(smem_u32(idle));
      drain_phase(smem_u32(idle), 0);
    }
  } else {
    // ── epilogue: each thread two pixels (its TMEM lane in both accumulators) ──
    const int q = warp & 3;
    int i = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      if (!wait_phase(smem_u32(tfull), i & 1, abort, &g_conv_timeouts)) break;
      tc_fence_after();
      int64_t m0;
      int n0;
      coord(t, m0, n0);
      for (int hf = 0; hf < 2; ++hf) {
        int64_t m = m0 + hf * 128 + q * 32 + lane;
        const bool mok = m < sh.mtot;
        int x = 0;
        if (sh.owp && mok) {
          const int img = (int)(m / ((int64_t)sh.ho * sh.wo));
          const int rem = (int)(m - (int64_t)img * sh.ho * sh.wo);
          const int y = rem / sh.wo;
          x = rem - y * sh.wo;
          m = ((int64_t)img * sh.ho + y) * sh.wso + sh.owp + x;  // stored output pixel
        }
        const int margin = sh.owp && mok && (x == 0 || x == sh.wo - 1) ? (x == 0 ? -1 : 1) : 0;
        __nv_bfloat16* orow = out + m * sh.cout + n0;
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(hf * 256);
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          if (mok) {
            uint32_t pk[16];
            pack_bf16x32(r, relu, pk);
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
            for (int e = 1; margin && e <= sh.owp; ++e) {
              uint4* z = reinterpret_cast<uint4*>(orow + (int64_t)margin * e * sh.cout + c * 32);
#pragma unroll
              for (int v = 0; v < 4; ++v) z[v] = make_uint4(0, 0, 0, 0);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(tempty));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
}

// ── stride-1 convolution over a flat halo (A_HALO) ──
// For stride 1 with the input stored with `pad` zero columns on each side,
// output pixel (y, x) at stored position q = y*ws + x + pad reads, for filter
// tap (r, c), the stored pixel q + (r - pad)*ws + (c - pad): every tap is the
// same run of positions shifted by a constant. A tile is 128 consecutive
// stored positions q0.. of one image (margin positions included, their
// results discarded or written as zeros); per 64-channel block ONE tiled TMA
// load brings the halo run q0 - pad*ws - pad .. q0 + 127 + pad*ws + pad
// (rows above and below the image are out of range, so zero), and each tap's
// A operand is that run shifted by r*ws + c rows: the shared-memory
// descriptor's start moves by whole 128-byte rows. The 128-byte swizzle is a
// function of the shared-memory address bits (chunk bits 4-6 XOR row bits
// 7-9), for the TMA writes and the MMA reads alike, so a start that is not
// 1024-byte aligned reads the rows the TMA wrote with base offset 0 (measured:
// every tap exact with 0; with (start >> 7) & 7 all but the aligned tap wrong). The weights of this CTA's
// BN-column block stay resident in shared memory for the whole kernel
// (taps * Cin/64 K blocks of 64 x BN). Roles as in conv_bf16_kernel: warp 0
// loads, warp 1 issues tcgen05.mma into two TMEM accumulators, warps 2-5 read
// them back.
//
// Stride 2 (3x3, padding 1) over the plain NHWC input: the input splits into
// four parity planes (row parity pr, column parity pc), each a tensor map
// over the same memory with pixel stride 2 and row stride 2 (no copy). Output
// pixel (y, x) reads, for tap (r, c), plane row y - 1 (r = 0, odd rows), y
// (r = 1, even rows; r = 2, odd rows) and plane column x - 1 (c = 0, odd
// columns), x (c = 1, even; c = 2, odd). A tile is ph_rows output rows; per
// plane and 64-channel block one TMA load brings the frame of plane rows
// y0 - 1 .. y0 + ph_rows and columns -1 .. Wo - 1 (pq = Wo + 1 positions per
// row; row -1 and column -1 lie outside the input: zeros, the padding). MMA
// row m is output (y0 + m / pq, m % pq) (m % pq == Wo: no pixel), and tap (r,
// c) reads frame position m + (r != 0) * pq + (c != 0): again one shifted run.
template <int BN>
struct HaloCfg {
  static constexpr uint32_t kBBlock = 64 * BN * 2;  // one K block of weights
  // two issuing threads (warps 1 and 6) take alternate tiles, each with two
  // accumulators: four in TMEM
  static constexpr uint32_t kTmemCols = 4 * BN;
  static_assert(4 * BN <= 512, "four accumulators must fit the 512 TMEM columns");
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, BN, false, true);
};

__host__ __device__ inline uint32_t halo_smem_bytes(const ConvShape& sh, uint32_t bblock) {
  return 1024 + (uint32_t)sh.kblocks * bblock + (uint32_t)(sh.halo_stages * sh.halo_stage_bytes) + 256 +
         (sh.halo_stg ? 4 * 2048 : 0);
}

// The epilogue of one halo tile (t-th of the grid), accumulator a, this
// warp's 32 rows (lane quarter q): ReLU, bf16, NHWC stores and margin zeros.
template <int BN, bool PH>
__device__ __forceinline__ void halo_store_tile(const ConvShape& sh, uint32_t tmem, int a, int q, int lane, int64_t t,
                                                __nv_bfloat16* __restrict__ out, int n0, int relu,
                                                unsigned char* stg) {
  const int pitch = PH ? sh.pq : sh.ws;
  const int grid_pos = sh.h * sh.ws;  // stride 1: positions of one image's stored grid
  const int img = (int)(t / sh.halo_tiles);
  const int tt = (int)(t - (int64_t)img * sh.halo_tiles);
  const int m = q * 32 + lane;
  // the output pixel of MMA row m, and whether it is one
  int y, xo;
  bool inner;
  if (PH) {
    const int row = m / pitch;
    y = tt * sh.ph_rows + row;
    xo = m - row * pitch;
    inner = row < sh.ph_rows && y < sh.ho && xo < sh.wo;
  } else {
    const int pos = tt * 128 + m;  // stored position
    y = pos / pitch;
    xo = pos - y * pitch - sh.pad;
    inner = pos < grid_pos && xo >= 0 && xo < sh.wo;
  }
  // Where the row goes (-1: nowhere) and the margin pixels it zeros:
  //   stride 1 with margins == padding: every stored position of the
  //     image, zeros at the margins;
  //   otherwise the output pixel with `owp` margins, the first and last
  //     pixel of a row also zeroing that row's margin (owp <= 1 here).
  int64_t dpos = -1, zpos = -1, zpos2 = -1;
  if (!PH && sh.owp) {
    const int pos = tt * 128 + m;
    if (pos < grid_pos) {
      if (inner)
        dpos = (int64_t)img * grid_pos + pos;
      else
        zpos = (int64_t)img * grid_pos + pos;
    }
  } else if (inner) {
    const int64_t rowb = ((int64_t)img * sh.ho + y) * sh.wso;
    dpos = rowb + sh.owp + xo;
    if (sh.owp && xo == 0) zpos = rowb;
    if (sh.owp && xo == sh.wo - 1) zpos2 = rowb + sh.owp + sh.wo;
  }
  const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN);
  __nv_bfloat16* drow = out + (dpos >= 0 ? dpos : 0) * sh.cout + n0;
  if (stg) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN / 32; c0 += 2) {  // two chunks' TMEM loads in flight before one wait
      uint32_t rr[2][32];
      tmem_ld32_nowait(tbase + c0 * 32, rr[0]);
      tmem_ld32_nowait(tbase + (c0 + 1) * 32, rr[1]);
      tmem_wait_ld();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[16];
        pack_bf16x32(rr[h], relu, pk);
        stage_store_chunk(stg, lane, dpos >= 0 ? reinterpret_cast<uint4*>(drow + (c0 + h) * 32) : nullptr, pk);
      }
    }
  }
#pragma unroll 1
  for (int c = 0; c < (stg ? 0 : BN / 32); ++c) {
    uint32_t r[32];
    tmem_ld32(tbase + c * 32, r);
    if (dpos >= 0) {
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
      uint4* dst = reinterpret_cast<uint4*>(drow + c * 32);
#pragma unroll
      for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
    }
  }
  // margin pixels: zeros over this column block
#pragma unroll 1
  for (int zz = 0; zz < 2; ++zz) {
    const int64_t zp = zz ? zpos2 : zpos;
    if (zp < 0) continue;
    uint4* z = reinterpret_cast<uint4*>(out + zp * sh.cout + n0);
#pragma unroll
    for (int v = 0; v < BN / 8; ++v) z[v] = make_uint4(0, 0, 0, 0);
  }
}

// Taps of phase plane p = 2 * row parity + column parity for a 3x3 stride-2
// filter with padding 1: row parity 0 holds filter row 1, parity 1 rows 0 and
// 2 (row 0 one plane row up); columns likewise (column 0 one plane column
// left, into the zero column 0).
__host__ __device__ constexpr int ph_ntaps(int p) { return ((p >> 1) ? 2 : 1) * ((p & 1) ? 2 : 1); }
__host__ __device__ constexpr int ph_tap_r(int p, int t) {
  return (p >> 1) ? ((t / ((p & 1) ? 2 : 1)) ? 2 : 0) : 1;
}
__host__ __device__ constexpr int ph_tap_c(int p, int t) { return (p & 1) ? ((t % 2) ? 2 : 0) : 1; }

// The A-operand maps of a halo convolution: [0] the stored rows (stride 1),
// or the four parity planes pr * 2 + pc (stride 2).
struct HaloMaps {
  CUtensorMap m[4];
};

template <int BN, bool PH>
__global__ void __launch_bounds__(224, 1)
    conv_halo_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ HaloMaps tmA,
                     __nv_bfloat16* __restrict__ out, const ConvShape sh, int relu) {
  using Cfg = HaloCfg<BN>;
  extern __shared__ unsigned char hsm_raw[];
  unsigned char* bres =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(hsm_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* astage = bres + (size_t)sh.kblocks * Cfg::kBBlock;
  const int S = sh.halo_stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(astage + (size_t)S * sh.halo_stage_bytes);
  uint64_t* full = bars;           // [S], S <= 8
  uint64_t* empty = bars + 8;      // [S]
  uint64_t* tfull = bars + 16;     // [4] accumulator ready
  uint64_t* tempty = bars + 20;    // [4] accumulator drained
  uint64_t* bfull = bars + 24;     // resident weights landed
  uint64_t* idle = bars + 25;      // [2] an issuer's MMAs all done (drain before exit)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 27);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* prog = reinterpret_cast<volatile int*>(tmem_holder + 2);  // [2] loads each issuer has waited for
  unsigned char* stg_base = reinterpret_cast<unsigned char*>(bars) + 256;  // [4] x 2 KiB epilogue staging

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int cblocks = sh.cin / 64;
  const int nb = blockIdx.x % sh.nblk, n0 = nb * BN;
  const int64_t first = blockIdx.x / sh.nblk, step = gridDim.x / sh.nblk;
  const int64_t mtiles = (int64_t)sh.n * sh.halo_tiles;
  // positions per row of the tiled grid: stored input rows (stride 1; the
  // halo run starts pad*ws + pad positions before the tile), or frame rows
  // (stride 2)
  const int pitch = PH ? sh.pq : sh.ws;
  const int halo0 = sh.pad * sh.ws + sh.pad;
  constexpr int kLoads = PH ? 4 : 1;  // stages per (tile, channel block): the planes
  const uint32_t load_bytes = PH ? (uint32_t)sh.ph_box_bytes : (uint32_t)sh.halo_rows * 128;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), 1);
    }
    for (int a = 0; a < 4; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 4);
    }
    mbar_init(smem_u32(bfull), 1);
    mbar_init(smem_u32(&idle[0]), 1);
    mbar_init(smem_u32(&idle[1]), 1);
    *abort = 0;
    prog[0] = prog[1] = 0;
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
  pdl_wait();  // the input (and the output's previous readers) are the last kernel's
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // the weights of column block nb, once
      mbar_expect_tx(smem_u32(bfull), (uint32_t)sh.kblocks * Cfg::kBBlock);
      for (int kb = 0; kb < sh.kblocks; ++kb)
#pragma unroll
        for (int c = 0; c < BN / 64; ++c)
          tma_load_3d(smem_u32(bres + (size_t)kb * Cfg::kBBlock + c * 8192), &tmW, n0 + c * 64, kb * 64, 0,
                      smem_u32(bfull));
      int s = 0;
      uint32_t ph = 0;
      int64_t loads = 0;
      for (int64_t t = first; t < mtiles; t += step) {
        const int64_t tg = PH ? mtiles - 1 - t : t;  // the grid tile (stride 2: last image first)
        const int img = (int)(tg / sh.halo_tiles);
        const int tt = (int)(tg - (int64_t)img * sh.halo_tiles);
        for (int cb = 0; cb < cblocks; ++cb)
          for (int p = 0; p < kLoads; ++p) {
            if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) goto p_done;
            const uint32_t fb = smem_u32(&full[s]);
            const uint32_t dst = smem_u32(astage + (size_t)s * sh.halo_stage_bytes);
            mbar_expect_tx(fb, load_bytes);
            if (PH)  // plane p's frame: rows y0 - 1 .., columns -1 ..
              tma_load_4d(dst, &tmA.m[p], cb * 64, -1, tt * sh.ph_rows - 1, img, fb);
            else
              tma_load_3d(dst, &tmA.m[0], cb * 64, tt * 128 - halo0, img, fb);
            ++loads;
            if (++s == S) {
              s = 0;
              ph ^= 1;
            }
          }
      }
    p_done:
      // no load may still be landing when the CTA leaves (an aborted run):
      // wait for the last phase armed on each stage used
      for (int u = 0; u < S && u < loads; ++u) {
        const int64_t g = loads - 1 - u;  // the last load into stage g % S
        drain_phase(smem_u32(&full[g % S]), (uint32_t)((g / S) & 1));
      }
      drain_phase(smem_u32(bfull), 0);
    }
  } else if (warp == 1 || warp == 6) {
    // Issuer j takes tiles i = j, j + 2, ... (the CTA's i-th tile is first +
    // i * step): one thread issuing N = 64 MMAs leaves the tensor core idle
    // between them, two keep it fed. The g-th load of the producer sits in
    // stage g mod S; tile i's accumulator is i mod 4. Both issuers wait on the
    // same stages, so before waiting for load g an issuer makes sure load g - S
    // (the stage's previous phase) has been waited for: when that was the
    // other issuer's, it checks the other's progress (a parity wait on a stage
    // two phases behind would pass at once).
    const int j = warp == 1 ? 0 : 1;
    const int per_tile = cblocks * kLoads;
    // Load k of a tile (k < S) follows load k - S of the tile ceil((S - k) /
    // per_tile) back: the other issuer's when that is odd (bit k of `cross`;
    // loads k >= S follow one of the same tile).
    uint32_t cross = 0;
    for (int k = 0; k < S && k < per_tile; ++k)
      if (((S - k + per_tile - 1) / per_tile) & 1) cross |= 1u << k;
    if (lane == 0 && wait_phase(smem_u32(bfull), 0, abort, &g_conv_timeouts)) {
      tc_fence_after();
      // descriptors as offsets in 16-byte units from stage 0 / weight block 0
      // (two adds per MMA; see conv_bf16_kernel)
      const uint64_t adesc = smem_desc(smem_u32(astage), 16, 1024);
      const uint64_t bdesc = smem_desc(smem_u32(bres), 64 * 128, 1024);
      const uint32_t bstep = (uint32_t)cblocks * (Cfg::kBBlock >> 4);  // next tap's weights
      const uint32_t prow = (uint32_t)pitch * 8;                          // one grid row of 128 B rows
      for (int i = j; first + (int64_t)i * step < mtiles; i += 2) {
        const int a = i & 3;
        if (!wait_phase(smem_u32(&tempty[a]), ((i >> 2) & 1) ^ 1, abort, &g_conv_timeouts)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(a * BN);
        bool ok = true;
        for (int cb = 0; cb < cblocks && ok; ++cb) {
          const uint64_t bc = bdesc + (uint64_t)((uint32_t)cb * (Cfg::kBBlock >> 4));  // weights of (tap 0, cb)
#pragma unroll
          for (int p = 0; p < kLoads; ++p) {
            const int k = cb * kLoads + p;
            const int g = i * per_tile + k;
            const int s = g % S;
            if (k < S && ((cross >> k) & 1) && g >= S &&
                !wait_progress(&prog[1 - j], g - S + 1, abort, &g_conv_timeouts)) {
              ok = false;
              break;
            }
            if (!wait_phase(smem_u32(&full[s]), (uint32_t)((g / S) & 1), abort, &g_conv_timeouts)) {
              ok = false;
              break;
            }
            prog[j] = g + 1;
            tc_fence_after();
            const uint64_t as = adesc + (uint64_t)(((uint32_t)s * (uint32_t)sh.halo_stage_bytes) >> 4);
            if (!PH) {
              // 3x3 stride 1: all 36 MMAs unrolled, tap (r, c) at r*ws + c rows of 128 B
#pragma unroll
              for (int tap = 0; tap < 9; ++tap) {
                const uint64_t at = as + (uint64_t)((uint32_t)(tap / 3) * prow + (tap % 3) * 8);
                const uint64_t b = bc + (uint64_t)((uint32_t)tap * bstep);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                  if (tap == 0 && kk == 0)
                    tc_mma(d, at, b, Cfg::kIdesc, cb != 0);
                  else
                    tc_mma_acc(d, at + kk * 2, b + kk * 128, Cfg::kIdesc);
                }
              }
            } else {
              // plane p's taps, each at frame position m + (r != 0) * pq + (c != 0)
#pragma unroll
              for (int t = 0; t < ph_ntaps(p); ++t) {
                const int r = ph_tap_r(p, t), c = ph_tap_c(p, t);
                const uint32_t start = (uint32_t)(r == 0 ? 0 : pitch) + (c == 0 ? 0u : 1u);  // rows of 128 B
                const uint64_t at = as + (uint64_t)(start * 8);
                const uint64_t b = bc + (uint64_t)((uint32_t)(r * 3 + c) * bstep);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                  if (p == 0 && t == 0 && kk == 0)
                    tc_mma(d, at, b, Cfg::kIdesc, cb != 0);
                  else
                    tc_mma_acc(d, at + kk * 2, b + kk * 128, Cfg::kIdesc);
                }
              }
            }
            tc_commit(smem_u32(&empty[s]));
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&tfull[a]));
      }
    }
    if (lane == 0) {
      // every MMA this thread issued has finished before TMEM is freed
      tc_commit(smem_u32(&idle[j]));
      drain_phase(smem_u32(&idle[j]), 0);
    }
    __syncwarp();
  } else if (warp < 6) {
    const int q = warp & 3;
    int i = 0;
    for (int64_t t = first; t < mtiles; t += step, ++i) {
      const int a = i & 3;
      if (!wait_phase(smem_u32(&tfull[a]), (i >> 2) & 1, abort, &g_conv_timeouts)) break;
      tc_fence_after();
      halo_store_tile<BN, PH>(sh, tmem, a, q, lane, PH ? mtiles - 1 - t : t, out, n0, relu,
                              sh.halo_stg ? stg_base + q * 2048 : nullptr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[a]));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmemCols) : "memory");
}

// ── epilogue through shared memory and TMA stores ──
// One warp's 32 accumulator rows (TMEM lane quarter) x BN columns: ReLU,
// bf16, written as BN/64 chunks of 32 rows x 128 bytes in the 128-byte-swizzled
// layout (16-byte piece j of row i at position j ^ (i & 7): conflict-free
// shared stores) into `stage` (1024-byte aligned, BN/64 x 4 KiB), then lane 0
// stores each chunk with one TMA store of box {64, 32, 1} at (c0 + 64*chunk,
// c1, c2); rows past the map's second extent are clipped by the TMA. The
// caller takes kRowsStg staging buffers per warp in turn and calls
// epi_stage_acquire() before reusing one (three: with two the stem's epilogue
// warps waited 16 % of their time for a store to finish reading).
constexpr int kRowsStg = 3;
__device__ __forceinline__ void epi_stage_acquire(int lane) {
  if (lane == 0) bulk_wait_read<kRowsStg - 1>();
  __syncwarp();
}

template <int BN>
__device__ __forceinline__ void epi_tma_store(uint32_t tbase, int relu, unsigned char* stage, const CUtensorMap* tmO,
                                              int c0, int c1, int c2, int lane) {
  // every chunk's TMEM load in flight before one wait
  uint32_t rr[BN / 32][32];
#pragma unroll
  for (int c = 0; c < BN / 32; ++c) tmem_ld32_nowait(tbase + c * 32, rr[c]);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < BN / 32; ++c) {
    const uint32_t (&r)[32] = rr[c];
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
    unsigned char* row = stage + (c / 2) * 4096 + lane * 128;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int piece = (c % 2) * 4 + v;
      *reinterpret_cast<uint4*>(row + ((piece ^ (lane & 7)) << 4)) =
          make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) {
#pragma unroll
    for (int c = 0; c < BN / 64; ++c) tma_store_3d(tmO, smem_u32(stage + c * 4096), c0 + c * 64, c1, c2);
    bulk_commit();
  }
}

// ── strided convolution over raw input rows (A_ROWS) ──
// For stride * Cin * 2 == 16 bytes (the 4-channel stem at stride 2) with the
// input stored with `pad` zero columns each side: output pixel x of output row
// oh reads, for filter row r, the 8 stored pixels s*x .. s*x + 7 of input row
// s*oh - pad + r, i.e. the bytes 16*x .. 16*x + 8*Cin*2 - 1 of that stored row.
// As a K-major matrix without swizzle (core matrices of 8 rows x 16 bytes)
// that is row stride 16 B, K-chunk stride (LBO) 16 B and 8-row-group stride
// (SBO) 128 B: the overlapping windows are read straight from the raw row, no
// window copy. A tile is one output row (M = 128 >= Wo; rows past Wo read into
// the next stored row or the stage's slack and are discarded); a stage holds
// the s*(G-1) + k input rows of G consecutive output rows, brought by ONE bulk
// copy (rows outside the image are not copied; their filter rows are skipped).
// The weights of the CTA's 64-column block stay resident (k filter rows of
// 8*Cin K rows, the 8th column zero). The epilogue goes through shared memory
// and TMA stores.
constexpr int kRowsG = 8;  // output rows per stage

__host__ __device__ inline uint32_t rows_smem_bytes(const ConvShape& sh) {
  // 1 KiB alignment slack, resident weights, stages, staging (4 warps x kRowsStg x 4 KiB), barriers
  return 1024 + (uint32_t)sh.kblocks * 8192 + (uint32_t)(sh.halo_stages * sh.halo_stage_bytes) +
         4 * kRowsStg * 4096 + 256;
}

// With SRC_C > 0 the input is the network's NCHW tensor with SRC_C <= CIN
// channels instead: the producer bulk-copies the stage's rows of each channel
// plane into a raw buffer (two, alternating), and a converter warp writes the
// stage's padded NHWC rows from them (margins and the padding channels zero),
// fences the async proxy and signals the stage full: the NCHW -> NHWC pass
// never touches HBM.
__host__ __device__ inline uint32_t rows_raw_bytes(const ConvShape& sh, int src_c) {
  const int hrows = sh.stride * (kRowsG - 1) + sh.k;
  return ((uint32_t)hrows * sh.w * 2 * src_c + 1023) & ~1023u;
}

// Two MMA-issuing warps (1 and kRowsIssuer2) take alternate output rows of
// each stage, each with two of the four TMEM accumulators. From NCHW input two
// converter warps (6 and 8) take alternate rows of each stage (one converter
// was busy 94 % of the time, the issuers waiting 17 % for its rows).
template <int SRC_C>
constexpr int rows_threads() { return SRC_C ? 288 : 224; }

template <int CIN, int KT, int SRC_C>  // KT: the filter size when known at compile time (its interior rows fully unrolled), else 0
__global__ void __launch_bounds__(rows_threads<SRC_C>(), 1)
    conv_rows_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmO,
                     const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, const ConvShape sh,
                     int relu) {
  constexpr int BN = 64;
  constexpr int KQ = CIN / 2;  // K16 steps per filter row (8 pixels x CIN channels)
  constexpr uint32_t kIdesc = idesc_bf16_f32(128, BN, false, true);
  extern __shared__ unsigned char rsm_raw[];
  unsigned char* bres =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(rsm_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* astage = bres + (size_t)sh.kblocks * 8192;
  const int S = sh.halo_stages;
  unsigned char* staging = astage + (size_t)S * sh.halo_stage_bytes;  // [4 warps][kRowsStg][4 KiB]
  unsigned char* raw = staging + 4 * kRowsStg * 4096;                   // SRC_C: [2][raw bytes]
  const uint32_t raw_bytes = SRC_C ? rows_raw_bytes(sh, SRC_C) : 0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + 2 * raw_bytes);
  uint64_t* full = bars;         // [S]
  uint64_t* empty = bars + 4;    // [S], S <= 4; both issuers release a stage
  uint64_t* tfull = bars + 8;    // [4]
  uint64_t* tempty = bars + 12;  // [4]
  uint64_t* bfull = bars + 16;
  uint64_t* raw_full = bars + 17;   // [2]
  uint64_t* raw_empty = bars + 19;  // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 21);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nb = blockIdx.x % sh.nblk, n0 = nb * BN;
  const int64_t first = blockIdx.x / sh.nblk, step = gridDim.x / sh.nblk;
  const int groups = (sh.ho + kRowsG - 1) / kRowsG;
  const int64_t units = (int64_t)sh.n * groups;
  const uint32_t rowbytes = (uint32_t)sh.ws * CIN * 2;
  const int hrows = sh.stride * (kRowsG - 1) + sh.k;  // input rows of a stage

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), SRC_C ? 2 : 1);  // the two converters, or the producer's load
      mbar_init(smem_u32(&empty[i]), 2);
    }
    for (int a = 0; a < 4; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 4);
    }
    mbar_init(smem_u32(bfull), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&raw_full[b]), 1);
      mbar_init(smem_u32(&raw_empty[b]), 2);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(4 * BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // the input (and the output's previous readers) are the last kernel's
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // resident weights: K blocks of 64 rows (8/CIN filter rows of 8*CIN)
      mbar_expect_tx(smem_u32(bfull), (uint32_t)sh.kblocks * 8192);
      for (int kb = 0; kb < sh.kblocks; ++kb)
        tma_load_4d(smem_u32(bres + (size_t)kb * 8192), &tmW, n0, 0, 0, kb * (8 / CIN), smem_u32(bfull));
      int s = 0;
      uint32_t ph = 0;
      for (int64_t u = first; u < units; u += step) {
        const int img = (int)(u / groups);
        const int oh0 = (int)(u - (int64_t)img * groups) * kRowsG;
        const int r0 = oh0 * sh.stride - sh.pad;  // input row of stage row 0
        const int lo = max(r0, 0), hi = min(r0 + hrows, sh.h);
        if (SRC_C) {
          // the stage's rows of each channel plane into raw buffer s % 2 (s counts units here)
          if (!wait_phase(smem_u32(&raw_empty[s]), ph ^ 1, abort, &g_conv_timeouts)) break;
          const uint32_t fb = smem_u32(&raw_full[s]);
          const uint32_t plane = (uint32_t)(hi - lo) * sh.w * 2;
          mbar_expect_tx(fb, plane * SRC_C);
          for (int c = 0; c < SRC_C; ++c)
            bulk_load(smem_u32(raw + (size_t)s * raw_bytes + (size_t)c * hrows * sh.w * 2),
                      in + (((int64_t)img * SRC_C + c) * sh.h + lo) * sh.w, plane, fb);
          if (++s == 2) {
            s = 0;
            ph ^= 1;
          }
          continue;
        }
        if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) break;
        const uint32_t fb = smem_u32(&full[s]);
        const uint32_t bytes = (uint32_t)(hi - lo) * rowbytes;
        mbar_expect_tx(fb, bytes);
        bulk_load(smem_u32(astage + (size_t)s * sh.halo_stage_bytes + (size_t)(lo - r0) * rowbytes),
                  in + ((int64_t)img * sh.h + lo) * sh.ws * CIN, bytes, fb);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1 || warp == (SRC_C ? 7 : 6)) {
    // issuer j: rows t = j, j + 2, ... of every stage; its c-th tile uses
    // accumulator j + 2 * (c & 1)
    const int j = warp == 1 ? 0 : 1;
    if (lane == 0 && wait_phase(smem_u32(bfull), 0, abort, &g_conv_timeouts)) {
      tc_fence_after();
      int s = 0;
      uint32_t ph = 0;
      int c = 0;
      const uint64_t adesc = smem_desc_noswizzle(smem_u32(astage), 16, 128);
      const uint64_t bdesc = smem_desc(smem_u32(bres), 64 * 128, 1024);
      bool ok = true;
      for (int64_t u = first; u < units && ok; u += step) {
        const int img = (int)(u / groups);
        const int oh0 = (int)(u - (int64_t)img * groups) * kRowsG;
        if (!wait_phase(smem_u32(&full[s]), ph, abort, &g_conv_timeouts)) break;
        tc_fence_after();
        const uint64_t as = adesc + (uint64_t)(((uint32_t)s * (uint32_t)sh.halo_stage_bytes) >> 4);
        bool issued = false;
        for (int t = j; t < kRowsG && oh0 + t < sh.ho; t += 2, ++c) {
          const int a = j + 2 * (c & 1);
          if (!wait_phase(smem_u32(&tempty[a]), ((c >> 1) & 1) ^ 1, abort, &g_conv_timeouts)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(a * BN);
          const int ir0 = (oh0 + t) * sh.stride - sh.pad;  // input row of filter row 0
          // filter rows inside the image (the padding rows contribute nothing)
          const int rlo = max(0, -ir0), rhi = min(sh.k, sh.h - ir0);
          const uint64_t at = as + (uint64_t)(((uint32_t)(sh.stride * t) * rowbytes) >> 4);
          const uint32_t arow = rowbytes >> 4;
          constexpr uint32_t brow = 8 * CIN * 8;  // 8*CIN K rows of 128 B per filter row
          if (KT > 0 && rlo == 0 && rhi == KT) {
#pragma unroll
            for (int r = 0; r < KT; ++r)
#pragma unroll
              for (int q = 0; q < KQ; ++q) {
                if (r == 0 && q == 0)
                  tc_mma(d, at, bdesc, kIdesc, 0);
                else
                  tc_mma_acc(d, at + r * arow + q * 2, bdesc + r * brow + q * 128, kIdesc);
              }
          } else {
            uint32_t acc = 0;
            for (int r = rlo; r < rhi; ++r) {
#pragma unroll
              for (int q = 0; q < KQ; ++q) {
                tc_mma(d, at + r * arow + q * 2, bdesc + r * brow + q * 128, kIdesc, acc);
                acc = 1;
              }
            }
          }
          tc_commit(smem_u32(&tfull[a]));
          issued = true;
        }
        if (!ok) break;
        // both issuers release the stage; one with no row here (a short last
        // stage) has nothing in flight on it
        if (issued)
          tc_commit(smem_u32(&empty[s]));
        else
          mbar_arrive(smem_u32(&empty[s]));
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (SRC_C && (warp == 6 || warp == 8)) {
    // ── converters: raw channel-plane rows -> the stage's padded NHWC rows,
    // warp 6 the even rows of a stage, warp 8 the odd ones ──
    const int half = warp == 6 ? 0 : 1;
    int s = 0, rb = 0;
    uint32_t ph = 0, rph = 0;
    for (int64_t u = first; u < units; u += step) {
      const int img = (int)(u / groups);
      const int oh0 = (int)(u - (int64_t)img * groups) * kRowsG;
      const int r0 = oh0 * sh.stride - sh.pad;
      const int lo = max(r0, 0), hi = min(r0 + hrows, sh.h);
      (void)img;
      if (!wait_phase(smem_u32(&raw_full[rb]), rph, abort, &g_conv_timeouts)) break;
      if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) break;
      // lane m of a row converts image pixels 4m..4m+3: one 8-byte load per
      // channel plane, four 8-byte pixel stores; lanes past the row zero the
      // margin pixels
      const unsigned char* src = raw + (size_t)rb * raw_bytes;
      unsigned char* dst = astage + (size_t)s * sh.halo_stage_bytes + (size_t)(lo - r0) * rowbytes;
      const int quads = sh.w / 4;
      const size_t plane = (size_t)hrows * sh.w * 2;
      for (int j = half; j < hi - lo; j += 2) {
        const unsigned char* srow = src + (size_t)j * sh.w * 2;
        unsigned char* drow = dst + (size_t)j * rowbytes;
        for (int m = lane; m < quads; m += 32) {
          uint2 pl[4];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            pl[c] = c < SRC_C ? *reinterpret_cast<const uint2*>(srow + c * plane + (size_t)m * 8) : make_uint2(0, 0);
          // pixel i of the quad: channel c is the i-th bf16 of plane c's load
          uint2 px[4];
          px[0] = make_uint2(__byte_perm(pl[0].x, pl[1].x, 0x5410), __byte_perm(pl[2].x, pl[3].x, 0x5410));
          px[1] = make_uint2(__byte_perm(pl[0].x, pl[1].x, 0x7632), __byte_perm(pl[2].x, pl[3].x, 0x7632));
          px[2] = make_uint2(__byte_perm(pl[0].y, pl[1].y, 0x5410), __byte_perm(pl[2].y, pl[3].y, 0x5410));
          px[3] = make_uint2(__byte_perm(pl[0].y, pl[1].y, 0x7632), __byte_perm(pl[2].y, pl[3].y, 0x7632));
#pragma unroll
          for (int i = 0; i < 4; ++i) *reinterpret_cast<uint2*>(drow + (size_t)(sh.wpad + 4 * m + i) * 8) = px[i];
        }
        if (lane < 2 * sh.wpad) {  // margins: stored pixels 0..wpad-1 and wpad+w..ws-1
          const int x = lane < sh.wpad ? lane : sh.w + lane;
          *reinterpret_cast<uint2*>(drow + (size_t)x * 8) = make_uint2(0, 0);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&full[s]));
        mbar_arrive(smem_u32(&raw_empty[rb]));
      }
      if (++s == S) {
        s = 0;
        ph ^= 1;
      }
      if (++rb == 2) {
        rb = 0;
        rph ^= 1;
      }
    }
  } else if (warp >= 2 && warp < 6) {
    // ── epilogue: one output row per tile, through shared memory and TMA stores ──
    const int q = warp & 3;
    unsigned char* my_stage = staging + (warp - 2) * kRowsStg * 4096;
    int i = 0;
    int cnt[2] = {0, 0};  // tiles seen per issuer
    bool ok = true;
    for (int64_t u = first; u < units && ok; u += step) {
      const int img = (int)(u / groups);
      const int oh0 = (int)(u - (int64_t)img * groups) * kRowsG;
      for (int t = 0; t < kRowsG && oh0 + t < sh.ho; ++t, ++i) {
        const int j = t & 1, c = cnt[j]++;
        const int a = j + 2 * (c & 1);
        if (!wait_phase(smem_u32(&tfull[a]), (c >> 1) & 1, abort, &g_conv_timeouts)) {
          ok = false;
          break;
        }
        tc_fence_after();
        unsigned char* buf = my_stage + (i % kRowsStg) * 4096;
        epi_stage_acquire(lane);
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN);
        const int orow = img * sh.ho + oh0 + t;
        const int x = q * 32 + lane;
        epi_tma_store<BN>(tbase, relu, buf, &tmO, n0, q * 32, orow, lane);
        if (sh.owp && (x == 0 || x == sh.wo - 1)) {  // zero this output row's margin pixels
          __nv_bfloat16* p = out + ((int64_t)orow * sh.wso + sh.owp + x) * sh.cout + n0;
          for (int e = 1; e <= sh.owp; ++e) {
            uint4* z = reinterpret_cast<uint4*>(p + (int64_t)(x == 0 ? -e : e) * sh.cout);
#pragma unroll
            for (int v = 0; v < BN / 8; ++v) z[v] = make_uint4(0, 0, 0, 0);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tempty[a]));
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(4 * BN) : "memory");
}

// ── the 4-channel stride-2 stem with its weights in tensor memory (Cout = 64) ──
// In conv_rows_kernel the MMA's A operand is 128 output pixels and B the 64
// output channels: an M = 128, N = 64, K = 16 MMA reads 6 KiB of operands from
// shared memory for 32 cycles of tensor work. Here the roles swap. A is the
// weights, written once into tensor memory, and B is the overlapping windows
// of one output row's pixels straight from the stage (N = Wo rounded up to 16,
// the same 16-byte row stride trick), so an MMA reads only N x 32 bytes of
// shared memory and does 1.75x the work. A's 128 rows are the 64 filters
// twice: row 64*s + co holds filter co shifted down by s*stride input rows,
// over K = (k + stride) input rows of 8 pixels x 4 channels, so one chain of
// MMAs over those rows computes output rows oh and oh + 1 together. The
// accumulator then holds channels in TMEM lanes and pixels in columns; the
// epilogue reads it back in the mma fragment layout (.16x256b) and writes it
// transposed with stmatrix, one pixel's 8 channels per 16-byte row.
// Measured on B200 (batch 256, 224 x 224): 108-110 us against 143 us for
// conv_rows_kernel. A clock64 trace per role shows what bounds it: the MMAs
// themselves, about 105 cycles each (a row pair's 18 complete ~1900 cycles
// apart) against 56 of nominal tensor work at N = 112, with the two issuers
// (one thread issues a tcgen05.mma about every 75 cycles) and the epilogue
// keeping ahead of them. Roles: warp 0 loads (the weights,
// then the stages), warps 1 and kPairIssuer2 issue, warps 2 .. kPairEpi + 1
// write A into tensor memory and then drain the accumulators, the last two
// warps convert NCHW rows as in conv_rows_kernel.
constexpr int kPairEpi = 8;  // epilogue warps: kPairGroups per TMEM lane quarter, taking alternate 32-pixel chunks
constexpr int kPairGroups = kPairEpi / 4;
constexpr int kPairStg = 2;  // staging chunks of 32 channels x 32 pixels (2 KiB) per epilogue warp
// Converter warps (NCHW input), taking every kPairConv-th row of a stage, and
// raw-row buffers (each holds one stage's channel-plane rows from its bulk copy
// until converted). Measured on B200 at batch 256: 2 or 4 converters and 2 or
// 3 buffers, 108-110 us alike.
constexpr int kPairConv = 2;
constexpr int kPairRaw = 2;

__host__ __device__ inline uint32_t pair_wbytes(const ConvShape& sh) {
  return ((uint32_t)sh.k * sh.k * 4 * 64 * 2 + 1023) & ~1023u;
}
__host__ __device__ inline uint32_t pair_smem_bytes(const ConvShape& sh, int src_c) {
  return 1024 + pair_wbytes(sh) + (uint32_t)(sh.halo_stages * sh.halo_stage_bytes) + kPairEpi * kPairStg * 2048 +
         kPairRaw * rows_raw_bytes(sh, src_c) + 256;
}
// warps: 0 loads, 1 and kPairIssuer2 issue the MMAs, 2 .. kPairEpi + 1 drain the accumulators, the
// kPairConv after kPairIssuer2 convert (NCHW input)
constexpr int kPairIssuer2 = 2 + kPairEpi;
// TMEM accumulators in rotation (pair i into i % kPairAcc); 2 and 3 measured
// alike (108.9 and 108.7-109.1 us), 2 leaves room for rows of 128 pixels
constexpr int kPairAcc = 2;
constexpr int kPairConv0 = kPairIssuer2 + 1;
template <int SRC_C>
constexpr int pair_threads() { return 32 * (kPairConv0 + (SRC_C ? kPairConv : 0)); }

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes, from registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// tcgen05.mma with the A operand in tensor memory (row m in lane m, two bf16
// of K per 32-bit column, the lower K index in the low half).
__device__ __forceinline__ void tc_mma_ta(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma_ta_acc(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, 1, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc)
      : "memory");
}

// 16 TMEM lanes x 32 columns in the mma accumulator-fragment layout
// (.16x256b, four 8-column blocks): block g's registers 4g .. 4g + 3 hold
// (lane t/4, columns 8g + 2(t%4) and + 1) and (lane 8 + t/4, the same columns).
__device__ __forceinline__ void tmem_ld16x256b_x4(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ uint32_t relu_pack_bf16(uint32_t a, uint32_t b, int relu) {
  float x0 = __uint_as_float(a), x1 = __uint_as_float(b);
  if (relu) {
    x0 = fmaxf(x0, 0.f);
    x1 = fmaxf(x1, 0.f);
  }
  const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One 32-pixel chunk of this warp's 32 channels (TMEM lanes from tb, columns
// = pixels): the two 16-lane halves come back in the fragment layout, so each
// 8-channel x 8-pixel block is one stmatrix operand (thread t: channel t/4,
// pixels 2(t%4) and + 1), and stmatrix .trans writes its columns — one pixel's
// 8 channels, 16 bytes — as rows. The staging rows are 64 bytes (32 channels)
// with the 64-byte swizzle (16-byte piece c of pixel row p at c ^ ((p >> 1) &
// 3), which also keeps the eight rows of each block in distinct banks), stored
// by one TMA box {32, 32, 1} at (c0, p0, orow).
__device__ __forceinline__ void pair_chunk_store(uint32_t tb, int relu, unsigned char* buf, const CUtensorMap* tmO,
                                                 int c0, int p0, int orow, int lane) {
  uint32_t lo[16], hi[16];
  tmem_ld16x256b_x4(tb, lo);                           // channels 0-15 of the warp
  tmem_ld16x256b_x4(tb + ((uint32_t)16 << 16), hi);  // channels 16-31
  tmem_wait_ld();
  const int i = lane >> 3, r = lane & 7;  // this lane addresses row r of matrix i
  const uint32_t rowaddr = smem_u32(buf) + (uint32_t)r * 64 + (uint32_t)((i ^ ((r >> 1) & 3)) << 4);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t m0 = relu_pack_bf16(lo[4 * g], lo[4 * g + 1], relu);
    const uint32_t m1 = relu_pack_bf16(lo[4 * g + 2], lo[4 * g + 3], relu);
    const uint32_t m2 = relu_pack_bf16(hi[4 * g], hi[4 * g + 1], relu);
    const uint32_t m3 = relu_pack_bf16(hi[4 * g + 2], hi[4 * g + 3], relu);
    asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(rowaddr + g * 512),
                 "r"(m0), "r"(m1), "r"(m2), "r"(m3)
                 : "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(tmO, smem_u32(buf), c0, p0, orow);
    bulk_commit();
  }
}

template <int KT, int SRC_C>  // KT: the filter size when known at compile time, else 0
__global__ void __launch_bounds__(pair_threads<SRC_C>(), 1)
    conv_rows_pair_kernel(const __grid_constant__ CUtensorMap tmO, const __nv_bfloat16* __restrict__ in,
                          const __nv_bfloat16* __restrict__ wgt, __nv_bfloat16* __restrict__ out, const ConvShape sh,
                          int relu) {
  constexpr int CIN = 4;
  const int nmma = (sh.wo + 15) & ~15;
  const uint32_t idesc = idesc_bf16_f32(128, nmma, false, false);
  const int KR = sh.k + sh.stride;  // input rows under one pair of output rows
  // TMEM: kPairAcc accumulators at columns 0, 128, ... (measured: one at
  // column 112 instead of 128 makes the stem 5 % slower), A in the last
  // 16*KR columns (its position does not matter)
  const uint32_t kAcol = 512 - 16 * (uint32_t)KR;
  extern __shared__ unsigned char psm_raw[];
  unsigned char* wsm =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(psm_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* astage = wsm + pair_wbytes(sh);
  const int S = sh.halo_stages;
  unsigned char* staging = astage + (size_t)S * sh.halo_stage_bytes;  // [kPairEpi warps][kPairStg][2 KiB]
  unsigned char* raw = staging + kPairEpi * kPairStg * 2048;           // SRC_C: [kPairRaw][raw bytes]
  const uint32_t raw_bytes = SRC_C ? rows_raw_bytes(sh, SRC_C) : 0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + kPairRaw * raw_bytes);
  uint64_t* full = bars;         // [S], S <= 4
  uint64_t* empty = bars + 4;    // [S]
  uint64_t* tfull = bars + 8;    // [kPairAcc]
  uint64_t* tempty = bars + 11;  // [kPairAcc]
  uint64_t* bfull = bars + 14;   // the weights in shared memory
  uint64_t* afull = bars + 15;   // A in tensor memory
  uint64_t* raw_full = bars + 16;   // [kPairRaw], kPairRaw <= 4
  uint64_t* raw_empty = bars + 20;  // [kPairRaw]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t first = blockIdx.x, step = gridDim.x;
  const int groups = (sh.ho + kRowsG - 1) / kRowsG;
  const int64_t units = (int64_t)sh.n * groups;
  const uint32_t rowbytes = (uint32_t)sh.ws * CIN * 2;
  const int hrows = sh.stride * (kRowsG - 1) + sh.k;  // input rows of a stage

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), SRC_C ? kPairConv : 1);  // the converters, or the producer's load
      mbar_init(smem_u32(&empty[i]), 2);  // both issuers
    }
    for (int a = 0; a < kPairAcc; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), kPairEpi);
    }
    mbar_init(smem_u32(bfull), 1);
    mbar_init(smem_u32(afull), kPairEpi);
    for (int b = 0; b < kPairRaw; ++b) {
      mbar_init(smem_u32(&raw_full[b]), 1);
      mbar_init(smem_u32(&raw_empty[b]), kPairConv);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // the input, the weights (and the output's previous readers) are the last kernel's
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t wbytes = (uint32_t)sh.k * sh.k * CIN * 64 * 2;
      mbar_expect_tx(smem_u32(bfull), wbytes);
      bulk_load(smem_u32(wsm), wgt, wbytes, smem_u32(bfull));
      int s = 0;
      uint32_t ph = 0;
      int64_t g = 0;  // loads issued (raw buffers with NCHW input, else stages)
      for (int64_t u = first; u < units; u += step, ++g) {
        const int img = (int)(u / groups);
        const int oh0 = (int)(u - (int64_t)img * groups) * kRowsG;
        const int r0 = oh0 * sh.stride - sh.pad;  // input row of stage row 0
        const int lo = max(r0, 0), hi = min(r0 + hrows, sh.h);
        if (SRC_C) {
          // the stage's rows of each channel plane into raw buffer s (s counts units here)
          if (!wait_phase(smem_u32(&raw_empty[s]), ph ^ 1, abort, &g_conv_timeouts)) break;  // (g not issued)
          const uint32_t fb = smem_u32(&raw_full[s]);
          const uint32_t plane = (uint32_t)(hi - lo) * sh.w * 2;
          mbar_expect_tx(fb, plane * SRC_C);
          for (int c = 0; c < SRC_C; ++c)
            bulk_load(smem_u32(raw + (size_t)s * raw_bytes + (size_t)c * hrows * sh.w * 2),
                      in + (((int64_t)img * SRC_C + c) * sh.h + lo) * sh.w, plane, fb);
          if (++s == kPairRaw) {
            s = 0;
            ph ^= 1;
          }
          continue;
        }
        if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) break;
        const uint32_t fb = smem_u32(&full[s]);
        const uint32_t bytes = (uint32_t)(hi - lo) * rowbytes;
        mbar_expect_tx(fb, bytes);
        bulk_load(smem_u32(astage + (size_t)s * sh.halo_stage_bytes + (size_t)(lo - r0) * rowbytes),
                  in + ((int64_t)img * sh.h + lo) * sh.ws * CIN, bytes, fb);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
      // leaving on an abort: the loads in flight land before the CTA's shared
      // memory is released (the last kPairRaw or S of them)
      if (*abort) {
        const int nb = SRC_C ? kPairRaw : S;
        for (int64_t q = g > nb ? g - nb : 0; q < g; ++q)
          drain_phase(smem_u32(SRC_C ? &raw_full[q % nb] : &full[q % nb]), (uint32_t)((q / nb) & 1));
      }
    }
  } else if (warp == 1 || warp == kPairIssuer2) {
    // two issuers take alternate row pairs (issuing tcgen05.mma from one
    // thread is the slower side here: about 75 cycles an MMA against 56 of
    // tensor work); pair i goes into accumulator i % kPairAcc
    const int j = warp == 1 ? 0 : 1;
    if (lane == 0 && wait_phase(smem_u32(afull), 0, abort, &g_conv_timeouts)) {
      tc_fence_after();
      int s = 0, i = 0;
      uint32_t ph = 0;
      const uint64_t bdesc = smem_desc_noswizzle(smem_u32(astage), 16, 128);
      const uint32_t arow = rowbytes >> 4;
      const uint32_t abase = tmem + kAcol;
      bool ok = true;
      int last = -1;  // the last pair whose MMAs this thread committed
      for (int64_t u = first; u < units && ok; u += step) {
        const int img = (int)(u / groups);
        const int oh0 = (int)(u - (int64_t)img * groups) * kRowsG;
        if (!wait_phase(smem_u32(&full[s]), ph, abort, &g_conv_timeouts)) break;
        tc_fence_after();
        const uint64_t bs = bdesc + (uint64_t)(((uint32_t)s * (uint32_t)sh.halo_stage_bytes) >> 4);
        bool issued = false;
        for (int t = 0; t < kRowsG && oh0 + t < sh.ho; t += 2, ++i) {
          if ((i & 1) != j) continue;
          const int a = i % kPairAcc;
          if (!wait_phase(smem_u32(&tempty[a]), ((i / kPairAcc) & 1) ^ 1, abort, &g_conv_timeouts)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(a * 128);
          const int ir0 = (oh0 + t) * sh.stride - sh.pad;  // input row of K row 0 (filter row 0 of row oh0 + t)
          const int rlo = max(0, -ir0), rhi = min(KR, sh.h - ir0);  // K rows inside the image
          const uint64_t bt = bs + (uint64_t)(((uint32_t)(sh.stride * t) * rowbytes) >> 4);
          if (KT > 0 && rlo == 0 && rhi == KT + 2) {
#pragma unroll
            for (int r = 0; r < KT + 2; ++r)
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                if (r == 0 && q == 0)
                  tc_mma_ta(d, abase, bt, idesc, 0);
                else
                  tc_mma_ta_acc(d, abase + (uint32_t)(16 * r + 8 * q), bt + r * arow + q * 2, idesc);
              }
          } else {
            uint32_t acc = 0;
            for (int r = rlo; r < rhi; ++r)
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                tc_mma_ta(d, abase + (uint32_t)(16 * r + 8 * q), bt + r * arow + q * 2, idesc, acc);
                acc = 1;
              }
          }
          tc_commit(smem_u32(&tfull[a]));
          issued = true;
          last = i;
        }
        if (!ok) break;
        // both issuers release the stage; one with no pair here (a short last
        // stage) has nothing in flight on it
        if (issued)
          tc_commit(smem_u32(&empty[s]));
        else
          mbar_arrive(smem_u32(&empty[s]));
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
      // leaving on an abort: this thread's MMAs finish before the TMEM is freed
      if (*abort && last >= 0) drain_phase(smem_u32(&tfull[last % kPairAcc]), (uint32_t)((last / kPairAcc) & 1));
    }
  } else if (SRC_C && warp >= kPairConv0) {
    // ── converters: raw channel-plane rows -> the stage's padded NHWC rows,
    // converter i taking rows i, i + kPairConv, ... of a stage ──
    const int half = warp - kPairConv0;
    int s = 0, rb = 0;
    uint32_t ph = 0, rph = 0;
    for (int64_t u = first; u < units; u += step) {
      const int img = (int)(u / groups);
      const int oh0 = (int)(u - (int64_t)img * groups) * kRowsG;
      const int r0 = oh0 * sh.stride - sh.pad;
      const int lo = max(r0, 0), hi = min(r0 + hrows, sh.h);
      (void)img;
      if (!wait_phase(smem_u32(&raw_full[rb]), rph, abort, &g_conv_timeouts)) break;
      if (!wait_phase(smem_u32(&empty[s]), ph ^ 1, abort, &g_conv_timeouts)) break;
      const unsigned char* src = raw + (size_t)rb * raw_bytes;
      unsigned char* dst = astage + (size_t)s * sh.halo_stage_bytes + (size_t)(lo - r0) * rowbytes;
      const int quads = sh.w / 4;
      const size_t plane = (size_t)hrows * sh.w * 2;
      for (int jr = half; jr < hi - lo; jr += kPairConv) {
        const unsigned char* srow = src + (size_t)jr * sh.w * 2;
        unsigned char* drow = dst + (size_t)jr * rowbytes;
        for (int m = lane; m < quads; m += 32) {
          uint2 pl[4];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            pl[c] = c < SRC_C ? *reinterpret_cast<const uint2*>(srow + c * plane + (size_t)m * 8) : make_uint2(0, 0);
          uint2 px[4];
          px[0] = make_uint2(__byte_perm(pl[0].x, pl[1].x, 0x5410), __byte_perm(pl[2].x, pl[3].x, 0x5410));
          px[1] = make_uint2(__byte_perm(pl[0].x, pl[1].x, 0x7632), __byte_perm(pl[2].x, pl[3].x, 0x7632));
          px[2] = make_uint2(__byte_perm(pl[0].y, pl[1].y, 0x5410), __byte_perm(pl[2].y, pl[3].y, 0x5410));
          px[3] = make_uint2(__byte_perm(pl[0].y, pl[1].y, 0x7632), __byte_perm(pl[2].y, pl[3].y, 0x7632));
#pragma unroll
          for (int i = 0; i < 4; ++i) *reinterpret_cast<uint2*>(drow + (size_t)(sh.wpad + 4 * m + i) * 8) = px[i];
        }
        if (lane < 2 * sh.wpad) {  // margins: stored pixels 0..wpad-1 and wpad+w..ws-1
          const int x = lane < sh.wpad ? lane : sh.w + lane;
          *reinterpret_cast<uint2*>(drow + (size_t)x * 8) = make_uint2(0, 0);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&full[s]));
        mbar_arrive(smem_u32(&raw_empty[rb]));
      }
      if (++s == S) {
        s = 0;
        ph ^= 1;
      }
      if (++rb == kPairRaw) {
        rb = 0;
        rph ^= 1;
      }
    }
  } else if (warp >= 2 && warp < 2 + kPairEpi) {
    // TMEM lanes 32q .. 32q + 31: A rows (and accumulator rows) 64 * srow + co;
    // epilogue warp group h takes the 32-pixel chunks h, h + kPairGroups, ...
    const int q = warp & 3, h = (warp - 2) / 4;
    const int m = 32 * q + lane, srow = m >> 6, co = m & 63;
    const uint32_t lanes = (uint32_t)(32 * q) << 16;
    bool ok = wait_phase(smem_u32(bfull), 0, abort, &g_conv_timeouts);
    if (ok) {
      // A row m, K row r: column jc holds K elements 2jc and 2jc + 1 (pixel
      // jc/2 of the window, channels 2(jc&1) and 2(jc&1) + 1) of filter row
      // r - srow*stride; the two halves write alternate K rows
      const uint16_t* wl = reinterpret_cast<const uint16_t*>(wsm);  // HWIO [k][k][4][64]
      for (int r = h; r < KR; r += kPairGroups) {
        const int fr = r - srow * sh.stride;
        uint32_t pk[16];
#pragma unroll
        for (int jc = 0; jc < 16; ++jc) {
          const int px = jc >> 1, ch = (jc & 1) * 2;
          uint32_t v = 0;
          if (fr >= 0 && fr < sh.k && px < sh.k) {
            const int e = ((fr * sh.k + px) * CIN + ch) * 64 + co;
            v = (uint32_t)wl[e] | ((uint32_t)wl[e + 64] << 16);
          }
          pk[jc] = v;
        }
        tmem_st16(tmem + lanes + kAcol + (uint32_t)(16 * r), pk);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(afull));
    // ── epilogue: per pair of output rows, this warp's 32 channels of row srow ──
    unsigned char* my_stage = staging + (warp - 2) * kPairStg * 2048;
    int sb = 0, i = 0;
    const int nch = (sh.wo + 31) / 32;  // 32-pixel chunks of a row (at most 4)
    for (int64_t u = first; u < units && ok; u += step) {
      const int img = (int)(u / groups);
      const int oh0 = (int)(u - (int64_t)img * groups) * kRowsG;
      for (int t = 0; t < kRowsG && oh0 + t < sh.ho; t += 2, ++i) {
        const int a = i % kPairAcc;
        if (!wait_phase(smem_u32(&tfull[a]), (i / kPairAcc) & 1, abort, &g_conv_timeouts)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int oh = oh0 + t + srow;
        if (oh < sh.ho && h < nch) {
          const int orow = img * sh.ho + oh;
          const uint32_t tb = tmem + lanes + (uint32_t)(a * 128);
          for (int ck = h; ck < nch; ck += kPairGroups) {
            unsigned char* buf = my_stage + (sb++ % kPairStg) * 2048;
            if (lane == 0) bulk_wait_read<kPairStg - 1>();
            __syncwarp();
            pair_chunk_store(tb + 32 * ck, relu, buf, &tmO, 32 * (q & 1), 32 * ck, orow, lane);
          }
          if (sh.owp) {  // this row's margin pixels, this warp's channels (group 0 writes them)
            if (h == 0) {
              __nv_bfloat16* p = out + (int64_t)orow * sh.wso * 64 + co;
              for (int e = 0; e < sh.owp; ++e) {
                p[(int64_t)e * 64] = __float2bfloat16(0.f);
                p[(int64_t)(sh.owp + sh.wo + e) * 64] = __float2bfloat16(0.f);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tempty[a]));
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
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

// Vector form for W a multiple of 8, C <= CP and CP = 4 or 8: a thread
// converts 8 consecutive pixels of one row (one 16-byte load per channel
// plane, one CP-channel store per pixel); thread group w/8 of each row writes
// the 2*wpad margin pixels.
template <int CP>
__global__ void nchw_to_nhwc_vec_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int c,
                                        int h, int w, int wpad, int64_t rows) {
  using Px = typename std::conditional<CP == 8, uint4, uint2>::type;
  const int groups = w / 8 + 1;
  const int ws = w + 2 * wpad;
  const int64_t hw = (int64_t)h * w;
  const int64_t total = rows * groups;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    const int64_t row = t / groups;
    const int g = (int)(t - row * groups);
    Px* orow = reinterpret_cast<Px*>(out + row * ws * CP);
    if (g == w / 8) {
      Px z;
      memset(&z, 0, sizeof z);
      for (int x = 0; x < wpad; ++x) {
        orow[x] = z;
        orow[wpad + w + x] = z;
      }
      continue;
    }
    const int64_t img = row / h, y = row - img * h;
    const __nv_bfloat16* src = in + img * c * hw + y * w + g * 8;
    __align__(16) __nv_bfloat16 plane[CP][8];  // [channel][pixel]
#pragma unroll
    for (int k = 0; k < CP; ++k) {
      if (k < c)
        *reinterpret_cast<uint4*>(plane[k]) = __ldcs(reinterpret_cast<const uint4*>(src + k * hw));
      else
        *reinterpret_cast<uint4*>(plane[k]) = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int px = 0; px < 8; ++px) {
      __align__(16) __nv_bfloat16 v[CP];
#pragma unroll
      for (int k = 0; k < CP; ++k) v[k] = plane[k][px];
      orow[wpad + g * 8 + px] = *reinterpret_cast<const Px*>(v);
    }
  }
}

// ── global average pool + fully connected ──
// Two kernels. gap_kernel: one CTA per image; its threads split the channels
// into V-pair (4V-byte) units and the pixels into G interleaved groups, each
// thread summing its unit over its pixels (fp32, loads independent of one
// another), then the G partial sums per channel are added in group order into
// the mean (scratch). fc_kernel: logits = means · W with W stored [C][classes]
// (below).
constexpr int kGapMaxGroups = 8;

// blockIdx.y: a slice of cw = c / gridDim.y channels (one slice for large
// batches; several when the images alone leave SMs idle).
template <int V>
__global__ void __launch_bounds__(256) gap_kernel(const __nv_bfloat16* __restrict__ act, float* __restrict__ mean,
                                                  int hw, int c) {
  extern __shared__ float part[];  // [G][cw]
  const int img = blockIdx.x;
  const int cw = c / (int)gridDim.y, c0 = (int)blockIdx.y * cw;
  pdl_wait();
  pdl_trigger();
  const int units = cw / (2 * V);
  const int G = max(1, min(kGapMaxGroups, (int)blockDim.x / units));
  const __nv_bfloat16* a = act + (int64_t)img * hw * c + c0;
  for (int idx = threadIdx.x; idx < G * units; idx += blockDim.x) {
    const int g = idx / units, u = idx - (idx / units) * units;
    float sum[2 * V];
#pragma unroll
    for (int e = 0; e < 2 * V; ++e) sum[e] = 0.f;
    const __nv_bfloat16* src = a + u * 2 * V;
#pragma unroll 4
    for (int p = g; p < hw; p += G) {
      if (V == 4) {
        const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src + (int64_t)p * c));
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[e]));
          sum[2 * e] += f.x;
          sum[2 * e + 1] += f.y;
        }
      } else {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + (int64_t)p * c));
        sum[0] += f.x;
        sum[1] += f.y;
      }
    }
#pragma unroll
    for (int e = 0; e < 2 * V; ++e) part[g * cw + u * 2 * V + e] = sum[e];
  }
  __syncthreads();
  const float inv = 1.f / (float)hw;
  for (int ch = threadIdx.x; ch < cw; ch += blockDim.x) {
    float t = 0.f;
    for (int g = 0; g < G; ++g) t += part[g * cw + ch];
    mean[(int64_t)img * c + c0 + ch] = t * inv;
  }
}

// fc_kernel: a cluster of kFcSplit CTAs computes one 32-image x 256-class tile
// of logits, CTA z of the cluster summing channels [z*kc, (z+1)*kc) (kc = C/8
// rounded up to 4, or to 8 with POOL). Each thread keeps 4 images x 8 classes
// in registers over 64-channel slices staged in shared memory; the partial
// tiles then meet over distributed shared memory, CTA z adding images [4z,
// 4z+4) of the tile from all eight partials in rank order (so the result does
// not depend on timing). POOL: the kernel pools its own slices from the
// activations instead of reading gap_kernel's means — thread (image t/8,
// channel octet t%8) adds its 8 channels over the HW pixels in pixel order
// with 16-byte loads, the weight slice's loads issued first — so pooling and
// FC are one launch and each image's means are computed by the CTAs that use
// them (four class blocks each read the 12.8 MB of a batch-256 network once,
// from L2). Measured on B200 in the batch-256 CNN the two forms take the same
// step time within 0.5 %, so the two-kernel form stays the default and
// MTL_GAPFC_FUSED=1 selects this one.
constexpr int kFcImg = 32, kFcCls = 256, kFcKc = 64, kFcSplit = 8;
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// d = a * b + d on both 32-bit halves (sm_100 packed FP32)
__device__ __forceinline__ void fma_f32x2(uint64_t& d, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}
constexpr int kFcSmem = (kFcKc * kFcImg + kFcKc * kFcCls) * 4;  // 72 KiB; the partial tile reuses it

// CLS: classes per tile, 256 (the thread's eight classes 4jg.., 128+4jg..) or
// 64 for small batches (the thread's two classes 2jg, 2jg + 1: four times the
// CTAs over the same work). Each logit is summed in the same order either way.
template <bool POOL, int CLS = kFcCls>
__global__ void __cluster_dims__(1, 1, kFcSplit) __launch_bounds__(256)
    fc_kernel(const float* __restrict__ mean, const __nv_bfloat16* __restrict__ act, int hw,
              const float* __restrict__ w, float* __restrict__ logits, int nimg, int c, int classes, int vec) {
  static_assert(CLS == 256 || (CLS == 64 && !POOL), "class tiles of 256, or 64 without pooling");
  constexpr int NQ = CLS / 64;  // class pairs a thread
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) float fsm[];
  float* sm = fsm;                   // [k][image]
  float* sw = fsm + kFcKc * kFcImg;  // [k][class]
  const int i0 = blockIdx.x * kFcImg, j0 = blockIdx.y * CLS;
  const int z = (int)cluster.block_rank();
  const int ig = threadIdx.x / 32, jg = threadIdx.x % 32;  // images 4ig..4ig+3; classes as above
  const int kc = POOL ? (((c + kFcSplit - 1) / kFcSplit) + 7) & ~7 : (((c + kFcSplit - 1) / kFcSplit) + 3) & ~3;
  const int kbeg = min(c, z * kc), kend = min(c, kbeg + kc);
  uint64_t acc2[4][NQ];  // images 4ig + r; class pairs of the thread
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < NQ; ++q) acc2[r][q] = 0;
  auto load_w = [&](int k0, int kn) {
#pragma unroll
    for (int it = 0; it < kFcKc * CLS / 4 / 256; ++it) {
      const int e = threadIdx.x + it * 256;
      const int kk = e / (CLS / 4), jj = 4 * (e % (CLS / 4));
      const float4 v = kk < kn && j0 + jj < classes
                           ? *reinterpret_cast<const float4*>(w + (int64_t)(k0 + kk) * classes + j0 + jj)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(sw + kk * CLS + jj) = v;
    }
  };
  pdl_wait();
  pdl_trigger();
  for (int k0 = kbeg; k0 < kend; k0 += kFcKc) {
    const int kn = min(kFcKc, kend - k0);
    if (POOL) {  // vec holds; kn, C multiples of 8
      load_w(k0, kn);
      const int ii = threadIdx.x >> 3, o = threadIdx.x & 7;
      float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (i0 + ii < nimg && 8 * o < kn) {
        const __nv_bfloat16* src = act + (int64_t)(i0 + ii) * hw * c + k0 + 8 * o;
#pragma unroll 7
        for (int p = 0; p < hw; ++p) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + (int64_t)p * c));
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[e]));
            s8[2 * e] += f.x;
            s8[2 * e + 1] += f.y;
          }
        }
      }
      const float inv = 1.f / (float)hw;
#pragma unroll
      for (int e = 0; e < 8; ++e) sm[(8 * o + e) * kFcImg + ii] = s8[e] * inv;
    } else if (vec) {  // kn, C and classes multiples of 4: whole float4s are in or out of range
      // fixed trip counts, fully unrolled: every load of the slice is in flight at once
#pragma unroll
      for (int it = 0; it < kFcImg * kFcKc / 4 / 256; ++it) {
        const int e = threadIdx.x + it * 256;
        const int ii = e / (kFcKc / 4), kk = 4 * (e % (kFcKc / 4));
        const float4 v = i0 + ii < nimg && kk < kn ? *reinterpret_cast<const float4*>(mean + (int64_t)(i0 + ii) * c + k0 + kk)
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        sm[(kk + 0) * kFcImg + ii] = v.x;
        sm[(kk + 1) * kFcImg + ii] = v.y;
        sm[(kk + 2) * kFcImg + ii] = v.z;
        sm[(kk + 3) * kFcImg + ii] = v.w;
      }
      load_w(k0, kn);
    } else {
      for (int e = threadIdx.x; e < kFcImg * kFcKc; e += 256) {
        const int ii = e / kFcKc, kk = e % kFcKc;
        sm[kk * kFcImg + ii] = i0 + ii < nimg && kk < kn ? mean[(int64_t)(i0 + ii) * c + k0 + kk] : 0.f;
      }
      for (int e = threadIdx.x; e < kFcKc * CLS; e += 256) {
        const int kk = e / CLS, jj = e % CLS;
        sw[kk * CLS + jj] = kk < kn && j0 + jj < classes ? w[(int64_t)(k0 + kk) * classes + j0 + jj] : 0.f;
      }
    }
    __syncthreads();
    // packed f32x2 FMAs (two classes an instruction; each half is an IEEE
    // fma, so the sums are those of one fmaf per product in channel order)
#pragma unroll 4
    for (int kk = 0; kk < kFcKc; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(sm + kk * kFcImg + 4 * ig);
      uint64_t b2[NQ];
      if constexpr (CLS == 256) {
        const float4 b0 = *reinterpret_cast<const float4*>(sw + kk * CLS + 4 * jg);
        const float4 b1 = *reinterpret_cast<const float4*>(sw + kk * CLS + 128 + 4 * jg);
        b2[0] = pack_f32x2(b0.x, b0.y);
        b2[1] = pack_f32x2(b0.z, b0.w);
        b2[2] = pack_f32x2(b1.x, b1.y);
        b2[3] = pack_f32x2(b1.z, b1.w);
      } else {
        const float2 b = *reinterpret_cast<const float2*>(sw + kk * CLS + 2 * jg);
        b2[0] = pack_f32x2(b.x, b.y);
      }
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint64_t a2 = pack_f32x2(av[r], av[r]);
#pragma unroll
        for (int q = 0; q < NQ; ++q) fma_f32x2(acc2[r][q], a2, b2[q]);
      }
    }
    __syncthreads();
  }
  float acc[4][2 * NQ];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < NQ; ++q) unpack_f32x2(acc2[r][q], acc[r][2 * q], acc[r][2 * q + 1]);
  // the partial tile [image][class] into this CTA's shared memory
  float* part = fsm;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float* row = part + (4 * ig + r) * CLS;
    if constexpr (CLS == 256) {
      *reinterpret_cast<float4*>(row + 4 * jg) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
      *reinterpret_cast<float4*>(row + 128 + 4 * jg) = make_float4(acc[r][4], acc[r][5], acc[r][6], acc[r][7]);
    } else {
      *reinterpret_cast<float2*>(row + 2 * jg) = make_float2(acc[r][0], acc[r][1]);
    }
  }
  cluster.sync();
  // all of a thread's remote loads in flight before the in-order sums
  constexpr int kOut = 4 * CLS / 256;  // outputs a thread: CTA z adds images [4z, 4z + 4) of the tile
  float pv[kOut][kFcSplit];
#pragma unroll
  for (int it = 0; it < kOut; ++it) {
    const int e = threadIdx.x + it * 256;
    const int ii = 4 * z + e / CLS, jj = e % CLS;
#pragma unroll
    for (int rk = 0; rk < kFcSplit; ++rk) pv[it][rk] = cluster.map_shared_rank(part, rk)[ii * CLS + jj];
  }
#pragma unroll
  for (int it = 0; it < kOut; ++it) {
    const int e = threadIdx.x + it * 256;
    const int ii = 4 * z + e / CLS, jj = e % CLS;
    float sum = 0.f;
#pragma unroll
    for (int rk = 0; rk < kFcSplit; ++rk) sum += pv[it][rk];
    if (i0 + ii < nimg && j0 + jj < classes) logits[(int64_t)(i0 + ii) * classes + j0 + jj] = sum;
  }
  cluster.sync();  // no CTA leaves while another still reads its partial tile
}

// ── host side ────────────────────────────────────────────────────────────────
// conv2d_bf16 arguments: out (B), in (B), w (B), H, W, Cin, Cout, k, stride,
// pad, relu, in_wpad, out_wpad (i); ndrange = number of images. in_wpad: zero
// columns the input buffer stores on each side of every row (its rows are
// W + 2*in_wpad pixels long); the convolution's own padding is still `pad`.
// out_wpad: the same for the output rows, which the kernel writes as zeros.
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
  sh.wpad = la.a[11].i32;
  sh.owp = la.a[12].i32;
  sh.ws = sh.w + 2 * sh.wpad;
  if (sh.stride > 0) {
    sh.ho = (sh.h + 2 * sh.pad - sh.k) / sh.stride + 1;
    sh.wo = (sh.w + 2 * sh.pad - sh.k) / sh.stride + 1;
  }
  sh.wso = sh.wo + 2 * sh.owp;
  sh.taps = sh.k * sh.k;
  sh.cpt = sh.cin / 8;
  sh.kblocks = (sh.taps * sh.cin + 63) / 64;
  sh.mtot = (int64_t)sh.n * sh.ho * sh.wo;
  return sh;
}

static int conv_amode(ConvShape& sh);

mtl_status conv_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.ndim != 1) return fail(MTL_ERR_ARGUMENT, "conv2d: ndrange must be one-dimensional (the image count)");
  ConvShape sh = conv_shape(la);
  if (sh.n < 0 || sh.h <= 0 || sh.w <= 0 || sh.k <= 0 || sh.stride <= 0 || sh.pad < 0 || sh.cin <= 0 || sh.cout <= 0 ||
      sh.wpad < 0 || sh.owp < 0 || sh.owp > 64)
    return fail(MTL_ERR_ARGUMENT, "conv2d: sizes must be positive (paddings non-negative, out_wpad at most 64)");
  if (sh.ho <= 0 || sh.wo <= 0) return fail(MTL_ERR_ARGUMENT, "conv2d: the filter does not fit the padded input");
  const int am = conv_amode(sh);
  if (sh.cin % 8 && !(sh.cin == 4 && (am == A_WINDOW4 || am == A_WINDOW4_RECT || am == A_ROWS)))
    return fail(MTL_ERR_UNSUPPORTED,
                "conv2d: Cin must be a multiple of 8 (pad the channels), or 4 for an input stored with its padding "
                "columns (at least 128 KiB), got %d",
                sh.cin);
  if (sh.cout % 64) return fail(MTL_ERR_UNSUPPORTED, "conv2d: Cout must be a multiple of 64, got %d", sh.cout);
  const uint64_t need[3] = {(uint64_t)sh.n * sh.ho * sh.wso * sh.cout * 2, (uint64_t)sh.n * sh.h * sh.ws * sh.cin * 2,
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
    // "Pixels" of 8 stored pixels (8*Cin elements: 128 B at Cin = 8, 64 B at
    // Cin = 4) starting every `stride` stored pixels: pixel u covers stored
    // columns stride*u .. stride*u + 7, the widened filter row of output column u.
    dims[0] = (cuuint64_t)8 * sh.cin;
    dims[1] = (cuuint64_t)sh.wo;
    strides[0] = (cuuint64_t)sh.stride * sh.cin * 2;
    lower[0] = 0;
    upper[0] = 0;
    estr[1] = 1;
  }
  const CUtensorMapSwizzle sw = !swizzle ? CU_TENSOR_MAP_SWIZZLE_NONE
                                : cpp * 2 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(in), dims, strides, lower, upper, cpp, 128,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTL_ERR_ARGUMENT, "conv2d: im2col tensor map rejected (CUresult %d)", (int)r);
  return MTL_OK;
}

// Weights [k][k][Cin][cout] read as {cout, ci, filter column, filter row} with
// box {64, Cin, 8, 8/Cin}: 64 K rows = one (Cin = 8) or two (Cin = 4) filter
// rows widened to 8 columns; the 8th column and rows past k are out of range
// and so zero.
static mtl_status make_window_weight_map(CUtensorMap* map, const void* w, const ConvShape& sh) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(MTL_ERR_CUDA, "conv2d: cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t ci = (cuuint64_t)sh.cin;
  cuuint64_t dims[4] = {(cuuint64_t)sh.cout, ci, (cuuint64_t)sh.k, (cuuint64_t)sh.k};
  cuuint64_t strides[3] = {(cuuint64_t)sh.cout * 2, (cuuint64_t)sh.cout * ci * 2, (cuuint64_t)sh.cout * ci * sh.k * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)ci, 8, (cuuint32_t)(8 / ci)};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTL_ERR_ARGUMENT, "conv2d: weight tensor map rejected (CUresult %d)", (int)r);
  return MTL_OK;
}

template <int BN, int AM>
static cudaError_t launch_conv(const CUtensorMap& tw, const CUtensorMap& ta, const void* in, void* out,
                               const ConvShape& sh, int relu, int sm_count, cudaStream_t s, float* part = nullptr,
                               int ks = 1) {
  using Cfg = ConvCfg<BN, AM>;
  cudaError_t e =
      cudaFuncSetAttribute(conv_bf16_kernel<BN, AM>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  if (e != cudaSuccess) return e;
  if (AM == A_GATHER) ks = 1;
  const int64_t mtiles = is_rect(AM) ? (int64_t)sh.n * sh.tiles_x * sh.tiles_y : (sh.mtot + 127) / 128;
  const int64_t items = mtiles * (sh.cout / BN) * ks;
  const int grid = (int)std::min<int64_t>(items, (int64_t)sm_count * Cfg::kCtasPerSm);
  e = launch_pdl(conv_bf16_kernel<BN, AM>, grid, Cfg::kThreads, Cfg::kSmem, s, tw, ta,
                 reinterpret_cast<const __nv_bfloat16*>(in), reinterpret_cast<__nv_bfloat16*>(out), sh, relu, part,
                 ks);
  if (e != cudaSuccess || ks == 1) return e;
  const int64_t groups = sh.mtot * (sh.cout / 8);
  const int rgrid = (int)std::min<int64_t>((groups + 255) / 256, (int64_t)sm_count * 8);
  conv_splitk_reduce_kernel<<<rgrid, 256, 0, s>>>(part, reinterpret_cast<__nv_bfloat16*>(out), sh, relu, ks);
  return cudaGetLastError();
}

// K parts per tile for a one-run layer with fewer tiles than SMs (1: no
// split): the largest count, up to 8, that leaves every part at least 4 K
// blocks and keeps the work items to one round over the SMs. Taken when
// it is at least three parts and saves more than 28 K blocks a tile: the
// parts' fp32 planes and the reduction launch cost about 10 us, which only the
// deep layers win back (measured at batch 32: 7x7x512 layers 38 -> 24 us and
// 26 -> 22 us with five parts; a 14x14x256 layer with three parts 20 -> 23
// us; at batch 64 two parts made the 7x7x512 layers slower). Small batches,
// such as one GPU's share of a batch split over eight, leave most SMs idle on
// those layers without it. MTL_CONV_SPLITK=0 keeps every layer whole.
static int conv_split(const ConvShape& sh, int bn, bool rect, int sm_count) {
  static const bool off = [] {
    const char* v = std::getenv("MTL_CONV_SPLITK");
    return v && v[0] == '0';
  }();
  const int64_t mtiles = rect ? (int64_t)sh.n * sh.tiles_x * sh.tiles_y : (sh.mtot + 127) / 128;
  const int64_t tiles = mtiles * (sh.cout / bn);
  if (off || tiles >= sm_count) return 1;
  auto cost = [&](int ks) { return (double)((tiles * ks + sm_count - 1) / sm_count) / ks; };
  int best = 1;
  for (int ks = 2; ks <= 8 && sh.kblocks / ks >= 4 && tiles * ks <= sm_count; ++ks)  // one round of items
    if (cost(ks) < cost(best)) best = ks;
  const double saved = sh.kblocks * (1.0 - cost(best) / cost(1));
  return best >= 3 && saved > 28.0 ? best : 1;
}

static uint64_t split_bytes(const ConvShape& sh, int ks) {
  return ks > 1 ? (uint64_t)ks * (uint64_t)sh.mtot * (uint64_t)sh.cout * 4 : 0;
}

// The four parity planes of a plain NHWC input for the stride-2 halo path:
// plane pr * 2 + pc is {Cin, columns of parity pc, rows of parity pr, N} with
// pixel stride 2 * Cin, row stride 2 * W * Cin, starting at pixel (pr, pc);
// box {64, pq, ph_rows + 1, 1} (one frame).
static mtl_status make_plane_maps(HaloMaps* maps, const void* in, const ConvShape& sh) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(MTL_ERR_CUDA, "conv2d: cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t px = (cuuint64_t)sh.cin * 2;
  for (int p = 0; p < 4; ++p) {
    const int pr = p >> 1, pc = p & 1;
    cuuint64_t dims[4] = {(cuuint64_t)sh.cin, (cuuint64_t)(sh.w - pc + 1) / 2, (cuuint64_t)(sh.h - pr + 1) / 2,
                          (cuuint64_t)sh.n};
    cuuint64_t strides[3] = {2 * px, 2 * (cuuint64_t)sh.w * px, (cuuint64_t)sh.h * sh.w * px};
    cuuint32_t box[4] = {64, (cuuint32_t)sh.pq, (cuuint32_t)(sh.ph_rows + 1), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const void* base = reinterpret_cast<const __nv_bfloat16*>(in) + ((int64_t)pr * sh.w + pc) * sh.cin;
    CUresult r = enc(&maps->m[p], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(MTL_ERR_ARGUMENT, "conv2d: parity-plane tensor map rejected (CUresult %d)", (int)r);
  }
  return MTL_OK;
}

// The output as {Cout, Wo, N*Ho} (pixel stride Cout, row stride (Wo + 2*owp)
// * Cout, starting after the left margin) for TMA stores of {64, 32, 1} from
// 128-byte-swizzled staging, or (narrow) of {32, 32, 1} from 64-byte rows
// with the 64-byte swizzle (conv_rows_pair_kernel).
static mtl_status make_out_map(CUtensorMap* map, void* out, const ConvShape& sh, bool narrow = false) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(MTL_ERR_CUDA, "conv2d: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {(cuuint64_t)sh.cout, (cuuint64_t)sh.wo, (cuuint64_t)sh.n * sh.ho};
  cuuint64_t strides[2] = {(cuuint64_t)sh.cout * 2, (cuuint64_t)sh.wso * sh.cout * 2};
  cuuint32_t box[3] = {narrow ? 32u : 64u, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  void* base = reinterpret_cast<__nv_bfloat16*>(out) + (int64_t)sh.owp * sh.cout;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   narrow ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTL_ERR_ARGUMENT, "conv2d: output tensor map rejected (CUresult %d)", (int)r);
  return MTL_OK;
}

template <int CIN, int KT, int SRC_C>
static cudaError_t launch_rows(const CUtensorMap& tw, const CUtensorMap& to, const void* in, void* out,
                               const ConvShape& sh, int relu, int sm_count, cudaStream_t s) {
  const uint32_t smem = rows_smem_bytes(sh) + 2 * rows_raw_bytes(sh, SRC_C);
  cudaError_t e =
      cudaFuncSetAttribute(conv_rows_kernel<CIN, KT, SRC_C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t units = (int64_t)sh.n * ((sh.ho + kRowsG - 1) / kRowsG) * sh.nblk;
  int grid = (int)std::min<int64_t>(units, sm_count);
  grid = std::max(sh.nblk, grid - grid % sh.nblk);
  return launch_pdl(conv_rows_kernel<CIN, KT, SRC_C>, grid, rows_threads<SRC_C>(), smem, s, tw, to,
                    reinterpret_cast<const __nv_bfloat16*>(in), reinterpret_cast<__nv_bfloat16*>(out), sh, relu);
}

template <int KT, int SRC_C>
static cudaError_t launch_pair(const CUtensorMap& to, const void* in, const void* w, void* out, const ConvShape& sh,
                               int relu, int sm_count, cudaStream_t s) {
  const uint32_t smem = pair_smem_bytes(sh, SRC_C);
  cudaError_t e =
      cudaFuncSetAttribute(conv_rows_pair_kernel<KT, SRC_C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t units = (int64_t)sh.n * ((sh.ho + kRowsG - 1) / kRowsG);
  const int grid = (int)std::min<int64_t>(units, sm_count);
  return launch_pdl(conv_rows_pair_kernel<KT, SRC_C>, grid, pair_threads<SRC_C>(), smem, s, to,
                    reinterpret_cast<const __nv_bfloat16*>(in), reinterpret_cast<const __nv_bfloat16*>(w),
                    reinterpret_cast<__nv_bfloat16*>(out), sh, relu);
}

template <int BN, bool PH>
static cudaError_t launch_halo(const CUtensorMap& tw, const HaloMaps& ta, void* out, const ConvShape& sh, int relu,
                               int sm_count, cudaStream_t s) {
  const uint32_t smem = halo_smem_bytes(sh, HaloCfg<BN>::kBBlock);
  cudaError_t e = cudaFuncSetAttribute(conv_halo_kernel<BN, PH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t tiles = (int64_t)sh.n * sh.halo_tiles * sh.nblk;
  // whole column-block groups: CTA b serves column block b % nblk
  int grid = (int)std::min<int64_t>(tiles, sm_count);
  grid = std::max(sh.nblk, grid - grid % sh.nblk);
  return launch_pdl(conv_halo_kernel<BN, PH>, grid, 224, smem, s, tw, ta, reinterpret_cast<__nv_bfloat16*>(out), sh,
                    relu);
}

// Whether two 128-pixel runs per CTA beat one for a 256-wide im2col layer:
// a two-run tile takes about 1.7 times a one-run tile (measured on the
// 14x14x256 and 7x7x512 layers at batch 256), so it pays when halving the
// tile count saves a whole round of tiles over the SMs.
static bool m2_pays(const ConvShape& sh, int sm_count) {
  const int64_t t1 = (sh.mtot + 127) / 128 * (sh.cout / 256), t2 = (sh.mtot + 255) / 256 * (sh.cout / 256);
  const int64_t r1 = (t1 + sm_count - 1) / sm_count, r2 = (t2 + sm_count - 1) / sm_count;
  return 1.7 * (double)r2 < (double)r1;
}

static cudaError_t launch_m2(const CUtensorMap& tw, const CUtensorMap& ta, void* out, const ConvShape& sh, int relu,
                             int sm_count, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(conv_m2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kM2Smem);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((sh.mtot + 255) / 256) * (sh.cout / 256);
  const int grid = (int)std::min<int64_t>(tiles, sm_count);
  return launch_pdl(conv_m2_kernel, grid, 192, kM2Smem, s, tw, ta, reinterpret_cast<__nv_bfloat16*>(out), sh, relu);
}

template <int AM>
static cudaError_t launch_conv_bn(int bn, const CUtensorMap& tw, const CUtensorMap& ta, const void* in, void* out,
                                  const ConvShape& sh, int relu, int sm_count, cudaStream_t s, float* part = nullptr,
                                  int ks = 1) {
  return bn == 256   ? launch_conv<256, AM>(tw, ta, in, out, sh, relu, sm_count, s, part, ks)
         : bn == 128 ? launch_conv<128, AM>(tw, ta, in, out, sh, relu, sm_count, s, part, ks)
                     : launch_conv<64, AM>(tw, ta, in, out, sh, relu, sm_count, s, part, ks);
}

// The rectangle th x tw (th * tw <= 128 output pixels) that wastes the fewest
// MMA rows over an ho x wo image, the wider one on ties, with the TMA box
// limits tw * sx <= 256 and th * sy <= 256 (sx, sy: traversal strides).
// Returns the fraction of the tiles' 128 rows that hold output pixels.
static double pick_rect(ConvShape& sh, int sx, int sy) {
  double best = 0.0;
  for (int tw = std::min(sh.wo, 128); tw >= 1; --tw) {
    const int th = std::min(128 / tw, sh.ho);
    if (tw * sx > 256 || th * sy > 256) continue;
    const int tx = (sh.wo + tw - 1) / tw, ty = (sh.ho + th - 1) / th;
    const double use = (double)sh.ho * sh.wo / ((double)tx * ty * 128.0);
    if (use > best + 1e-9) {
      best = use;
      sh.tw = tw;
      sh.th = th;
      sh.tiles_x = tx;
      sh.tiles_y = ty;
    }
  }
  return best;
}

// The flat-halo plan (A_HALO) for a 3x3 convolution with padding 1 and Cin a
// multiple of 64: at stride 1 over an input that stores its padding column on
// each side, at stride 2 over plain rows (no stored margins) whose output rows
// have at most 126 pixels; either way the tiles' unused positions must waste
// under 15 % of the MMA rows (measured at stride 2: 77 % busy rows over the
// 28 x 28 x 128 input took 67 us against 36 us for rectangles). The widest BN
// dividing Cout whose resident weights leave room for at least two halo
// stages in the 227 KiB of shared memory, where the halo fits one TMA box (at
// most 256 rows). Returns BN, or 0.
static int halo_plan(ConvShape& sh) {
  if (sh.cin % 64 || sh.k != 3 || sh.pad != 1) return 0;
  int rows, tiles, max_stages;
  if (sh.stride == 2) {
    if (sh.wpad != 0 || sh.owp > 1 || sh.h < 2 || sh.w < 2) return 0;
    sh.pq = sh.wo + 1;
    if (sh.pq > 127) return 0;
    sh.ph_rows = std::min(128 / sh.pq, sh.ho);
    tiles = (sh.ho + sh.ph_rows - 1) / sh.ph_rows;
    if ((double)sh.ho * sh.wo < 0.85 * tiles * 128.0) return 0;
    rows = 128 + sh.pq + 1;  // the frame ((ph_rows + 1) * pq) and every MMA row's reads
    sh.ph_box_bytes = 64 * 2 * sh.pq * (sh.ph_rows + 1);
    max_stages = 8;  // four loads (planes) per tile and channel block
  } else {
    if (sh.stride != 1 || sh.wpad != 1) return 0;
    if (sh.owp != 0 && sh.owp != sh.pad) return 0;
    rows = 128 + 2 * (sh.pad * sh.ws + sh.pad);
    tiles = (sh.h * sh.ws + 127) / 128;
    if ((double)sh.h * sh.w < 0.85 * tiles * 128.0) return 0;
    max_stages = 4;
  }
  if (rows > 256) return 0;
  const int stage = (rows * 128 + 1023) & ~1023;
  const int kblocks = sh.taps * sh.cin / 64;
  for (int bn = 128; bn >= 64; bn /= 2) {  // four accumulators of 4 * bn <= 512 TMEM columns
    if (sh.cout % bn) continue;
    const int64_t avail = 232448 - 1024 - 256 - (int64_t)kblocks * 64 * bn * 2;
    const int stages = (int)std::min<int64_t>(max_stages, avail / stage);
    if (stages < 2) continue;
    // staged epilogue stores where the 8 KiB of staging cost no stage
    sh.halo_stg = std::min<int64_t>(max_stages, (avail - 4 * 2048) / stage) == stages;
    sh.kblocks = kblocks;
    sh.halo_rows = rows;
    sh.halo_tiles = tiles;
    sh.halo_stages = stages;
    sh.halo_stage_bytes = stage;
    sh.nblk = sh.cout / bn;
    return bn;
  }
  return 0;
}

// The raw-row plan (A_ROWS): 4 channels at stride 2 (16 bytes per output
// step), a filter row that fits the 8-pixel window, stored padding columns, one output
// row per 128-row tile, the windows of valid outputs inside the stored row,
// and resident weights plus two or more stages in shared memory.
static bool rows_plan(ConvShape& sh, int src_c = 0) {
  if (sh.cin != 4 || sh.stride != 2) return false;  // the 4-channel stride-2 stem
  if (sh.k > 8 || sh.wpad != sh.pad || sh.wo > 128 || sh.stride * (sh.wo - 1) + 8 > sh.ws) return false;
  const int64_t rowbytes = (int64_t)sh.ws * sh.cin * 2;
  if (rowbytes % 16 || sh.cout % 64) return false;
  const int hrows = sh.stride * (kRowsG - 1) + sh.k;
  // the last stage row's windows of the 128 tile rows: 127 * 16 + 16 * Cin bytes
  const int64_t stage = (hrows * rowbytes + 127 * 16 + 16 * sh.cin + 1023) & ~int64_t(1023);
  const int kblocks = (sh.k * 8 * sh.cin + 63) / 64;
  const int64_t avail =
      232448 - 1024 - (int64_t)kblocks * 8192 - 4 * kRowsStg * 4096 - 256 - 2 * (int64_t)rows_raw_bytes(sh, src_c);
  const int stages = (int)std::min<int64_t>(4, avail / stage);
  if (stages < 2) return false;
  sh.kblocks = kblocks;
  sh.halo_stages = stages;
  sh.halo_stage_bytes = (int)stage;
  sh.nblk = sh.cout / 64;
  return true;
}

// The plan of conv_rows_pair_kernel: the raw-row conditions with Cout = 64
// (two output rows fill the 128 TMEM lanes) and pad < k (every output row
// overlaps the image), its own shared-memory budget. MTL_CONV_STEM_PAIR=0
// turns it off (conv_rows_kernel then runs these shapes).
static bool pair_plan(ConvShape& sh, int src_c = 0) {
  const char* env = std::getenv("MTL_CONV_STEM_PAIR");
  if (env && env[0] == '0') return false;
  if (sh.cin != 4 || sh.stride != 2 || sh.cout != 64 || sh.pad >= sh.k) return false;
  if (sh.k > 8 || sh.wpad != sh.pad || sh.wo > 128 || sh.stride * (sh.wo - 1) + 8 > sh.ws) return false;
  // TMEM: the accumulators (128 columns apart) and A (16 columns per K row) in 512 columns
  if ((kPairAcc - 1) * 128 + ((sh.wo + 15) & ~15) + 16 * (sh.k + sh.stride) > 512) return false;
  const int64_t rowbytes = (int64_t)sh.ws * sh.cin * 2;
  if (rowbytes % 16) return false;
  const int hrows = sh.stride * (kRowsG - 1) + sh.k;
  // the last stage row's windows of up to 128 pixels: 127 * 16 + 16 * Cin bytes
  const int64_t stage = (hrows * rowbytes + 127 * 16 + 16 * sh.cin + 1023) & ~int64_t(1023);
  const int64_t avail = 232448 - 1024 - (int64_t)pair_wbytes(sh) - kPairEpi * kPairStg * 2048 - 256 -
                        kPairRaw * (int64_t)rows_raw_bytes(sh, src_c);
  const int stages = (int)std::min<int64_t>(4, avail / stage);
  if (stages < 2) return false;
  sh.kblocks = 0;
  sh.halo_stages = stages;
  sh.halo_stage_bytes = (int)stage;
  sh.nblk = 1;
  return true;
}

// Which A path a convolution takes (and, for the rectangle paths, its tile
// shape in sh). Rectangles where they keep at least 85 % of the MMA rows busy
// (wide outputs); flat 128-pixel im2col runs otherwise. The im2col paths need
// the im2col corners to fit the 4-D encoding ([-128, 127]) and, as a
// precaution, an input of at least 128 KiB (CUTLASS patches im2col
// descriptors of smaller tensors on drivers up to 13.1; those small inputs
// take the gather path instead).
static int conv_amode(ConvShape& sh) {
  const uint64_t in_bytes = (uint64_t)sh.n * sh.h * sh.ws * sh.cin * 2;
  const bool corners_ok = sh.pad + sh.wpad <= 127 && sh.pad - (sh.k - 1) - sh.wpad >= -128;
  if (!corners_ok || in_bytes < (128u << 10) || sh.stride > 8) return A_GATHER;
  {
    ConvShape t = sh;
    if (halo_plan(t)) {
      sh = t;
      return A_HALO;
    }
    t = sh;
    if (rows_plan(t)) {
      sh = t;
      return A_ROWS;
    }
  }
  if (sh.cin % 64 == 0) {
    ConvShape t = sh;
    if (pick_rect(t, sh.stride, sh.stride) >= 0.85) {
      sh = t;
      return A_RECT;
    }
    return A_IM2COL;
  }
  // windows: 16-byte steps between windows and rows (TMA strides)
  const bool window = sh.k <= 8 && sh.wpad == sh.pad && sh.stride * (sh.wo - 1) + 8 <= sh.ws &&
                      (sh.stride * sh.cin * 2) % 16 == 0 && ((int64_t)sh.ws * sh.cin * 2) % 16 == 0;
  if (sh.cin == 8 && window) return A_WINDOW;
  if (sh.cin == 4 && window) {
    ConvShape t = sh;
    if (pick_rect(t, 1, sh.stride) >= 0.85) {
      sh = t;
      return A_WINDOW4_RECT;
    }
    return A_WINDOW4;
  }
  if (sh.cin == 8) return A_IM2COL_CHUNK;
  return A_GATHER;
}

// Tiled map for the rectangle paths. A_RECT: the NHWC input {C, stored W, H,
// N} with box {64, tw*s, th*s, 1} and traversal strides {1, s, s, 1}, so one
// load brings th x tw pixels x 64 channels of one filter tap (128-byte rows,
// 128-byte swizzle). A_WINDOW4_RECT: the window view {8 pixels x Cin, wo
// windows, H, N} (windows `stride` pixels apart) with box {8*Cin, tw, th*s, 1},
// traversal {1, 1, s, 1}: th x tw windows of one filter row (64-byte rows,
// 64-byte swizzle).
static mtl_status make_rect_map(CUtensorMap* map, const void* in, const ConvShape& sh, bool window) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(MTL_ERR_CUDA, "conv2d: cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t px = (cuuint64_t)sh.cin * 2;  // bytes per stored pixel
  cuuint64_t dims[4] = {(cuuint64_t)sh.cin, (cuuint64_t)sh.ws, (cuuint64_t)sh.h, (cuuint64_t)sh.n};
  cuuint64_t strides[3] = {px, (cuuint64_t)sh.ws * px, (cuuint64_t)sh.h * sh.ws * px};
  cuuint32_t box[4] = {64, (cuuint32_t)(sh.tw * sh.stride), (cuuint32_t)(sh.th * sh.stride), 1};
  cuuint32_t estr[4] = {1, (cuuint32_t)sh.stride, (cuuint32_t)sh.stride, 1};
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if (window) {
    dims[0] = (cuuint64_t)8 * sh.cin;
    dims[1] = (cuuint64_t)sh.wo;
    strides[0] = (cuuint64_t)sh.stride * px;
    box[0] = (cuuint32_t)(8 * sh.cin);
    box[1] = (cuuint32_t)sh.tw;
    estr[1] = 1;
    sw = CU_TENSOR_MAP_SWIZZLE_64B;
  }
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(in), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTL_ERR_ARGUMENT, "conv2d: tiled activation map rejected (CUresult %d)", (int)r);
  return MTL_OK;
}

// Scratch of a conv2d_bf16 launch: the K parts' fp32 planes when a one-run
// layer (flat im2col runs or rectangles) has fewer tiles than SMs and splits
// its K blocks (conv_split); none otherwise. A launch given less runs whole.
uint64_t conv_workspace(const LaunchArgs& la) {
  ConvShape sh = conv_shape(la);
  if (sh.mtot == 0 || sh.mtot > (int64_t)1 << 31) return 0;
  const int BN = sh.cout % 256 == 0 ? 256 : sh.cout % 128 == 0 ? 128 : 64;
  const int am = conv_amode(sh);
  if (am != A_IM2COL && am != A_RECT) return 0;
  if (am == A_IM2COL && BN == 256 && m2_pays(sh, la.sm_count)) return 0;
  return split_bytes(sh, conv_split(sh, BN, am == A_RECT, la.sm_count));
}

mtl_status conv_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream) {
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
  if (am == A_RECT)
    if (mtl_status st = make_rect_map(&ta, in, sh, false)) return st;
  if (am == A_WINDOW4_RECT)
    if (mtl_status st = make_rect_map(&ta, in, sh, true)) return st;
  if (am == A_WINDOW || am == A_WINDOW4)
    if (mtl_status st = make_im2col_map(&ta, in, sh, 8 * sh.cin, true, true)) return st;
  if (am == A_WINDOW || am == A_WINDOW4 || am == A_WINDOW4_RECT) {
    if (mtl_status st = make_window_weight_map(&tw, reinterpret_cast<const void*>(la.a[2].ptr), sh)) return st;
    sh.kblocks = am == A_WINDOW ? sh.k : (sh.k + 1) / 2;  // one or two filter rows per K block
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (am == A_ROWS) {
    CUtensorMap to;
    ConvShape ps = sh;
    if (pair_plan(ps)) {
      if (mtl_status st = make_out_map(&to, out, ps, true)) return st;
      const void* w = reinterpret_cast<const void*>(la.a[2].ptr);
      cudaError_t e = ps.k == 7 ? launch_pair<7, 0>(to, in, w, out, ps, relu, la.sm_count, s)
                                : launch_pair<0, 0>(to, in, w, out, ps, relu, la.sm_count, s);
      if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
      return MTL_OK;
    }
    if (mtl_status st = make_window_weight_map(&tw, reinterpret_cast<const void*>(la.a[2].ptr), sh)) return st;
    if (mtl_status st = make_out_map(&to, out, sh)) return st;
    cudaError_t e = sh.k == 7 ? launch_rows<4, 7, 0>(tw, to, in, out, sh, relu, la.sm_count, s)
                              : launch_rows<4, 0, 0>(tw, to, in, out, sh, relu, la.sm_count, s);
    if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
    return MTL_OK;
  }
  if (am == A_HALO) {
    ConvShape hs = sh;
    const int bn = halo_plan(hs);
    HaloMaps maps;
    memset(&maps, 0, sizeof maps);
    const bool ph = sh.stride == 2;
    if (ph) {
      if (mtl_status st = make_plane_maps(&maps, in, hs)) return st;
    } else if (mtl_status st = make_bf16_map(&maps.m[0], in, (uint64_t)sh.cin, (uint64_t)sh.h * sh.ws, (uint64_t)sh.n,
                                             (uint32_t)hs.halo_rows)) {
      return st;
    }
    cudaError_t e = ph ? (bn == 128 ? launch_halo<128, true>(tw, maps, out, hs, relu, la.sm_count, s)
                                    : launch_halo<64, true>(tw, maps, out, hs, relu, la.sm_count, s))
                       : (bn == 128 ? launch_halo<128, false>(tw, maps, out, hs, relu, la.sm_count, s)
                                    : launch_halo<64, false>(tw, maps, out, hs, relu, la.sm_count, s));
    if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
    return MTL_OK;
  }
  if (am == A_IM2COL && BN == 256 && m2_pays(sh, la.sm_count)) {
    cudaError_t e = launch_m2(tw, ta, out, sh, relu, la.sm_count, s);
    if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
    return MTL_OK;
  }
  // a one-run layer with fewer tiles than SMs splits its K blocks when given
  // the scratch for the parts (conv_workspace)
  int ks = am == A_IM2COL || am == A_RECT ? conv_split(sh, BN, am == A_RECT, la.sm_count) : 1;
  if (!ws || ws_bytes < split_bytes(sh, ks) || (reinterpret_cast<uintptr_t>(ws) & 15)) ks = 1;
  float* part = reinterpret_cast<float*>(ws);
  if (am == A_IM2COL && ks > 1) {
    cudaError_t e = launch_conv_bn<A_IM2COL>(BN, tw, ta, in, out, sh, relu, la.sm_count, s, part, ks);
    if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
    return MTL_OK;
  }
  if (am == A_RECT && ks > 1) {
    cudaError_t e = launch_conv_bn<A_RECT>(BN, tw, ta, in, out, sh, relu, la.sm_count, s, part, ks);
    if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
    return MTL_OK;
  }
  cudaError_t e = am == A_IM2COL         ? launch_conv_bn<A_IM2COL>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                  : am == A_IM2COL_CHUNK ? launch_conv_bn<A_IM2COL_CHUNK>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                  : am == A_WINDOW       ? launch_conv_bn<A_WINDOW>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                  : am == A_WINDOW4      ? launch_conv_bn<A_WINDOW4>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                  : am == A_RECT         ? launch_conv_bn<A_RECT>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                  : am == A_WINDOW4_RECT ? launch_conv_bn<A_WINDOW4_RECT>(BN, tw, ta, in, out, sh, relu, la.sm_count, s)
                                         : launch_conv_bn<A_GATHER>(BN, tw, ta, in, out, sh, relu, la.sm_count, s);
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d: %s", cudaGetErrorString(e));
  return MTL_OK;
}

// conv2d_nchw_bf16 arguments: out (B), in (B, NCHW bf16), w (B, HWIO with 4
// input channels, those past C zero), H, W, C, Cout, k, stride, pad, relu,
// out_wpad (i); ndrange = images. The first convolution of a network straight
// from its NCHW input: the raw-row kernel with the NCHW -> NHWC conversion in
// shared memory (C <= 4, stride 2, k <= 8, W a multiple of 8, output rows of
// at most 128 pixels, Cout a multiple of 64).
static ConvShape nchw_conv_shape(const LaunchArgs& la) {
  ConvShape sh{};
  sh.n = (int)la.nd[0];
  sh.h = la.a[3].i32;
  sh.w = la.a[4].i32;
  sh.cin = 4;
  sh.cout = la.a[6].i32;
  sh.k = la.a[7].i32;
  sh.stride = la.a[8].i32;
  sh.pad = la.a[9].i32;
  sh.wpad = sh.pad;
  sh.owp = la.a[11].i32;
  sh.ws = sh.w + 2 * sh.wpad;
  if (sh.stride > 0) {
    sh.ho = (sh.h + 2 * sh.pad - sh.k) / sh.stride + 1;
    sh.wo = (sh.w + 2 * sh.pad - sh.k) / sh.stride + 1;
  }
  sh.wso = sh.wo + 2 * sh.owp;
  sh.taps = sh.k * sh.k;
  sh.cpt = 1;
  sh.mtot = (int64_t)sh.n * sh.ho * sh.wo;
  return sh;
}

mtl_status nchwconv_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.ndim != 1) return fail(MTL_ERR_ARGUMENT, "conv2d_nchw: ndrange must be one-dimensional (the image count)");
  ConvShape sh = nchw_conv_shape(la);
  const int c = la.a[5].i32;
  if (sh.n < 0 || sh.h <= 0 || sh.w <= 0 || sh.k <= 0 || sh.stride <= 0 || sh.pad < 0 || c <= 0 || sh.cout <= 0 ||
      sh.owp < 0 || sh.owp > 64 || sh.ho <= 0 || sh.wo <= 0)
    return fail(MTL_ERR_ARGUMENT, "conv2d_nchw: bad sizes");
  if (c > 4 || sh.stride != 2 || sh.w % 8 || sh.ws % 2 || sh.cout % 64 || !rows_plan(sh, c))
    return fail(MTL_ERR_UNSUPPORTED,
                "conv2d_nchw: needs C <= 4, stride 2, k <= 8, W a multiple of 8, output rows of at most 128 pixels "
                "and Cout a multiple of 64");
  const uint64_t need[3] = {(uint64_t)sh.n * sh.ho * sh.wso * sh.cout * 2, (uint64_t)sh.n * c * sh.h * sh.w * 2,
                            (uint64_t)sh.taps * 4 * sh.cout * 2};
  const char* what[3] = {"the output", "the input", "the weights"};
  for (int i = 0; i < 3; ++i) {
    if (bytes[i] && bytes[i] < need[i])
      return fail(MTL_ERR_ARGUMENT, "conv2d_nchw: %s has %llu bytes, the launch touches %llu", what[i],
                  (unsigned long long)bytes[i], (unsigned long long)need[i]);
    if (la.a[i].ptr & 15) return fail(MTL_ERR_ARGUMENT, "conv2d_nchw: %s must be 16-byte aligned", what[i]);
  }
  return MTL_OK;
}

mtl_status nchwconv_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  ConvShape sh = nchw_conv_shape(la);
  if (sh.mtot == 0) return MTL_OK;
  const int c = la.a[5].i32;
  if (!rows_plan(sh, c)) return fail(MTL_ERR_UNSUPPORTED, "conv2d_nchw: shape not supported");
  const int relu = la.a[10].i32 != 0;
  void* out = reinterpret_cast<void*>(la.a[0].ptr);
  const void* in = reinterpret_cast<const void*>(la.a[1].ptr);
  CUtensorMap tw, to;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  ConvShape ps = sh;
  if (pair_plan(ps, c)) {
    if (mtl_status st = make_out_map(&to, out, ps, true)) return st;
    const void* w = reinterpret_cast<const void*>(la.a[2].ptr);
    if (c == 3)
      e = ps.k == 7 ? launch_pair<7, 3>(to, in, w, out, ps, relu, la.sm_count, s)
                    : launch_pair<0, 3>(to, in, w, out, ps, relu, la.sm_count, s);
    else if (c == 4)
      e = launch_pair<0, 4>(to, in, w, out, ps, relu, la.sm_count, s);
    else if (c == 2)
      e = launch_pair<0, 2>(to, in, w, out, ps, relu, la.sm_count, s);
    else
      e = launch_pair<0, 1>(to, in, w, out, ps, relu, la.sm_count, s);
    if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d_nchw: %s", cudaGetErrorString(e));
    return MTL_OK;
  }
  if (mtl_status st = make_window_weight_map(&tw, reinterpret_cast<const void*>(la.a[2].ptr), sh)) return st;
  if (mtl_status st = make_out_map(&to, out, sh)) return st;
  if (c == 3)
    e = sh.k == 7 ? launch_rows<4, 7, 3>(tw, to, in, out, sh, relu, la.sm_count, s)
                  : launch_rows<4, 0, 3>(tw, to, in, out, sh, relu, la.sm_count, s);
  else if (c == 4)
    e = launch_rows<4, 0, 4>(tw, to, in, out, sh, relu, la.sm_count, s);
  else if (c == 2)
    e = launch_rows<4, 0, 2>(tw, to, in, out, sh, relu, la.sm_count, s);
  else
    e = launch_rows<4, 0, 1>(tw, to, in, out, sh, relu, la.sm_count, s);
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "conv2d_nchw: %s", cudaGetErrorString(e));
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
  const int c = la.a[2].i32, cp = la.a[5].i32;
  if (w % 8 == 0 && c <= cp && (cp == 8 || cp == 4) && (la.a[1].ptr & 15) == 0 && (la.a[0].ptr & 15) == 0) {
    const int64_t rows = la.nd[0] * h, work = rows * (w / 8 + 1);
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)la.sm_count * 16);
    auto* src = reinterpret_cast<const __nv_bfloat16*>(la.a[1].ptr);
    auto* dst = reinterpret_cast<__nv_bfloat16*>(la.a[0].ptr);
    if (cp == 8)
      nchw_to_nhwc_vec_kernel<8><<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(src, dst, c, h, w, wp, rows);
    else
      nchw_to_nhwc_vec_kernel<4><<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(src, dst, c, h, w, wp, rows);
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
  const auto* act = reinterpret_cast<const __nv_bfloat16*>(la.a[1].ptr);
  const bool v4 = c % 8 == 0 && (la.a[1].ptr & 15) == 0;
  // float4 loads need C, classes and each CTA's channel range (a multiple of 4
  // by construction) to keep rows 16-byte aligned
  const int vec = c % 4 == 0 && classes % 4 == 0 && (la.a[2].ptr & 15) == 0;
  dim3 grid((unsigned)((n + kFcImg - 1) / kFcImg), (unsigned)((classes + kFcCls - 1) / kFcCls), kFcSplit);
  const float* w = reinterpret_cast<const float*>(la.a[2].ptr);
  float* logits = reinterpret_cast<float*>(la.a[0].ptr);
  const char* env = std::getenv("MTL_GAPFC_FUSED");  // "1": pooling inside the FC kernel
  if (v4 && vec && env && env[0] == '1') {
    cudaFuncSetAttribute(fc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFcSmem);
    fc_kernel<true><<<grid, 256, kFcSmem, s>>>(nullptr, act, hw, w, logits, (int)n, c, classes, 1);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "gap_fc: %s", cudaGetErrorString(e));
  }
  // channel slices per image while the images alone fill under two CTAs an
  // SM (each slice a whole number of units and at least 64 channels); batch
  // sizes that fill the SMs keep one slice
  const int unit = v4 ? 8 : 2;
  int slices = 1;
  while (slices < 8 && n * slices * 2 <= 2 * (int64_t)la.sm_count && c % (2 * slices * unit) == 0 &&
         c / (2 * slices) >= 64)
    slices *= 2;
  const int cw = c / slices;
  const int units = cw / unit;
  const int groups = std::max(1, std::min(kGapMaxGroups, 256 / units));
  const size_t gsm = (size_t)groups * cw * 4;  // at most 8 x 1536 floats = 48 KiB
  const dim3 ggrid((unsigned)n, (unsigned)slices);
  if (v4)
    gap_kernel<4><<<ggrid, 256, gsm, s>>>(act, mean, hw, c);
  else
    gap_kernel<1><<<ggrid, 256, gsm, s>>>(act, mean, hw, c);
  // a batch whose 32-image x 256-class clusters fill under the SMs takes
  // 64-class tiles: four times the CTAs, each a quarter of the work
  if ((int64_t)grid.x * grid.y * kFcSplit < la.sm_count) {
    constexpr int kSmall = (kFcKc * kFcImg + kFcKc * 64) * 4;
    const dim3 g64(grid.x, (unsigned)((classes + 63) / 64), kFcSplit);
    cudaFuncSetAttribute(fc_kernel<false, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmall);
    fc_kernel<false, 64><<<g64, 256, kSmall, s>>>(mean, nullptr, hw, w, logits, (int)n, c, classes, vec);
  } else {
    cudaFuncSetAttribute(fc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFcSmem);
    fc_kernel<false><<<grid, 256, kFcSmem, s>>>(mean, nullptr, hw, w, logits, (int)n, c, classes, vec);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "gap_fc: %s", cudaGetErrorString(e));
}

// Host: read (and with reset, clear) this file's count of bounded waits that
// ran out on the current device.
// Host: the bounded waits' limit of this file's kernels on the current device.
cudaError_t conv_set_wait_limit(unsigned long long ns) { return set_wait_limit_this_file(ns); }

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

