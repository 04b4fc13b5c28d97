// The arithmetic of the reference's point-cloud and image-chain passes as CUDA
// kernels, headless (no graphics API): a framebuffer is a device buffer.
//
//   advect_points  bench/two_scatters.jl:46-62 (advect!): p = pos + v*dt; if
//                  |p| > radius, put p on the sphere and reflect v.
//   clear_rgba     the render pass's clear to a colour (M.Clear).
//   splat_points   the SCATTER pipeline (bench/two_scatters.jl:11-26): each
//                  point is projected by the MVP, covers the pixels whose
//                  centres lie in the s×s square around it, and adds its
//                  colour to them (additive blend). Float32 RGBA framebuffer,
//                  [H][W] rows; colours and sizes are per point or shared
//                  (stride 1 or 0, the reference's scol/ssiz).
//   pack_bgra8     the framebuffer as 8-bit BGRA (what an image-to-buffer copy
//                  of a BGRA8 target yields): round(clamp(x, 0, 1) * 255).
//   unpack_bgra8   unpack! (bench/chain.jl:27-31): BGRA8 bytes to RGBA/255
//                  with alpha 1, transposed to [W][H] (h contiguous).
//   blur3x3        blur! (bench/chain.jl:33-40): 3×3 box blur with
//                  clamp-to-edge on the [W][H] layout, nine adds in the
//                  reference's order (di fastest), then /9.
//
// Every float operation is an explicit round-to-nearest intrinsic in the
// order written, so the C oracle (built without FP contraction) reproduces
// advect, coverage, unpack and blur bit for bit; only the splat's atomic sums
// depend on the order in which points land.

#include <cuda_runtime.h>

#include <algorithm>

#include "../mtl_internal.hpp"

namespace mtl {

__global__ void advect_kernel(float* __restrict__ pos, float* __restrict__ vel, float dt, float radius, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float* P = pos + 3 * i;
    float* V = vel + 3 * i;
    const float v0 = V[0], v1 = V[1], v2 = V[2];
    float p0 = __fadd_rn(P[0], __fmul_rn(v0, dt));
    float p1 = __fadd_rn(P[1], __fmul_rn(v1, dt));
    float p2 = __fadd_rn(P[2], __fmul_rn(v2, dt));
    const float r = __fsqrt_rn(__fadd_rn(__fadd_rn(__fmul_rn(p0, p0), __fmul_rn(p1, p1)), __fmul_rn(p2, p2)));
    if (r > radius) {
      const float n0 = __fdiv_rn(p0, r), n1 = __fdiv_rn(p1, r), n2 = __fdiv_rn(p2, r);
      p0 = __fmul_rn(n0, radius);
      p1 = __fmul_rn(n1, radius);
      p2 = __fmul_rn(n2, radius);
      const float d = __fadd_rn(__fadd_rn(__fmul_rn(v0, n0), __fmul_rn(v1, n1)), __fmul_rn(v2, n2));
      const float d2 = __fmul_rn(2.f, d);
      V[0] = __fsub_rn(v0, __fmul_rn(d2, n0));
      V[1] = __fsub_rn(v1, __fmul_rn(d2, n1));
      V[2] = __fsub_rn(v2, __fmul_rn(d2, n2));
    }
    P[0] = p0;
    P[1] = p1;
    P[2] = p2;
  }
}

__global__ void clear_rgba_kernel(float4* __restrict__ fb, float4 c, int64_t npix) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < npix; i += stride) fb[i] = c;
}

// MVP is 16 floats, column-major (element (r, c) at m[4c + r]).
__global__ void splat_kernel(float* __restrict__ fb, const float* __restrict__ pos, const float* __restrict__ col,
                             const float* __restrict__ size, const float* __restrict__ mvp, int w, int h,
                             int col_stride, int size_stride, int64_t n) {
  __shared__ float m[16];
  if (threadIdx.x < 16) m[threadIdx.x] = mvp[threadIdx.x];
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float x = pos[3 * i], y = pos[3 * i + 1], z = pos[3 * i + 2];
    float cl[4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
      cl[r] = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(m[r], x), __fmul_rn(m[4 + r], y)), __fmul_rn(m[8 + r], z)),
                        m[12 + r]);
    const float cw = cl[3];
    // the clip volume: -w <= x, y <= w, 0 <= z <= w (NaN fails every test)
    if (!(cw > 0.f && cl[0] >= -cw && cl[0] <= cw && cl[1] >= -cw && cl[1] <= cw && cl[2] >= 0.f && cl[2] <= cw))
      continue;
    const float hw = 0.5f * (float)w, hh = 0.5f * (float)h;
    const float fx = __fadd_rn(__fmul_rn(__fdiv_rn(cl[0], cw), hw), hw);
    const float fy = __fadd_rn(__fmul_rn(__fdiv_rn(cl[1], cw), hh), hh);
    const float s = size[size_stride * i];
    const float half = fminf(__fmul_rn(0.5f, s), 1e6f);  // larger squares cover the image anyway
    if (!(half > 0.f)) continue;
    // pixels whose centre px + 0.5 lies in [f - s/2, f + s/2)
    const int x0 = max(0, (int)ceilf(__fsub_rn(__fsub_rn(fx, half), 0.5f)));
    const int x1 = min(w - 1, (int)ceilf(__fsub_rn(__fadd_rn(fx, half), 0.5f)) - 1);
    const int y0 = max(0, (int)ceilf(__fsub_rn(__fsub_rn(fy, half), 0.5f)));
    const int y1 = min(h - 1, (int)ceilf(__fsub_rn(__fadd_rn(fy, half), 0.5f)) - 1);
    const float* c = col + 4 * col_stride * i;
    const float c0 = c[0], c1 = c[1], c2 = c[2], c3 = c[3];
    for (int py = y0; py <= y1; ++py)
      for (int px = x0; px <= x1; ++px) {
        float* dst = fb + 4 * ((int64_t)py * w + px);
        atomicAdd(dst, c0);
        atomicAdd(dst + 1, c1);
        atomicAdd(dst + 2, c2);
        atomicAdd(dst + 3, c3);
      }
  }
}

__device__ __forceinline__ uint32_t to_unorm8(float x) {
  x = fminf(fmaxf(x, 0.f), 1.f);
  return (uint32_t)__float2int_rn(__fmul_rn(x, 255.f));
}

__global__ void pack_bgra8_kernel(uint32_t* __restrict__ dst, const float4* __restrict__ src, int64_t npix) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < npix; i += stride) {
    const float4 c = src[i];
    dst[i] = to_unorm8(c.z) | (to_unorm8(c.y) << 8) | (to_unorm8(c.x) << 16) | (to_unorm8(c.w) << 24);
  }
}

// Thread (j, i) of a 32 x 8 block: j walks the contiguous H dimension.
__global__ void unpack_bgra8_kernel(float4* __restrict__ dst, const uchar4* __restrict__ src, int w, int h) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y * blockDim.y + threadIdx.y;
  if (i >= w || j >= h) return;
  const uchar4 b = src[(int64_t)j * w + i];  // bytes B, G, R, A
  dst[(int64_t)i * h + j] = make_float4(__fdiv_rn((float)b.z, 255.f), __fdiv_rn((float)b.y, 255.f),
                                        __fdiv_rn((float)b.x, 255.f), 1.f);
}

__global__ void blur3x3_kernel(float4* __restrict__ dst, const float4* __restrict__ src, int w, int h) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y * blockDim.y + threadIdx.y;
  if (i >= w || j >= h) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int dj = -1; dj <= 1; ++dj) {
    const int jj = min(max(j + dj, 0), h - 1);
#pragma unroll
    for (int di = -1; di <= 1; ++di) {
      const int ii = min(max(i + di, 0), w - 1);
      const float4 v = __ldg(src + (int64_t)ii * h + jj);
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
  }
  dst[(int64_t)i * h + j] =
      make_float4(__fdiv_rn(acc.x, 9.f), __fdiv_rn(acc.y, 9.f), __fdiv_rn(acc.z, 9.f), __fdiv_rn(acc.w, 9.f));
}

// ── host side ────────────────────────────────────────────────────────────────
static int64_t grid_for(int64_t n, int sm) { return std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sm * 8)); }

static mtl_status launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static mtl_status need(const uint64_t* bytes, int i, uint64_t b, const char* kern, const char* what) {
  if (bytes[i] && bytes[i] < b)
    return fail(MTL_ERR_ARGUMENT, "%s: %s has %llu bytes, the launch touches %llu", kern, what,
                (unsigned long long)bytes[i], (unsigned long long)b);
  return MTL_OK;
}

// advect_points: pos (B, 3 floats per point), vel (B), dt (f), radius (f); ndrange = points.
mtl_status advect_check(const LaunchArgs& la, const uint64_t* bytes) {
  const uint64_t n = (uint64_t)la.nd[0];
  if (mtl_status s = need(bytes, 0, 12 * n, "advect_points", "pos")) return s;
  return need(bytes, 1, 12 * n, "advect_points", "vel");
}
mtl_status advect_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = la.nd[0];
  if (n <= 0) return MTL_OK;
  advect_kernel<<<(unsigned)grid_for(n, la.sm_count), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float*>(la.a[0].ptr), reinterpret_cast<float*>(la.a[1].ptr), la.a[2].f32, la.a[3].f32, n);
  return launched("advect_points");
}

// clear_rgba: fb (B, float RGBA), r, g, b, a (f); ndrange = pixels.
mtl_status clear_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.a[0].ptr & 15) return fail(MTL_ERR_ARGUMENT, "clear_rgba: the framebuffer must be 16-byte aligned");
  return need(bytes, 0, 16 * (uint64_t)la.nd[0], "clear_rgba", "the framebuffer");
}
mtl_status clear_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = la.nd[0];
  if (n <= 0) return MTL_OK;
  clear_rgba_kernel<<<(unsigned)grid_for(n, la.sm_count), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float4*>(la.a[0].ptr), make_float4(la.a[1].f32, la.a[2].f32, la.a[3].f32, la.a[4].f32), n);
  return launched("clear_rgba");
}

// splat_points: fb (B), pos (B), col (B), size (B), mvp (B, 16 floats), W, H,
// col_stride, size_stride (i); ndrange = points.
mtl_status splat_check(const LaunchArgs& la, const uint64_t* bytes) {
  const uint64_t n = (uint64_t)la.nd[0];
  const int w = la.a[5].i32, h = la.a[6].i32, cs = la.a[7].i32, ss = la.a[8].i32;
  if (w <= 0 || h <= 0) return fail(MTL_ERR_ARGUMENT, "splat_points: the framebuffer must be at least 1x1");
  if ((cs != 0 && cs != 1) || (ss != 0 && ss != 1))
    return fail(MTL_ERR_ARGUMENT, "splat_points: colour and size strides are 0 (shared) or 1 (per point)");
  if (mtl_status s = need(bytes, 0, 16ull * w * h, "splat_points", "the framebuffer")) return s;
  if (mtl_status s = need(bytes, 1, 12 * n, "splat_points", "pos")) return s;
  if (mtl_status s = need(bytes, 2, 16 * (cs ? n : 1), "splat_points", "col")) return s;
  if (mtl_status s = need(bytes, 3, 4 * (ss ? n : 1), "splat_points", "size")) return s;
  return need(bytes, 4, 64, "splat_points", "mvp");
}
mtl_status splat_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = la.nd[0];
  if (n <= 0) return MTL_OK;
  splat_kernel<<<(unsigned)grid_for(n, la.sm_count), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float*>(la.a[0].ptr), reinterpret_cast<const float*>(la.a[1].ptr),
      reinterpret_cast<const float*>(la.a[2].ptr), reinterpret_cast<const float*>(la.a[3].ptr),
      reinterpret_cast<const float*>(la.a[4].ptr), la.a[5].i32, la.a[6].i32, la.a[7].i32, la.a[8].i32, n);
  return launched("splat_points");
}

// pack_bgra8: dst (B, 4 bytes per pixel), src (B, float RGBA); ndrange = pixels.
mtl_status pack_check(const LaunchArgs& la, const uint64_t* bytes) {
  const uint64_t n = (uint64_t)la.nd[0];
  if ((la.a[0].ptr & 3) || (la.a[1].ptr & 15)) return fail(MTL_ERR_ARGUMENT, "pack_bgra8: misaligned buffers");
  if (mtl_status s = need(bytes, 0, 4 * n, "pack_bgra8", "dst")) return s;
  return need(bytes, 1, 16 * n, "pack_bgra8", "src");
}
mtl_status pack_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int64_t n = la.nd[0];
  if (n <= 0) return MTL_OK;
  pack_bgra8_kernel<<<(unsigned)grid_for(n, la.sm_count), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<uint32_t*>(la.a[0].ptr), reinterpret_cast<const float4*>(la.a[1].ptr), n);
  return launched("pack_bgra8");
}

// unpack_bgra8 / blur3x3: dst (B), src (B), W, H (i); ndrange = (W, H).
static mtl_status image_check(const LaunchArgs& la, const uint64_t* bytes, const char* kern, uint64_t src_px) {
  if (la.ndim != 2 || la.nd[0] != la.a[2].i32 || la.nd[1] != la.a[3].i32)
    return fail(MTL_ERR_ARGUMENT, "%s: ndrange must be (W, H)", kern);
  const uint64_t npix = (uint64_t)la.nd[0] * la.nd[1];
  if ((la.a[0].ptr & 15) || (la.a[1].ptr & (src_px - 1))) return fail(MTL_ERR_ARGUMENT, "%s: misaligned buffers", kern);
  if (mtl_status s = need(bytes, 0, 16 * npix, kern, "dst")) return s;
  return need(bytes, 1, src_px * npix, kern, "src");
}
mtl_status unpack_check(const LaunchArgs& la, const uint64_t* bytes) { return image_check(la, bytes, "unpack_bgra8", 4); }
mtl_status blur_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (mtl_status s = image_check(la, bytes, "blur3x3", 16)) return s;
  const uint64_t nb = 16ull * la.nd[0] * la.nd[1], d = la.a[0].ptr, x = la.a[1].ptr;
  if (d < x + nb && x < d + nb) return fail(MTL_ERR_ARGUMENT, "blur3x3: dst and src overlap (it reads neighbours)");
  return MTL_OK;
}

mtl_status unpack_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int w = la.a[2].i32, h = la.a[3].i32;
  if (w <= 0 || h <= 0) return MTL_OK;
  dim3 block(32, 8), grid((h + 31) / 32, (w + 7) / 8);
  unpack_bgra8_kernel<<<grid, block, 0, (cudaStream_t)stream>>>(reinterpret_cast<float4*>(la.a[0].ptr),
                                                               reinterpret_cast<const uchar4*>(la.a[1].ptr), w, h);
  return launched("unpack_bgra8");
}
mtl_status blur_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int w = la.a[2].i32, h = la.a[3].i32;
  if (w <= 0 || h <= 0) return MTL_OK;
  dim3 block(32, 8), grid((h + 31) / 32, (w + 7) / 8);
  blur3x3_kernel<<<grid, block, 0, (cudaStream_t)stream>>>(reinterpret_cast<float4*>(la.a[0].ptr),
                                                          reinterpret_cast<const float4*>(la.a[1].ptr), w, h);
  return launched("blur3x3");
}

}  // namespace mtl
