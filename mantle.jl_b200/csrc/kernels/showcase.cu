// The compute passes of the reference's deferred-shading showcase
// (bench/showcase.jl) as CUDA kernels, headless: the g-buffer and the shadow
// map are device buffers (the raster passes that fill them in the reference
// need a graphics stack; here they are inputs), and the composite writes a
// float RGBA buffer instead of the swapchain.
//
//   sc_move_lights  move_lights! (showcase.jl:214-229)
//   sc_cull         cull! (:187-201) with frustum_plane (:156-163)
//   sc_write_draw   write_draw! (:203-205)
//   sc_tile_lights  tile_lights! (:331-376)
//   sc_shade        shade! (:380-454) with ggx (:307-326), sky (:298-305),
//                   sunshadow (:270-287), unproject (:289-292)
//   sc_ssao         ssao! (:471-523) with hash01 (:456-461)
//   sc_ao_blur      ao_blur! (:527-542)
//   sc_bright       bright! (:550-565)
//   sc_blur         blur! (:568-583)
//   sc_composite    composite_fragment (:593-617) as a compute pass
//
// Scene constants come in one float buffer P (matrices column-major, see
// the SC_* offsets below), uploaded per frame like the reference's Refs.
// This file is compiled without FMA contraction: every +, -, *, / and sqrt is
// one IEEE operation in the order written, as in the C oracle (built without
// contraction), so results agree bit for bit except where expf, powf, sinf or
// cosf round differently in the last place.
//
// Layouts: images are [H][W] rows (x fastest), g-buffer channels packed as
// RGBA8 in a uint32 (r in the low byte), depth float in [0, 1] (1 = sky),
// lights float4 (xyz, radius) and (rgb, intensity), instances float4.

#include <cuda_runtime.h>

#include <algorithm>

#include "../mtl_internal.hpp"

namespace mtl {

// offsets into the scene-constant buffer P
enum : int {
  SC_VP = 0,         // camera view-projection (16, column-major)
  SC_INVVP = 16,     // its inverse
  SC_SUNVP = 32,     // the sun's view-projection
  SC_EYE = 48,       // eye position (4)
  SC_SUN = 52,       // sun direction (4)
  SC_SUNCOL = 56,    // sun colour rgb and intensity (4)
  SC_FOG = 60,
  SC_EMIT = 61,      // emission scale
  SC_STEXEL = 62,    // a shadow texel in world units
  SC_SBIAS = 63,     // shadow depth bias
  SC_AOAMB = 64,     // occlusion on the ambient term
  SC_AODIRECT = 65,  // share of occlusion on point lights
  SC_AORADIUS = 66,
  SC_AOBIAS = 67,
  SC_THRESHOLD = 68,  // bloom threshold
  SC_EXPOSURE = 69,
  SC_BLOOM = 70,      // bloom amount
  SC_AOSHARP = 71,    // bilateral depth sharpness
  SC_TIME = 72,
  SC_PARAMS = 80      // floats in P
};

struct v3 {
  float x, y, z;
};
__device__ __forceinline__ v3 mk(float x, float y, float z) { return v3{x, y, z}; }
__device__ __forceinline__ v3 operator+(v3 a, v3 b) { return mk(a.x + b.x, a.y + b.y, a.z + b.z); }
__device__ __forceinline__ v3 operator-(v3 a, v3 b) { return mk(a.x - b.x, a.y - b.y, a.z - b.z); }
__device__ __forceinline__ v3 operator*(v3 a, float s) { return mk(a.x * s, a.y * s, a.z * s); }
__device__ __forceinline__ v3 mul(v3 a, v3 b) { return mk(a.x * b.x, a.y * b.y, a.z * b.z); }
__device__ __forceinline__ float dot3(v3 a, v3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ v3 cross3(v3 a, v3 b) {
  return mk(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
// x / |x| component by component (the reference's normalize)
__device__ __forceinline__ v3 unit(v3 a) {
  const float n = sqrtf(a.x * a.x + a.y * a.y + a.z * a.z);
  return mk(a.x / n, a.y / n, a.z / n);
}
__device__ __forceinline__ float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }
__device__ __forceinline__ int clampi(int x, int lo, int hi) { return min(max(x, lo), hi); }

// M * (x, y, z, w) for a column-major 4x4 M
__device__ __forceinline__ float4 mat4(const float* M, float x, float y, float z, float w) {
  return make_float4(M[0] * x + M[4] * y + M[8] * z + M[12] * w, M[1] * x + M[5] * y + M[9] * z + M[13] * w,
                     M[2] * x + M[6] * y + M[10] * z + M[14] * w, M[3] * x + M[7] * y + M[11] * z + M[15] * w);
}

__device__ __forceinline__ float unpack8(uint32_t px, int shift) { return (float)((px >> shift) & 0xffu) * (1.f / 255.f); }

// screen position (pixels) and depth -> world
__device__ __forceinline__ v3 unproject(const float* invvp, float fx, float fy, float d, int w, int h) {
  const float4 q = mat4(invvp, 2.f * fx / (float)w - 1.f, 2.f * fy / (float)h - 1.f, d, 1.f);
  return mk(q.x / q.w, q.y / q.w, q.z / q.w);
}

// the packed normal: 2 * channel - 1, normalized
__device__ __forceinline__ v3 normal_of(uint32_t nn) {
  return unit(mk(2.f * unpack8(nn, 0) - 1.f, 2.f * unpack8(nn, 8) - 1.f, 2.f * unpack8(nn, 16) - 1.f));
}

// dusk sky: horizon to zenith by the ray's height, plus a sun glow
__device__ v3 sky(v3 dir, v3 sundir, v3 suncol) {
  const float t = clampf(0.5f * (dir.y + 1.f), 0.f, 1.f);
  const v3 horizon = mk(0.115f, 0.085f, 0.105f), zenith = mk(0.012f, 0.020f, 0.055f);
  const v3 base = horizon + (zenith - horizon) * powf(t, 0.55f);
  const float c = fmaxf(0.f, dir.x * sundir.x + dir.y * sundir.y + dir.z * sundir.z);
  return base + suncol * (powf(c, 220.f) * 7.f + powf(c, 12.f) * 0.10f);
}

// Cook-Torrance with the GGX distribution, Smith-Schlick geometry and Schlick
// Fresnel; returns the reflected radiance factor times n.l
__device__ v3 ggx(v3 n, v3 v, v3 l, v3 albedo, float rough, float metal) {
  const float ndl = n.x * l.x + n.y * l.y + n.z * l.z;
  const float ndv = n.x * v.x + n.y * v.y + n.z * v.z;
  if (ndl <= 0.f || ndv <= 0.f) return mk(0.f, 0.f, 0.f);
  const v3 hv = unit(v + l);
  const float ndh = fmaxf(0.f, n.x * hv.x + n.y * hv.y + n.z * hv.z);
  const float vdh = fmaxf(0.f, v.x * hv.x + v.y * hv.y + v.z * hv.z);
  const float a = fmaxf(1e-3f, rough * rough);
  const float a2 = a * a;
  const float dd = ndh * ndh * (a2 - 1.f) + 1.f;
  const float D = a2 / (3.14159274f * dd * dd);
  const float k = a * 0.5f;
  const float G = (ndl / (ndl * (1.f - k) + k)) * (ndv / (ndv * (1.f - k) + k));
  const v3 f0 = mk(0.04f, 0.04f, 0.04f) + (albedo - mk(0.04f, 0.04f, 0.04f)) * metal;
  const float om = 1.f - vdh;
  const float fr = om * om * om * om * om;  // (1 - v.h)^5 as four products, left to right
  const v3 F = f0 + (mk(1.f, 1.f, 1.f) - f0) * fr;
  const v3 spec = F * (D * G / fmaxf(1e-4f, 4.f * ndl * ndv));
  const v3 kd = (mk(1.f, 1.f, 1.f) - F) * (1.f - metal);
  return (mul(kd, albedo) * (1.f / 3.14159274f) + spec) * ndl;
}

// 3x3 percentage-closer lookup with slope-scaled normal offset and bias
__device__ float sunshadow(const float* __restrict__ smap, const float* sunvp, v3 world, v3 n, float ndl, int res,
                           float texel, float bias) {
  const float slope = clampf(sqrtf(fmaxf(0.f, 1.f - ndl * ndl)) / fmaxf(ndl, 0.08f), 0.f, 10.f);
  const v3 w = world + n * (texel * (1.6f + 2.2f * slope));
  const float4 q = mat4(sunvp, w.x, w.y, w.z, 1.f);
  if (fabsf(q.x) > 1.f || fabsf(q.y) > 1.f || q.z < 0.f || q.z > 1.f) return 1.f;
  const float fx = (0.5f * q.x + 0.5f) * (float)res;
  const float fy = (0.5f * q.y + 0.5f) * (float)res;
  const float ref = q.z - bias * (1.f + slope);
  float lit = 0.f;
  for (int dy = -1; dy <= 1; ++dy)
    for (int dx = -1; dx <= 1; ++dx) {
      const int sx = clampi((int)fx + dx, 0, res - 1);
      const int sy = clampi((int)fy + dy, 0, res - 1);
      lit += smap[(int64_t)sy * res + sx] > ref ? 1.f : 0.f;
    }
  return lit * (1.f / 9.f);
}

// ── per-instance passes ─────────────────────────────────────────────────────
// Light i (0-based) moves on its orbit around home[i]; the instance that
// stands for it (first + i) follows, and its emission is the light's intensity.
__global__ void sc_move_lights_kernel(float4* __restrict__ pos, float4* __restrict__ centers,
                                      float4* __restrict__ params, const float4* __restrict__ home,
                                      const float4* __restrict__ lcol, const float* __restrict__ P, int first,
                                      int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float t = P[SC_TIME];
  const float4 h = home[i];
  const float ph = 0.7f * (float)(i + 1);  // the reference counts lights from 1
  const float4 p = make_float4(h.x + 7.f * sinf(0.42f * t + ph), h.y + 1.6f * sinf(0.9f * t + ph),
                               h.z + 7.f * cosf(0.33f * t + ph), h.w);
  pos[i] = p;
  centers[first + i] = make_float4(p.x, p.y, p.z, centers[first + i].w);
  params[first + i] = make_float4(0.f, lcol[i].w, 0.f, 0.f);
}

// plane k (0..5) of the frustum of the column-major view-projection M:
// w ± x, w ± y, z, w - z, scaled to a unit normal
__device__ __forceinline__ float4 frustum_plane(const float* M, int k) {
  const float4 rw = make_float4(M[3], M[7], M[11], M[15]);
  const int r = k < 4 ? k / 2 : 2;
  const float4 ri = make_float4(M[r], M[4 + r], M[8 + r], M[12 + r]);
  float4 p;
  if (k == 4)
    p = ri;
  else if (k % 2 == 0 && k < 4)
    p = make_float4(rw.x + ri.x, rw.y + ri.y, rw.z + ri.z, rw.w + ri.w);
  else
    p = make_float4(rw.x - ri.x, rw.y - ri.y, rw.z - ri.z, rw.w - ri.w);
  const float len = sqrtf(p.x * p.x + p.y * p.y + p.z * p.z);
  return make_float4(p.x / len, p.y / len, p.z / len, p.w / len);
}

// Instances whose bounding sphere (centre xyz, radius w) is not outside any
// plane get a slot from the counter; the slot holds the instance's 1-based id.
// Warp-aggregated: one atomic per warp for its survivors.
__global__ void sc_cull_kernel(uint32_t* __restrict__ visible, uint32_t* __restrict__ counter,
                               const float4* __restrict__ centers, const float* __restrict__ P, int mat, int n) {
  __shared__ float planes[6][4];
  if (threadIdx.x < 6) {
    const float4 p = frustum_plane(P + mat, threadIdx.x);
    planes[threadIdx.x][0] = p.x;
    planes[threadIdx.x][1] = p.y;
    planes[threadIdx.x][2] = p.z;
    planes[threadIdx.x][3] = p.w;
  }
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  bool keep = false;
  if (i < n) {
    const float4 c = centers[i];
    keep = true;
    for (int k = 0; k < 6; ++k)
      keep &= planes[k][0] * c.x + planes[k][1] * c.y + planes[k][2] * c.z + planes[k][3] >= -c.w;
  }
  const unsigned mask = __ballot_sync(0xffffffffu, keep);
  if (!mask) return;
  const int lane = threadIdx.x % 32, leader = __ffs(mask) - 1;
  uint32_t base = 0;
  if (lane == leader) base = atomicAdd(counter, (uint32_t)__popc(mask));
  base = __shfl_sync(0xffffffffu, base, leader);
  // A counter that was not cleared would walk off the list: those slots are
  // dropped (the count still says how many survived), never written past n.
  const uint32_t slot = base + __popc(mask & ((1u << lane) - 1));
  if (keep && slot < (uint32_t)n) visible[slot] = (uint32_t)(i + 1);
}

// the indirect draw command {vertex count, instances 1, 0, 0}
__global__ void sc_write_draw_kernel(uint32_t* __restrict__ cmd, const uint32_t* __restrict__ counter, uint32_t vpb) {
  cmd[0] = counter[0] * vpb;
  cmd[1] = 1;
  cmd[2] = 0;
  cmd[3] = 0;
}

// ── tiled light lists ───────────────────────────────────────────────────────
// One CTA per screen tile (tile x tile pixels, tile <= 32): the tile's depth
// range over covered pixels (d < 1), its world-space box from the eight
// unprojected corners, and the lights whose sphere reaches the box, in light
// order, at most pertile of them (the block's threads test lights in parallel
// and compact with ballots, which keeps the order).
__global__ void __launch_bounds__(256) sc_tile_lights_kernel(uint32_t* __restrict__ tilelights,
                                                             uint32_t* __restrict__ tilecount,
                                                             const float* __restrict__ dep,
                                                             const float4* __restrict__ lpos,
                                                             const float* __restrict__ P, int w, int h, int tile,
                                                             int nlight, int pertile) {
  __shared__ float smin[8], smax[8];
  __shared__ float box[6];
  __shared__ uint32_t wcount[8];
  const int tx = blockIdx.x, ty = blockIdx.y, ntx = gridDim.x;
  const int ti = ty * ntx + tx;
  const int x0 = tx * tile, y0 = ty * tile;
  const int x1 = min(x0 + tile, w), y1 = min(y0 + tile, h);
  // this thread's light, loaded early so its latency overlaps the depth pass
  float4 mylight = make_float4(0.f, 0.f, 0.f, -1.f);
  if (threadIdx.x < nlight) mylight = lpos[threadIdx.x];
  float dmin = 1.f, dmax = 0.f;
  for (int e = threadIdx.x; e < tile * tile; e += blockDim.x) {
    const int px = x0 + e % tile, py = y0 + e / tile;
    if (px < x1 && py < y1) {
      const float d = dep[(int64_t)py * w + px];
      if (d < 1.f) {
        dmin = fminf(dmin, d);
        dmax = fmaxf(dmax, d);
      }
    }
  }
  for (int o = 16; o; o >>= 1) {
    dmin = fminf(dmin, __shfl_xor_sync(0xffffffffu, dmin, o));
    dmax = fmaxf(dmax, __shfl_xor_sync(0xffffffffu, dmax, o));
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarp = blockDim.x / 32;
  if (lane == 0) {
    smin[warp] = dmin;
    smax[warp] = dmax;
  }
  __syncthreads();
  if (warp == 0) {
    // every lane of warp 0 folds the per-warp ranges; lanes 0-7 then unproject
    // one corner each and the box is their min / max (fminf / fmaxf are exact,
    // so the order of folding does not matter)
    dmin = 1.f;
    dmax = 0.f;
    for (int k = 0; k < nwarp; ++k) {
      dmin = fminf(dmin, smin[k]);
      dmax = fmaxf(dmax, smax[k]);
    }
    const int c = lane & 7;
    const v3 p = unproject(P + SC_INVVP, (float)((c & 1) == 0 ? x0 : x1), (float)((c & 2) == 0 ? y0 : y1),
                           (c & 4) == 0 ? dmin : dmax, w, h);
    float lo[3] = {p.x, p.y, p.z}, hi[3] = {p.x, p.y, p.z};
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        lo[j] = fminf(lo[j], __shfl_xor_sync(0xffffffffu, lo[j], o));
        hi[j] = fmaxf(hi[j], __shfl_xor_sync(0xffffffffu, hi[j], o));
      }
    __syncwarp();
    if (lane == 0) {
      smin[0] = dmin;
      smax[0] = dmax;
      box[0] = lo[0], box[1] = lo[1], box[2] = lo[2], box[3] = hi[0], box[4] = hi[1], box[5] = hi[2];
    }
  }
  __syncthreads();
  if (!(smax[0] > 0.f)) {
    if (threadIdx.x == 0) tilecount[ti] = 0;
    return;
  }
  uint32_t total = 0;
  for (int l0 = 0; l0 < nlight; l0 += blockDim.x) {
    const int l = l0 + threadIdx.x;
    bool hit = false;
    if (l < nlight) {
      const float4 lp = l0 == 0 ? mylight : lpos[l];
      const float dx = fmaxf(0.f, fmaxf(box[0] - lp.x, lp.x - box[3]));
      const float dy = fmaxf(0.f, fmaxf(box[1] - lp.y, lp.y - box[4]));
      const float dz = fmaxf(0.f, fmaxf(box[2] - lp.z, lp.z - box[5]));
      hit = dx * dx + dy * dy + dz * dz <= lp.w * lp.w;
    }
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) wcount[warp] = __popc(m);
    __syncthreads();
    uint32_t before = total;
    for (int k = 0; k < warp; ++k) before += wcount[k];
    const uint32_t slot = before + __popc(m & ((1u << lane) - 1));
    if (hit && slot < (uint32_t)pertile) tilelights[(int64_t)ti * pertile + slot] = (uint32_t)(l + 1);
    for (int k = 0; k < nwarp; ++k) total += wcount[k];
    __syncthreads();
  }
  if (threadIdx.x == 0) tilecount[ti] = min(total, (uint32_t)pertile);
}

// ── deferred lighting ───────────────────────────────────────────────────────
// One thread per pixel: sky behind empty pixels; on surfaces an ambient term
// (sky above, ground bounce below, darkened by the bilinear half-resolution
// occlusion), the sun through GGX and the shadow map, the tile's point lights
// through GGX with a squared falloff, emission, and distance fog towards the
// sky. HDR out (alpha 1), no tone map.
__global__ void __launch_bounds__(256) sc_shade_kernel(
    float4* __restrict__ hdr, const uint32_t* __restrict__ alb, const uint32_t* __restrict__ mat,
    const uint32_t* __restrict__ nrm, const float* __restrict__ dep, const float4* __restrict__ lpos,
    const float4* __restrict__ lcol, const uint32_t* __restrict__ tilelights, const uint32_t* __restrict__ tilecount,
    const float* __restrict__ smap, const float* __restrict__ aomap, const float* __restrict__ P, int w, int h,
    int tile, int pertile, int smapres, int aow, int aoh) {
  const int px = blockIdx.x * blockDim.x + threadIdx.x, py = blockIdx.y * blockDim.y + threadIdx.y;
  if (px >= w || py >= h) return;
  const int64_t i = (int64_t)py * w + px;
  const float d = dep[i];
  const v3 sundir = mk(P[SC_SUN], P[SC_SUN + 1], P[SC_SUN + 2]);
  const v3 sunrgb = mk(P[SC_SUNCOL], P[SC_SUNCOL + 1], P[SC_SUNCOL + 2]) * P[SC_SUNCOL + 3];
  const v3 world = unproject(P + SC_INVVP, (float)px + 0.5f, (float)py + 0.5f, fminf(d, 0.999999f), w, h);
  const v3 eyep = mk(P[SC_EYE], P[SC_EYE + 1], P[SC_EYE + 2]);
  const v3 ray = unit(world - eyep);
  const v3 skyc = sky(ray, sundir, sunrgb);  // the background, and the fog's colour below
  v3 out = skyc;
  if (d < 1.f) {
    const uint32_t a = alb[i], m = mat[i];
    const v3 albedo = mk(unpack8(a, 0), unpack8(a, 8), unpack8(a, 16));
    const float rough = fmaxf(0.04f, unpack8(a, 24));
    const float metal = unpack8(m, 0), emit = unpack8(m, 8);
    const v3 n = normal_of(nrm[i]);
    const v3 view = mk(-ray.x, -ray.y, -ray.z);
    // bilinear on the half-resolution occlusion
    const float fax = ((float)px + 0.5f) * 0.5f - 0.5f, fay = ((float)py + 0.5f) * 0.5f - 0.5f;
    const int ax0 = clampi((int)fax, 0, aow - 1), ay0 = clampi((int)fay, 0, aoh - 1);
    const int ax1 = min(ax0 + 1, aow - 1), ay1 = min(ay0 + 1, aoh - 1);
    const float atx = clampf(fax - (float)ax0, 0.f, 1.f), aty = clampf(fay - (float)ay0, 0.f, 1.f);
    const float a00 = aomap[(int64_t)ay0 * aow + ax0], a10 = aomap[(int64_t)ay0 * aow + ax1];
    const float a01 = aomap[(int64_t)ay1 * aow + ax0], a11 = aomap[(int64_t)ay1 * aow + ax1];
    const float top = a00 + (a10 - a00) * atx;
    const float occ = top + ((a01 + (a11 - a01) * atx) - top) * aty;
    const float ao = clampf(1.f - occ * P[SC_AOAMB], 0.f, 1.f);
    const float aol = 1.f - P[SC_AODIRECT] * (1.f - ao);
    const float up = 0.5f * n.y + 0.5f;
    const v3 amb = (mk(0.055f, 0.070f, 0.115f) * up + mk(0.020f, 0.017f, 0.016f) * (1.f - up)) *
                   (1.f - 0.7f * metal) * ao;
    const float ndl = fmaxf(0.f, n.x * sundir.x + n.y * sundir.y + n.z * sundir.z);
    const float shd = ndl > 0.f ? sunshadow(smap, P + SC_SUNVP, world, n, ndl, smapres, P[SC_STEXEL], P[SC_SBIAS])
                                : 1.f;
    v3 acc = mul(albedo, amb) + mul(ggx(n, view, sundir, albedo, rough, metal), sunrgb) * shd;
    const int ntx = (w + tile - 1) / tile;
    const int64_t ti = (int64_t)(py / tile) * ntx + px / tile;
    const int cnt = (int)tilecount[ti];
    for (int k = 0; k < cnt; ++k) {
      const int l = (int)tilelights[ti * pertile + k] - 1;
      const float4 lp = lpos[l];
      const v3 dv = mk(lp.x - world.x, lp.y - world.y, lp.z - world.z);
      const float dist = sqrtf(dv.x * dv.x + dv.y * dv.y + dv.z * dv.z) + 1e-4f;
      const float fall = fmaxf(0.f, 1.f - dist / lp.w);
      if (fall > 0.f) {
        const float4 c = lcol[l];
        const v3 ldir = mk(dv.x / dist, dv.y / dist, dv.z / dist);
        acc = acc + mul(ggx(n, view, ldir, albedo, rough, metal), mk(c.x, c.y, c.z) * (c.w * fall * fall * aol));
      }
    }
    acc = acc + albedo * (emit * P[SC_EMIT]);
    const v3 de = world - eyep;
    const float dist = sqrtf(de.x * de.x + de.y * de.y + de.z * de.z);
    const float f = 1.f - expf(-dist * P[SC_FOG]);
    out = acc + (skyc - acc) * f;
  }
  hdr[i] = make_float4(out.x, out.y, out.z, 1.f);
}

// ── ambient occlusion ───────────────────────────────────────────────────────
__device__ __forceinline__ float hash01(int x, int y) {
  uint32_t hh = (uint32_t)x * 0x9e3779b9u + (uint32_t)y * 0x85ebca6bu;
  hh ^= hh >> 15;
  hh *= 0x2545f491u;
  return (float)(hh & 0x00ffffffu) * (1.f / 16777216.f);
}

// One thread per half-resolution pixel (the full-resolution pixel 2ix, 2iy):
// nsample points on a cosine-weighted, per-pixel rotated spiral in the
// hemisphere around the normal; a point counts as occluded when the g-buffer
// surface where it projects is nearer the eye than the point (by more than
// bias), weighted down with the gap between that surface and the pixel's.
// Writes (occlusion / nsample, depth).
__global__ void __launch_bounds__(256) sc_ssao_kernel(float2* __restrict__ ao, const float* __restrict__ dep,
                                                      const uint32_t* __restrict__ nrm, const float* __restrict__ P,
                                                      int w, int h, int aow, int aoh, int nsample) {
  const int ix = blockIdx.x * blockDim.x + threadIdx.x, iy = blockIdx.y * blockDim.y + threadIdx.y;
  if (ix >= aow || iy >= aoh) return;
  const int px = 2 * ix, py = 2 * iy;
  const int64_t i = (int64_t)py * w + px;
  const float d = dep[i];
  float occ = 0.f;
  if (d < 1.f) {
    const float* vp = P + SC_VP;
    const float* inv = P + SC_INVVP;
    const float radius = P[SC_AORADIUS], bias = P[SC_AOBIAS];
    const v3 n = normal_of(nrm[i]);
    const v3 p = unproject(inv, (float)px + 0.5f, (float)py + 0.5f, d, w, h);
    const v3 ep = mk(P[SC_EYE], P[SC_EYE + 1], P[SC_EYE + 2]);
    const v3 upv = fabsf(n.z) < 0.9f ? mk(0.f, 0.f, 1.f) : mk(1.f, 0.f, 0.f);
    const v3 t = unit(cross3(upv, n));
    const v3 b = cross3(n, t);
    const float rot = hash01(px, py) * 6.2831854f;
    for (int k = 0; k < nsample; ++k) {
      const float a = ((float)k + 0.5f) / (float)nsample;
      const float rr = sqrtf(a);
      const float phi = (float)k * 2.3999632f + rot;
      const v3 dir = t * (rr * cosf(phi)) + b * (rr * sinf(phi)) + n * sqrtf(fmaxf(0.f, 1.f - a));
      const v3 sp = p + dir * (radius * (0.3f + 0.7f * a));
      const float4 q = mat4(vp, sp.x, sp.y, sp.z, 1.f);
      if (q.w > 0.f) {
        const float sx = (0.5f * q.x / q.w + 0.5f) * (float)w;
        const float sy = (0.5f * q.y / q.w + 0.5f) * (float)h;
        if (sx >= 0.f && sx < (float)w && sy >= 0.f && sy < (float)h) {
          const float ds = dep[(int64_t)(int)sy * w + (int)sx];
          if (ds < 1.f) {
            const v3 ps = unproject(inv, sx, sy, ds, w, h);
            const v3 e1 = ps - ep, e2 = sp - ep, g = ps - p;
            const float dp = sqrtf(e1.x * e1.x + e1.y * e1.y + e1.z * e1.z);
            const float dsamp = sqrtf(e2.x * e2.x + e2.y * e2.y + e2.z * e2.z);
            if (dp < dsamp - bias) {
              const float gap = sqrtf(g.x * g.x + g.y * g.y + g.z * g.z);
              occ += clampf(radius / fmaxf(1e-4f, gap), 0.f, 1.f);
            }
          }
        }
      }
    }
  }
  ao[(int64_t)iy * aow + ix] = make_float2(occ / (float)nsample, d);
}

// 5x5 bilateral blur of the occlusion, clamp to edge, weights exp(-|dd| * sharp)
__global__ void __launch_bounds__(256) sc_ao_blur_kernel(float* __restrict__ dst, const float2* __restrict__ src,
                                                         const float* __restrict__ P, int aow, int aoh) {
  const int ix = blockIdx.x * blockDim.x + threadIdx.x, iy = blockIdx.y * blockDim.y + threadIdx.y;
  if (ix >= aow || iy >= aoh) return;
  const float sharp = P[SC_AOSHARP];
  const float d0 = src[(int64_t)iy * aow + ix].y;
  float acc = 0.f, wsum = 0.f;
  for (int dy = -2; dy <= 2; ++dy)
    for (int dx = -2; dx <= 2; ++dx) {
      const int sx = clampi(ix + dx, 0, aow - 1), sy = clampi(iy + dy, 0, aoh - 1);
      const float2 v = src[(int64_t)sy * aow + sx];
      const float g = expf(-fabsf(v.y - d0) * sharp);
      acc += v.x * g;
      wsum += g;
    }
  dst[(int64_t)iy * aow + ix] = acc / wsum;
}

// ── bloom and composite ─────────────────────────────────────────────────────
// Four taps (offsets 0 and shift/2 per axis) of the HDR image per bloom pixel,
// each keeping the part of its colour above the threshold (by its max channel).
__global__ void __launch_bounds__(256) sc_bright_kernel(float4* __restrict__ dst, const float4* __restrict__ hdr,
                                                        const float* __restrict__ P, int w, int h, int bw, int bh,
                                                        int shift) {
  const int ix = blockIdx.x * blockDim.x + threadIdx.x, iy = blockIdx.y * blockDim.y + threadIdx.y;
  if (ix >= bw || iy >= bh) return;
  const float thr = P[SC_THRESHOLD];
  const int half = shift / 2;
  v3 acc = mk(0.f, 0.f, 0.f);
  for (int ty = 0; ty < 2; ++ty)
    for (int tx = 0; tx < 2; ++tx) {
      const int sx = min(ix * shift + (tx ? half : 0), w - 1);
      const int sy = min(iy * shift + (ty ? half : 0), h - 1);
      const float4 c = hdr[(int64_t)sy * w + sx];
      const float m = fmaxf(c.x, fmaxf(c.y, c.z));
      acc = acc + mk(c.x, c.y, c.z) * (m > thr ? (m - thr) / m : 0.f);
    }
  dst[(int64_t)iy * bw + ix] = make_float4(acc.x * 0.25f, acc.y * 0.25f, acc.z * 0.25f, 1.f);
}

// 13-tap Gaussian (weights exp(-k^2 / 16)) along (dx, dy), clamp to edge
__global__ void __launch_bounds__(256) sc_blur_kernel(float4* __restrict__ dst, const float4* __restrict__ src,
                                                      int bw, int bh, int dx, int dy) {
  const int ix = blockIdx.x * blockDim.x + threadIdx.x, iy = blockIdx.y * blockDim.y + threadIdx.y;
  if (ix >= bw || iy >= bh) return;
  v3 acc = mk(0.f, 0.f, 0.f);
  float wsum = 0.f;
  for (int k = -6; k <= 6; ++k) {
    const int sx = clampi(ix + k * dx, 0, bw - 1), sy = clampi(iy + k * dy, 0, bh - 1);
    const float4 c = src[(int64_t)sy * bw + sx];
    const float g = expf(-(float)(k * k) * (1.f / 16.f));
    acc = acc + mk(c.x, c.y, c.z) * g;
    wsum += g;
  }
  dst[(int64_t)iy * bw + ix] = make_float4(acc.x / wsum, acc.y / wsum, acc.z / wsum, 1.f);
}

// HDR plus the bilinear bloom, times exposure, Reinhard v / (1 + v)
__global__ void __launch_bounds__(256) sc_composite_kernel(float4* __restrict__ out, const float4* __restrict__ hdr,
                                                           const float4* __restrict__ bloom,
                                                           const float* __restrict__ P, int w, int h, int bw, int bh,
                                                           int shift) {
  const int px = blockIdx.x * blockDim.x + threadIdx.x, py = blockIdx.y * blockDim.y + threadIdx.y;
  if (px >= w || py >= h) return;
  const float4 c = hdr[(int64_t)py * w + px];
  const float fx = ((float)px + 0.5f) / (float)shift - 0.5f, fy = ((float)py + 0.5f) / (float)shift - 0.5f;
  const int x0 = clampi((int)fx, 0, bw - 1), y0 = clampi((int)fy, 0, bh - 1);
  const int x1 = min(x0 + 1, bw - 1), y1 = min(y0 + 1, bh - 1);
  const float tx = clampf(fx - (float)x0, 0.f, 1.f), ty = clampf(fy - (float)y0, 0.f, 1.f);
  const float4 b00 = bloom[(int64_t)y0 * bw + x0], b10 = bloom[(int64_t)y0 * bw + x1];
  const float4 b01 = bloom[(int64_t)y1 * bw + x0], b11 = bloom[(int64_t)y1 * bw + x1];
  const v3 bt = mk(b00.x, b00.y, b00.z) + (mk(b10.x, b10.y, b10.z) - mk(b00.x, b00.y, b00.z)) * tx;
  const v3 bb = mk(b01.x, b01.y, b01.z) + (mk(b11.x, b11.y, b11.z) - mk(b01.x, b01.y, b01.z)) * tx;
  const v3 b = bt + (bb - bt) * ty;
  const float amount = P[SC_BLOOM], exposure = P[SC_EXPOSURE];
  const v3 v = mk(c.x + b.x * amount, c.y + b.y * amount, c.z + b.z * amount) * exposure;
  out[(int64_t)py * w + px] = make_float4(v.x / (1.f + v.x), v.y / (1.f + v.y), v.z / (1.f + v.z), 1.f);
}

// ── host side ───────────────────────────────────────────────────────────────
// Argument lists (B buffer, i int); ndrange in parentheses.
//   sc_move_lights  pos, centers, params, home, lcol, P, first        (lights)
//   sc_cull         visible, counter, centers, P, matrix offset in P  (instances)
//   sc_write_draw   cmd, counter, vertices per instance               (1)
//   sc_tile_lights  tilelights, tilecount, depth, lpos, P, W, H, tile, nlight, pertile  (tiles x, tiles y)
//   sc_ssao         ao, depth, normal, P, W, H, nsample              (aow, aoh)
//   sc_ao_blur      dst, src, P                                       (aow, aoh)
//   sc_shade        hdr, albedo, matter, normal, depth, lpos, lcol, tilelights, tilecount,
//                   shadow map, ao map, P, tile, pertile, smap res    (W, H)
//   sc_bright       dst, hdr, P, W, H, shift                          (bw, bh)
//   sc_blur         dst, src, dx, dy                                  (bw, bh)
//   sc_composite    out, hdr, bloom, P, bw, bh, shift                 (W, H)
static mtl_status sc_launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MTL_OK : fail(MTL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}
static mtl_status sc_need(const uint64_t* bytes, int i, uint64_t b, const char* kern) {
  if (bytes[i] && bytes[i] < b)
    return fail(MTL_ERR_ARGUMENT, "%s: argument %d has %llu bytes, the launch touches %llu", kern, i + 1,
                (unsigned long long)bytes[i], (unsigned long long)b);
  return MTL_OK;
}
static mtl_status sc_align(const LaunchArgs& la, int i, uint64_t a, const char* kern) {
  if (la.a[i].ptr % a) return fail(MTL_ERR_ARGUMENT, "%s: argument %d must be %llu-byte aligned", kern, i + 1,
                                   (unsigned long long)a);
  return MTL_OK;
}
static dim3 grid2(int64_t x, int64_t y, dim3 b) {
  return dim3((unsigned)((x + b.x - 1) / b.x), (unsigned)((y + b.y - 1) / b.y));
}
static bool dims2(const LaunchArgs& la) { return la.ndim == 2 && la.nd[0] >= 0 && la.nd[1] >= 0; }

mtl_status sc_move_lights_check(const LaunchArgs& la, const uint64_t* bytes) {
  const uint64_t n = (uint64_t)la.nd[0], first = (uint64_t)la.a[6].i32;
  if (la.ndim != 1 || la.a[6].i32 < 0) return fail(MTL_ERR_ARGUMENT, "sc_move_lights: ndrange = lights, first >= 0");
  for (int i : {0, 3, 4})
    if (mtl_status st = sc_need(bytes, i, 16 * n, "sc_move_lights")) return st;
  for (int i : {1, 2})
    if (mtl_status st = sc_need(bytes, i, 16 * (first + n), "sc_move_lights")) return st;
  if (mtl_status st = sc_need(bytes, 5, 4 * SC_PARAMS, "sc_move_lights")) return st;
  for (int i : {0, 1, 2, 3, 4})
    if (mtl_status st = sc_align(la, i, 16, "sc_move_lights")) return st;
  return MTL_OK;
}
mtl_status sc_move_lights_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int n = (int)la.nd[0];
  if (n == 0) return MTL_OK;
  sc_move_lights_kernel<<<(n + 127) / 128, 128, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float4*>(la.a[0].ptr), reinterpret_cast<float4*>(la.a[1].ptr),
      reinterpret_cast<float4*>(la.a[2].ptr), reinterpret_cast<const float4*>(la.a[3].ptr),
      reinterpret_cast<const float4*>(la.a[4].ptr), reinterpret_cast<const float*>(la.a[5].ptr), la.a[6].i32, n);
  return sc_launched("sc_move_lights");
}

mtl_status sc_cull_check(const LaunchArgs& la, const uint64_t* bytes) {
  const uint64_t n = (uint64_t)la.nd[0];
  const int off = la.a[4].i32;
  if (la.ndim != 1) return fail(MTL_ERR_ARGUMENT, "sc_cull: ndrange = instances");
  if (off < 0 || off + 16 > SC_PARAMS) return fail(MTL_ERR_ARGUMENT, "sc_cull: matrix offset %d outside P", off);
  if (mtl_status st = sc_need(bytes, 0, 4 * n, "sc_cull")) return st;
  if (mtl_status st = sc_need(bytes, 1, 4, "sc_cull")) return st;
  if (mtl_status st = sc_need(bytes, 2, 16 * n, "sc_cull")) return st;
  if (mtl_status st = sc_need(bytes, 3, 4 * SC_PARAMS, "sc_cull")) return st;
  return sc_align(la, 2, 16, "sc_cull");
}
mtl_status sc_cull_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int n = (int)la.nd[0];
  if (n == 0) return MTL_OK;
  sc_cull_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<uint32_t*>(la.a[0].ptr), reinterpret_cast<uint32_t*>(la.a[1].ptr),
      reinterpret_cast<const float4*>(la.a[2].ptr), reinterpret_cast<const float*>(la.a[3].ptr), la.a[4].i32, n);
  return sc_launched("sc_cull");
}

mtl_status sc_write_draw_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (mtl_status st = sc_need(bytes, 0, 16, "sc_write_draw")) return st;
  return sc_need(bytes, 1, 4, "sc_write_draw");
}
mtl_status sc_write_draw_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  sc_write_draw_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(reinterpret_cast<uint32_t*>(la.a[0].ptr),
                                                          reinterpret_cast<const uint32_t*>(la.a[1].ptr),
                                                          (uint32_t)la.a[2].i32);
  return sc_launched("sc_write_draw");
}

mtl_status sc_tile_lights_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int w = la.a[5].i32, h = la.a[6].i32, tile = la.a[7].i32, nl = la.a[8].i32, pt = la.a[9].i32;
  if (!dims2(la) || w <= 0 || h <= 0 || tile <= 0 || tile > 32 || nl < 0 || pt <= 0)
    return fail(MTL_ERR_ARGUMENT, "sc_tile_lights: ndrange (tiles x, tiles y), 0 < tile <= 32, pertile > 0");
  if (la.nd[0] != (w + tile - 1) / tile || la.nd[1] != (h + tile - 1) / tile)
    return fail(MTL_ERR_ARGUMENT, "sc_tile_lights: ndrange must be (ceil(W/tile), ceil(H/tile))");
  const uint64_t nt = (uint64_t)la.nd[0] * la.nd[1];
  if (mtl_status st = sc_need(bytes, 0, 4 * nt * pt, "sc_tile_lights")) return st;
  if (mtl_status st = sc_need(bytes, 1, 4 * nt, "sc_tile_lights")) return st;
  if (mtl_status st = sc_need(bytes, 2, 4ull * w * h, "sc_tile_lights")) return st;
  if (mtl_status st = sc_need(bytes, 3, 16ull * nl, "sc_tile_lights")) return st;
  if (mtl_status st = sc_need(bytes, 4, 4 * SC_PARAMS, "sc_tile_lights")) return st;
  return sc_align(la, 3, 16, "sc_tile_lights");
}
mtl_status sc_tile_lights_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  if (la.nd[0] == 0 || la.nd[1] == 0) return MTL_OK;
  sc_tile_lights_kernel<<<dim3((unsigned)la.nd[0], (unsigned)la.nd[1]), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<uint32_t*>(la.a[0].ptr), reinterpret_cast<uint32_t*>(la.a[1].ptr),
      reinterpret_cast<const float*>(la.a[2].ptr), reinterpret_cast<const float4*>(la.a[3].ptr),
      reinterpret_cast<const float*>(la.a[4].ptr), la.a[5].i32, la.a[6].i32, la.a[7].i32, la.a[8].i32,
      la.a[9].i32);
  return sc_launched("sc_tile_lights");
}

mtl_status sc_ssao_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int w = la.a[4].i32, h = la.a[5].i32, ns = la.a[6].i32;
  if (!dims2(la) || w <= 0 || h <= 0 || ns <= 0)
    return fail(MTL_ERR_ARGUMENT, "sc_ssao: ndrange (aow, aoh), W, H, nsample > 0");
  if (la.nd[0] != (w + 1) / 2 || la.nd[1] != (h + 1) / 2)
    return fail(MTL_ERR_ARGUMENT, "sc_ssao: ndrange must be (ceil(W/2), ceil(H/2))");
  if (mtl_status st = sc_need(bytes, 0, 8ull * la.nd[0] * la.nd[1], "sc_ssao")) return st;
  if (mtl_status st = sc_need(bytes, 1, 4ull * w * h, "sc_ssao")) return st;
  if (mtl_status st = sc_need(bytes, 2, 4ull * w * h, "sc_ssao")) return st;
  if (mtl_status st = sc_need(bytes, 3, 4 * SC_PARAMS, "sc_ssao")) return st;
  return sc_align(la, 0, 8, "sc_ssao");
}
mtl_status sc_ssao_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const dim3 b(32, 8);
  sc_ssao_kernel<<<grid2(la.nd[0], la.nd[1], b), b, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float2*>(la.a[0].ptr), reinterpret_cast<const float*>(la.a[1].ptr),
      reinterpret_cast<const uint32_t*>(la.a[2].ptr), reinterpret_cast<const float*>(la.a[3].ptr), la.a[4].i32,
      la.a[5].i32, (int)la.nd[0], (int)la.nd[1], la.a[6].i32);
  return sc_launched("sc_ssao");
}

mtl_status sc_ao_blur_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (!dims2(la)) return fail(MTL_ERR_ARGUMENT, "sc_ao_blur: ndrange (aow, aoh)");
  const uint64_t n = (uint64_t)la.nd[0] * la.nd[1];
  if (mtl_status st = sc_need(bytes, 0, 4 * n, "sc_ao_blur")) return st;
  if (mtl_status st = sc_need(bytes, 1, 8 * n, "sc_ao_blur")) return st;
  if (mtl_status st = sc_need(bytes, 2, 4 * SC_PARAMS, "sc_ao_blur")) return st;
  return sc_align(la, 1, 8, "sc_ao_blur");
}
mtl_status sc_ao_blur_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  if (la.nd[0] == 0 || la.nd[1] == 0) return MTL_OK;
  const dim3 b(32, 8);
  sc_ao_blur_kernel<<<grid2(la.nd[0], la.nd[1], b), b, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float*>(la.a[0].ptr), reinterpret_cast<const float2*>(la.a[1].ptr),
      reinterpret_cast<const float*>(la.a[2].ptr), (int)la.nd[0], (int)la.nd[1]);
  return sc_launched("sc_ao_blur");
}

mtl_status sc_shade_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int tile = la.a[12].i32, pt = la.a[13].i32, res = la.a[14].i32;
  if (!dims2(la) || tile <= 0 || pt <= 0 || res <= 0)
    return fail(MTL_ERR_ARGUMENT, "sc_shade: ndrange (W, H), tile, pertile, shadow-map size > 0");
  const uint64_t w = (uint64_t)la.nd[0], h = (uint64_t)la.nd[1], npx = w * h;
  const uint64_t nt = ((w + tile - 1) / tile) * ((h + tile - 1) / tile);
  const uint64_t aon = ((w + 1) / 2) * ((h + 1) / 2);
  if (mtl_status st = sc_need(bytes, 0, 16 * npx, "sc_shade")) return st;
  for (int i : {1, 2, 3, 4})
    if (mtl_status st = sc_need(bytes, i, 4 * npx, "sc_shade")) return st;
  if (mtl_status st = sc_need(bytes, 7, 4 * nt * pt, "sc_shade")) return st;
  if (mtl_status st = sc_need(bytes, 8, 4 * nt, "sc_shade")) return st;
  if (mtl_status st = sc_need(bytes, 9, 4ull * res * res, "sc_shade")) return st;
  if (mtl_status st = sc_need(bytes, 10, 4 * aon, "sc_shade")) return st;
  if (mtl_status st = sc_need(bytes, 11, 4 * SC_PARAMS, "sc_shade")) return st;
  for (int i : {0, 5, 6})
    if (mtl_status st = sc_align(la, i, 16, "sc_shade")) return st;
  return MTL_OK;
}
mtl_status sc_shade_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  const int w = (int)la.nd[0], h = (int)la.nd[1];
  if (w == 0 || h == 0) return MTL_OK;
  const dim3 b(16, 16);  // one light tile of 16 x 16 per CTA at the reference's tile size
  sc_shade_kernel<<<grid2(w, h, b), b, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float4*>(la.a[0].ptr), reinterpret_cast<const uint32_t*>(la.a[1].ptr),
      reinterpret_cast<const uint32_t*>(la.a[2].ptr), reinterpret_cast<const uint32_t*>(la.a[3].ptr),
      reinterpret_cast<const float*>(la.a[4].ptr), reinterpret_cast<const float4*>(la.a[5].ptr),
      reinterpret_cast<const float4*>(la.a[6].ptr), reinterpret_cast<const uint32_t*>(la.a[7].ptr),
      reinterpret_cast<const uint32_t*>(la.a[8].ptr), reinterpret_cast<const float*>(la.a[9].ptr),
      reinterpret_cast<const float*>(la.a[10].ptr), reinterpret_cast<const float*>(la.a[11].ptr), w, h, la.a[12].i32,
      la.a[13].i32, la.a[14].i32, (w + 1) / 2, (h + 1) / 2);
  return sc_launched("sc_shade");
}

mtl_status sc_bright_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int w = la.a[3].i32, h = la.a[4].i32, shift = la.a[5].i32;
  if (!dims2(la) || w <= 0 || h <= 0 || shift <= 0) return fail(MTL_ERR_ARGUMENT, "sc_bright: bad sizes");
  if (la.nd[0] != (w + shift - 1) / shift || la.nd[1] != (h + shift - 1) / shift)
    return fail(MTL_ERR_ARGUMENT, "sc_bright: ndrange must be (ceil(W/shift), ceil(H/shift))");
  if (mtl_status st = sc_need(bytes, 0, 16ull * la.nd[0] * la.nd[1], "sc_bright")) return st;
  if (mtl_status st = sc_need(bytes, 1, 16ull * w * h, "sc_bright")) return st;
  if (mtl_status st = sc_need(bytes, 2, 4 * SC_PARAMS, "sc_bright")) return st;
  for (int i : {0, 1})
    if (mtl_status st = sc_align(la, i, 16, "sc_bright")) return st;
  return MTL_OK;
}
mtl_status sc_bright_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  if (la.nd[0] == 0 || la.nd[1] == 0) return MTL_OK;
  const dim3 b(32, 8);
  sc_bright_kernel<<<grid2(la.nd[0], la.nd[1], b), b, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float4*>(la.a[0].ptr), reinterpret_cast<const float4*>(la.a[1].ptr),
      reinterpret_cast<const float*>(la.a[2].ptr), la.a[3].i32, la.a[4].i32, (int)la.nd[0], (int)la.nd[1],
      la.a[5].i32);
  return sc_launched("sc_bright");
}

mtl_status sc_blur_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (!dims2(la)) return fail(MTL_ERR_ARGUMENT, "sc_blur: ndrange (bw, bh)");
  const uint64_t n = 16ull * la.nd[0] * la.nd[1];
  if (mtl_status st = sc_need(bytes, 0, n, "sc_blur")) return st;
  if (mtl_status st = sc_need(bytes, 1, n, "sc_blur")) return st;
  const uint64_t d = la.a[0].ptr, x = la.a[1].ptr;
  if (d < x + n && x < d + n) return fail(MTL_ERR_ARGUMENT, "sc_blur: dst and src overlap (it reads neighbours)");
  for (int i : {0, 1})
    if (mtl_status st = sc_align(la, i, 16, "sc_blur")) return st;
  return MTL_OK;
}
mtl_status sc_blur_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  if (la.nd[0] == 0 || la.nd[1] == 0) return MTL_OK;
  const dim3 b(32, 8);
  sc_blur_kernel<<<grid2(la.nd[0], la.nd[1], b), b, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float4*>(la.a[0].ptr), reinterpret_cast<const float4*>(la.a[1].ptr), (int)la.nd[0],
      (int)la.nd[1], la.a[2].i32, la.a[3].i32);
  return sc_launched("sc_blur");
}

mtl_status sc_composite_check(const LaunchArgs& la, const uint64_t* bytes) {
  const int bw = la.a[4].i32, bh = la.a[5].i32, shift = la.a[6].i32;
  if (!dims2(la) || bw <= 0 || bh <= 0 || shift <= 0) return fail(MTL_ERR_ARGUMENT, "sc_composite: bad sizes");
  const uint64_t npx = (uint64_t)la.nd[0] * la.nd[1];
  if (mtl_status st = sc_need(bytes, 0, 16 * npx, "sc_composite")) return st;
  if (mtl_status st = sc_need(bytes, 1, 16 * npx, "sc_composite")) return st;
  if (mtl_status st = sc_need(bytes, 2, 16ull * bw * bh, "sc_composite")) return st;
  if (mtl_status st = sc_need(bytes, 3, 4 * SC_PARAMS, "sc_composite")) return st;
  for (int i : {0, 1, 2})
    if (mtl_status st = sc_align(la, i, 16, "sc_composite")) return st;
  return MTL_OK;
}
mtl_status sc_composite_run(const LaunchArgs& la, void*, uint64_t, void* stream) {
  if (la.nd[0] == 0 || la.nd[1] == 0) return MTL_OK;
  const dim3 b(32, 8);
  sc_composite_kernel<<<grid2(la.nd[0], la.nd[1], b), b, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<float4*>(la.a[0].ptr), reinterpret_cast<const float4*>(la.a[1].ptr),
      reinterpret_cast<const float4*>(la.a[2].ptr), reinterpret_cast<const float*>(la.a[3].ptr), (int)la.nd[0],
      (int)la.nd[1], la.a[4].i32, la.a[5].i32, la.a[6].i32);
  return sc_launched("sc_composite");
}

}  // namespace mtl
