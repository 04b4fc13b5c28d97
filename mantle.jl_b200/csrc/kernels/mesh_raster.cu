// Headless triangle rasterisation of instanced meshes: the g-buffer and shadow
// passes of the reference's deferred renderers (bench/showcase.jl:231-257
// gbuffer_vertex/gbuffer_fragment, :259-270 shadow_vertex; bench/deferred.jl
// :121-145), written as CUDA kernels instead of a graphics pipeline.
//
// What one launch draws: every instance named by the culled list `visible`
// (1-based instance indices, `counter[0]` of them, as the cull pass writes
// them), each a copy of the prototype triangle list (V vertices, T = V/3
// triangles) scaled by sizes.xyz, turned by the yaw sizes.w and moved to
// centers.xyz, seen through the 4x4 matrix P[mat..mat+15] (column-major).
// The rules of the Vulkan pipeline the reference describes:
//   * clip volume 0 <= z <= w (near and far are clipped, Sutherland-Hodgman in
//     clip space; x and y are clipped only against a guard band of 16 w, the
//     rest is the scissor);
//   * viewport (0, 0, W, H): x_f = x_ndc*W/2 + W/2, y_f = y_ndc*H/2 + H/2,
//     depth z_ndc; samples at pixel centres;
//   * back faces culled, front face counter-clockwise: a triangle is kept when
//     Vulkan's a = -1/2 sum(x_i y_i+1 - x_i+1 y_i) over framebuffer
//     coordinates is positive;
//   * depth test LESS against a depth cleared to 1;
//   * perspective-correct interpolation of the varyings.
// Coverage is decided exactly: vertices are snapped to 1/256 pixel and the
// edge functions are 64-bit integers, with a tie rule for samples exactly on
// an edge that gives a shared edge to exactly one of its two triangles.
//
// Visibility first, attributes after. Every covered sample proposes the key
// (depth bits << 32) | primitive (positive float depths order like their bits;
// primitive = ((instance * T + triangle) << 3) | clipped piece) and the pixel
// keeps the smallest (atomicMin): the nearest surface, ties to the smaller
// primitive, whatever order the triangles ran in. A resolve pass then
// recomputes the winning triangle at each pixel and evaluates the fragment.
//
// Work split: a setup kernel transforms, clips, snaps and culls one prototype
// triangle per thread and sorts the pieces by screen size: those whose box is
// at most 64 x 64 pixels go to a list rasterised one warp per piece (lanes over
// the box), the others to a list rasterised per 16 x 16 screen tile by a CTA
// that first selects the big pieces meeting its tile, then tests them one
// pixel per thread, keeping its minimum in a register and merging once.
//
// Modes: 0 the showcase's g-buffer (albedo + roughness, metalness + emission,
// normal, each RGBA8 packed R in the low byte, and depth), 1 depth only (the
// shadow map), 2 deferred.jl's g-buffer (albedo, normal as given, and depth).
//
// Compiled without FMA contraction (-fmad=false): every float operation
// rounds once, in the order written, as in the CPU oracle.

#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdint>

#include "../mtl_internal.hpp"

namespace mtl {

constexpr float kGuard = 16.f;
constexpr int kSub = 256;           // subpixel steps per pixel
constexpr int kWarpBox = 64 * 64;   // pieces with a box up to this many pixels go to the warp list
constexpr int kTile = 16;           // big pieces: 16 x 16 pixel tiles, one CTA each
constexpr int kMaxPoly = 9;         // a triangle clipped by six planes
constexpr int kSetupThreads = 128;

struct RasterArgs {
  float* depth;
  uint32_t* out0;
  uint32_t* out1;
  uint32_t* out2;
  const float4* ppos;
  const float4* pnrm;
  const uint32_t* visible;
  const uint32_t* counter;
  const float4* centers;
  const float4* sizes;
  const float4* colors;
  const float4* params;
  const float* M;  // the 4x4 matrix, column-major
  int mode, W, H, T, ninst;
};

// One clipped, snapped piece of a triangle, oriented so that its edge
// functions are positive inside.
struct Piece {
  int32_t X[3], Y[3];
  float z[3];
  uint16_t bx0, by0, bx1, by1;  // inclusive pixel box
  uint32_t prim;
};
static_assert(sizeof(Piece) == 48, "piece layout");

struct Scratch {
  unsigned long long* vis;  // W*H keys
  uint32_t* counts;         // [0] warp list, [1] big list
  Piece* warp_list;
  Piece* big_list;
  uint2* big_box;           // the big pieces' boxes, packed (x0 | y0 << 16, x1 | y1 << 16)
  uint64_t cap;             // pieces per list
};

struct CV {  // a clip-space vertex and its barycentric coordinates in the prototype triangle
  float x, y, z, w, u0, u1, u2;
};

__device__ __forceinline__ float4 mat4v(const float* M, float x, float y, float z, float w) {
  float4 q;
  q.x = M[0] * x + M[4] * y + M[8] * z + M[12] * w;
  q.y = M[1] * x + M[5] * y + M[9] * z + M[13] * w;
  q.z = M[2] * x + M[6] * y + M[10] * z + M[14] * w;
  q.w = M[3] * x + M[7] * y + M[11] * z + M[15] * w;
  return q;
}

// The yaw of an instance: cos and sin in double, rounded to float, so the
// result does not depend on which float sine the platform has.
__device__ __forceinline__ void yaw_of(float a, float* ca, float* sa) {
  double s, c;
  sincos((double)a, &s, &c);
  *ca = (float)c;
  *sa = (float)s;
}

// World position of prototype vertex lp in instance (c, s); showcase.jl:238-242.
__device__ __forceinline__ float4 world_of(float4 c, float4 s, float4 lp, float ca, float sa) {
  const float px = lp.x * s.x, py = lp.y * s.y, pz = lp.z * s.z;
  return make_float4(c.x + ca * px + sa * pz, c.y + py, c.z - sa * px + ca * pz, 1.f);
}

// Signed distance of v to clip plane k (inside when >= 0).
__device__ __forceinline__ float plane_d(const CV& v, int k) {
  switch (k) {
    case 0: return v.z;
    case 1: return v.w - v.z;
    case 2: return kGuard * v.w - v.x;
    case 3: return kGuard * v.w + v.x;
    case 4: return kGuard * v.w - v.y;
    default: return kGuard * v.w + v.y;
  }
}
__device__ __forceinline__ CV lerp_cv(const CV& a, const CV& b, float t) {
  CV r;
  r.x = a.x + t * (b.x - a.x);
  r.y = a.y + t * (b.y - a.y);
  r.z = a.z + t * (b.z - a.z);
  r.w = a.w + t * (b.w - a.w);
  r.u0 = a.u0 + t * (b.u0 - a.u0);
  r.u1 = a.u1 + t * (b.u1 - a.u1);
  r.u2 = a.u2 + t * (b.u2 - a.u2);
  return r;
}

// Clip a triangle to the six planes; returns the polygon's vertex count (0 when
// nothing is left). Planes a polygon is wholly inside are skipped.
__device__ int clip_poly(CV (&poly)[kMaxPoly]) {
  int n = 3;
  CV tmp[kMaxPoly];
  for (int k = 0; k < 6 && n > 0; ++k) {
    bool all_in = true;
    for (int i = 0; i < n; ++i) all_in &= plane_d(poly[i], k) >= 0.f;
    if (all_in) continue;
    int m = 0;
    for (int i = 0; i < n; ++i) {
      const CV& a = poly[i];
      const CV& b = poly[i + 1 == n ? 0 : i + 1];
      const float da = plane_d(a, k), db = plane_d(b, k);
      if (da >= 0.f) tmp[m++] = a;
      if ((da >= 0.f) != (db >= 0.f)) tmp[m++] = lerp_cv(a, b, da / (da - db));
    }
    n = m;
    for (int i = 0; i < n; ++i) poly[i] = tmp[i];
  }
  return n;
}

struct Snap {
  int32_t X, Y;
  float z, iw;
};
__device__ __forceinline__ Snap snap(const CV& v, int W, int H) {
  Snap s;
  const float xn = v.x / v.w, yn = v.y / v.w;
  s.z = v.z / v.w;
  s.iw = 1.f / v.w;
  const float hw = 0.5f * (float)W, hh = 0.5f * (float)H;
  s.X = (int32_t)rintf((xn * hw + hw) * (float)kSub);
  s.Y = (int32_t)rintf((yn * hh + hh) * (float)kSub);
  return s;
}
__device__ __forceinline__ int64_t edge(int32_t ax, int32_t ay, int32_t bx, int32_t by, int64_t px, int64_t py) {
  return (int64_t)(bx - ax) * (py - ay) - (int64_t)(by - ay) * (px - ax);
}
// A sample exactly on edge a->b belongs to this triangle when the edge runs
// down the framebuffer, or along it to the left.
__device__ __forceinline__ bool owns_edge(int32_t ax, int32_t ay, int32_t bx, int32_t by) {
  const int32_t dx = bx - ax, dy = by - ay;
  return dy > 0 || (dy == 0 && dx < 0);
}
__device__ __forceinline__ bool inside(int64_t e, bool own) { return e > 0 || (e == 0 && own); }

// The three prototype vertices of triangle t of instance o, in clip space.
__device__ __forceinline__ void triangle_cv(const RasterArgs& a, int o, int t, CV (&poly)[kMaxPoly]) {
  const float4 c = a.centers[o], s = a.sizes[o];
  float ca, sa;
  yaw_of(s.w, &ca, &sa);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float4 wp = world_of(c, s, a.ppos[3 * t + i], ca, sa);
    const float4 q = mat4v(a.M, wp.x, wp.y, wp.z, wp.w);
    poly[i] = CV{q.x, q.y, q.z, q.w, i == 0 ? 1.f : 0.f, i == 1 ? 1.f : 0.f, i == 2 ? 1.f : 0.f};
  }
}

__device__ __forceinline__ int floor_div(int32_t a, int32_t b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }
__device__ __forceinline__ int ceil_div(int32_t a, int32_t b) { return -floor_div(-a, b); }

// Piece `sub` of the clipped polygon (a fan from vertex 0), snapped, culled
// and oriented. Returns false when it is culled or covers no pixel centre.
__device__ bool make_piece(const CV (&poly)[kMaxPoly], int n, int sub, int W, int H, Snap (&sv)[3], int (&vi)[3],
                           int* bx0, int* by0, int* bx1, int* by1) {
  if (sub + 2 >= n) return false;
  vi[0] = 0;
  vi[1] = sub + 1;
  vi[2] = sub + 2;
  for (int i = 0; i < 3; ++i) {
    if (!(poly[vi[i]].w > 0.f)) return false;  // only the clip volume's apex, (0, 0, 0, 0), has no position
    sv[i] = snap(poly[vi[i]], W, H);
  }
  const int64_t S = edge(sv[0].X, sv[0].Y, sv[1].X, sv[1].Y, sv[2].X, sv[2].Y);
  if (S >= 0) return false;  // a <= 0: a back face, or no area
  // positive orientation for the edge functions
  Snap t = sv[1];
  sv[1] = sv[2];
  sv[2] = t;
  int u = vi[1];
  vi[1] = vi[2];
  vi[2] = u;
  const int32_t xmin = min(sv[0].X, min(sv[1].X, sv[2].X)), xmax = max(sv[0].X, max(sv[1].X, sv[2].X));
  const int32_t ymin = min(sv[0].Y, min(sv[1].Y, sv[2].Y)), ymax = max(sv[0].Y, max(sv[1].Y, sv[2].Y));
  // pixel p's sample is at p*256 + 128: the pixels whose samples lie in
  // [min, max] are ceil((min - 128) / 256) .. floor((max - 128) / 256)
  *bx0 = max(0, ceil_div(xmin - kSub / 2, kSub));
  *by0 = max(0, ceil_div(ymin - kSub / 2, kSub));
  *bx1 = min(W - 1, floor_div(xmax - kSub / 2, kSub));
  *by1 = min(H - 1, floor_div(ymax - kSub / 2, kSub));
  return *bx0 <= *bx1 && *by0 <= *by1;
}

// Depth from the three edge values at a sample of a positively oriented
// piece: the barycentric weights e_i / S (S = e0 + e1 + e2, twice the
// piece's area in subpixels, the same at every sample) applied to the
// vertices' depths, as ((e0 z0 + e1 z1) + e2 z2) * (1 / S). -1 when the depth
// is outside [0, 1) (the clip range, and the test LESS against 1).
__device__ __forceinline__ float depth_of(float f0, float f1, float f2, const float (&z)[3], float inv_s) {
  const float d = (f0 * z[0] + f1 * z[1] + f2 * z[2]) * inv_s + 0.f;  // + 0: a depth of -0 becomes +0
  return (d >= 0.f && d < 1.f) ? d : -1.f;
}
__device__ __forceinline__ float inv_area(const int32_t (&X)[3], const int32_t (&Y)[3]) {
  return 1.f / (float)edge(X[0], Y[0], X[1], Y[1], X[2], Y[2]);
}
// Depth at sample (sx, sy) of a positively oriented piece, or -1 when the
// sample is not covered (or the depth is out of range).
__device__ __forceinline__ float piece_depth(const int32_t (&X)[3], const int32_t (&Y)[3], const float (&z)[3],
                                             float inv_s, int64_t sx, int64_t sy) {
  const int64_t e0 = edge(X[1], Y[1], X[2], Y[2], sx, sy);
  const int64_t e1 = edge(X[2], Y[2], X[0], Y[0], sx, sy);
  const int64_t e2 = edge(X[0], Y[0], X[1], Y[1], sx, sy);
  if (!inside(e0, owns_edge(X[1], Y[1], X[2], Y[2])) || !inside(e1, owns_edge(X[2], Y[2], X[0], Y[0])) ||
      !inside(e2, owns_edge(X[0], Y[0], X[1], Y[1])))
    return -1.f;
  return depth_of((float)e0, (float)e1, (float)e2, z, inv_s);
}
__device__ __forceinline__ unsigned long long key_of(float d, uint32_t prim) {
  return ((unsigned long long)__float_as_uint(d) << 32) | prim;
}

// ── setup: one prototype triangle of one visible instance per thread ────────
__global__ void __launch_bounds__(kSetupThreads) raster_setup_kernel(RasterArgs a, Scratch s) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t count = min(a.counter[0], (uint32_t)a.ninst);
  if (tid >= (int64_t)count * a.T) return;
  const int slot = (int)(tid / a.T), t = (int)(tid % a.T);
  const uint32_t vis1 = a.visible[slot];
  if (vis1 == 0 || vis1 > (uint32_t)a.ninst) return;  // not an instance: nothing to draw
  const int o = (int)vis1 - 1;
  CV poly[kMaxPoly];
  triangle_cv(a, o, t, poly);
  const int n = clip_poly(poly);
  for (int sub = 0; sub + 2 < n; ++sub) {
    Snap sv[3];
    int vi[3], bx0, by0, bx1, by1;
    if (!make_piece(poly, n, sub, a.W, a.H, sv, vi, &bx0, &by0, &bx1, &by1)) continue;
    Piece p;
    for (int i = 0; i < 3; ++i) {
      p.X[i] = sv[i].X;
      p.Y[i] = sv[i].Y;
      p.z[i] = sv[i].z;
    }
    p.bx0 = (uint16_t)bx0;
    p.by0 = (uint16_t)by0;
    p.bx1 = (uint16_t)bx1;
    p.by1 = (uint16_t)by1;
    p.prim = ((uint32_t)(o * a.T + t) << 3) | (uint32_t)sub;
    const int64_t area = (int64_t)(bx1 - bx0 + 1) * (by1 - by0 + 1);
    const bool big = area > kWarpBox;
    const uint32_t at = atomicAdd(&s.counts[big ? 1 : 0], 1u);
    if (at < s.cap) {
      (big ? s.big_list : s.warp_list)[at] = p;
      if (big) s.big_box[at] = make_uint2((uint32_t)bx0 | ((uint32_t)by0 << 16), (uint32_t)bx1 | ((uint32_t)by1 << 16));
    }
  }
}

// ── the warp list: one warp per piece, lanes over its box ───────────────────
// The edge values step by constants from pixel to pixel: e(x0 + dx, y0 + dy) =
// e(x0, y0) + A dx + B dy. When every value over the box fits 32 bits (a box
// of at most 64 x 64 pixels whose vertices lie near it) the lanes step in
// 32-bit integers; otherwise they evaluate each edge in 64 bits. The values
// are the same integers either way.
__global__ void __launch_bounds__(256) raster_warp_kernel(Scratch s, int W) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const uint32_t n = min(s.counts[0], (uint32_t)s.cap);
  for (int64_t e = warp; e < n; e += nwarps) {
    const Piece p = s.warp_list[e];
    const int bw = p.bx1 - p.bx0 + 1;
    const int area = bw * (p.by1 - p.by0 + 1);
    const float inv_s = inv_area(p.X, p.Y);
    const int64_t sx0 = (int64_t)p.bx0 * kSub + kSub / 2, sy0 = (int64_t)p.by0 * kSub + kSub / 2;
    int64_t E0[3], A[3], B[3];
    int32_t bias[3];
    int64_t bound = 0;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int a = k == 0 ? 1 : (k == 1 ? 2 : 0), b = k == 0 ? 2 : (k == 1 ? 0 : 1);
      E0[k] = edge(p.X[a], p.Y[a], p.X[b], p.Y[b], sx0, sy0);
      A[k] = -(int64_t)(p.Y[b] - p.Y[a]) * kSub;
      B[k] = (int64_t)(p.X[b] - p.X[a]) * kSub;
      bias[k] = owns_edge(p.X[a], p.Y[a], p.X[b], p.Y[b]) ? 0 : 1;  // inside: e >= bias
      const int64_t bk = (E0[k] < 0 ? -E0[k] : E0[k]) + (A[k] < 0 ? -A[k] : A[k]) * (bw - 1) +
                         (B[k] < 0 ? -B[k] : B[k]) * (p.by1 - p.by0);
      bound = bk > bound ? bk : bound;
    }
    const bool narrow = bound < (int64_t)INT32_MAX;
    // i / bw as a multiply-high (exact for i < 4096 and any bw <= 4096: the
    // error of the rounded-up reciprocal stays below 2^-20, the gap below the
    // next integer is at least 1/bw)
    const uint32_t mag = bw > 1 ? (uint32_t)((0x100000000ull + (uint32_t)bw - 1) / (uint32_t)bw) : 0u;
    unsigned long long* vrow = s.vis + (int64_t)p.by0 * W + p.bx0;
    if (narrow) {  // every edge value over the box fits 32 bits
      const int32_t e0 = (int32_t)E0[0], e1 = (int32_t)E0[1], e2 = (int32_t)E0[2];
      const int32_t a0 = (int32_t)A[0], a1 = (int32_t)A[1], a2 = (int32_t)A[2];
      const int32_t b0 = (int32_t)B[0], b1 = (int32_t)B[1], b2 = (int32_t)B[2];
      for (int i = lane; i < area; i += 32) {
        const int dy = bw > 1 ? (int)__umulhi((uint32_t)i, mag) : i, dx = i - dy * bw;
        const int32_t v0 = e0 + a0 * dx + b0 * dy, v1 = e1 + a1 * dx + b1 * dy, v2 = e2 + a2 * dx + b2 * dy;
        if (v0 < bias[0] || v1 < bias[1] || v2 < bias[2]) continue;
        const float d = depth_of((float)v0, (float)v1, (float)v2, p.z, inv_s);
        if (d < 0.f) continue;
        const unsigned long long k = key_of(d, p.prim);
        unsigned long long* v = vrow + (int64_t)dy * W + dx;
        if (k < *v) atomicMin(v, k);
      }
    } else {
      for (int i = lane; i < area; i += 32) {
        const int dy = bw > 1 ? (int)__umulhi((uint32_t)i, mag) : i, dx = i - dy * bw;
        int64_t ev[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) ev[k] = E0[k] + A[k] * dx + B[k] * dy;
        if (ev[0] < bias[0] || ev[1] < bias[1] || ev[2] < bias[2]) continue;
        const float d = depth_of((float)ev[0], (float)ev[1], (float)ev[2], p.z, inv_s);
        if (d < 0.f) continue;
        const unsigned long long k = key_of(d, p.prim);
        unsigned long long* v = vrow + (int64_t)dy * W + dx;
        if (k < *v) atomicMin(v, k);
      }
    }
  }
}

// ── the big list: one CTA per 16 x 16 tile, one pixel per thread ─────────────
// The CTA first picks out, all threads together, the big pieces whose boxes
// meet its tile (from the packed boxes, 8 bytes a piece), then tests only
// those against its pixels, in rounds of kFilter pieces.
constexpr int kFilter = 1024;
__global__ void __launch_bounds__(kTile* kTile) raster_big_kernel(Scratch s, int W, int H) {
  __shared__ uint32_t hits[kFilter];
  __shared__ int nhits;
  const int px = blockIdx.x * kTile + threadIdx.x % kTile, py = blockIdx.y * kTile + threadIdx.x / kTile;
  const uint32_t tx0 = blockIdx.x * kTile, ty0 = blockIdx.y * kTile;
  const uint32_t tx1 = tx0 + kTile - 1, ty1 = ty0 + kTile - 1;
  const uint32_t n = min(s.counts[1], (uint32_t)s.cap);
  unsigned long long best = ~0ull;
  const int64_t sx = (int64_t)px * kSub + kSub / 2, sy = (int64_t)py * kSub + kSub / 2;
  for (uint32_t base = 0; base < n; base += kFilter) {
    const uint32_t m = min((uint32_t)kFilter, n - base);
    if (threadIdx.x == 0) nhits = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
      const uint2 b = s.big_box[base + i];
      const uint32_t bx0 = b.x & 0xffffu, by0 = b.x >> 16, bx1 = b.y & 0xffffu, by1 = b.y >> 16;
      if (bx1 >= tx0 && bx0 <= tx1 && by1 >= ty0 && by0 <= ty1) hits[atomicAdd(&nhits, 1)] = base + i;
    }
    __syncthreads();
    const int nh = nhits;
    for (int j = 0; j < nh; ++j) {
      const Piece& p = s.big_list[hits[j]];
      if (px > p.bx1 || px < p.bx0 || py > p.by1 || py < p.by0) continue;
      const float d = piece_depth(p.X, p.Y, p.z, inv_area(p.X, p.Y), sx, sy);
      if (d < 0.f) continue;
      const unsigned long long k = key_of(d, p.prim);
      best = k < best ? k : best;
    }
    __syncthreads();
  }
  if (px < W && py < H && best != ~0ull) atomicMin(s.vis + (int64_t)py * W + px, best);
}

__device__ __forceinline__ uint32_t q8(float x) { return __float2uint_rn(fminf(fmaxf(x, 0.f), 1.f) * 255.f); }
__device__ __forceinline__ uint32_t pack4(float r, float g, float b, float al) {
  return q8(r) | (q8(g) << 8) | (q8(b) << 16) | (q8(al) << 24);
}

// ── resolve: the winning piece at each pixel, its fragment evaluated ─────────
__global__ void __launch_bounds__(256) raster_resolve_kernel(RasterArgs a, Scratch s) {
  const int px = blockIdx.x * 16 + threadIdx.x % 16, py = blockIdx.y * 16 + threadIdx.x / 16;
  if (px >= a.W || py >= a.H) return;
  const int64_t pix = (int64_t)py * a.W + px;
  const unsigned long long k = s.vis[pix];
  if (k == ~0ull) {
    a.depth[pix] = 1.f;
    if (a.mode != 1) {
      a.out0[pix] = 0xff000000u;  // albedo cleared to (0, 0, 0, 1)
      a.out1[pix] = 0u;
      if (a.mode == 0) a.out2[pix] = 0u;
    }
    return;
  }
  const float d = __uint_as_float((uint32_t)(k >> 32));
  a.depth[pix] = d;
  if (a.mode == 1) return;
  const uint32_t prim = (uint32_t)k;
  const int sub = (int)(prim & 7u), ot = (int)(prim >> 3);
  const int o = ot / a.T, t = ot % a.T;
  CV poly[kMaxPoly];
  triangle_cv(a, o, t, poly);
  const int n = clip_poly(poly);
  Snap sv[3];
  int vi[3], bx0, by0, bx1, by1;
  if (!make_piece(poly, n, sub, a.W, a.H, sv, vi, &bx0, &by0, &bx1, &by1)) return;  // cannot happen: it won
  const int64_t sx = (int64_t)px * kSub + kSub / 2, sy = (int64_t)py * kSub + kSub / 2;
  const int64_t e0 = edge(sv[1].X, sv[1].Y, sv[2].X, sv[2].Y, sx, sy);
  const int64_t e1 = edge(sv[2].X, sv[2].Y, sv[0].X, sv[0].Y, sx, sy);
  const int64_t e2 = edge(sv[0].X, sv[0].Y, sv[1].X, sv[1].Y, sx, sy);
  // perspective-correct weights of the piece's vertices (the screen-space
  // weights e_i / S over w_i, normalised: S cancels), then of the prototype
  // triangle's
  const float q0 = (float)e0 * sv[0].iw, q1 = (float)e1 * sv[1].iw, q2 = (float)e2 * sv[2].iw;
  const float qs = q0 + q1 + q2;
  const float b0 = q0 / qs, b1 = q1 / qs, b2 = q2 / qs;
  const CV& v0 = poly[vi[0]];
  const CV& v1 = poly[vi[1]];
  const CV& v2 = poly[vi[2]];
  const float U0 = b0 * v0.u0 + b1 * v1.u0 + b2 * v2.u0;
  const float U1 = b0 * v0.u1 + b1 * v1.u1 + b2 * v2.u1;
  const float U2 = b0 * v0.u2 + b1 * v1.u2 + b2 * v2.u2;
  const float4 col = a.colors[o];
  // the vertex normals, as the vertex stage outputs them
  float3 nv[3];
  const float4 sz = a.sizes[o];
  float ca, sa;
  yaw_of(sz.w, &ca, &sa);
  for (int i = 0; i < 3; ++i) {
    const float4 ln = a.pnrm[3 * t + i];
    if (a.mode == 0) {  // inverse scale, then the yaw (showcase.jl:243-246)
      const float nx = ln.x / sz.x, ny = ln.y / sz.y, nz = ln.z / sz.z;
      const float rx = ca * nx + sa * nz, ry = ny, rz = -sa * nx + ca * nz;
      const float len = sqrtf(rx * rx + ry * ry + rz * rz);
      nv[i] = make_float3(rx / len, ry / len, rz / len);
    } else {  // as given (deferred.jl:135)
      nv[i] = make_float3(ln.x, ln.y, ln.z);
    }
  }
  float nx = U0 * nv[0].x + U1 * nv[1].x + U2 * nv[2].x;
  float ny = U0 * nv[0].y + U1 * nv[1].y + U2 * nv[2].y;
  float nz = U0 * nv[0].z + U1 * nv[1].z + U2 * nv[2].z;
  if (a.mode == 0) {
    const float len = sqrtf(nx * nx + ny * ny + nz * nz);
    nx = nx / len;
    ny = ny / len;
    nz = nz / len;
    const float4 par = a.params[o];
    a.out0[pix] = pack4(col.x, col.y, col.z, col.w);
    a.out1[pix] = pack4(par.x, fminf(1.f, par.y), 0.f, 1.f);
    a.out2[pix] = pack4(0.5f * nx + 0.5f, 0.5f * ny + 0.5f, 0.5f * nz + 0.5f, 1.f);
  } else {
    a.out0[pix] = pack4(col.x, col.y, col.z, col.w);
    a.out1[pix] = pack4(0.5f * nx + 0.5f, 0.5f * ny + 0.5f, 0.5f * nz + 0.5f, 1.f);
  }
}

// ── host side ────────────────────────────────────────────────────────────────
// Arguments: depth (B), out0 (b), out1 (b), out2 (b), proto positions (B),
// proto normals (b), visible (B), counter (B), centers (B), sizes (B),
// colors (b), params (b), P (B), mat, mode, W, H, nverts (i); ndrange = the
// number of instances (the length of visible, centers, sizes, ...).
static void unpack(const LaunchArgs& la, RasterArgs& a) {
  auto F4 = [&](int i) { return reinterpret_cast<const float4*>(la.a[i].kind == MTL_ARG_PTR ? la.a[i].ptr : 0); };
  auto U = [&](int i) { return reinterpret_cast<uint32_t*>(la.a[i].kind == MTL_ARG_PTR ? la.a[i].ptr : 0); };
  a.depth = reinterpret_cast<float*>(la.a[0].ptr);
  a.out0 = U(1);
  a.out1 = U(2);
  a.out2 = U(3);
  a.ppos = F4(4);
  a.pnrm = F4(5);
  a.visible = U(6);
  a.counter = U(7);
  a.centers = F4(8);
  a.sizes = F4(9);
  a.colors = F4(10);
  a.params = F4(11);
  a.M = reinterpret_cast<const float*>(la.a[12].ptr) + la.a[13].i32;
  a.mode = la.a[14].i32;
  a.W = la.a[15].i32;
  a.H = la.a[16].i32;
  a.T = la.a[17].i32 / 3;
  a.ninst = (int)la.nd[0];
}

static uint64_t pieces_cap(const LaunchArgs& la) {
  // every prototype triangle of every instance, clipped into at most seven pieces
  return (uint64_t)la.nd[0] * (uint64_t)(la.a[17].i32 / 3) * 7;
}
static uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

uint64_t raster_workspace(const LaunchArgs& la) {
  const uint64_t W = (uint64_t)std::max(la.a[15].i32, 0), H = (uint64_t)std::max(la.a[16].i32, 0);
  return align256(W * H * 8) + 256 + 2 * align256(pieces_cap(la) * sizeof(Piece)) + align256(pieces_cap(la) * 8);
}

mtl_status raster_check(const LaunchArgs& la, const uint64_t* bytes) {
  if (la.ndim != 1) return fail(MTL_ERR_ARGUMENT, "raster_instances: ndrange must be the instance count");
  const int mode = la.a[14].i32, W = la.a[15].i32, H = la.a[16].i32, nv = la.a[17].i32;
  const int64_t ninst = la.nd[0];
  if (mode < 0 || mode > 2) return fail(MTL_ERR_ARGUMENT, "raster_instances: mode %d (0 g-buffer, 1 depth, 2 deferred)", mode);
  if (W <= 0 || H <= 0 || W > 16384 || H > 16384)
    return fail(MTL_ERR_ARGUMENT, "raster_instances: %d x %d pixels (1..16384 each)", W, H);
  if (nv <= 0 || nv % 3 || nv / 3 > 1024) return fail(MTL_ERR_ARGUMENT, "raster_instances: %d prototype vertices", nv);
  if (ninst < 0 || (uint64_t)ninst * (nv / 3) >= (1ull << 29))
    return fail(MTL_ERR_ARGUMENT, "raster_instances: %lld instances of %d triangles exceed 2^29 primitives",
                (long long)ninst, nv / 3);
  if (la.a[13].i32 < 0) return fail(MTL_ERR_ARGUMENT, "raster_instances: negative matrix offset");
  const bool colour = mode != 1;
  struct Need {
    int i;
    uint64_t b;
    bool needed;
    const char* what;
  } need[] = {{0, (uint64_t)W * H * 4, true, "depth"},
              {1, (uint64_t)W * H * 4, colour, "out0"},
              {2, (uint64_t)W * H * 4, colour, "out1"},
              {3, (uint64_t)W * H * 4, mode == 0, "out2"},
              {4, (uint64_t)nv * 16, true, "prototype positions"},
              {5, (uint64_t)nv * 16, colour, "prototype normals"},
              {6, (uint64_t)ninst * 4, true, "visible"},
              {7, 4, true, "counter"},
              {8, (uint64_t)ninst * 16, true, "centers"},
              {9, (uint64_t)ninst * 16, true, "sizes"},
              {10, (uint64_t)ninst * 16, colour, "colors"},
              {11, (uint64_t)ninst * 16, mode == 0, "params"},
              {12, (uint64_t)(la.a[13].i32 + 16) * 4, true, "the matrix buffer"}};
  for (const Need& n : need) {
    if (!n.needed) continue;
    if (la.a[n.i].kind != MTL_ARG_PTR || la.a[n.i].ptr == 0)
      return fail(MTL_ERR_ARGUMENT, "raster_instances: mode %d needs %s", mode, n.what);
    if (bytes[n.i] && bytes[n.i] < n.b)
      return fail(MTL_ERR_ARGUMENT, "raster_instances: %s has %llu bytes, the launch touches %llu", n.what,
                  (unsigned long long)bytes[n.i], (unsigned long long)n.b);
  }
  for (int i : {4, 5, 8, 9, 10, 11})
    if (la.a[i].kind == MTL_ARG_PTR && (la.a[i].ptr & 15))
      return fail(MTL_ERR_ARGUMENT, "raster_instances: argument %d must be 16-byte aligned (float4)", i + 1);
  return MTL_OK;
}

mtl_status raster_run(const LaunchArgs& la, void* ws, uint64_t ws_bytes, void* stream) {
  RasterArgs a;
  unpack(la, a);
  cudaStream_t st = (cudaStream_t)stream;
  const uint64_t need = raster_workspace(la);
  if (!ws || ws_bytes < need)
    return fail(MTL_ERR_ARGUMENT, "raster_instances: needs %llu bytes of scratch, got %llu", (unsigned long long)need,
                (unsigned long long)ws_bytes);
  Scratch s;
  unsigned char* p = reinterpret_cast<unsigned char*>(ws);
  s.vis = reinterpret_cast<unsigned long long*>(p);
  p += align256((uint64_t)a.W * a.H * 8);
  s.counts = reinterpret_cast<uint32_t*>(p);
  p += 256;
  s.cap = pieces_cap(la);
  s.warp_list = reinterpret_cast<Piece*>(p);
  p += align256(s.cap * sizeof(Piece));
  s.big_list = reinterpret_cast<Piece*>(p);
  p += align256(s.cap * sizeof(Piece));
  s.big_box = reinterpret_cast<uint2*>(p);
  cudaError_t e = cudaMemsetAsync(s.vis, 0xff, (size_t)a.W * a.H * 8, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(s.counts, 0, 256, st);
  const int64_t threads = (int64_t)a.ninst * a.T;
  if (e == cudaSuccess && threads > 0) {
    raster_setup_kernel<<<(unsigned)((threads + kSetupThreads - 1) / kSetupThreads), kSetupThreads, 0, st>>>(a, s);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && threads > 0) {
    raster_warp_kernel<<<(unsigned)la.sm_count * 8, 256, 0, st>>>(s, a.W);
    e = cudaGetLastError();
  }
  dim3 tiles((unsigned)((a.W + kTile - 1) / kTile), (unsigned)((a.H + kTile - 1) / kTile));
  if (e == cudaSuccess && threads > 0) {
    raster_big_kernel<<<tiles, kTile * kTile, 0, st>>>(s, a.W, a.H);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    raster_resolve_kernel<<<tiles, 256, 0, st>>>(a, s);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return fail(MTL_ERR_CUDA, "raster_instances: %s", cudaGetErrorString(e));
  return MTL_OK;
}

}  // namespace mtl
