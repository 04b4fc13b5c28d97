/*
 * raster_oracle.c — CPU restatement of the headless triangle rasteriser
 * (the g-buffer and shadow passes of bench/showcase.jl:231-270 and the
 * g-buffer of bench/deferred.jl:121-145). TEST INFRASTRUCTURE ONLY: the parity
 * tests call it as the checker; the product never links or calls it.
 *
 * The rules (Vulkan's, as the reference's pipelines use them): clip volume
 * 0 <= z <= w plus a guard band of 16 w in x and y (Sutherland-Hodgman in clip
 * space, fan triangulation of what is left); viewport x_f = x_ndc*W/2 + W/2,
 * y_f = y_ndc*H/2 + H/2; vertices snapped to 1/256 pixel; 64-bit integer edge
 * functions with samples at pixel centres; back faces culled with a
 * counter-clockwise front face (kept when sum(x_i y_i+1 - x_i+1 y_i) < 0 in
 * framebuffer coordinates); a sample exactly on an edge a->b belongs to the
 * triangle when dy > 0, or dy == 0 and dx < 0; depth LESS against 1; the
 * nearest key (depth bits << 32 | ((instance*T + triangle) << 3 | piece))
 * wins; varyings perspective-correct.
 *
 * Built with -ffp-contract=off: every float operation rounds once, in the
 * order written, which is the order of the CUDA kernels (built without FMA
 * contraction). The yaw's cosine and sine are taken in double and rounded to
 * float on both sides. Parity with the reference itself is unpinned: it
 * rasterises on a Vulkan device, and no golden image exists.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define GUARD 16.f
#define SUB 256
#define MAXPOLY 9

typedef struct {
  float x, y, z, w, u0, u1, u2;
} CV;
typedef struct {
  int32_t X, Y;
  float z, iw;
} Snap;
typedef struct {
  float x, y, z, w;
} F4;

static F4 mat4v(const float* M, float x, float y, float z, float w) {
  F4 q;
  q.x = M[0] * x + M[4] * y + M[8] * z + M[12] * w;
  q.y = M[1] * x + M[5] * y + M[9] * z + M[13] * w;
  q.z = M[2] * x + M[6] * y + M[10] * z + M[14] * w;
  q.w = M[3] * x + M[7] * y + M[11] * z + M[15] * w;
  return q;
}
static void yaw_of(float a, float* ca, float* sa) {
  *ca = (float)cos((double)a);
  *sa = (float)sin((double)a);
}
static float plane_d(const CV* v, int k) {
  switch (k) {
    case 0: return v->z;
    case 1: return v->w - v->z;
    case 2: return GUARD * v->w - v->x;
    case 3: return GUARD * v->w + v->x;
    case 4: return GUARD * v->w - v->y;
    default: return GUARD * v->w + v->y;
  }
}
static CV lerp_cv(const CV* a, const CV* b, float t) {
  CV r;
  r.x = a->x + t * (b->x - a->x);
  r.y = a->y + t * (b->y - a->y);
  r.z = a->z + t * (b->z - a->z);
  r.w = a->w + t * (b->w - a->w);
  r.u0 = a->u0 + t * (b->u0 - a->u0);
  r.u1 = a->u1 + t * (b->u1 - a->u1);
  r.u2 = a->u2 + t * (b->u2 - a->u2);
  return r;
}
static int clip_poly(CV* poly) {
  int n = 3;
  CV tmp[MAXPOLY];
  for (int k = 0; k < 6 && n > 0; ++k) {
    int all_in = 1;
    for (int i = 0; i < n; ++i) all_in &= plane_d(&poly[i], k) >= 0.f;
    if (all_in) continue;
    int m = 0;
    for (int i = 0; i < n; ++i) {
      const CV* a = &poly[i];
      const CV* b = &poly[i + 1 == n ? 0 : i + 1];
      const float da = plane_d(a, k), db = plane_d(b, k);
      if (da >= 0.f) tmp[m++] = *a;
      if ((da >= 0.f) != (db >= 0.f)) tmp[m++] = lerp_cv(a, b, da / (da - db));
    }
    n = m;
    for (int i = 0; i < n; ++i) poly[i] = tmp[i];
  }
  return n;
}
static Snap snap(const CV* v, int W, int H) {
  Snap s;
  const float xn = v->x / v->w, yn = v->y / v->w;
  s.z = v->z / v->w;
  s.iw = 1.f / v->w;
  const float hw = 0.5f * (float)W, hh = 0.5f * (float)H;
  s.X = (int32_t)rintf((xn * hw + hw) * (float)SUB);
  s.Y = (int32_t)rintf((yn * hh + hh) * (float)SUB);
  return s;
}
static int64_t edge(int32_t ax, int32_t ay, int32_t bx, int32_t by, int64_t px, int64_t py) {
  return (int64_t)(bx - ax) * (py - ay) - (int64_t)(by - ay) * (px - ax);
}
static int owns_edge(int32_t ax, int32_t ay, int32_t bx, int32_t by) {
  const int32_t dx = bx - ax, dy = by - ay;
  return dy > 0 || (dy == 0 && dx < 0);
}
static int inside(int64_t e, int own) { return e > 0 || (e == 0 && own); }
static int floor_div(int32_t a, int32_t b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }
static int ceil_div(int32_t a, int32_t b) { return -floor_div(-a, b); }
static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

typedef struct {
  const float* ppos;  /* V x 4 */
  const float* pnrm;
  const float* centers; /* ninst x 4 */
  const float* sizes;
  const float* colors;
  const float* params;
  const float* M;
  int mode, W, H, T, ninst;
} Args;

static void triangle_cv(const Args* a, int o, int t, CV* poly) {
  const float* c = a->centers + 4 * o;
  const float* s = a->sizes + 4 * o;
  float ca, sa;
  yaw_of(s[3], &ca, &sa);
  for (int i = 0; i < 3; ++i) {
    const float* lp = a->ppos + 4 * (3 * t + i);
    const float px = lp[0] * s[0], py = lp[1] * s[1], pz = lp[2] * s[2];
    const float wx = c[0] + ca * px + sa * pz, wy = c[1] + py, wz = c[2] - sa * px + ca * pz;
    const F4 q = mat4v(a->M, wx, wy, wz, 1.f);
    CV v = {q.x, q.y, q.z, q.w, i == 0 ? 1.f : 0.f, i == 1 ? 1.f : 0.f, i == 2 ? 1.f : 0.f};
    poly[i] = v;
  }
}

static int make_piece(const CV* poly, int n, int sub, int W, int H, Snap* sv, int* vi, int* bx0, int* by0, int* bx1,
                      int* by1) {
  if (sub + 2 >= n) return 0;
  vi[0] = 0;
  vi[1] = sub + 1;
  vi[2] = sub + 2;
  for (int i = 0; i < 3; ++i) {
    if (!(poly[vi[i]].w > 0.f)) return 0;
    sv[i] = snap(&poly[vi[i]], W, H);
  }
  const int64_t S = edge(sv[0].X, sv[0].Y, sv[1].X, sv[1].Y, sv[2].X, sv[2].Y);
  if (S >= 0) return 0;
  Snap t = sv[1];
  sv[1] = sv[2];
  sv[2] = t;
  int u = vi[1];
  vi[1] = vi[2];
  vi[2] = u;
  const int32_t xmin = imin(sv[0].X, imin(sv[1].X, sv[2].X)), xmax = imax(sv[0].X, imax(sv[1].X, sv[2].X));
  const int32_t ymin = imin(sv[0].Y, imin(sv[1].Y, sv[2].Y)), ymax = imax(sv[0].Y, imax(sv[1].Y, sv[2].Y));
  *bx0 = imax(0, ceil_div(xmin - SUB / 2, SUB));
  *by0 = imax(0, ceil_div(ymin - SUB / 2, SUB));
  *bx1 = imin(W - 1, floor_div(xmax - SUB / 2, SUB));
  *by1 = imin(H - 1, floor_div(ymax - SUB / 2, SUB));
  return *bx0 <= *bx1 && *by0 <= *by1;
}

/* depth from the edge values: ((e0 z0 + e1 z1) + e2 z2) * (1 / S), S = e0 + e1 + e2 */
static float piece_depth(const Snap* sv, int64_t sx, int64_t sy) {
  const int64_t e0 = edge(sv[1].X, sv[1].Y, sv[2].X, sv[2].Y, sx, sy);
  const int64_t e1 = edge(sv[2].X, sv[2].Y, sv[0].X, sv[0].Y, sx, sy);
  const int64_t e2 = edge(sv[0].X, sv[0].Y, sv[1].X, sv[1].Y, sx, sy);
  if (!inside(e0, owns_edge(sv[1].X, sv[1].Y, sv[2].X, sv[2].Y)) ||
      !inside(e1, owns_edge(sv[2].X, sv[2].Y, sv[0].X, sv[0].Y)) ||
      !inside(e2, owns_edge(sv[0].X, sv[0].Y, sv[1].X, sv[1].Y)))
    return -1.f;
  const float inv_s = 1.f / (float)edge(sv[0].X, sv[0].Y, sv[1].X, sv[1].Y, sv[2].X, sv[2].Y);
  const float d = ((float)e0 * sv[0].z + (float)e1 * sv[1].z + (float)e2 * sv[2].z) * inv_s + 0.f;
  return (d >= 0.f && d < 1.f) ? d : -1.f;
}
static uint32_t fbits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static float bitsf(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t q8(float x) { return (uint32_t)rintf(fminf(fmaxf(x, 0.f), 1.f) * 255.f); }
static uint32_t pack4(float r, float g, float b, float al) {
  return q8(r) | (q8(g) << 8) | (q8(b) << 16) | (q8(al) << 24);
}

/* Draw `count` instances of `visible` (1-based indices into the ninst
 * instances). Outputs: depth (W*H floats), out0/out1/out2 (W*H packed RGBA8,
 * mode 0: albedo+roughness, metal+emission, normal; mode 2: albedo, normal;
 * mode 1 writes depth only). Returns the number of pieces rasterised. */
int64_t oracle_raster_instances(float* depth, uint32_t* out0, uint32_t* out1, uint32_t* out2, const float* ppos,
                                const float* pnrm, const uint32_t* visible, uint32_t count, const float* centers,
                                const float* sizes, const float* colors, const float* params, const float* M,
                                int mode, int W, int H, int nverts, int ninst) {
  Args a = {ppos, pnrm, centers, sizes, colors, params, M, mode, W, H, nverts / 3, ninst};
  const int64_t npix = (int64_t)W * H;
  uint64_t* vis = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)npix);
  for (int64_t i = 0; i < npix; ++i) vis[i] = ~0ull;
  int64_t pieces = 0;
  if (count > (uint32_t)ninst) count = (uint32_t)ninst;
  for (uint32_t slot = 0; slot < count; ++slot) {
    const uint32_t v1 = visible[slot];
    if (v1 == 0 || v1 > (uint32_t)ninst) continue;
    const int o = (int)v1 - 1;
    for (int t = 0; t < a.T; ++t) {
      CV poly[MAXPOLY];
      triangle_cv(&a, o, t, poly);
      const int n = clip_poly(poly);
      for (int sub = 0; sub + 2 < n; ++sub) {
        Snap sv[3];
        int vi[3], bx0, by0, bx1, by1;
        if (!make_piece(poly, n, sub, W, H, sv, vi, &bx0, &by0, &bx1, &by1)) continue;
        ++pieces;
        const uint32_t prim = ((uint32_t)(o * a.T + t) << 3) | (uint32_t)sub;
        for (int py = by0; py <= by1; ++py)
          for (int px = bx0; px <= bx1; ++px) {
            const float d = piece_depth(sv, (int64_t)px * SUB + SUB / 2, (int64_t)py * SUB + SUB / 2);
            if (d < 0.f) continue;
            const uint64_t k = ((uint64_t)fbits(d) << 32) | prim;
            uint64_t* vp = vis + (int64_t)py * W + px;
            if (k < *vp) *vp = k;
          }
      }
    }
  }
  for (int py = 0; py < H; ++py)
    for (int px = 0; px < W; ++px) {
      const int64_t pix = (int64_t)py * W + px;
      const uint64_t k = vis[pix];
      if (k == ~0ull) {
        depth[pix] = 1.f;
        if (mode != 1) {
          out0[pix] = 0xff000000u;
          out1[pix] = 0u;
          if (mode == 0) out2[pix] = 0u;
        }
        continue;
      }
      depth[pix] = bitsf((uint32_t)(k >> 32));
      if (mode == 1) continue;
      const uint32_t prim = (uint32_t)k;
      const int sub = (int)(prim & 7u), ot = (int)(prim >> 3);
      const int o = ot / a.T, t = ot % a.T;
      CV poly[MAXPOLY];
      triangle_cv(&a, o, t, poly);
      const int n = clip_poly(poly);
      Snap sv[3];
      int vi[3], bx0, by0, bx1, by1;
      if (!make_piece(poly, n, sub, W, H, sv, vi, &bx0, &by0, &bx1, &by1)) continue;
      const int64_t sx = (int64_t)px * SUB + SUB / 2, sy = (int64_t)py * SUB + SUB / 2;
      const int64_t e0 = edge(sv[1].X, sv[1].Y, sv[2].X, sv[2].Y, sx, sy);
      const int64_t e1 = edge(sv[2].X, sv[2].Y, sv[0].X, sv[0].Y, sx, sy);
      const int64_t e2 = edge(sv[0].X, sv[0].Y, sv[1].X, sv[1].Y, sx, sy);
      const float q0 = (float)e0 * sv[0].iw, q1 = (float)e1 * sv[1].iw, q2 = (float)e2 * sv[2].iw;
      const float qs = q0 + q1 + q2;
      const float b0 = q0 / qs, b1 = q1 / qs, b2 = q2 / qs;
      const CV* v0 = &poly[vi[0]];
      const CV* v1 = &poly[vi[1]];
      const CV* v2 = &poly[vi[2]];
      const float U0 = b0 * v0->u0 + b1 * v1->u0 + b2 * v2->u0;
      const float U1 = b0 * v0->u1 + b1 * v1->u1 + b2 * v2->u1;
      const float U2 = b0 * v0->u2 + b1 * v1->u2 + b2 * v2->u2;
      const float* col = colors + 4 * o;
      const float* sz = sizes + 4 * o;
      float ca, sa;
      yaw_of(sz[3], &ca, &sa);
      float nv[3][3];
      for (int i = 0; i < 3; ++i) {
        const float* ln = pnrm + 4 * (3 * t + i);
        if (mode == 0) {
          const float nx = ln[0] / sz[0], ny = ln[1] / sz[1], nz = ln[2] / sz[2];
          const float rx = ca * nx + sa * nz, ry = ny, rz = -sa * nx + ca * nz;
          const float len = sqrtf(rx * rx + ry * ry + rz * rz);
          nv[i][0] = rx / len;
          nv[i][1] = ry / len;
          nv[i][2] = rz / len;
        } else {
          nv[i][0] = ln[0];
          nv[i][1] = ln[1];
          nv[i][2] = ln[2];
        }
      }
      float nx = U0 * nv[0][0] + U1 * nv[1][0] + U2 * nv[2][0];
      float ny = U0 * nv[0][1] + U1 * nv[1][1] + U2 * nv[2][1];
      float nz = U0 * nv[0][2] + U1 * nv[1][2] + U2 * nv[2][2];
      if (mode == 0) {
        const float len = sqrtf(nx * nx + ny * ny + nz * nz);
        nx = nx / len;
        ny = ny / len;
        nz = nz / len;
        const float* par = params + 4 * o;
        out0[pix] = pack4(col[0], col[1], col[2], col[3]);
        out1[pix] = pack4(par[0], fminf(1.f, par[1]), 0.f, 1.f);
        out2[pix] = pack4(0.5f * nx + 0.5f, 0.5f * ny + 0.5f, 0.5f * nz + 0.5f, 1.f);
      } else {
        out0[pix] = pack4(col[0], col[1], col[2], col[3]);
        out1[pix] = pack4(0.5f * nx + 0.5f, 0.5f * ny + 0.5f, 0.5f * nz + 0.5f, 1.f);
      }
    }
  free(vis);
  return pieces;
}
