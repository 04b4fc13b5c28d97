/*
 * showcase_oracle.c — CPU restatement of the compute passes of the
 * reference's deferred-shading showcase (bench/showcase.jl). TEST
 * INFRASTRUCTURE ONLY: the parity tests call it as the checker; the product
 * never links or calls it.
 *
 * Restated (bench/showcase.jl): move_lights! :214-229, cull! :187-201 with
 * frustum_plane :156-163, write_draw! :203-205, tile_lights! :331-376, shade!
 * :380-454 with ggx :307-326, sky :298-305, sunshadow :270-287, unproject
 * :289-292, unpack8 :259, ssao! :471-523 with hash01 :456-461, ao_blur!
 * :527-542, bright! :550-565, blur! :568-583, composite_fragment :593-617.
 *
 * Built with -ffp-contract=off: every +, -, *, / and sqrtf rounds once, in the
 * order written, which is also the order of the CUDA kernels (compiled without
 * FMA contraction). expf, powf, sinf and cosf are the C library's; the GPU's
 * may differ in the last place. Parity with the reference itself is unpinned:
 * the reference runs these passes in Julia on a Vulkan device, absent here.
 *
 * Scene constants P use the offsets of the CUDA file (SC_* below).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>

enum {
  SC_VP = 0, SC_INVVP = 16, SC_SUNVP = 32, SC_EYE = 48, SC_SUN = 52, SC_SUNCOL = 56, SC_FOG = 60, SC_EMIT = 61,
  SC_STEXEL = 62, SC_SBIAS = 63, SC_AOAMB = 64, SC_AODIRECT = 65, SC_AORADIUS = 66, SC_AOBIAS = 67,
  SC_THRESHOLD = 68, SC_EXPOSURE = 69, SC_BLOOM = 70, SC_AOSHARP = 71, SC_TIME = 72
};

typedef struct {
  float x, y, z;
} V3;
static V3 V(float x, float y, float z) { V3 r = {x, y, z}; return r; }
static V3 add(V3 a, V3 b) { return V(a.x + b.x, a.y + b.y, a.z + b.z); }
static V3 sub(V3 a, V3 b) { return V(a.x - b.x, a.y - b.y, a.z - b.z); }
static V3 scl(V3 a, float s) { return V(a.x * s, a.y * s, a.z * s); }
static V3 hmul(V3 a, V3 b) { return V(a.x * b.x, a.y * b.y, a.z * b.z); }
static V3 crs(V3 a, V3 b) { return V(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x); }
static V3 nrmz(V3 a) {
  const float n = sqrtf(a.x * a.x + a.y * a.y + a.z * a.z);
  return V(a.x / n, a.y / n, a.z / n);
}
static float clampf_(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }
static int clampi_(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }
static int mini(int a, int b) { return a < b ? a : b; }

/* column-major M times (x, y, z, w) */
static void m4(const float* M, float x, float y, float z, float w, float* q) {
  q[0] = M[0] * x + M[4] * y + M[8] * z + M[12] * w;
  q[1] = M[1] * x + M[5] * y + M[9] * z + M[13] * w;
  q[2] = M[2] * x + M[6] * y + M[10] * z + M[14] * w;
  q[3] = M[3] * x + M[7] * y + M[11] * z + M[15] * w;
}
static float unpack8(uint32_t px, int shift) { return (float)((px >> shift) & 0xffu) * (1.f / 255.f); }
static V3 unproject(const float* inv, float fx, float fy, float d, int w, int h) {
  float q[4];
  m4(inv, 2.f * fx / (float)w - 1.f, 2.f * fy / (float)h - 1.f, d, 1.f, q);
  return V(q[0] / q[3], q[1] / q[3], q[2] / q[3]);
}
static V3 normal_of(uint32_t nn) {
  return nrmz(V(2.f * unpack8(nn, 0) - 1.f, 2.f * unpack8(nn, 8) - 1.f, 2.f * unpack8(nn, 16) - 1.f));
}
static V3 sky(V3 dir, V3 sundir, V3 suncol) {
  const float t = clampf_(0.5f * (dir.y + 1.f), 0.f, 1.f);
  const V3 horizon = V(0.115f, 0.085f, 0.105f), zenith = V(0.012f, 0.020f, 0.055f);
  const V3 base = add(horizon, scl(sub(zenith, horizon), powf(t, 0.55f)));
  const float c = fmaxf(0.f, dir.x * sundir.x + dir.y * sundir.y + dir.z * sundir.z);
  return add(base, scl(suncol, powf(c, 220.f) * 7.f + powf(c, 12.f) * 0.10f));
}
static V3 ggx(V3 n, V3 v, V3 l, V3 albedo, float rough, float metal) {
  const float ndl = n.x * l.x + n.y * l.y + n.z * l.z;
  const float ndv = n.x * v.x + n.y * v.y + n.z * v.z;
  if (ndl <= 0.f || ndv <= 0.f) return V(0.f, 0.f, 0.f);
  const V3 hv = nrmz(add(v, l));
  const float ndh = fmaxf(0.f, n.x * hv.x + n.y * hv.y + n.z * hv.z);
  const float vdh = fmaxf(0.f, v.x * hv.x + v.y * hv.y + v.z * hv.z);
  const float a = fmaxf(1e-3f, rough * rough);
  const float a2 = a * a;
  const float dd = ndh * ndh * (a2 - 1.f) + 1.f;
  const float D = a2 / (3.14159274f * dd * dd);
  const float k = a * 0.5f;
  const float G = (ndl / (ndl * (1.f - k) + k)) * (ndv / (ndv * (1.f - k) + k));
  const V3 f0 = add(V(0.04f, 0.04f, 0.04f), scl(sub(albedo, V(0.04f, 0.04f, 0.04f)), metal));
  const float om = 1.f - vdh;
  const float fr = om * om * om * om * om;  // (1 - v.h)^5 as four products, left to right
  const V3 F = add(f0, scl(sub(V(1.f, 1.f, 1.f), f0), fr));
  const V3 spec = scl(F, D * G / fmaxf(1e-4f, 4.f * ndl * ndv));
  const V3 kd = scl(sub(V(1.f, 1.f, 1.f), F), 1.f - metal);
  return scl(add(scl(hmul(kd, albedo), 1.f / 3.14159274f), spec), ndl);
}
static float sunshadow(const float* smap, const float* sunvp, V3 world, V3 n, float ndl, int res, float texel,
                       float bias) {
  const float slope = clampf_(sqrtf(fmaxf(0.f, 1.f - ndl * ndl)) / fmaxf(ndl, 0.08f), 0.f, 10.f);
  const V3 w = add(world, scl(n, texel * (1.6f + 2.2f * slope)));
  float q[4];
  m4(sunvp, w.x, w.y, w.z, 1.f, q);
  if (fabsf(q[0]) > 1.f || fabsf(q[1]) > 1.f || q[2] < 0.f || q[2] > 1.f) return 1.f;
  const float fx = (0.5f * q[0] + 0.5f) * (float)res;
  const float fy = (0.5f * q[1] + 0.5f) * (float)res;
  const float ref = q[2] - bias * (1.f + slope);
  float lit = 0.f;
  for (int dy = -1; dy <= 1; ++dy)
    for (int dx = -1; dx <= 1; ++dx) {
      const int sx = clampi_((int)fx + dx, 0, res - 1), sy = clampi_((int)fy + dy, 0, res - 1);
      lit += smap[(int64_t)sy * res + sx] > ref ? 1.f : 0.f;
    }
  return lit * (1.f / 9.f);
}

void oracle_sc_move_lights(float* pos, float* centers, float* params, const float* home, const float* lcol,
                           const float* P, int first, int n) {
  const float t = P[SC_TIME];
  for (int i = 0; i < n; ++i) {
    const float* h = home + 4 * i;
    const float ph = 0.7f * (float)(i + 1);
    float* p = pos + 4 * i;
    p[0] = h[0] + 7.f * sinf(0.42f * t + ph);
    p[1] = h[1] + 1.6f * sinf(0.9f * t + ph);
    p[2] = h[2] + 7.f * cosf(0.33f * t + ph);
    p[3] = h[3];
    float* c = centers + 4 * (first + i);
    c[0] = p[0], c[1] = p[1], c[2] = p[2];
    float* q = params + 4 * (first + i);
    q[0] = 0.f, q[1] = lcol[4 * i + 3], q[2] = 0.f, q[3] = 0.f;
  }
}

/* keep[i] = 1 when instance i survives the frustum of M (the list order on the
   GPU depends on atomics; the test compares sets) */
void oracle_sc_cull(uint8_t* keep, const float* centers, const float* M, int n) {
  float pl[6][4];
  for (int k = 0; k < 6; ++k) {
    const float w[4] = {M[3], M[7], M[11], M[15]};
    const int r = k < 4 ? k / 2 : 2;
    const float ri[4] = {M[r], M[4 + r], M[8 + r], M[12 + r]};
    float p[4];
    for (int j = 0; j < 4; ++j) p[j] = k == 4 ? ri[j] : (k % 2 == 0 && k < 4 ? w[j] + ri[j] : w[j] - ri[j]);
    const float len = sqrtf(p[0] * p[0] + p[1] * p[1] + p[2] * p[2]);
    for (int j = 0; j < 4; ++j) pl[k][j] = p[j] / len;
  }
  for (int i = 0; i < n; ++i) {
    const float* c = centers + 4 * i;
    int ok = 1;
    for (int k = 0; k < 6; ++k) ok &= pl[k][0] * c[0] + pl[k][1] * c[1] + pl[k][2] * c[2] + pl[k][3] >= -c[3];
    keep[i] = (uint8_t)ok;
  }
}

void oracle_sc_tile_lights(uint32_t* tilelights, uint32_t* tilecount, const float* dep, const float* lpos,
                           const float* P, int w, int h, int tile, int nlight, int pertile) {
  const int ntx = (w + tile - 1) / tile, nty = (h + tile - 1) / tile;
#pragma omp parallel for schedule(static)
  for (int ti = 0; ti < ntx * nty; ++ti) {
    const int tx = ti % ntx, ty = ti / ntx;
    const int x0 = tx * tile, y0 = ty * tile, x1 = mini(x0 + tile, w), y1 = mini(y0 + tile, h);
    float dmin = 1.f, dmax = 0.f;
    for (int py = y0; py < y1; ++py)
      for (int px = x0; px < x1; ++px) {
        const float d = dep[(int64_t)py * w + px];
        if (d < 1.f) {
          dmin = fminf(dmin, d);
          dmax = fmaxf(dmax, d);
        }
      }
    uint32_t n = 0;
    if (dmax > 0.f) {
      V3 lo = V(1e30f, 1e30f, 1e30f), hi = V(-1e30f, -1e30f, -1e30f);
      for (int c = 0; c < 8; ++c) {
        const V3 p = unproject(P + SC_INVVP, (float)((c & 1) == 0 ? x0 : x1), (float)((c & 2) == 0 ? y0 : y1),
                               (c & 4) == 0 ? dmin : dmax, w, h);
        lo = V(fminf(lo.x, p.x), fminf(lo.y, p.y), fminf(lo.z, p.z));
        hi = V(fmaxf(hi.x, p.x), fmaxf(hi.y, p.y), fmaxf(hi.z, p.z));
      }
      for (int l = 0; l < nlight; ++l) {
        const float* lp = lpos + 4 * l;
        const float dx = fmaxf(0.f, fmaxf(lo.x - lp[0], lp[0] - hi.x));
        const float dy = fmaxf(0.f, fmaxf(lo.y - lp[1], lp[1] - hi.y));
        const float dz = fmaxf(0.f, fmaxf(lo.z - lp[2], lp[2] - hi.z));
        if (dx * dx + dy * dy + dz * dz <= lp[3] * lp[3] && n < (uint32_t)pertile)
          tilelights[(int64_t)ti * pertile + n++] = (uint32_t)(l + 1);
      }
    }
    tilecount[ti] = n;
  }
}

void oracle_sc_shade(float* hdr, const uint32_t* alb, const uint32_t* mat, const uint32_t* nrm, const float* dep,
                     const float* lpos, const float* lcol, const uint32_t* tilelights, const uint32_t* tilecount,
                     const float* smap, const float* aomap, const float* P, int w, int h, int tile, int pertile,
                     int smapres) {
  const int aow = (w + 1) / 2, aoh = (h + 1) / 2, ntx = (w + tile - 1) / tile;
  const V3 sundir = V(P[SC_SUN], P[SC_SUN + 1], P[SC_SUN + 2]);
  const V3 sunrgb = scl(V(P[SC_SUNCOL], P[SC_SUNCOL + 1], P[SC_SUNCOL + 2]), P[SC_SUNCOL + 3]);
  const V3 eyep = V(P[SC_EYE], P[SC_EYE + 1], P[SC_EYE + 2]);
#pragma omp parallel for schedule(static)
  for (int py = 0; py < h; ++py)
    for (int px = 0; px < w; ++px) {
      const int64_t i = (int64_t)py * w + px;
      const float d = dep[i];
      const V3 world = unproject(P + SC_INVVP, (float)px + 0.5f, (float)py + 0.5f, fminf(d, 0.999999f), w, h);
      const V3 ray = nrmz(sub(world, eyep));
      const V3 skyc = sky(ray, sundir, sunrgb);
      V3 out = skyc;
      if (d < 1.f) {
        const uint32_t a = alb[i], m = mat[i];
        const V3 albedo = V(unpack8(a, 0), unpack8(a, 8), unpack8(a, 16));
        const float rough = fmaxf(0.04f, unpack8(a, 24));
        const float metal = unpack8(m, 0), emit = unpack8(m, 8);
        const V3 n = normal_of(nrm[i]);
        const V3 view = V(-ray.x, -ray.y, -ray.z);
        const float fax = ((float)px + 0.5f) * 0.5f - 0.5f, fay = ((float)py + 0.5f) * 0.5f - 0.5f;
        const int ax0 = clampi_((int)fax, 0, aow - 1), ay0 = clampi_((int)fay, 0, aoh - 1);
        const int ax1 = mini(ax0 + 1, aow - 1), ay1 = mini(ay0 + 1, aoh - 1);
        const float atx = clampf_(fax - (float)ax0, 0.f, 1.f), aty = clampf_(fay - (float)ay0, 0.f, 1.f);
        const float a00 = aomap[(int64_t)ay0 * aow + ax0], a10 = aomap[(int64_t)ay0 * aow + ax1];
        const float a01 = aomap[(int64_t)ay1 * aow + ax0], a11 = aomap[(int64_t)ay1 * aow + ax1];
        const float top = a00 + (a10 - a00) * atx;
        const float occ = top + ((a01 + (a11 - a01) * atx) - top) * aty;
        const float ao = clampf_(1.f - occ * P[SC_AOAMB], 0.f, 1.f);
        const float aol = 1.f - P[SC_AODIRECT] * (1.f - ao);
        const float up = 0.5f * n.y + 0.5f;
        const V3 amb = scl(scl(add(scl(V(0.055f, 0.070f, 0.115f), up), scl(V(0.020f, 0.017f, 0.016f), 1.f - up)),
                               1.f - 0.7f * metal),
                           ao);
        const float ndl = fmaxf(0.f, n.x * sundir.x + n.y * sundir.y + n.z * sundir.z);
        const float shd = ndl > 0.f ? sunshadow(smap, P + SC_SUNVP, world, n, ndl, smapres, P[SC_STEXEL], P[SC_SBIAS])
                                    : 1.f;
        V3 acc = add(hmul(albedo, amb), scl(hmul(ggx(n, view, sundir, albedo, rough, metal), sunrgb), shd));
        const int64_t ti = (int64_t)(py / tile) * ntx + px / tile;
        const int cnt = (int)tilecount[ti];
        for (int k = 0; k < cnt; ++k) {
          const int l = (int)tilelights[ti * pertile + k] - 1;
          const float* lp = lpos + 4 * l;
          const V3 dv = V(lp[0] - world.x, lp[1] - world.y, lp[2] - world.z);
          const float dist = sqrtf(dv.x * dv.x + dv.y * dv.y + dv.z * dv.z) + 1e-4f;
          const float fall = fmaxf(0.f, 1.f - dist / lp[3]);
          if (fall > 0.f) {
            const float* c = lcol + 4 * l;
            const V3 ldir = V(dv.x / dist, dv.y / dist, dv.z / dist);
            acc = add(acc, hmul(ggx(n, view, ldir, albedo, rough, metal), scl(V(c[0], c[1], c[2]), c[3] * fall * fall * aol)));
          }
        }
        acc = add(acc, scl(albedo, emit * P[SC_EMIT]));
        const V3 de = sub(world, eyep);
        const float dist = sqrtf(de.x * de.x + de.y * de.y + de.z * de.z);
        const float f = 1.f - expf(-dist * P[SC_FOG]);
        out = add(acc, scl(sub(skyc, acc), f));
      }
      float* o = hdr + 4 * i;
      o[0] = out.x, o[1] = out.y, o[2] = out.z, o[3] = 1.f;
    }
}

static float hash01(int x, int y) {
  uint32_t hh = (uint32_t)x * 0x9e3779b9u + (uint32_t)y * 0x85ebca6bu;
  hh ^= hh >> 15;
  hh *= 0x2545f491u;
  return (float)(hh & 0x00ffffffu) * (1.f / 16777216.f);
}

/* ao: (occlusion / nsample, depth) per half-resolution pixel, interleaved */
void oracle_sc_ssao(float* ao, const float* dep, const uint32_t* nrm, const float* P, int w, int h, int nsample) {
  const int aow = (w + 1) / 2, aoh = (h + 1) / 2;
  const float radius = P[SC_AORADIUS], bias = P[SC_AOBIAS];
  const V3 ep = V(P[SC_EYE], P[SC_EYE + 1], P[SC_EYE + 2]);
#pragma omp parallel for schedule(static)
  for (int iy = 0; iy < aoh; ++iy)
    for (int ix = 0; ix < aow; ++ix) {
      const int px = 2 * ix, py = 2 * iy;
      const int64_t i = (int64_t)py * w + px;
      const float d = dep[i];
      float occ = 0.f;
      if (d < 1.f) {
        const V3 n = normal_of(nrm[i]);
        const V3 p = unproject(P + SC_INVVP, (float)px + 0.5f, (float)py + 0.5f, d, w, h);
        const V3 upv = fabsf(n.z) < 0.9f ? V(0.f, 0.f, 1.f) : V(1.f, 0.f, 0.f);
        const V3 t = nrmz(crs(upv, n));
        const V3 b = crs(n, t);
        const float rot = hash01(px, py) * 6.2831854f;
        for (int k = 0; k < nsample; ++k) {
          const float a = ((float)k + 0.5f) / (float)nsample;
          const float rr = sqrtf(a);
          const float phi = (float)k * 2.3999632f + rot;
          const V3 dir = add(add(scl(t, rr * cosf(phi)), scl(b, rr * sinf(phi))), scl(n, sqrtf(fmaxf(0.f, 1.f - a))));
          const V3 sp = add(p, scl(dir, radius * (0.3f + 0.7f * a)));
          float q[4];
          m4(P + SC_VP, sp.x, sp.y, sp.z, 1.f, q);
          if (q[3] > 0.f) {
            const float sx = (0.5f * q[0] / q[3] + 0.5f) * (float)w;
            const float sy = (0.5f * q[1] / q[3] + 0.5f) * (float)h;
            if (sx >= 0.f && sx < (float)w && sy >= 0.f && sy < (float)h) {
              const float ds = dep[(int64_t)(int)sy * w + (int)sx];
              if (ds < 1.f) {
                const V3 ps = unproject(P + SC_INVVP, sx, sy, ds, w, h);
                const V3 e1 = sub(ps, ep), e2 = sub(sp, ep), g = sub(ps, p);
                const float dp = sqrtf(e1.x * e1.x + e1.y * e1.y + e1.z * e1.z);
                const float dsamp = sqrtf(e2.x * e2.x + e2.y * e2.y + e2.z * e2.z);
                if (dp < dsamp - bias) {
                  const float gap = sqrtf(g.x * g.x + g.y * g.y + g.z * g.z);
                  occ += clampf_(radius / fmaxf(1e-4f, gap), 0.f, 1.f);
                }
              }
            }
          }
        }
      }
      ao[2 * ((int64_t)iy * aow + ix)] = occ / (float)nsample;
      ao[2 * ((int64_t)iy * aow + ix) + 1] = d;
    }
}

void oracle_sc_ao_blur(float* dst, const float* src, const float* P, int aow, int aoh) {
  const float sharp = P[SC_AOSHARP];
  for (int iy = 0; iy < aoh; ++iy)
    for (int ix = 0; ix < aow; ++ix) {
      const float d0 = src[2 * ((int64_t)iy * aow + ix) + 1];
      float acc = 0.f, wsum = 0.f;
      for (int dy = -2; dy <= 2; ++dy)
        for (int dx = -2; dx <= 2; ++dx) {
          const int sx = clampi_(ix + dx, 0, aow - 1), sy = clampi_(iy + dy, 0, aoh - 1);
          const float* v = src + 2 * ((int64_t)sy * aow + sx);
          const float g = expf(-fabsf(v[1] - d0) * sharp);
          acc += v[0] * g;
          wsum += g;
        }
      dst[(int64_t)iy * aow + ix] = acc / wsum;
    }
}

void oracle_sc_bright(float* dst, const float* hdr, const float* P, int w, int h, int shift) {
  const int bw = (w + shift - 1) / shift, bh = (h + shift - 1) / shift, half = shift / 2;
  const float thr = P[SC_THRESHOLD];
  for (int iy = 0; iy < bh; ++iy)
    for (int ix = 0; ix < bw; ++ix) {
      V3 acc = V(0.f, 0.f, 0.f);
      for (int ty = 0; ty < 2; ++ty)
        for (int tx = 0; tx < 2; ++tx) {
          const int sx = mini(ix * shift + (tx ? half : 0), w - 1), sy = mini(iy * shift + (ty ? half : 0), h - 1);
          const float* c = hdr + 4 * ((int64_t)sy * w + sx);
          const float m = fmaxf(c[0], fmaxf(c[1], c[2]));
          acc = add(acc, scl(V(c[0], c[1], c[2]), m > thr ? (m - thr) / m : 0.f));
        }
      float* o = dst + 4 * ((int64_t)iy * bw + ix);
      o[0] = acc.x * 0.25f, o[1] = acc.y * 0.25f, o[2] = acc.z * 0.25f, o[3] = 1.f;
    }
}

void oracle_sc_blur(float* dst, const float* src, int bw, int bh, int dx, int dy) {
  for (int iy = 0; iy < bh; ++iy)
    for (int ix = 0; ix < bw; ++ix) {
      V3 acc = V(0.f, 0.f, 0.f);
      float wsum = 0.f;
      for (int k = -6; k <= 6; ++k) {
        const int sx = clampi_(ix + k * dx, 0, bw - 1), sy = clampi_(iy + k * dy, 0, bh - 1);
        const float* c = src + 4 * ((int64_t)sy * bw + sx);
        const float g = expf(-(float)(k * k) * (1.f / 16.f));
        acc = add(acc, scl(V(c[0], c[1], c[2]), g));
        wsum += g;
      }
      float* o = dst + 4 * ((int64_t)iy * bw + ix);
      o[0] = acc.x / wsum, o[1] = acc.y / wsum, o[2] = acc.z / wsum, o[3] = 1.f;
    }
}

void oracle_sc_composite(float* out, const float* hdr, const float* bloom, const float* P, int w, int h, int bw,
                         int bh, int shift) {
  const float amount = P[SC_BLOOM], exposure = P[SC_EXPOSURE];
  for (int py = 0; py < h; ++py)
    for (int px = 0; px < w; ++px) {
      const float* c = hdr + 4 * ((int64_t)py * w + px);
      const float fx = ((float)px + 0.5f) / (float)shift - 0.5f, fy = ((float)py + 0.5f) / (float)shift - 0.5f;
      const int x0 = clampi_((int)fx, 0, bw - 1), y0 = clampi_((int)fy, 0, bh - 1);
      const int x1 = mini(x0 + 1, bw - 1), y1 = mini(y0 + 1, bh - 1);
      const float tx = clampf_(fx - (float)x0, 0.f, 1.f), ty = clampf_(fy - (float)y0, 0.f, 1.f);
      const float* b00 = bloom + 4 * ((int64_t)y0 * bw + x0);
      const float* b10 = bloom + 4 * ((int64_t)y0 * bw + x1);
      const float* b01 = bloom + 4 * ((int64_t)y1 * bw + x0);
      const float* b11 = bloom + 4 * ((int64_t)y1 * bw + x1);
      const V3 bt = add(V(b00[0], b00[1], b00[2]), scl(sub(V(b10[0], b10[1], b10[2]), V(b00[0], b00[1], b00[2])), tx));
      const V3 bb = add(V(b01[0], b01[1], b01[2]), scl(sub(V(b11[0], b11[1], b11[2]), V(b01[0], b01[1], b01[2])), tx));
      const V3 b = add(bt, scl(sub(bb, bt), ty));
      const V3 v = scl(V(c[0] + b.x * amount, c[1] + b.y * amount, c[2] + b.z * amount), exposure);
      float* o = out + 4 * ((int64_t)py * w + px);
      o[0] = v.x / (1.f + v.x), o[1] = v.y / (1.f + v.y), o[2] = v.z / (1.f + v.z), o[3] = 1.f;
    }
}
