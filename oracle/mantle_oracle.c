/*
 * mantle_oracle.c — CPU restatement of the data-parallel work the Mantle
 * graphs of this backend carry. TEST INFRASTRUCTURE ONLY: the parity tests,
 * the smoke check and bench.py's CPU-baseline / reference arm call it as the
 * checker or as the CPU timing. The product never links or calls it.
 *
 * Built with -ffp-contract=off so every expression rounds exactly as written,
 * in the order written (the GPU kernels use explicit round-to-nearest
 * intrinsics for the same reason).
 *
 * Sources restated:
 *   touch1!..touch3!   bench/stress.jl:30-45   a = a*1.0001 + b (+ c)
 *   mix!               bench/fuzz.jl:19-22     dst = a*0.5 + b*0.25 + k
 *   stir!              bench/independent.jl:37-40
 *   touch4!            bench/stress.jl:42-45
 *   transpose_scale!, frombytes!   test/test_window.jl:30-33, 84-87
 *   advect!            bench/two_scatters.jl:46-62
 *   unpack!, blur!     bench/chain.jl:27-40
 *   point splat        bench/two_scatters.jl:11-26 (SCATTER: MVP projection,
 *                      s x s point square, additive blend), restated headless
 *   the eight-op chain, the scatter-add/histogram and the batched FFT are
 *   stated by the workload definitions (no reference kernel exists for them:
 *   parity with the reference is unpinned there, and this file is the
 *   definition; the FFT checker is itself checked against numpy.fft).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static int nthreads(int t) { return t > 0 ? t : omp_get_max_threads(); }

/* out = 2*sqrt(|fma(((0.5x+y)*z)+y, x, z)|) - x, one rounding per op. */
void oracle_chain8(const float* x, const float* y, const float* z, float* out, int64_t n, int threads) {
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float t1 = 0.5f * x[i];
    t1 = t1 + y[i];
    float t2 = t1 * z[i];
    float t3 = t2 + y[i];
    float t4 = fmaf(t3, x[i], z[i]);
    float t5 = fabsf(t4);
    float t6 = sqrtf(fabsf(t5));
    float t7 = 2.0f * t6;
    out[i] = t7 - x[i];
  }
}

/* The chain as eight separate passes over memory, as the unfused graph runs it
 * (axpy, mul, add, fma, abs, sqrt(abs), scale, sub), with intermediates in
 * `tmp` (n floats each, 7 of them). Same values as oracle_chain8. */
void oracle_chain8_passes(const float* x, const float* y, const float* z, float* out, float* tmp,
                          int64_t n, int threads) {
  float *t1 = tmp, *t2 = tmp + n, *t3 = tmp + 2 * n, *t4 = tmp + 3 * n, *t5 = tmp + 4 * n,
        *t6 = tmp + 5 * n, *t7 = tmp + 6 * n;
  int nt = nthreads(threads);
#pragma omp parallel num_threads(nt)
  {
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) t1[i] = 0.5f * x[i] + y[i];
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) t2[i] = t1[i] * z[i];
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) t3[i] = t2[i] + y[i];
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) t4[i] = fmaf(t3[i], x[i], z[i]);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) t5[i] = fabsf(t4[i]);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) t6[i] = sqrtf(fabsf(t5[i]));
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) t7[i] = 2.0f * t6[i];
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = t7[i] - x[i];
  }
}

/* Three in-place updates with read-after-write order (touch1!, touch2!,
 * touch3!): b = b*1.0001 + 1; b = b*1.0001 + c; b = b*1.0001 + c + d. */
void oracle_touch3(float* b, const float* c, const float* d, int64_t n, int threads) {
  int nt = nthreads(threads);
#pragma omp parallel num_threads(nt)
  {
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      float t = b[i] * 1.0001f;
      b[i] = t + 1.0f;
    }
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      float t = b[i] * 1.0001f;
      b[i] = t + c[i];
    }
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      float t = b[i] * 1.0001f;
      t = t + c[i];
      b[i] = t + d[i];
    }
  }
}

/* Scatter-add checker: acc[b] = sum of v[i] with idx[i] == b, in double, and
 * the exact count per bin. Indices outside [0, nbins) are skipped. Per-thread
 * private bins, reduced in thread order. acc may be NULL (histogram only),
 * hist may be NULL. */
void oracle_scatter_f64(const float* v, const int32_t* idx, int64_t n, int32_t nbins, double* acc,
                        uint32_t* hist, int threads) {
  int nt = nthreads(threads);
  double* pa = acc ? (double*)calloc((size_t)nt * nbins, sizeof(double)) : NULL;
  uint32_t* ph = hist ? (uint32_t*)calloc((size_t)nt * nbins, sizeof(uint32_t)) : NULL;
#pragma omp parallel num_threads(nt)
  {
    int t = omp_get_thread_num();
    double* a = pa ? pa + (size_t)t * nbins : NULL;
    uint32_t* h = ph ? ph + (size_t)t * nbins : NULL;
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      int32_t b = idx[i];
      if ((uint32_t)b >= (uint32_t)nbins) continue;
      if (a) a[b] += (double)v[i];
      if (h) h[b] += 1u;
    }
  }
  for (int32_t b = 0; b < nbins; ++b) {
    if (acc) {
      double s = 0;
      for (int t = 0; t < nt; ++t) s += pa[(size_t)t * nbins + b];
      acc[b] = s;
    }
    if (hist) {
      uint32_t s = 0;
      for (int t = 0; t < nt; ++t) s += ph[(size_t)t * nbins + b];
      hist[b] = s;
    }
  }
  free(pa);
  free(ph);
}

/* The same scatter in float, as a CPU implementation of the workload would run
 * it (private float bins per thread, reduced in thread order). `scratch` holds
 * threads*nbins floats and threads*nbins uint32 (caller-allocated, so the timed
 * region allocates nothing). */
void oracle_scatter_f32(const float* v, const int32_t* idx, int64_t n, int32_t nbins, float* acc,
                        uint32_t* hist, float* scratch_f, uint32_t* scratch_u, int threads) {
  int nt = nthreads(threads);
#pragma omp parallel num_threads(nt)
  {
    int t = omp_get_thread_num();
    float* a = acc ? scratch_f + (size_t)t * nbins : NULL;
    uint32_t* h = hist ? scratch_u + (size_t)t * nbins : NULL;
    if (a) memset(a, 0, sizeof(float) * (size_t)nbins);
    if (h) memset(h, 0, sizeof(uint32_t) * (size_t)nbins);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      int32_t b = idx[i];
      if ((uint32_t)b >= (uint32_t)nbins) continue;
      if (a) a[b] += v[i];
      if (h) h[b] += 1u;
    }
#pragma omp barrier
#pragma omp for schedule(static)
    for (int32_t b = 0; b < nbins; ++b) {
      if (acc) {
        float s = 0;
        for (int k = 0; k < nt; ++k) s += scratch_f[(size_t)k * nbins + b];
        acc[b] = s;
      }
      if (hist) {
        uint32_t s = 0;
        for (int k = 0; k < nt; ++k) s += scratch_u[(size_t)k * nbins + b];
        hist[b] = s;
      }
    }
  }
}

/* stir!(dst, src, k) over n elements (bench/independent.jl:37-40):
 * dst = src*k + sin(src), in float. */
void oracle_stir(float* dst, const float* src, float k, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float t = src[i] * k;
    dst[i] = t + sinf(src[i]);
  }
}

/* touch4!(a, b, c, d) (bench/stress.jl:42-45): a = a*1.0001 + b + c + d, left
 * to right. */
void oracle_touch4(float* a, const float* b, const float* c, const float* d, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float t = a[i] * 1.0001f;
    t = t + b[i];
    t = t + c[i];
    a[i] = t + d[i];
  }
}

/* transpose_scale!(dst, src, w, h, a) over the ndrange (nx, ny)
 * (test/test_window.jl:30-33), 0-based: dst[ix*h + iy] = src[iy*w + ix]*a. */
void oracle_transpose_scale(float* dst, const float* src, int32_t w, int32_t h, float a, int64_t nx,
                            int64_t ny) {
  for (int64_t iy = 0; iy < ny; ++iy)
    for (int64_t ix = 0; ix < nx; ++ix) dst[ix * h + iy] = src[iy * w + ix] * a;
}

/* frombytes!(dst, src) (test/test_window.jl:84-87): dst = Float32(src & 0xff). */
void oracle_frombytes(float* dst, const uint32_t* src, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = (float)(src[i] & 0xffu);
}

/* mix!(dst, a, b, k) over n elements (bench/fuzz.jl:19-22). */
void oracle_mix(float* dst, const float* a, const float* b, float k, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float t = a[i] * 0.5f;
    float u = b[i] * 0.25f;
    dst[i] = (t + u) + k;
  }
}

/* Batched complex DFT of length n (a power of two), interleaved re/im:
 *   forward  X[k] = sum_j x[j] e^{-2 pi i jk/n},  inverse  (1/n) sum_j x[j] e^{+2 pi i jk/n}.
 * Iterative radix-2 Cooley-Tukey (bit-reversal permutation, then log2 n
 * butterfly stages), one transform per loop iteration across threads. The
 * checker runs it in double (oracle_fft_f64); oracle_fft_f32 is the same
 * algorithm in float with double-precision twiddles, the CPU timing leg. */
#define FFT_BODY(T, in, out, batch, n, inverse, threads)                                          \
  do {                                                                                            \
    int lg = 0;                                                                                   \
    while ((1 << lg) < n) ++lg;                                                                   \
    const double sgn = inverse ? 1.0 : -1.0;                                                      \
    T* tw = (T*)malloc(sizeof(T) * (size_t)n);                                                    \
    for (int k = 0; k < n / 2; ++k) {                                                             \
      double a = 6.283185307179586476925286766559 * (double)k / (double)n;                        \
      tw[2 * k] = (T)cos(a);                                                                      \
      tw[2 * k + 1] = (T)(sgn * sin(a));                                                          \
    }                                                                                             \
    _Pragma("omp parallel for num_threads(nthreads(threads)) schedule(static)")                   \
    for (int64_t b = 0; b < batch; ++b) {                                                         \
      T* y = out + (size_t)b * 2 * n;                                                             \
      const float* x = in + (size_t)b * 2 * n;                                                    \
      for (int j = 0; j < n; ++j) {                                                               \
        int r = 0;                                                                                \
        for (int q = 0; q < lg; ++q) r |= ((j >> q) & 1) << (lg - 1 - q);                         \
        y[2 * r] = (T)x[2 * j];                                                                   \
        y[2 * r + 1] = (T)x[2 * j + 1];                                                           \
      }                                                                                           \
      for (int len = 2; len <= n; len <<= 1) {                                                    \
        const int half = len >> 1, step = n / len;                                                \
        for (int s0 = 0; s0 < n; s0 += len)                                                       \
          for (int k = 0; k < half; ++k) {                                                        \
            T wr = tw[2 * k * step], wi = tw[2 * k * step + 1];                                   \
            T* u = y + 2 * (s0 + k);                                                              \
            T* v = y + 2 * (s0 + k + half);                                                       \
            T tr = v[0] * wr - v[1] * wi, ti = v[0] * wi + v[1] * wr;                             \
            v[0] = u[0] - tr;                                                                     \
            v[1] = u[1] - ti;                                                                     \
            u[0] = u[0] + tr;                                                                     \
            u[1] = u[1] + ti;                                                                     \
          }                                                                                       \
      }                                                                                           \
      if (inverse)                                                                                \
        for (int j = 0; j < 2 * n; ++j) y[j] = y[j] / (T)n;                                       \
    }                                                                                             \
    free(tw);                                                                                     \
  } while (0)

void oracle_fft_f64(const float* in, double* out, int64_t batch, int n, int inverse, int threads) {
  FFT_BODY(double, in, out, batch, n, inverse, threads);
}

void oracle_fft_f32(const float* in, float* out, int64_t batch, int n, int inverse, int threads) {
  FFT_BODY(float, in, out, batch, n, inverse, threads);
}

/* Dense GEMM checker: C[b][i][:] = sum_k A[b][i][k] * B[b][k][:] in double, for
 * rows i in [row0, row0 + rows) of every batch b. A (M x K) and B (K x N) are
 * row-major bfloat16 bit patterns (the top 16 bits of a float32); C is
 * batch x rows x N doubles. Products of two bfloat16 values are exact in double,
 * and the double sum is far inside the tolerance the GPU result is held to. */
static inline double bf16_to_double(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}

void oracle_gemm_bf16(const uint16_t* A, const uint16_t* B, double* C, int64_t M, int64_t N, int64_t K,
                      int64_t batch, int64_t row0, int64_t rows, int threads) {
  double* Bd = (double*)malloc(sizeof(double) * (size_t)K * (size_t)N);
  for (int64_t b = 0; b < batch; ++b) {
    const uint16_t* Bb = B + (size_t)b * K * N;
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
    for (int64_t x = 0; x < K * N; ++x) Bd[x] = bf16_to_double(Bb[x]);
#pragma omp parallel for num_threads(nthreads(threads)) schedule(dynamic, 1)
    for (int64_t r = 0; r < rows; ++r) {
      const uint16_t* a = A + ((size_t)b * M + (size_t)(row0 + r)) * K;
      double* c = C + ((size_t)b * rows + (size_t)r) * N;
      for (int64_t n = 0; n < N; ++n) c[n] = 0.0;
      for (int64_t k = 0; k < K; ++k) {
        const double av = bf16_to_double(a[k]);
        if (av == 0.0) continue;
        const double* bk = Bd + (size_t)k * N;
        for (int64_t n = 0; n < N; ++n) c[n] += av * bk[n];
      }
    }
  }
  free(Bd);
}

static inline uint16_t double_to_bf16(double d) {
  float f = (float)d;
  uint32_t u;
  memcpy(&u, &f, 4);
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
  return (uint16_t)u;
}

/* NHWC convolution, bf16 bit patterns in, double accumulation:
 *   out[n][oh][ow][co] = sum_{r,c,ci} in[n][oh*s-p+r][ow*s-p+c][ci] * w[r][c][ci][co]
 * (zero outside the image), then ReLU when relu != 0. `out_d` (may be NULL)
 * receives the double result, `out_h` (may be NULL) the result rounded once
 * to bfloat16 (nearest even) — the form the next layer reads. */
void oracle_conv_bf16(const uint16_t* in, const uint16_t* w, double* out_d, uint16_t* out_h, int n, int h, int wd,
                      int cin, int cout, int k, int stride, int pad, int relu, int threads) {
  const int ho = (h + 2 * pad - k) / stride + 1, wo = (wd + 2 * pad - k) / stride + 1;
  const int64_t wsz = (int64_t)k * k * cin * cout;
  double* wf = (double*)malloc(sizeof(double) * (size_t)wsz);
  for (int64_t x = 0; x < wsz; ++x) wf[x] = bf16_to_double(w[x]);
#pragma omp parallel num_threads(nthreads(threads))
  {
    double* acc = (double*)malloc(sizeof(double) * (size_t)cout);
#pragma omp for schedule(static) collapse(2)
    for (int b = 0; b < n; ++b)
      for (int oh = 0; oh < ho; ++oh)
        for (int ow = 0; ow < wo; ++ow) {
          for (int co = 0; co < cout; ++co) acc[co] = 0.0;
          for (int r = 0; r < k; ++r) {
            const int ih = oh * stride - pad + r;
            if (ih < 0 || ih >= h) continue;
            for (int c = 0; c < k; ++c) {
              const int iw = ow * stride - pad + c;
              if (iw < 0 || iw >= wd) continue;
              const uint16_t* px = in + (((int64_t)b * h + ih) * wd + iw) * cin;
              const double* wr = wf + ((int64_t)(r * k + c) * cin) * cout;
              for (int ci = 0; ci < cin; ++ci) {
                const double a = bf16_to_double(px[ci]);
                if (a == 0.0) continue;
                const double* wc = wr + (int64_t)ci * cout;
                for (int co = 0; co < cout; ++co) acc[co] += a * wc[co];
              }
            }
          }
          const int64_t o = (((int64_t)b * ho + oh) * wo + ow) * cout;
          for (int co = 0; co < cout; ++co) {
            double v = acc[co];
            if (relu && v < 0) v = 0;
            if (out_d) out_d[o + co] = v;
            if (out_h) out_h[o + co] = double_to_bf16(v);
          }
        }
    free(acc);
  }
  free(wf);
}

/* Global average pool over hw pixels of NHWC bf16 activations, then logits[j]
 * = sum_ch mean[ch] * w[ch][j] (w is c x classes, float), all in double. */
void oracle_gap_fc(const uint16_t* act, const float* w, double* logits, int n, int hw, int c, int classes,
                   int threads) {
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
  for (int b = 0; b < n; ++b) {
    double* mean = (double*)malloc(sizeof(double) * (size_t)c);
    for (int ch = 0; ch < c; ++ch) {
      double s = 0;
      for (int p = 0; p < hw; ++p) s += bf16_to_double(act[((int64_t)b * hw + p) * c + ch]);
      mean[ch] = s / hw;
    }
    for (int j = 0; j < classes; ++j) {
      double s = 0;
      for (int ch = 0; ch < c; ++ch) s += mean[ch] * (double)w[(int64_t)ch * classes + j];
      logits[(int64_t)b * classes + j] = s;
    }
    free(mean);
  }
}

/* advect!: p = pos + v*dt; if |p| > radius: n = p/r, p = n*radius,
 * v = v - (2*(v.n))*n. pos, vel: 3 floats per point. */
void oracle_advect(float* pos, float* vel, float dt, float radius, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float* P = pos + 3 * i;
    float* V = vel + 3 * i;
    const float v0 = V[0], v1 = V[1], v2 = V[2];
    float p0 = P[0] + v0 * dt, p1 = P[1] + v1 * dt, p2 = P[2] + v2 * dt;
    const float r = sqrtf((p0 * p0 + p1 * p1) + p2 * p2);
    if (r > radius) {
      const float n0 = p0 / r, n1 = p1 / r, n2 = p2 / r;
      p0 = n0 * radius;
      p1 = n1 * radius;
      p2 = n2 * radius;
      const float d = (v0 * n0 + v1 * n1) + v2 * n2;
      const float d2 = 2.0f * d;
      V[0] = v0 - d2 * n0;
      V[1] = v1 - d2 * n1;
      V[2] = v2 - d2 * n2;
    }
    P[0] = p0;
    P[1] = p1;
    P[2] = p2;
  }
}

/* The pixels a point covers: project by the column-major MVP (the sum over
 * columns left to right), clip to -w <= x, y <= w, 0 <= z <= w, map NDC to the
 * W x H framebuffer, and take the pixels whose centres px + 0.5 lie in
 * [f - s/2, f + s/2). Returns 0 when the point is clipped. */
static int point_rect(const float* m, const float* p, float s, int w, int h, int* x0, int* x1, int* y0, int* y1) {
  float cl[4];
  for (int r = 0; r < 4; ++r) cl[r] = ((m[r] * p[0] + m[4 + r] * p[1]) + m[8 + r] * p[2]) + m[12 + r];
  const float cw = cl[3];
  if (!(cw > 0.f && cl[0] >= -cw && cl[0] <= cw && cl[1] >= -cw && cl[1] <= cw && cl[2] >= 0.f && cl[2] <= cw))
    return 0;
  const float hw = 0.5f * (float)w, hh = 0.5f * (float)h;
  const float fx = (cl[0] / cw) * hw + hw, fy = (cl[1] / cw) * hh + hh;
  float half = 0.5f * s;
  if (half > 1e6f) half = 1e6f;
  if (!(half > 0.f)) return 0;
  int a = (int)ceilf((fx - half) - 0.5f), b = (int)ceilf((fx + half) - 0.5f) - 1;
  int c = (int)ceilf((fy - half) - 0.5f), d = (int)ceilf((fy + half) - 0.5f) - 1;
  *x0 = a < 0 ? 0 : a;
  *x1 = b > w - 1 ? w - 1 : b;
  *y0 = c < 0 ? 0 : c;
  *y1 = d > h - 1 ? h - 1 : d;
  return 1;
}

/* Additive point splat into a double RGBA framebuffer [h][w] (caller clears
 * it); colours/sizes per point (stride 1) or shared (stride 0). */
void oracle_splat(double* fb, const float* pos, const float* col, const float* size, const float* mvp, int w, int h,
                  int col_stride, int size_stride, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    int x0, x1, y0, y1;
    if (!point_rect(mvp, pos + 3 * i, size[size_stride * i], w, h, &x0, &x1, &y0, &y1)) continue;
    const float* c = col + 4 * col_stride * i;
    for (int py = y0; py <= y1; ++py)
      for (int px = x0; px <= x1; ++px)
        for (int k = 0; k < 4; ++k) fb[4 * ((int64_t)py * w + px) + k] += (double)c[k];
  }
}

/* Framebuffer (float RGBA) to BGRA8: round(clamp(x, 0, 1) * 255), ties to even. */
void oracle_pack_bgra8(uint8_t* dst, const float* src, int64_t npix) {
  for (int64_t i = 0; i < npix; ++i) {
    const int order[4] = {2, 1, 0, 3};
    for (int k = 0; k < 4; ++k) {
      float x = src[4 * i + order[k]];
      x = x < 0.f ? 0.f : (x > 1.f ? 1.f : x);
      dst[4 * i + k] = (uint8_t)nearbyintf(x * 255.0f);
    }
  }
}

/* unpack!: dst[i*h + j] = (R, G, B, 255)/255 from the BGRA8 pixel (i, j) at
 * byte (j*w + i)*4. */
void oracle_unpack_bgra8(float* dst, const uint8_t* src, int w, int h) {
  for (int i = 0; i < w; ++i)
    for (int j = 0; j < h; ++j) {
      const uint8_t* b = src + ((int64_t)j * w + i) * 4;
      float* d = dst + 4 * ((int64_t)i * h + j);
      d[0] = (float)b[2] / 255.0f;
      d[1] = (float)b[1] / 255.0f;
      d[2] = (float)b[0] / 255.0f;
      d[3] = 255.0f / 255.0f;
    }
}

/* blur!: 3x3 box with clamp-to-edge, nine adds (di fastest), then /9. */
void oracle_blur3x3(float* dst, const float* src, int w, int h) {
  for (int i = 0; i < w; ++i)
    for (int j = 0; j < h; ++j) {
      float acc[4] = {0, 0, 0, 0};
      for (int dj = -1; dj <= 1; ++dj) {
        int jj = j + dj;
        jj = jj < 0 ? 0 : (jj > h - 1 ? h - 1 : jj);
        for (int di = -1; di <= 1; ++di) {
          int ii = i + di;
          ii = ii < 0 ? 0 : (ii > w - 1 ? w - 1 : ii);
          const float* v = src + 4 * ((int64_t)ii * h + jj);
          for (int k = 0; k < 4; ++k) acc[k] = acc[k] + v[k];
        }
      }
      float* d = dst + 4 * ((int64_t)i * h + j);
      for (int k = 0; k < 4; ++k) d[k] = acc[k] / 9.0f;
    }
}

int oracle_max_threads(void) { return omp_get_max_threads(); }
