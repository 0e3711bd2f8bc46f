/*
 * rnb_cpu_fast.c -- vectorised CPU baseline of the sparse-MoE block.
 *
 * BENCHMARK AND TEST INFRASTRUCTURE.  bench.py times it as the CPU baseline
 * and as the reference arm, because MLX's CPU backend (the reference's own
 * CPU path: src/runnel/mlx.py:57-82 over mlx.core gather_qmm) is not
 * installable here; tests/ check it against the exact-order oracle
 * (rnb_oracle.c).  The product path (runnel_b200) never links or calls it.
 *
 * The block is the oracle's, with the same routing, computed the way a CPU
 * runs it fast:
 *   - router: fp64 dot products four wide (bf16 x bf16 products are exact in
 *     fp64, so the bf16-rounded logits are the oracle's), one (token, expert)
 *     pair per work item; softmax, top-k and renormalisation as the oracle;
 *   - experts grouped: every (token, slot) entry is listed under its expert,
 *     and the shared expert takes every token, so each weight panel is
 *     dequantised once (scale * code + bias, fp32) and used by all of the
 *     expert's tokens;
 *   - gate/up: panels of 8 up rows and the matching 8 gate rows, register
 *     tiles of 4 rows x 3 tokens (AVX2 + FMA, 8 lanes), SwiGLU fused;
 *   - down: panels of 16 output rows over the entries' hidden rows;
 *   - combine: the slots in order, then the gated shared expert (the
 *     oracle's order).
 * After the router everything is fp32 in another summation order than the
 * oracle's, so outputs agree within the parity tolerance, not bit for bit.
 * The AVX2 kernels are chosen at run time (rnbc_simd); other hosts, or any
 * host with RNB_CPU_NO_SIMD=1 in the environment, run the same loops in
 * plain C.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__x86_64__)
#include <immintrin.h>
#define RNBC_X86 1
#endif

#include "rnb_oracle.h"

#define RNBC_PANEL 16 /* weight rows per dequantised panel */
#define RNBC_TR 4     /* rows per register tile */
#define RNBC_TT 3     /* tokens per register tile */

static float bf16f(uint16_t v) {
  const uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static int g_simd = -1;

int rnbc_simd(void) {
  if (g_simd < 0) {
#ifdef RNBC_X86
    __builtin_cpu_init();
    const char* off = getenv("RNB_CPU_NO_SIMD"); /* set: the plain C loops (tests cover both) */
    g_simd = !(off && off[0] && off[0] != '0') && __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
    g_simd = 0;
#endif
  }
  return g_simd;
}

/* ------------------------------------------------------------ kernels */

/* Rows [r0, r0 + n) of a packed affine matrix with K inputs per row into
 * dst [n][K] fp32: w = scale * code + bias per group. */
static void deq_rows_c(const uint32_t* w, const uint16_t* s, const uint16_t* b, int K, int bits,
                       int group, int r0, int n, float* dst) {
  const size_t ws = (size_t)K * bits / 32, ss = (size_t)K / group;
  for (int r = 0; r < n; ++r) {
    const uint32_t* wr = w + (size_t)(r0 + r) * ws;
    const uint16_t* sr = s + (size_t)(r0 + r) * ss;
    const uint16_t* br = b + (size_t)(r0 + r) * ss;
    float* o = dst + (size_t)r * K;
    for (int k = 0; k < K; ++k) {
      const uint32_t q = bits == 8 ? (wr[k >> 2] >> (8 * (k & 3))) & 0xFFu : (wr[k >> 3] >> (4 * (k & 7))) & 0xFu;
      o[k] = bf16f(sr[k / group]) * (float)q + bf16f(br[k / group]);
    }
  }
}

/* out[i][j] = dot(W row i, x row j) over K, 4 rows (stride K) x 3 tokens. */
static void tile_c(const float* W, int K, const float* const* xr, float out[RNBC_TR][RNBC_TT]) {
  for (int i = 0; i < RNBC_TR; ++i)
    for (int j = 0; j < RNBC_TT; ++j) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k) acc += W[(size_t)i * K + k] * xr[j][k];
      out[i][j] = acc;
    }
}

/* Router dot in fp64 of the token's fp32 (bf16-exact) values with row e
 * (e == E: the shared gate's weights). */
static double router_dot_c(const rnbo_block* d, const float* xf, int e) {
  const int H = d->H, shared = e == d->E;
  double acc = 0.0;
  if (d->router_bits == 8) {
    const uint32_t* q = shared ? d->sgate_q : d->router_q + (size_t)e * (H / 4);
    const uint16_t* sc = shared ? d->sgate_s : d->router_s + (size_t)e * (H / 64);
    const uint16_t* bi = shared ? d->sgate_b : d->router_b + (size_t)e * (H / 64);
    for (int h = 0; h < H; ++h) {
      const double code = (double)((q[h / 4] >> (8 * (h % 4))) & 0xFFu);
      acc += (double)xf[h] * ((double)bf16f(sc[h / 64]) * code + (double)bf16f(bi[h / 64]));
    }
  } else {
    const uint16_t* w = shared ? d->shared_gate_w : d->router_w + (size_t)e * H;
    for (int h = 0; h < H; ++h) acc += (double)xf[h] * (double)bf16f(w[h]);
  }
  return acc;
}

#ifdef RNBC_X86
__attribute__((target("avx2,fma"))) static inline float hsum8(__m256 v) {
  __m128 lo = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  lo = _mm_add_ps(lo, _mm_movehl_ps(lo, lo));
  lo = _mm_add_ss(lo, _mm_shuffle_ps(lo, lo, 1));
  return _mm_cvtss_f32(lo);
}

__attribute__((target("avx2,fma"))) static inline double hsum4d(__m256d v) {
  __m128d lo = _mm_add_pd(_mm256_castpd256_pd128(v), _mm256_extractf128_pd(v, 1));
  lo = _mm_add_sd(lo, _mm_unpackhi_pd(lo, lo));
  return _mm_cvtsd_f64(lo);
}

__attribute__((target("avx2,fma"))) static void deq_rows_avx2(const uint32_t* w, const uint16_t* s,
                                                              const uint16_t* b, int K, int bits, int group,
                                                              int r0, int n, float* dst) {
  const size_t ws = (size_t)K * bits / 32, ss = (size_t)K / group;
  const __m256i sh = _mm256_setr_epi32(0, 4, 8, 12, 16, 20, 24, 28), m4 = _mm256_set1_epi32(0xF);
  for (int r = 0; r < n; ++r) {
    const uint32_t* wr = w + (size_t)(r0 + r) * ws;
    const uint16_t* sr = s + (size_t)(r0 + r) * ss;
    const uint16_t* br = b + (size_t)(r0 + r) * ss;
    float* o = dst + (size_t)r * K;
    for (int g = 0; g < K / group; ++g) {
      const __m256 vs = _mm256_set1_ps(bf16f(sr[g])), vb = _mm256_set1_ps(bf16f(br[g]));
      for (int i = 0; i < group; i += 8) {
        const int k = g * group + i;
        __m256i q;
        if (bits == 8) {
          q = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i*)((const uint8_t*)wr + k)));
        } else {
          q = _mm256_and_si256(_mm256_srlv_epi32(_mm256_set1_epi32((int)wr[k >> 3]), sh), m4);
        }
        _mm256_storeu_ps(o + k, _mm256_fmadd_ps(_mm256_cvtepi32_ps(q), vs, vb));
      }
    }
  }
}

__attribute__((target("avx2,fma"))) static void tile_avx2(const float* W, int K, const float* const* xr,
                                                          float out[RNBC_TR][RNBC_TT]) {
  __m256 a00 = _mm256_setzero_ps(), a01 = a00, a02 = a00, a10 = a00, a11 = a00, a12 = a00;
  __m256 a20 = a00, a21 = a00, a22 = a00, a30 = a00, a31 = a00, a32 = a00;
  const float *w0 = W, *w1 = W + K, *w2 = W + 2 * (size_t)K, *w3 = W + 3 * (size_t)K;
  const float *x0 = xr[0], *x1 = xr[1], *x2 = xr[2];
  for (int k = 0; k < K; k += 8) {
    const __m256 v0 = _mm256_loadu_ps(x0 + k), v1 = _mm256_loadu_ps(x1 + k), v2 = _mm256_loadu_ps(x2 + k);
    __m256 w = _mm256_loadu_ps(w0 + k);
    a00 = _mm256_fmadd_ps(w, v0, a00);
    a01 = _mm256_fmadd_ps(w, v1, a01);
    a02 = _mm256_fmadd_ps(w, v2, a02);
    w = _mm256_loadu_ps(w1 + k);
    a10 = _mm256_fmadd_ps(w, v0, a10);
    a11 = _mm256_fmadd_ps(w, v1, a11);
    a12 = _mm256_fmadd_ps(w, v2, a12);
    w = _mm256_loadu_ps(w2 + k);
    a20 = _mm256_fmadd_ps(w, v0, a20);
    a21 = _mm256_fmadd_ps(w, v1, a21);
    a22 = _mm256_fmadd_ps(w, v2, a22);
    w = _mm256_loadu_ps(w3 + k);
    a30 = _mm256_fmadd_ps(w, v0, a30);
    a31 = _mm256_fmadd_ps(w, v1, a31);
    a32 = _mm256_fmadd_ps(w, v2, a32);
  }
  out[0][0] = hsum8(a00), out[0][1] = hsum8(a01), out[0][2] = hsum8(a02);
  out[1][0] = hsum8(a10), out[1][1] = hsum8(a11), out[1][2] = hsum8(a12);
  out[2][0] = hsum8(a20), out[2][1] = hsum8(a21), out[2][2] = hsum8(a22);
  out[3][0] = hsum8(a30), out[3][1] = hsum8(a31), out[3][2] = hsum8(a32);
}

/* One token: out[i] = dot(W row i, x) for 4 rows, two chains per row. */
__attribute__((target("avx2,fma"))) static void tile1_avx2(const float* W, int K, const float* x,
                                                           float out[RNBC_TR]) {
  __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0, b0 = a0, b1 = a0, b2 = a0, b3 = a0;
  const float *w0 = W, *w1 = W + K, *w2 = W + 2 * (size_t)K, *w3 = W + 3 * (size_t)K;
  int k = 0;
  for (; k + 16 <= K; k += 16) {
    const __m256 u = _mm256_loadu_ps(x + k), v = _mm256_loadu_ps(x + k + 8);
    a0 = _mm256_fmadd_ps(_mm256_loadu_ps(w0 + k), u, a0);
    b0 = _mm256_fmadd_ps(_mm256_loadu_ps(w0 + k + 8), v, b0);
    a1 = _mm256_fmadd_ps(_mm256_loadu_ps(w1 + k), u, a1);
    b1 = _mm256_fmadd_ps(_mm256_loadu_ps(w1 + k + 8), v, b1);
    a2 = _mm256_fmadd_ps(_mm256_loadu_ps(w2 + k), u, a2);
    b2 = _mm256_fmadd_ps(_mm256_loadu_ps(w2 + k + 8), v, b2);
    a3 = _mm256_fmadd_ps(_mm256_loadu_ps(w3 + k), u, a3);
    b3 = _mm256_fmadd_ps(_mm256_loadu_ps(w3 + k + 8), v, b3);
  }
  for (; k < K; k += 8) {
    const __m256 u = _mm256_loadu_ps(x + k);
    a0 = _mm256_fmadd_ps(_mm256_loadu_ps(w0 + k), u, a0);
    a1 = _mm256_fmadd_ps(_mm256_loadu_ps(w1 + k), u, a1);
    a2 = _mm256_fmadd_ps(_mm256_loadu_ps(w2 + k), u, a2);
    a3 = _mm256_fmadd_ps(_mm256_loadu_ps(w3 + k), u, a3);
  }
  out[0] = hsum8(_mm256_add_ps(a0, b0));
  out[1] = hsum8(_mm256_add_ps(a1, b1));
  out[2] = hsum8(_mm256_add_ps(a2, b2));
  out[3] = hsum8(_mm256_add_ps(a3, b3));
}

/* One token straight from the codes (no panel): out[r] = dot(row r0 + r, x)
 * for n rows (a multiple of 4), w = scale * code + bias per group. */
__attribute__((target("avx2,fma"))) static void rows_dot1_avx2(const uint32_t* w, const uint16_t* s,
                                                               const uint16_t* b, int K, int bits, int group,
                                                               int r0, int n, const float* x, float* out) {
  const size_t ws = (size_t)K * bits / 32, ss = (size_t)K / group;
  const __m256i sh = _mm256_setr_epi32(0, 4, 8, 12, 16, 20, 24, 28), m4 = _mm256_set1_epi32(0xF);
  for (int r = 0; r < n; r += 4) {
    __m256 acc[4];
    for (int i = 0; i < 4; ++i) acc[i] = _mm256_setzero_ps();
    for (int g = 0; g < K / group; ++g) {
      __m256 vs[4], vb[4];
      for (int i = 0; i < 4; ++i) {
        vs[i] = _mm256_set1_ps(bf16f(s[(size_t)(r0 + r + i) * ss + g]));
        vb[i] = _mm256_set1_ps(bf16f(b[(size_t)(r0 + r + i) * ss + g]));
      }
      for (int j = 0; j < group; j += 8) {
        const int k = g * group + j;
        const __m256 xv = _mm256_loadu_ps(x + k);
        for (int i = 0; i < 4; ++i) {
          const uint32_t* wr = w + (size_t)(r0 + r + i) * ws;
          const __m256i q = bits == 8
                                ? _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i*)((const uint8_t*)wr + k)))
                                : _mm256_and_si256(_mm256_srlv_epi32(_mm256_set1_epi32((int)wr[k >> 3]), sh), m4);
          acc[i] = _mm256_fmadd_ps(_mm256_fmadd_ps(_mm256_cvtepi32_ps(q), vs[i], vb[i]), xv, acc[i]);
        }
      }
    }
    for (int i = 0; i < 4; ++i) out[r + i] = hsum8(acc[i]);
  }
}

__attribute__((target("avx2,fma"))) static double router_dot_avx2(const rnbo_block* d, const float* xf, int e) {
  const int H = d->H, shared = e == d->E;
  __m256d a0 = _mm256_setzero_pd(), a1 = a0;
  if (d->router_bits == 8) {
    const uint32_t* q = shared ? d->sgate_q : d->router_q + (size_t)e * (H / 4);
    const uint16_t* sc = shared ? d->sgate_s : d->router_s + (size_t)e * (H / 64);
    const uint16_t* bi = shared ? d->sgate_b : d->router_b + (size_t)e * (H / 64);
    for (int g = 0; g < H / 64; ++g) {
      const __m256d vs = _mm256_set1_pd((double)bf16f(sc[g])), vb = _mm256_set1_pd((double)bf16f(bi[g]));
      for (int i = 0; i < 64; i += 8) {
        const int h = g * 64 + i;
        const __m256i c = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i*)((const uint8_t*)q + h)));
        const __m256d w0 = _mm256_fmadd_pd(_mm256_cvtepi32_pd(_mm256_castsi256_si128(c)), vs, vb);
        const __m256d w1 = _mm256_fmadd_pd(_mm256_cvtepi32_pd(_mm256_extracti128_si256(c, 1)), vs, vb);
        const __m256 x = _mm256_loadu_ps(xf + h);
        a0 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm256_castps256_ps128(x)), w0, a0);
        a1 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm256_extractf128_ps(x, 1)), w1, a1);
      }
    }
  } else {
    const uint16_t* w = shared ? d->shared_gate_w : d->router_w + (size_t)e * H;
    for (int h = 0; h < H; h += 8) {
      const __m256i wi = _mm256_slli_epi32(_mm256_cvtepu16_epi32(_mm_loadu_si128((const __m128i*)(w + h))), 16);
      const __m256 wf = _mm256_castsi256_ps(wi), x = _mm256_loadu_ps(xf + h);
      a0 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm256_castps256_ps128(x)), _mm256_cvtps_pd(_mm256_castps256_ps128(wf)), a0);
      a1 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm256_extractf128_ps(x, 1)), _mm256_cvtps_pd(_mm256_extractf128_ps(wf, 1)), a1);
    }
  }
  return hsum4d(_mm256_add_pd(a0, a1));
}
#endif

static void deq_rows(const uint32_t* w, const uint16_t* s, const uint16_t* b, int K, int bits, int group, int r0,
                     int n, float* dst) {
#ifdef RNBC_X86
  if (g_simd && group % 8 == 0) {
    deq_rows_avx2(w, s, b, K, bits, group, r0, n, dst);
    return;
  }
#endif
  deq_rows_c(w, s, b, K, bits, group, r0, n, dst);
}

/* nt live tokens (1 <= nt <= 3; the rest of xr repeats xr[0]). */
static void tile(const float* W, int K, const float* const* xr, int nt, float out[RNBC_TR][RNBC_TT]) {
#ifdef RNBC_X86
  if (g_simd && K % 8 == 0) {
    if (nt == 1) {
      float o[RNBC_TR];
      tile1_avx2(W, K, xr[0], o);
      for (int i = 0; i < RNBC_TR; ++i) out[i][0] = o[i];
    } else {
      tile_avx2(W, K, xr, out);
    }
    return;
  }
#endif
  tile_c(W, K, xr, out);
}

static double router_dot(const rnbo_block* d, const float* xf, int e) {
#ifdef RNBC_X86
  if (g_simd && d->H % 64 == 0) return router_dot_avx2(d, xf, e);
#endif
  return router_dot_c(d, xf, e);
}

#ifdef RNBC_X86
__attribute__((target("avx2,fma"))) static float dot_f32_avx2(const float* a, const float* b, int n) {
  __m256 acc = _mm256_setzero_ps();
  for (int i = 0; i < n; i += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc);
  return hsum8(acc);
}
#endif

static float dot_f32(const float* a, const float* b, int n) {
#ifdef RNBC_X86
  if (g_simd && n % 8 == 0) return dot_f32_avx2(a, b, n);
#endif
  float acc = 0.0f;
  for (int i = 0; i < n; ++i) acc += a[i] * b[i];
  return acc;
}

/* ------------------------------------------------------------- router */

/* Logits (bf16-rounded, as the oracle), top-k with ties to the lower index,
 * fp32 softmax over all E gathered at the picks and renormalised, and the
 * shared gate sigmoid(x . w_sg) in fp32. */
static void route(const rnbo_block* d, const float* xf, float* lg, int32_t* inds, float* scores, float* sg,
                  int nthreads) {
  const int T = d->T, H = d->H, E = d->E, K = d->k;
  const long pairs = (long)T * E;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (long te = 0; te < pairs; ++te) {
    const int t = (int)(te / E), e = (int)(te % E);
    lg[te] = rnbo_f64_to_bf16_f32(router_dot(d, xf + (size_t)t * H, e));
  }
  const int has_sg = d->router_bits == 8 ? d->sgate_q != NULL : d->shared_gate_w != NULL;
  float wsg[8192]; /* the shared gate's weights, fp32 (H <= 8192, checked by the caller) */
  for (int h = 0; h < H; ++h) {
    if (!has_sg) {
      wsg[h] = 0.0f;
    } else if (d->router_bits == 8) {
      const double code = (double)((d->sgate_q[h / 4] >> (8 * (h % 4))) & 0xFFu);
      wsg[h] = (float)((double)bf16f(d->sgate_s[h / 64]) * code + (double)bf16f(d->sgate_b[h / 64]));
    } else {
      wsg[h] = bf16f(d->shared_gate_w[h]);
    }
  }
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* l = lg + (size_t)t * E;
    float mx = l[0];
    for (int e = 1; e < E; ++e) mx = l[e] > mx ? l[e] : mx;
    float denom = 0.0f;
    for (int e = 0; e < E; ++e) denom += expf(l[e] - mx);
    float p[64], psum = 0.0f;
    int32_t* it = inds + (size_t)t * K;
    for (int s = 0; s < K; ++s) {
      int best = -1;
      for (int e = 0; e < E; ++e) {
        int used = 0;
        for (int j = 0; j < s; ++j) used |= it[j] == e;
        if (!used && (best < 0 || l[e] > l[best])) best = e;
      }
      it[s] = best;
      p[s] = expf(l[best] - mx) / denom;
      psum += p[s];
    }
    for (int s = 0; s < K; ++s) scores[(size_t)t * K + s] = p[s] / psum;
    sg[t] = has_sg ? 1.0f / (1.0f + expf(-dot_f32(xf + (size_t)t * H, wsg, H))) : 0.0f;
  }
}

/* -------------------------------------------------------------- block */

/* One expert's weights (e == E: the shared expert). */
typedef struct {
  const uint32_t *guw, *dnw;
  const uint16_t *gus, *gub, *dns, *dnb;
} expert_w;

static expert_w expert_at(const rnbo_block* d, int e) {
  expert_w w;
  if (e == d->E) {
    w.guw = d->sgu_w, w.gus = d->sgu_s, w.gub = d->sgu_b;
    w.dnw = d->sdn_w, w.dns = d->sdn_s, w.dnb = d->sdn_b;
    return w;
  }
  const size_t H = d->H, I = d->I, G = d->group, bits = d->bits;
  w.guw = d->gu_w + (size_t)e * 2 * I * H * bits / 32;
  w.gus = d->gu_s + (size_t)e * 2 * I * H / G;
  w.gub = d->gu_b + (size_t)e * 2 * I * H / G;
  w.dnw = d->dn_w + (size_t)e * H * I * bits / 32;
  w.dns = d->dn_s + (size_t)e * H * I / G;
  w.dnb = d->dn_b + (size_t)e * H * I / G;
  return w;
}

int rnbc_moe_block(const rnbo_block* d, float* out, int32_t* inds, float* scores, int nthreads) {
  if (!d || d->T < 0 || d->H <= 0 || d->I <= 0 || d->E <= 0 || d->k <= 0 || d->k > d->E || d->k > 64)
    return RNBO_EINVAL;
  if ((d->bits != 4 && d->bits != 8) || d->group <= 0 || d->H % d->group || d->I % d->group) return RNBO_EINVAL;
  if (d->I % 8 || d->H % RNBC_PANEL || d->H > 8192) return RNBO_EINVAL;
  if (d->router_bits == 8 && (!d->router_q || !d->router_s || !d->router_b || d->H % 64)) return RNBO_EINVAL;
  if (nthreads < 1) nthreads = 1;
  rnbc_simd();
  const int T = d->T, H = d->H, I = d->I, E = d->E, K = d->k, S = K + 1;
  const int shared = d->sgu_w != NULL, NE = E + 1;
  if (T == 0) return RNBO_OK;
  float* xf = (float*)malloc(sizeof(float) * (size_t)T * H);
  float* lg = (float*)malloc(sizeof(float) * (size_t)T * E);
  float* sg = (float*)malloc(sizeof(float) * T);
  int* cnt = (int*)calloc((size_t)NE + 1, sizeof(int));
  int* ent = (int*)malloc(sizeof(int) * (size_t)T * S); /* t * S + s, grouped by expert */
  float* hid = (float*)malloc(sizeof(float) * (size_t)T * S * I);
  float* y = (float*)malloc(sizeof(float) * (size_t)T * S * H);
  if (!xf || !lg || !sg || !cnt || !ent || !hid || !y) {
    free(xf), free(lg), free(sg), free(cnt), free(ent), free(hid), free(y);
    return RNBO_EINVAL;
  }
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (long i = 0; i < (long)T * H; ++i) xf[i] = bf16f(d->x[i]);
  route(d, xf, lg, inds, scores, sg, nthreads);

  /* entries grouped by expert (stable: token order, then slot) */
  for (int t = 0; t < T; ++t)
    for (int s = 0; s < K; ++s) cnt[inds[(size_t)t * K + s] + 1]++;
  if (shared) cnt[E + 1] = T;
  for (int e = 0; e < NE; ++e) cnt[e + 1] += cnt[e];
  {
    int* fill = (int*)malloc(sizeof(int) * NE);
    if (!fill) {
      free(xf), free(lg), free(sg), free(cnt), free(ent), free(hid), free(y);
      return RNBO_EINVAL;
    }
    memcpy(fill, cnt, sizeof(int) * NE);
    for (int t = 0; t < T; ++t) {
      for (int s = 0; s < K; ++s) ent[fill[inds[(size_t)t * K + s]]++] = t * S + s;
      if (shared) ent[fill[E]++] = t * S + K;
    }
    free(fill);
  }
  /* work items: (expert, panel); gate/up panels of 8 channels, down panels
   * of 16 output rows */
  const int gu_per = I / 8, dn_per = H / RNBC_PANEL;
  int n_act = 0;
  int* act = (int*)malloc(sizeof(int) * NE);
  if (!act) {
    free(xf), free(lg), free(sg), free(cnt), free(ent), free(hid), free(y);
    return RNBO_EINVAL;
  }
  for (int e = 0; e < NE; ++e)
    if (cnt[e + 1] > cnt[e]) act[n_act++] = e;

  int oom = 0;
#pragma omp parallel num_threads(nthreads)
  {
    const int kmax = H > I ? H : I;
    float* panel = (float*)malloc(sizeof(float) * (size_t)RNBC_PANEL * kmax);
    if (!panel) {
#pragma omp atomic write
      oom = 1;
    }
    float res[RNBC_TR][RNBC_TT];
    const float* xr[RNBC_TT];
#pragma omp for schedule(dynamic, 4)
    for (long it = 0; it < (long)n_act * gu_per; ++it) {
      if (!panel) continue;
      const int e = act[it / gu_per], c0 = (int)(it % gu_per) * 8;
      const expert_w w = expert_at(d, e);
#ifdef RNBC_X86
      if (g_simd && cnt[e + 1] - cnt[e] == 1 && d->group % 8 == 0) {
        /* one token: dot straight from the codes */
        const float* x1 = xf + (size_t)(ent[cnt[e]] / S) * H;
        float ug[16];
        rows_dot1_avx2(w.guw, w.gus, w.gub, H, d->bits, d->group, c0, 8, x1, ug);
        rows_dot1_avx2(w.guw, w.gus, w.gub, H, d->bits, d->group, I + c0, 8, x1, ug + 8);
        float* hr = hid + (size_t)ent[cnt[e]] * I + c0;
        for (int c = 0; c < 8; ++c) hr[c] = (ug[8 + c] / (1.0f + expf(-ug[8 + c]))) * ug[c];
        continue;
      }
#endif
      deq_rows(w.guw, w.gus, w.gub, H, d->bits, d->group, c0, 8, panel);               /* up rows */
      deq_rows(w.guw, w.gus, w.gub, H, d->bits, d->group, I + c0, 8, panel + 8 * (size_t)H); /* gate */
      for (int j0 = cnt[e]; j0 < cnt[e + 1]; j0 += RNBC_TT) {
        const int nj = cnt[e + 1] - j0 < RNBC_TT ? cnt[e + 1] - j0 : RNBC_TT;
        for (int j = 0; j < RNBC_TT; ++j) xr[j] = xf + (size_t)(ent[j0 + (j < nj ? j : 0)] / S) * H;
        float v[RNBC_PANEL][RNBC_TT];
        for (int q = 0; q < RNBC_PANEL / RNBC_TR; ++q) {
          tile(panel + (size_t)q * RNBC_TR * H, H, xr, nj, res);
          for (int i = 0; i < RNBC_TR; ++i)
            for (int j = 0; j < RNBC_TT; ++j) v[q * RNBC_TR + i][j] = res[i][j];
        }
        for (int j = 0; j < nj; ++j) {
          float* hr = hid + (size_t)ent[j0 + j] * I + c0;
          for (int c = 0; c < 8; ++c) {
            const float up = v[c][j], gate = v[8 + c][j];
            hr[c] = (gate / (1.0f + expf(-gate))) * up;
          }
        }
      }
    }
#pragma omp for schedule(dynamic, 4)
    for (long it = 0; it < (long)n_act * dn_per; ++it) {
      if (!panel) continue;
      const int e = act[it / dn_per], n0 = (int)(it % dn_per) * RNBC_PANEL;
      const expert_w w = expert_at(d, e);
#ifdef RNBC_X86
      if (g_simd && cnt[e + 1] - cnt[e] == 1 && d->group % 8 == 0) {
        const int en = ent[cnt[e]];
        rows_dot1_avx2(w.dnw, w.dns, w.dnb, I, d->bits, d->group, n0, RNBC_PANEL, hid + (size_t)en * I,
                       y + (size_t)en * H + n0);
        continue;
      }
#endif
      deq_rows(w.dnw, w.dns, w.dnb, I, d->bits, d->group, n0, RNBC_PANEL, panel);
      for (int j0 = cnt[e]; j0 < cnt[e + 1]; j0 += RNBC_TT) {
        const int nj = cnt[e + 1] - j0 < RNBC_TT ? cnt[e + 1] - j0 : RNBC_TT;
        for (int j = 0; j < RNBC_TT; ++j) xr[j] = hid + (size_t)ent[j0 + (j < nj ? j : 0)] * I;
        for (int q = 0; q < RNBC_PANEL / RNBC_TR; ++q) {
          tile(panel + (size_t)q * RNBC_TR * I, I, xr, nj, res);
          for (int j = 0; j < nj; ++j) {
            float* yr = y + (size_t)ent[j0 + j] * H + n0 + q * RNBC_TR;
            for (int i = 0; i < RNBC_TR; ++i) yr[i] = res[i][j];
          }
        }
      }
    }
    free(panel);
  }
  if (oom) {
    free(act);
    free(xf), free(lg), free(sg), free(cnt), free(ent), free(hid), free(y);
    return RNBO_EINVAL;
  }
  /* combine: the slots in order, then the gated shared expert */
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* sc = scores + (size_t)t * K;
    const float* yt = y + (size_t)t * S * H;
    float* o = out + (size_t)t * H;
    for (int n = 0; n < H; ++n) {
      float acc = 0.0f;
      for (int s = 0; s < K; ++s) acc += sc[s] * yt[(size_t)s * H + n];
      if (shared) acc += sg[t] * yt[(size_t)K * H + n];
      o[n] = acc;
    }
  }
  free(act);
  free(xf), free(lg), free(sg), free(cnt), free(ent), free(hid), free(y);
  return RNBO_OK;
}
