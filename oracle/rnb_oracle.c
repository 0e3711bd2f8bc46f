/*
 * rnb_oracle.c -- CPU restatement of Runnel's sparse-MoE block arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm load it.  The product path (runnel_b200) never links or calls it.
 *
 * What it restates (paths inside the waylake/runnel project):
 *   - MLX affine dequant-dot, fp32, sequential per 64-group:
 *       native/src/fused_moe_probe.mm:630-695   (row_dot, scale applied per group)
 *       native/src/quantized_qmv_probe.mm:404-431 (scale applied per element)
 *       native/src/quantized_qmm_probe.mm:281-305
 *   - packed routed gate/up layout (rows 0..I-1 = up, I..2I-1 = gate) and
 *     silu(gate)*up: src/runnel/mlx.py:38-48,76-78; native/shaders/fused_moe.metal:449,534-541
 *   - shared expert swiglu(x_gate, x_up) = silu(gate)*up, sigmoid gate:
 *       bench/mlx_lm_adapter.py:82-94
 *   - router softmax / top-k / renormalise of the mlx-lm Qwen3.5 sparse-MoE
 *     block (third-party mlx-lm @15bcf8b, not vendored; call site
 *     src/runnel/mlx.py:57-82).
 *   - the reference's synthetic data generators (xorshift64 + bf16 RNE) used
 *     to reproduce its recorded known-answer checksums:
 *       native/src/fused_moe_probe.mm:69-104,449-537,600-628
 *       native/src/quantized_qmv_probe.mm:64-101,365-431
 *       native/src/quantized_qmm_probe.mm:245-305
 *
 * Rounding points of the block oracle (the "fp32-accumulated result"):
 *   router logits are the correctly rounded bf16 (MLX's Linear output dtype)
 *   of the exact dot product (double accumulation of exact products), expert
 *   selection is top-k of those bf16 logits with ties broken
 *   toward the lower expert index, routing weights are the fp32 softmax over
 *   all E bf16 logits gathered at the selected experts and renormalised in
 *   fp32; everything after that (gate/up, SwiGLU, down, combine, shared
 *   expert and its sigmoid gate) stays fp32.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "rnb_oracle.h"

/* ---------------------------------------------------------------- bf16 */

uint16_t rnbo_f32_to_bf16(float value) {
  uint32_t bits;
  memcpy(&bits, &value, 4);
  if (((bits >> 23) & 0xFFu) == 0xFFu) return (uint16_t)(bits >> 16); /* inf/nan kept */
  bits += 0x7FFFu + ((bits >> 16) & 1u);                             /* round to nearest even */
  return (uint16_t)(bits >> 16);
}

float rnbo_bf16_to_f32(uint16_t value);

/* Round a double directly to bf16 (to nearest, ties to even), returned as
 * float; used for router logits so they are the correctly rounded bf16 of
 * the (double-accumulated) dot product.  Magnitudes below 2^-126 are rounded
 * through fp32; -0 becomes +0 (the selection compares values). */
float rnbo_f64_to_bf16_f32(double v) {
  if (v != v) return (float)v;
  if (fabs(v) < 0x1p-126) return rnbo_bf16_to_f32(rnbo_f32_to_bf16((float)v)) + 0.0f;
  uint64_t b;
  memcpy(&b, &v, 8);
  const uint64_t sign = b >> 63;
  int e = (int)((b >> 52) & 0x7FF);
  const uint64_t m = b & ((1ull << 52) - 1);
  uint64_t q = m >> 45;
  const uint64_t rem = m & ((1ull << 45) - 1), half = 1ull << 44;
  if (rem > half || (rem == half && (q & 1))) {
    if (++q == 128) {
      q = 0;
      ++e;
    }
  }
  const int fe = e - 1023 + 127;
  const uint32_t fb = fe >= 255 ? (uint32_t)(sign << 31) | 0x7F800000u
                                : (uint32_t)(sign << 31) | ((uint32_t)fe << 23) | (uint32_t)(q << 16);
  float out;
  memcpy(&out, &fb, 4);
  return out;
}

float rnbo_bf16_to_f32(uint16_t value) {
  uint32_t bits = (uint32_t)value << 16;
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

void rnbo_f32_to_bf16_array(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = rnbo_f32_to_bf16(in[i]);
}

void rnbo_bf16_to_f32_array(const uint16_t* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = rnbo_bf16_to_f32(in[i]);
}

/* ------------------------------------------------- affine dequant-dot */

static inline uint32_t code_at(const uint32_t* row, int bits, size_t k) {
  const size_t per = 32u / (unsigned)bits;
  const uint32_t mask = (bits == 8) ? 0xFFu : 0x0Fu;
  return (row[k / per] >> ((unsigned)bits * (k % per))) & mask;
}

/* One packed row against an fp32 vector: per group
 *   result += (sum_k q_k * x_k) * scale + (sum_k x_k) * bias
 * in fp32, k ascending (fused_moe_probe.mm:630-695).  The reference was built
 * by clang for arm64, which contracts `acc += a * b` into one fused
 * multiply-add and `a * b + c * d` into fma(a, b, c * d); the fmaf calls
 * below make that rounding explicit (it is what reproduces the recorded
 * QMM q8 checksum -12808.676; uncontracted fp32 gives -12808.682). */
float rnbo_affine_dot(const uint32_t* w_row, const uint16_t* s_row, const uint16_t* b_row,
                      const float* x, int K, int bits, int group) {
  float result = 0.0f;
  const int groups = K / group;
  for (int g = 0; g < groups; ++g) {
    const float scale = rnbo_bf16_to_f32(s_row[g]);
    const float bias = rnbo_bf16_to_f32(b_row[g]);
    float weighted = 0.0f, xsum = 0.0f;
    for (int i = 0; i < group; ++i) {
      const size_t k = (size_t)g * group + i;
      weighted = fmaf((float)code_at(w_row, bits, k), x[k], weighted);
      xsum += x[k];
    }
    result += fmaf(weighted, scale, xsum * bias);
  }
  return result;
}

/* Same contraction with the scale applied per element
 * (quantized_qmv_probe.mm:404-431): weighted += q * scale * x. */
static float affine_dot_scale_inside(const uint32_t* w_row, const uint16_t* s_row,
                                     const uint16_t* b_row, const float* x, int K, int bits,
                                     int group) {
  float result = 0.0f;
  const int groups = K / group;
  for (int g = 0; g < groups; ++g) {
    const float scale = rnbo_bf16_to_f32(s_row[g]);
    const float bias = rnbo_bf16_to_f32(b_row[g]);
    float weighted = 0.0f, xsum = 0.0f;
    for (int i = 0; i < group; ++i) {
      const size_t k = (size_t)g * group + i;
      weighted = fmaf((float)code_at(w_row, bits, k) * scale, x[k], weighted);
      xsum += x[k];
    }
    result += fmaf(xsum, bias, weighted);
  }
  return result;
}

/* y[r] = dot(row r, x) for a dense packed matrix [rows, K]. */
int rnbo_affine_matvec(const uint32_t* w, const uint16_t* s, const uint16_t* b, const float* x,
                       int rows, int K, int bits, int group, float* y, int nthreads) {
  if ((bits != 4 && bits != 8) || group <= 0 || K % group || K % (32 / bits)) return RNBO_EINVAL;
  const size_t wstride = (size_t)K * bits / 32, sstride = (size_t)K / group;
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(static)
  for (int r = 0; r < rows; ++r)
    y[r] = rnbo_affine_dot(w + r * wstride, s + r * sstride, b + r * sstride, x, K, bits, group);
  return RNBO_OK;
}

/* ------------------------------------------------------- MoE block */

/* Router weight (row e; e == E is the shared gate) at input h, exact in
 * double: bf16, or the 8-bit affine scale * code + bias (a bf16 times an
 * 8-bit integer plus a bf16 is exact in double). */
static double router_weight(const rnbo_block* d, int e, int h) {
  const int H = d->H, shared = e == d->E;
  if (d->router_bits == 8) {
    const uint32_t* q = shared ? d->sgate_q : d->router_q + (size_t)e * (H / 4);
    const uint16_t* sc = shared ? d->sgate_s : d->router_s + (size_t)e * (H / 64);
    const uint16_t* bi = shared ? d->sgate_b : d->router_b + (size_t)e * (H / 64);
    const double code = (double)((q[h / 4] >> (8 * (h % 4))) & 0xFFu);
    return (double)rnbo_bf16_to_f32(sc[h / 64]) * code + (double)rnbo_bf16_to_f32(bi[h / 64]);
  }
  const uint16_t* w = shared ? d->shared_gate_w : d->router_w + (size_t)e * H;
  return (double)rnbo_bf16_to_f32(w[h]);
}

static int block_valid(const rnbo_block* d) {
  if (!d || d->T < 0 || d->H <= 0 || d->I <= 0 || d->E <= 0 || d->k <= 0 || d->k > d->E) return 0;
  if (d->router_bits == 8 && (!d->router_q || !d->router_s || !d->router_b || d->H % 64)) return 0;
  if ((d->bits != 4 && d->bits != 8) || d->group <= 0) return 0;
  if (d->H % d->group || d->I % d->group) return 0;
  return 1;
}

static void x_row_f32(const rnbo_block* d, int t, float* xf) {
  for (int h = 0; h < d->H; ++h) xf[h] = rnbo_bf16_to_f32(d->x[(size_t)t * d->H + h]);
}

/* Router: bf16 logits, top-k (ties -> lower index), renormalised softmax
 * weights; slots ordered by descending (logit, -index).  shared_gate[t] is
 * sigmoid(x . w_sg) in fp32 when a shared expert is present. */
int rnbo_router(const rnbo_block* d, float* logits, int32_t* inds, float* scores,
                float* shared_gate, int nthreads) {
  if (!block_valid(d)) return RNBO_EINVAL;
  const int T = d->T, H = d->H, E = d->E, K = d->k;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float* xf = (float*)malloc(sizeof(float) * H);
    float* lg = (float*)malloc(sizeof(float) * E);
    unsigned char* taken = (unsigned char*)malloc(E);
#pragma omp for schedule(static)
    for (int t = 0; t < T; ++t) {
      x_row_f32(d, t, xf);
      for (int e = 0; e < E; ++e) {
        /* bf16 x bf16 products are exact in double and the double sum of
         * 2048 of them is far below bf16 resolution: the logit is the
         * correctly rounded bf16 of the exact dot product */
        double acc = 0.0;
        for (int h = 0; h < H; ++h) acc += (double)xf[h] * router_weight(d, e, h);
        lg[e] = rnbo_f64_to_bf16_f32(acc);
        if (logits) logits[(size_t)t * E + e] = lg[e];
      }
      /* softmax over all E in fp32 (mlx-lm: softmax(gates, precise=True)) */
      float mx = lg[0];
      for (int e = 1; e < E; ++e) mx = lg[e] > mx ? lg[e] : mx;
      float denom = 0.0f;
      for (int e = 0; e < E; ++e) denom += expf(lg[e] - mx);
      memset(taken, 0, E);
      float sel_sum = 0.0f;
      float sel_p[64];
      for (int s = 0; s < K; ++s) {
        int best = -1;
        for (int e = 0; e < E; ++e) {
          if (taken[e]) continue;
          if (best < 0 || lg[e] > lg[best]) best = e; /* strict: keeps the lower index on ties */
        }
        taken[best] = 1;
        inds[(size_t)t * K + s] = best;
        sel_p[s] = expf(lg[best] - mx) / denom;
        sel_sum += sel_p[s];
      }
      for (int s = 0; s < K; ++s) scores[(size_t)t * K + s] = sel_p[s] / sel_sum;
      if (shared_gate) {
        if (d->router_bits == 8 ? d->sgate_q != NULL : d->shared_gate_w != NULL) {
          /* fp32, the dequantised weight rounded to fp32 (exact for bf16) */
          float acc = 0.0f;
          for (int h = 0; h < H; ++h) acc += xf[h] * (float)router_weight(d, E, h);
          shared_gate[t] = 1.0f / (1.0f + expf(-acc));
        } else {
          shared_gate[t] = 0.0f;
        }
      }
    }
    free(xf);
    free(lg);
    free(taken);
  }
  return RNBO_OK;
}

/* gate/up -> silu(gate)*up -> down for one expert bank entry. */
static void expert_forward(int H, int I, int bits, int group, const uint32_t* guw,
                           const uint16_t* gus, const uint16_t* gub, const uint32_t* dnw,
                           const uint16_t* dns, const uint16_t* dnb, const float* xf, float* hbuf,
                           float* y) {
  const size_t gu_ws = (size_t)H * bits / 32, gu_ss = (size_t)H / group;
  const size_t dn_ws = (size_t)I * bits / 32, dn_ss = (size_t)I / group;
  for (int c = 0; c < I; ++c) {
    const float up = rnbo_affine_dot(guw + c * gu_ws, gus + c * gu_ss, gub + c * gu_ss, xf, H, bits, group);
    const size_t g = (size_t)(c + I);
    const float gate = rnbo_affine_dot(guw + g * gu_ws, gus + g * gu_ss, gub + g * gu_ss, xf, H, bits, group);
    hbuf[c] = (gate / (1.0f + expf(-gate))) * up;
  }
  for (int n = 0; n < H; ++n)
    y[n] = rnbo_affine_dot(dnw + n * dn_ws, dns + n * dn_ss, dnb + n * dn_ss, hbuf, I, bits, group);
}

/* SwitchGLU: per-slot, unweighted expert outputs y[t,s,:] (fp32) for the
 * caller's indices [T,k] (src/runnel/mlx.py:57-82 semantics). */
int rnbo_switchglu(const rnbo_block* d, const int32_t* inds, float* y, int nthreads) {
  if (!block_valid(d)) return RNBO_EINVAL;
  const int T = d->T, H = d->H, I = d->I, K = d->k, bits = d->bits, G = d->group;
  for (int i = 0; i < T * K; ++i)
    if (inds[i] < 0 || inds[i] >= d->E) return RNBO_EINVAL;
  const size_t gu_we = (size_t)2 * I * H * bits / 32, gu_se = (size_t)2 * I * H / G;
  const size_t dn_we = (size_t)H * I * bits / 32, dn_se = (size_t)H * I / G;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float* xf = (float*)malloc(sizeof(float) * H);
    float* hb = (float*)malloc(sizeof(float) * I);
#pragma omp for schedule(dynamic, 1)
    for (int ts = 0; ts < T * K; ++ts) {
      const int t = ts / K;
      const size_t e = (size_t)inds[ts];
      x_row_f32(d, t, xf);
      expert_forward(H, I, bits, G, d->gu_w + e * gu_we, d->gu_s + e * gu_se, d->gu_b + e * gu_se,
                     d->dn_w + e * dn_we, d->dn_s + e * dn_se, d->dn_b + e * dn_se, xf, hb,
                     y + (size_t)ts * H);
    }
    free(xf);
    free(hb);
  }
  return RNBO_OK;
}

/* Shared expert output (unweighted) per token: down(silu(gate.x)*(up.x)). */
int rnbo_shared_expert(const rnbo_block* d, float* y, int nthreads) {
  if (!block_valid(d) || !d->sgu_w) return RNBO_EINVAL;
  const int T = d->T, H = d->H, I = d->I;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float* xf = (float*)malloc(sizeof(float) * H);
    float* hb = (float*)malloc(sizeof(float) * I);
#pragma omp for schedule(dynamic, 1)
    for (int t = 0; t < T; ++t) {
      x_row_f32(d, t, xf);
      expert_forward(H, I, d->bits, d->group, d->sgu_w, d->sgu_s, d->sgu_b, d->sdn_w, d->sdn_s,
                     d->sdn_b, xf, hb, y + (size_t)t * H);
    }
    free(xf);
    free(hb);
  }
  return RNBO_OK;
}

/* ------------------------------------------- forward error bound */

/* gamma_n = n u / (1 - n u), u = 2^-24: the classical bound on the relative
 * error (to the sum of |terms|) of an n-term fp32 sum in any order. */
static double gamma_n(double n) {
  const double u = 0x1p-24;
  return n * u / (1.0 - n * u);
}

/* Dot product of one affine row with x, in double, plus sum |terms|. */
static double affine_dot_abs(const uint32_t* w_row, const uint16_t* s_row, const uint16_t* b_row,
                             const double* x, int K, int bits, int group, double* abs_sum) {
  double acc = 0.0, a = 0.0;
  for (int k = 0; k < K; ++k) {
    const int g = k / group;
    const double w = (double)rnbo_bf16_to_f32(s_row[g]) * (double)code_at(w_row, bits, (size_t)k) +
                     (double)rnbo_bf16_to_f32(b_row[g]);
    acc += w * x[k];
    a += fabs(w * x[k]);
  }
  *abs_sum = a;
  return acc;
}

/* One expert on one token: y[n] (double) and the first-order forward error
 * bound eb[n] of evaluating it in fp32 from the exact inputs, with every
 * dot product accumulated in any order:
 *   gate/up  g, u = W x (K = H terms):     |dg| <= gamma_H sum|W x|
 *   SwiGLU   h = silu(g) u:                 |dh| <= |silu'(g) u| |dg| + |silu(g)| |du| + 3u |h|
 *   down     y = W_dn h (I terms):          |dy| <= gamma_I sum|W_dn h| + sum |W_dn| |dh| */
static void expert_bound(int H, int I, int bits, int group, const uint32_t* guw, const uint16_t* gus,
                         const uint16_t* gub, const uint32_t* dnw, const uint16_t* dns, const uint16_t* dnb,
                         const double* xd, double* h, double* dh, double* y, double* eb) {
  const size_t gu_ws = (size_t)H * bits / 32, gu_ss = (size_t)H / group;
  const size_t dn_ws = (size_t)I * bits / 32, dn_ss = (size_t)I / group;
  const double gH = gamma_n(H), gI = gamma_n(I), u = 0x1p-24;
  for (int c = 0; c < I; ++c) {
    double au, ag;
    const double up = affine_dot_abs(guw + c * gu_ws, gus + c * gu_ss, gub + c * gu_ss, xd, H, bits, group, &au);
    const size_t r = (size_t)(c + I);
    const double gate = affine_dot_abs(guw + r * gu_ws, gus + r * gu_ss, gub + r * gu_ss, xd, H, bits, group, &ag);
    const double sig = 1.0 / (1.0 + exp(-gate));
    const double silu = gate * sig, dsilu = sig * (1.0 + gate * (1.0 - sig));
    h[c] = silu * up;
    dh[c] = fabs(dsilu * up) * gH * ag + fabs(silu) * gH * au + 3.0 * u * fabs(h[c]);
  }
  for (int n = 0; n < H; ++n) {
    const uint32_t* wr = dnw + n * dn_ws;
    const uint16_t* sr = dns + n * dn_ss;
    const uint16_t* br = dnb + n * dn_ss;
    double acc = 0.0, a = 0.0, prop = 0.0;
    for (int i = 0; i < I; ++i) {
      const int g = i / group;
      const double w = (double)rnbo_bf16_to_f32(sr[g]) * (double)code_at(wr, bits, (size_t)i) +
                       (double)rnbo_bf16_to_f32(br[g]);
      acc += w * h[i];
      a += fabs(w * h[i]);
      prop += fabs(w) * dh[i];
    }
    y[n] = acc;
    eb[n] = gI * a + prop;
  }
}

/* Forward error bound of every block output element: how far an fp32
 * evaluation of the block from the exact inputs (bf16 x and weights, the
 * oracle's routing) may land from the exact value, to first order, with
 * every sum accumulated in any order (gamma_n bounds, u = 2^-24):
 *   out[t,n] = sum_s w_s y_s[n] + sg y_shared[n]
 *   bound    = sum_s (|w_s| eb_s[n] + gamma_16 |w_s y_s[n]|)
 *              + |sg| eb_sh[n] + |d sg| |y_sh[n]| + gamma_9 sum |terms|
 * with the routing weights' own rounding (softmax, renormalisation) taken
 * as gamma_16 |w_s| and the shared gate's d sg = sg (1 - sg) gamma_H
 * sum_k |x_k w_sg,k| + 2u sg.  Without scores (scores == NULL) the bound is
 * that of each slot's unweighted SwitchGLU output: bound [T,k,H].  The
 * parity tests use it as the floor of their per-element tolerance. */
int rnbo_block_bound(const rnbo_block* d, const int32_t* inds, const float* scores, const float* sg,
                     float* bound, int nthreads) {
  if (!block_valid(d)) return RNBO_EINVAL;
  const int T = d->T, H = d->H, I = d->I, K = d->k, bits = d->bits, G = d->group;
  for (int i = 0; i < T * K; ++i)
    if (inds[i] < 0 || inds[i] >= d->E) return RNBO_EINVAL;
  const size_t gu_we = (size_t)2 * I * H * bits / 32, gu_se = (size_t)2 * I * H / G;
  const size_t dn_we = (size_t)H * I * bits / 32, dn_se = (size_t)H * I / G;
  const int per_slot = scores == NULL;
  const double g16 = gamma_n(16.0), g9 = gamma_n(9.0), gH = gamma_n(H), u = 0x1p-24;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    double* xd = (double*)malloc(sizeof(double) * H);
    double* h = (double*)malloc(sizeof(double) * I);
    double* dh = (double*)malloc(sizeof(double) * I);
    double* y = (double*)malloc(sizeof(double) * H);
    double* eb = (double*)malloc(sizeof(double) * H);
    double* acc = (double*)malloc(sizeof(double) * H);
    double* tabs = (double*)malloc(sizeof(double) * H);
#pragma omp for schedule(dynamic, 1)
    for (int t = 0; t < T; ++t) {
      for (int k = 0; k < H; ++k) xd[k] = (double)rnbo_bf16_to_f32(d->x[(size_t)t * H + k]);
      for (int n = 0; n < H; ++n) acc[n] = tabs[n] = 0.0;
      for (int s = 0; s < K; ++s) {
        const size_t e = (size_t)inds[(size_t)t * K + s];
        expert_bound(H, I, bits, G, d->gu_w + e * gu_we, d->gu_s + e * gu_se, d->gu_b + e * gu_se,
                     d->dn_w + e * dn_we, d->dn_s + e * dn_se, d->dn_b + e * dn_se, xd, h, dh, y, eb);
        if (per_slot) {
          for (int n = 0; n < H; ++n) bound[((size_t)t * K + s) * H + n] = (float)eb[n];
          continue;
        }
        const double wgt = fabs((double)scores[(size_t)t * K + s]);
        for (int n = 0; n < H; ++n) {
          acc[n] += wgt * eb[n] + g16 * wgt * fabs(y[n]);
          tabs[n] += wgt * fabs(y[n]);
        }
      }
      if (per_slot) continue;
      if (sg && d->sgu_w) {
        expert_bound(H, I, bits, G, d->sgu_w, d->sgu_s, d->sgu_b, d->sdn_w, d->sdn_s, d->sdn_b, xd, h, dh, y, eb);
        double a = 0.0;
        for (int k = 0; k < H; ++k) a += fabs(xd[k] * router_weight(d, d->E, k));
        const double g = fabs((double)sg[t]);
        const double dsg = g * (1.0 - g) * gH * a + 2.0 * u * g;
        for (int n = 0; n < H; ++n) {
          acc[n] += g * eb[n] + dsg * fabs(y[n]);
          tabs[n] += g * fabs(y[n]);
        }
      }
      for (int n = 0; n < H; ++n) bound[(size_t)t * H + n] = (float)(acc[n] + g9 * tabs[n]);
    }
    free(xd);
    free(h);
    free(dh);
    free(y);
    free(eb);
    free(acc);
    free(tabs);
  }
  return RNBO_OK;
}

/* Whole block: out[t] = sum_s score[t,s] * y[t,s] + sigmoid(x.w_sg) * shared(x). */
int rnbo_moe_block(const rnbo_block* d, float* out, int32_t* inds, float* scores,
                   float* logits, int nthreads) {
  if (!block_valid(d)) return RNBO_EINVAL;
  const int T = d->T, H = d->H, K = d->k;
  float* sg = (float*)malloc(sizeof(float) * (T > 0 ? T : 1));
  float* y = (float*)malloc(sizeof(float) * ((size_t)T * K * H + 1));
  float* ys = (float*)malloc(sizeof(float) * ((size_t)T * H + 1));
  int rc = rnbo_router(d, logits, inds, scores, sg, nthreads);
  if (rc == RNBO_OK) rc = rnbo_switchglu(d, inds, y, nthreads);
  if (rc == RNBO_OK && d->sgu_w) rc = rnbo_shared_expert(d, ys, nthreads);
  if (rc == RNBO_OK) {
    for (int t = 0; t < T; ++t)
      for (int n = 0; n < H; ++n) {
        float acc = 0.0f;
        for (int s = 0; s < K; ++s) acc += scores[(size_t)t * K + s] * y[((size_t)t * K + s) * H + n];
        if (d->sgu_w) acc += sg[t] * ys[(size_t)t * H + n];
        out[(size_t)t * H + n] = acc;
      }
  }
  free(sg);
  free(y);
  free(ys);
  return rc;
}

/* --------------------------- reference synthetic generators (KATs) */

typedef struct {
  uint64_t state;
} rnbo_xorshift;

static uint32_t xs_next(rnbo_xorshift* r) {
  r->state ^= r->state << 13;
  r->state ^= r->state >> 7;
  r->state ^= r->state << 17;
  return (uint32_t)(r->state >> 32);
}

/* lo + unit * (hi - lo), contracted to one fused multiply-add as the
 * reference's arm64 clang build does. */
static float xs_uniform(rnbo_xorshift* r, float lo, float hi) {
  const double unit = (double)xs_next(r) / 4294967295.0;
  return fmaf((float)unit, hi - lo, lo);
}

/* Codes are drawn one per byte, so for 4-bit data only the low nibble of
 * every byte is populated (fused_moe_probe.mm:620-625). */
static uint32_t xs_word(rnbo_xorshift* r, int bits) {
  const uint32_t mask = bits == 4 ? 0x0Fu : 0xFFu;
  uint32_t v = 0;
  for (int byte = 0; byte < 4; ++byte) v |= (xs_next(r) & mask) << (byte * 8);
  return v;
}

static float kat_scale_lo(int bits) { return bits == 4 ? 0.002f : 0.00005f; }
static float kat_scale_hi(int bits) { return bits == 4 ? 0.008f : 0.00015f; }

/* quantized_qmv_probe.mm:365-403 data: x[K], then (scale,bias) for every
 * (row,group) of the bank, then every packed word of the bank. */
int rnbo_kat_qmv_data(int bits, size_t K, size_t group, size_t bank_rows, uint32_t* w,
                      uint16_t* s, uint16_t* b, uint16_t* x) {
  if ((bits != 4 && bits != 8) || !group || K % group) return RNBO_EINVAL;
  rnbo_xorshift r = {bits == 4 ? 0x4A17C0DEull : 0x8A17C0DEull};
  for (size_t i = 0; i < K; ++i) x[i] = rnbo_f32_to_bf16(xs_uniform(&r, -1.0f, 1.0f));
  const size_t params = bank_rows * (K / group);
  for (size_t p = 0; p < params; ++p) {
    s[p] = rnbo_f32_to_bf16(xs_uniform(&r, kat_scale_lo(bits), kat_scale_hi(bits)));
    b[p] = rnbo_f32_to_bf16(xs_uniform(&r, -0.0005f, 0.0005f));
  }
  const size_t words = bank_rows * (K * bits / 32);
  for (size_t i = 0; i < words; ++i) w[i] = xs_word(&r, bits);
  return RNBO_OK;
}

/* Reference QMV outputs: active row r maps to bank row
 * sel[r / rows_per_expert] * rows_per_expert + r % rows_per_expert
 * (quantized_qmv_probe.mm:352-363); nsel == 0 means the identity map. */
int rnbo_kat_qmv_expected(int bits, size_t K, size_t group, size_t out_rows,
                          size_t rows_per_expert, const uint32_t* sel, size_t nsel,
                          const uint32_t* w, const uint16_t* s, const uint16_t* b,
                          const uint16_t* x, float* y, double* checksum) {
  float* xf = (float*)malloc(sizeof(float) * K);
  for (size_t i = 0; i < K; ++i) xf[i] = rnbo_bf16_to_f32(x[i]);
  const size_t ws = K * bits / 32, ss = K / group;
  double sum = 0.0;
  for (size_t r = 0; r < out_rows; ++r) {
    size_t row = r;
    if (nsel) row = (size_t)sel[r / rows_per_expert] * rows_per_expert + r % rows_per_expert;
    y[r] = affine_dot_scale_inside(w + row * ws, s + row * ss, b + row * ss, xf, (int)K, bits,
                                   (int)group);
    sum += y[r];
  }
  free(xf);
  if (checksum) *checksum = sum;
  return RNBO_OK;
}

/* quantized_qmm_probe.mm:245-305: x[tokens,K], then per output row its
 * (scale,bias) pairs followed by its packed words. */
int rnbo_kat_qmm_data(int bits, size_t tokens, size_t outputs, size_t K, size_t group,
                      uint32_t* w, uint16_t* s, uint16_t* b, uint16_t* x) {
  if ((bits != 4 && bits != 8) || !group || K % group) return RNBO_EINVAL;
  rnbo_xorshift r = {bits == 4 ? 0x4D4D4D01ull : 0x4D4D4D02ull};
  for (size_t i = 0; i < tokens * K; ++i) x[i] = rnbo_f32_to_bf16(xs_uniform(&r, -1.0f, 1.0f));
  const size_t groups = K / group, ws = K * bits / 32;
  for (size_t row = 0; row < outputs; ++row) {
    for (size_t g = 0; g < groups; ++g) {
      s[row * groups + g] = rnbo_f32_to_bf16(xs_uniform(&r, kat_scale_lo(bits), kat_scale_hi(bits)));
      b[row * groups + g] = rnbo_f32_to_bf16(xs_uniform(&r, -0.0005f, 0.0005f));
    }
    for (size_t p = 0; p < ws; ++p) w[row * ws + p] = xs_word(&r, bits);
  }
  return RNBO_OK;
}

int rnbo_kat_qmm_expected(int bits, size_t tokens, size_t outputs, size_t K, size_t group,
                          const uint32_t* w, const uint16_t* s, const uint16_t* b,
                          const uint16_t* x, float* y, double* checksum, int nthreads) {
  float* xf = (float*)malloc(sizeof(float) * tokens * K);
  for (size_t i = 0; i < tokens * K; ++i) xf[i] = rnbo_bf16_to_f32(x[i]);
  const size_t ws = K * bits / 32, ss = K / group;
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(static)
  for (long long t = 0; t < (long long)tokens; ++t)
    for (size_t o = 0; o < outputs; ++o)
      y[t * outputs + o] = rnbo_affine_dot(w + o * ws, s + o * ss, b + o * ss, xf + t * K,
                                           (int)K, bits, (int)group);
  double sum = 0.0;
  for (size_t i = 0; i < tokens * outputs; ++i) sum += y[i];
  free(xf);
  if (checksum) *checksum = sum;
  return RNBO_OK;
}

/* fused_moe_probe.mm:449-492: x[2048], the gate/up bank (per row: pairs then
 * words), the down bank (same), then 8 router weights U(0.5,1.5) normalised. */
int rnbo_kat_two_stage_data(int bits, size_t experts, size_t H, size_t I, size_t group,
                            size_t k, uint16_t* x, uint32_t* guw, uint16_t* gus, uint16_t* gub,
                            uint32_t* dnw, uint16_t* dns, uint16_t* dnb, float* route_w) {
  if ((bits != 4 && bits != 8) || !group || H % group || I % group) return RNBO_EINVAL;
  rnbo_xorshift r = {bits == 4 ? 0xF05EEDB1ull : 0xF05EEDB2ull};
  for (size_t i = 0; i < H; ++i) x[i] = rnbo_f32_to_bf16(xs_uniform(&r, -1.0f, 1.0f));
  const size_t banks[2][2] = {{experts * 2 * I, H}, {experts * H, I}};
  uint32_t* ws[2] = {guw, dnw};
  uint16_t* ss[2] = {gus, dns};
  uint16_t* bs[2] = {gub, dnb};
  for (int bank = 0; bank < 2; ++bank) {
    const size_t rows = banks[bank][0], red = banks[bank][1];
    const size_t groups = red / group, wstride = red * bits / 32;
    for (size_t row = 0; row < rows; ++row) {
      for (size_t g = 0; g < groups; ++g) {
        ss[bank][row * groups + g] =
            rnbo_f32_to_bf16(xs_uniform(&r, kat_scale_lo(bits), kat_scale_hi(bits)));
        bs[bank][row * groups + g] = rnbo_f32_to_bf16(xs_uniform(&r, -0.0005f, 0.0005f));
      }
      for (size_t p = 0; p < wstride; ++p) ws[bank][row * wstride + p] = xs_word(&r, bits);
    }
  }
  float total = 0.0f;
  for (size_t i = 0; i < k; ++i) {
    route_w[i] = xs_uniform(&r, 0.5f, 1.5f);
    total += route_w[i];
  }
  for (size_t i = 0; i < k; ++i) route_w[i] /= total;
  return RNBO_OK;
}

/* expected_direct_ of fused_moe_probe.mm:494-537: out = sum_s w_s * down_e(h_e). */
int rnbo_kat_two_stage_expected(int bits, size_t H, size_t I, size_t group, size_t k,
                                const uint32_t* sel, const uint16_t* x, const uint32_t* guw,
                                const uint16_t* gus, const uint16_t* gub, const uint32_t* dnw,
                                const uint16_t* dns, const uint16_t* dnb, const float* route_w,
                                float* out, double* checksum) {
  float* xf = (float*)malloc(sizeof(float) * H);
  float* hb = (float*)malloc(sizeof(float) * I);
  float* y = (float*)malloc(sizeof(float) * H);
  for (size_t i = 0; i < H; ++i) xf[i] = rnbo_bf16_to_f32(x[i]);
  for (size_t n = 0; n < H; ++n) out[n] = 0.0f;
  const size_t gu_we = 2 * I * H * bits / 32, gu_se = 2 * I * H / group;
  const size_t dn_we = H * I * bits / 32, dn_se = H * I / group;
  for (size_t s = 0; s < k; ++s) {
    const size_t e = sel[s];
    expert_forward((int)H, (int)I, bits, (int)group, guw + e * gu_we, gus + e * gu_se,
                   gub + e * gu_se, dnw + e * dn_we, dns + e * dn_se, dnb + e * dn_se, xf, hb, y);
    for (size_t n = 0; n < H; ++n) out[n] += route_w[s] * y[n];
  }
  double sum = 0.0;
  for (size_t n = 0; n < H; ++n) sum += out[n];
  free(xf);
  free(hb);
  free(y);
  if (checksum) *checksum = sum;
  return RNBO_OK;
}
