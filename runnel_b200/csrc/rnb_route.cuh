// rnb_route.cuh -- exact bf16 router logits and top-k selection.
//
// A router logit is defined as the correctly rounded bf16 of the exact dot
// product x . w_e (bf16 inputs; MLX's Linear returns bf16).  The kernels
// compute it fast on the tensor cores with fp32 accumulation, which is exact
// in every product but rounds partial sums, so the fp32 value L may sit on
// the other side of a bf16 rounding midpoint than the exact one.  Each fp32
// logit is therefore published as an interval of bf16 candidates
//     lo = bf16(L - B),  hi = bf16(L + B),  B = rel |x|_2 |w_e|_2 + 2^-21 |L|
// (|x|_2 |w_e|_2 >= sum |x_i w_i| by Cauchy-Schwarz; rel allows two fp32
// ulps of error per accumulation step at the largest possible partial sum,
// see kRouteRel*).  lo == hi certifies the rounding.  The
// selection warp recomputes, in fp64 from the bf16 inputs, exactly those
// uncertain logits that could still reach the top k; every selected logit
// is then the correctly rounded value, and so is the selection.
#pragma once

#include "rnb_common.cuh"

namespace rnb {

// Unique selection key: bf16 value order in the high half (-0 counts as +0,
// as a float comparison does), then the lower expert index.
__device__ __forceinline__ uint32_t route_key(uint16_t bits, int e) {
  if ((bits & 0x7FFFu) == 0) bits = 0;
  const uint32_t ord = (bits & 0x8000u) ? (~static_cast<uint32_t>(bits) & 0xFFFFu) : (static_cast<uint32_t>(bits) | 0x8000u);
  return (ord << 16) | (0xFFFFu - static_cast<uint32_t>(e));
}
__device__ __forceinline__ float route_key_value(uint32_t key) {
  const uint32_t ord = key >> 16;
  const uint32_t bits = (ord & 0x8000u) ? (ord & 0x7FFFu) : (~ord & 0xFFFFu);
  return __uint_as_float(bits << 16);
}
__device__ __forceinline__ int route_key_expert(uint32_t key) { return static_cast<int>(0xFFFFu - (key & 0xFFFFu)); }

// Round a double to bf16 (nearest, ties to even) in one step.  Magnitudes
// below 2^-126 are rounded through fp32.
__device__ __forceinline__ uint16_t f64_to_bf16_bits(double v) {
  if (v != v) return 0x7FC0u;
  if (fabs(v) < 0x1p-126) return __bfloat16_as_ushort(__float2bfloat16_rn(__double2float_rn(v)));
  const uint64_t b = static_cast<uint64_t>(__double_as_longlong(v));
  const uint32_t sign = static_cast<uint32_t>(b >> 63);
  int e = static_cast<int>((b >> 52) & 0x7FF);
  const uint64_t m = b & ((1ull << 52) - 1);
  uint32_t q = static_cast<uint32_t>(m >> 45);
  const uint64_t rem = m & ((1ull << 45) - 1), half = 1ull << 44;
  if (rem > half || (rem == half && (q & 1u))) {
    if (++q == 128) {
      q = 0;
      ++e;
    }
  }
  const int fe = e - 1023 + 127;
  if (fe >= 255) return static_cast<uint16_t>((sign << 15) | 0x7F80u);
  return static_cast<uint16_t>((sign << 15) | (static_cast<uint32_t>(fe) << 7) | q);
}

// Error allowances (multiples of sum |x_i w_i|): two fp32 ulps per MMA step
// and per cross-warp add.  Decode routers accumulate 8 k16 steps per warp
// and add 16 warp partials.  The prefill router (tcgen05) accumulates four K
// quarters of 32 steps each in fp32 and adds the quarters in fp64 (the fp64
// sum's rounding to fp32 is the 2^-21 |L| term of the bound).
constexpr float kRouteRelDecode = 0x1p-18f;
constexpr float kRouteRelTc = 0x1p-18f;
// 8-bit affine routers on the tensor cores: each dequantised weight w
// (fp32 s*code + b, one rounding) runs as two bf16 parts hi + lo, which leave
// a residual of at most 2^-17.9 |w|; the MMA steps double (hi and lo), and
// the norms come from hi (|w| <= (1 + 2^-8) |hi|).  2^-16 covers the sum.
constexpr float kRouteRelQ8 = 0x1p-16f;

// Packed candidate interval (lo | hi << 16) of an fp32 logit L with error
// allowance rel * sum |x_i w_i|.  Norms of the token (xn2 = sum x^2, xinf =
// max |x|) and of the router row (wn2 = sum w^2, wn1 = sum |w|), fp32: the
// bound uses |x|_2 |w|_2 when the squares cannot have underflowed, else
// |x|_inf |w|_1 (both >= sum |x_i w_i|; an all-zero token gets B = 0, its
// logits are exact zeros).
__device__ __forceinline__ uint32_t route_interval(float L, float xn2, float xinf, float wn2, float wn1, float rel) {
  float nb = xinf * wn1;
  if (xn2 >= 0x1p-100f && wn2 >= 0x1p-100f) nb = fminf(nb, sqrtf(xn2) * sqrtf(wn2));
  const float B = rel * 1.001f * nb + 0x1p-21f * fabsf(L);
  if (!(B <= 3.0e38f) || L != L) return 0xFF80u | (0x7F80u << 16);  // (-inf, +inf): recompute
  const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(L - B));
  const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(L + B));
  return lo | (hi << 16);
}

// Packed candidate interval of a logit accumulated in fp64 from bf16 inputs:
// every product is exact and each of the at most ~12 roundings of a partial
// sum (per-lane chain, shuffle tree, cross-warp tree) errs by at most 2^-53 of
// sum |x_i w_i|, so B = 2^-40 * (norm bound) covers the error with a wide
// margin and the interval is nearly always a single bf16 value (no fp64
// recompute needed).  Norms as for route_interval.
__device__ __forceinline__ uint32_t route_interval_f64(double L, float xn2, float xinf, float wn2, float wn1) {
  float nb = xinf * wn1;
  if (xn2 >= 0x1p-100f && wn2 >= 0x1p-100f) nb = fminf(nb, sqrtf(xn2) * sqrtf(wn2));
  const double B = 0x1p-40 * 1.001 * static_cast<double>(nb);
  if (!(B <= 3.0e38) || L != L) return 0xFF80u | (0x7F80u << 16);  // (-inf, +inf): recompute
  const uint32_t lo = f64_to_bf16_bits(L - B);
  const uint32_t hi = f64_to_bf16_bits(L + B);
  return lo | (hi << 16);
}

// Per-lane partial norms of a router tile in the mma.sync m16n8k16 layout:
// lane 4g+c sees, per 32-wide chunk, 8 activations of token g and 8 weights
// of each of the tile rows g and g+8.
struct RouterNorms {
  float xs2 = 0.f, xmx = 0.f, a2 = 0.f, a1 = 0.f, b2 = 0.f, b1 = 0.f;
  __device__ __forceinline__ void add(const uint4 x, const uint4 wa, const uint4 wb) {
    const uint32_t xv[4] = {x.x, x.y, x.z, x.w}, av[4] = {wa.x, wa.y, wa.z, wa.w}, bv[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float xf = __uint_as_float(h ? (xv[j] & 0xFFFF0000u) : (xv[j] << 16));
        const float af = __uint_as_float(h ? (av[j] & 0xFFFF0000u) : (av[j] << 16));
        const float bf = __uint_as_float(h ? (bv[j] & 0xFFFF0000u) : (bv[j] << 16));
        xs2 = fmaf(xf, xf, xs2);
        xmx = fmaxf(xmx, fabsf(xf));
        a2 = fmaf(af, af, a2);
        a1 += fabsf(af);
        b2 = fmaf(bf, bf, b2);
        b1 += fabsf(bf);
      }
    }
  }
  // sum over the four lanes of one g
  __device__ __forceinline__ void reduce_quad() {
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      xs2 += __shfl_xor_sync(0xffffffffu, xs2, o);
      xmx = fmaxf(xmx, __shfl_xor_sync(0xffffffffu, xmx, o));
      a2 += __shfl_xor_sync(0xffffffffu, a2, o);
      a1 += __shfl_xor_sync(0xffffffffu, a1, o);
      b2 += __shfl_xor_sync(0xffffffffu, b2, o);
      b1 += __shfl_xor_sync(0xffffffffu, b1, o);
    }
  }
  // one warp's 48 partials: token g at [g], [8+g]; row g at [16+g], [32+g]; row g+8 at [24+g], [40+g]
  __device__ __forceinline__ void store(float* dst, int g) const {
    dst[g] = xs2;
    dst[8 + g] = xmx;
    dst[16 + g] = a2;
    dst[24 + g] = b2;
    dst[32 + g] = a1;
    dst[40 + g] = b1;
  }
};

// Interval of tile row r (0..15), token n (0..7) from nw warps' partials.
__device__ __forceinline__ uint32_t router_interval_from(const float* part, int nw, int r, int n, float L,
                                                         float rel = kRouteRelDecode) {
  float xn2 = 0.f, xinf = 0.f, wn2 = 0.f, wn1 = 0.f;
  for (int w = 0; w < nw; ++w) {
    const float* q = part + w * 48;
    xn2 += q[n];
    xinf = fmaxf(xinf, q[8 + n]);
    wn2 += q[16 + r];  // rows 8..15 continue into [24, 32)
    wn1 += q[32 + r];
  }
  return route_interval(L, xn2, xinf, wn2, wn1, rel);
}

// fp64 dot product of two bf16 rows of length H (H % 8 == 0, 16-byte
// aligned), warp-cooperative; every lane returns the sum.  bf16 products are
// exact in fp64 and the fp64 sum of up to 2^11 of them errs by < 2^-42 of
// sum |x_i w_i|.  All of a 2048-wide chunk's loads are issued before any
// arithmetic (one memory round trip per chunk).
static __device__ __noinline__ double warp_dot_f64(const uint16_t* x, const uint16_t* w, int H, int lane) {
  double a0 = 0.0, a1 = 0.0;
  for (int k0 = 0; k0 < H; k0 += 2048) {
    uint4 xv[8], wv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j * 256 + lane * 8;
      xv[j] = k < H ? *reinterpret_cast<const uint4*>(x + k) : make_uint4(0, 0, 0, 0);  // x: global or shared
      wv[j] = k < H ? __ldg(reinterpret_cast<const uint4*>(w + k)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t xs[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w}, ws[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a0 = fma(static_cast<double>(__uint_as_float(xs[i] << 16)), static_cast<double>(__uint_as_float(ws[i] << 16)), a0);
        a1 = fma(static_cast<double>(__uint_as_float(xs[i] & 0xFFFF0000u)),
                 static_cast<double>(__uint_as_float(ws[i] & 0xFFFF0000u)), a1);
      }
    }
  }
  double s = a0 + a1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Router rows for the fp64 recompute: bf16 rows w [rows][H] (q == nullptr),
// or 8-bit affine rows: codes q [rows][H/4], bf16 scales s and biases b
// [rows][H/64]; row E_total is the shared gate (sq / ss / sb, or sw).
struct RouterSrc {
  const uint16_t* w;
  const uint32_t* q;
  const uint16_t* s;
  const uint16_t* b;
};

// fp64 dot product of a bf16 token row with router row e of an 8-bit affine
// router (H % 2048 == 0 or smaller H a multiple of 256), warp-cooperative;
// every lane returns the sum.  The dequantised weight s * code + b (a bf16
// times an 8-bit integer plus a bf16) is exact in fp64, and so is each
// product with a bf16 activation.
static __device__ __noinline__ double warp_dot_q8_f64(const uint16_t* x, const uint32_t* q, const uint16_t* s,
                                                       const uint16_t* b, int H, int lane) {
  double a0 = 0.0, a1 = 0.0;
  for (int k0 = 0; k0 < H; k0 += 2048) {
    uint4 xv[8];
    uint2 qv[8];
    uint32_t sb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j * 256 + lane * 8;
      const bool in = k < H;
      xv[j] = in ? *reinterpret_cast<const uint4*>(x + k) : make_uint4(0, 0, 0, 0);  // x: global or shared
      qv[j] = in ? __ldg(reinterpret_cast<const uint2*>(q + k / 4)) : make_uint2(0, 0);
      sb[j] = in ? (static_cast<uint32_t>(__ldg(s + k / 64)) | (static_cast<uint32_t>(__ldg(b + k / 64)) << 16)) : 0u;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const double sc = static_cast<double>(__uint_as_float(sb[j] << 16));
      const double bi = static_cast<double>(__uint_as_float(sb[j] & 0xFFFF0000u));
      const uint32_t xs[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t word = i < 2 ? qv[j].x : qv[j].y;
        const int sh = 16 * (i & 1);
        const double w0 = fma(sc, static_cast<double>((word >> sh) & 0xFFu), bi);
        const double w1 = fma(sc, static_cast<double>((word >> (sh + 8)) & 0xFFu), bi);
        a0 = fma(static_cast<double>(__uint_as_float(xs[i] << 16)), w0, a0);
        a1 = fma(static_cast<double>(__uint_as_float(xs[i] & 0xFFFF0000u)), w1, a1);
      }
    }
  }
  double r = a0 + a1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

__device__ __forceinline__ double warp_dot_router_f64(const uint16_t* x, const RouterSrc& rs, int e, int H, int lane) {
  if (rs.q)
    return warp_dot_q8_f64(x, rs.q + static_cast<size_t>(e) * (H / 4), rs.s + static_cast<size_t>(e) * (H / 64),
                           rs.b + static_cast<size_t>(e) * (H / 64), H, lane);
  return warp_dot_f64(x, rs.w + static_cast<size_t>(e) * H, H, lane);
}

// Compare-exchange for a descending order: a keeps the larger key.
__device__ __forceinline__ void cas_desc(uint32_t& a, uint32_t& b) {
  const uint32_t hi = max(a, b), lo = min(a, b);
  a = hi;
  b = lo;
}

// The K largest (K <= 16) of the warp's keys (8 per lane, unique, 0 =
// empty): lane s < K receives the s-th in `mine`; returns the K-th.  Each
// lane first sorts its 8 keys (Batcher's 19-comparator network, no
// cross-lane traffic); then every pick is one redux over the lanes' heads,
// and the lane that owned the winner shifts its list by one (branch-free).
__device__ __forceinline__ uint32_t warp_select_k(const uint32_t (&keys)[8], int K, int lane, uint32_t& mine) {
  uint32_t a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = keys[i];
  cas_desc(a[0], a[1]); cas_desc(a[2], a[3]); cas_desc(a[4], a[5]); cas_desc(a[6], a[7]);
  cas_desc(a[0], a[2]); cas_desc(a[1], a[3]); cas_desc(a[4], a[6]); cas_desc(a[5], a[7]);
  cas_desc(a[1], a[2]); cas_desc(a[5], a[6]);
  cas_desc(a[0], a[4]); cas_desc(a[1], a[5]); cas_desc(a[2], a[6]); cas_desc(a[3], a[7]);
  cas_desc(a[2], a[4]); cas_desc(a[3], a[5]);
  cas_desc(a[1], a[2]); cas_desc(a[3], a[4]); cas_desc(a[5], a[6]);
  uint32_t w = 0;
  mine = 0;
#pragma unroll
  for (int slot = 0; slot < 16; ++slot) {
    if (slot < K) {  // K is warp-uniform
      w = __reduce_max_sync(0xffffffffu, a[0]);
      mine = lane == slot ? w : mine;
      const bool hit = a[0] == w;  // keys are unique: one lane at most
#pragma unroll
      for (int i = 0; i < 7; ++i) a[i] = hit ? a[i + 1] : a[i];
      a[7] = hit ? 0u : a[7];
    }
  }
  return w;
}

// One token's routing, by one full warp.  ivl[e] (e < Et <= 256) holds the
// packed candidate interval of expert e's logit.  Lane s < K returns the
// s-th selected expert (descending logit, ties to the lower index) in *e_out
// and its weight in *score_out: exp(l_s - l_max) over the sum of that term
// for the K selected, which equals the softmax over all Et logits gathered
// at the selection and renormalised (the full denominator cancels; only the
// fp32 rounding differs).  The selection runs on the lower candidates; the
// uncertain logits that can still reach the top k are then resolved in fp64
// and, if there were any, the selection runs again.  With exact_all every
// uncertain logit is resolved and, if logits_row is non-null, all Et bf16
// logits are written there as fp32.  Returns the number of logits resolved.
// The uncertain candidates flagged in `need` (bit i: expert lane + 32 i) are
// resolved in fp64 and the selection runs again.  Out of line and not
// unrolled: it runs for a minority of tokens, and the common path stays
// small (its instructions are fetched once per token by the decode kernel).
static __device__ __noinline__ int route_resolve(uint32_t (&klo)[8], uint32_t need, int K, const uint16_t* xrow,
                                                 const RouterSrc rs, int H, int lane, uint32_t& mine) {
  int n = 0;
#pragma unroll 1
  for (int i = 0; i < 8; ++i) {
    uint32_t m = __ballot_sync(0xffffffffu, (need >> i) & 1u);
    n += __popc(m);
    while (m) {
      const int src = __ffs(m) - 1;
      m &= m - 1;
      const int e = src + 32 * i;
      const double d = warp_dot_router_f64(xrow, rs, e, H, lane);
      if (lane == src) klo[i] = route_key(f64_to_bf16_bits(d), e);
    }
  }
  if (n) warp_select_k(klo, K, lane, mine);
  return n;
}

__device__ __forceinline__ int warp_route_token_body(const uint32_t* ivl, int Et, int K, const uint16_t* xrow,
                                                     const RouterSrc rs, int H, int lane, bool exact_all,
                                                     float* logits_row, int* e_out, float* score_out) {
  uint32_t klo[8], vhi = 0;  // vhi bit i: lo != hi for expert lane + 32 i
  uint16_t hib[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    klo[i] = 0;
    hib[i] = 0;
    if (e < Et) {
      const uint32_t v = ivl[e];
      klo[i] = route_key(static_cast<uint16_t>(v & 0xFFFFu), e);
      hib[i] = static_cast<uint16_t>(v >> 16);
      if ((v & 0xFFFFu) != (v >> 16)) vhi |= 1u << i;
    }
  }
  uint32_t mine;
  const uint32_t theta = warp_select_k(klo, K, lane, mine);  // the K-th largest lower key
  // an expert whose upper key is below theta is beaten for certain by K others
  uint32_t need = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (((vhi >> i) & 1u) && (exact_all || route_key(hib[i], lane + 32 * i) >= theta)) need |= 1u << i;
  int n_exact = 0;
  if (__any_sync(0xffffffffu, need != 0)) n_exact = route_resolve(klo, need, K, xrow, rs, H, lane, mine);
  if (logits_row) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane + 32 * i < Et) logits_row[lane + 32 * i] = route_key_value(klo[i]);
  }
  const float mx = route_key_value(__shfl_sync(0xffffffffu, mine, 0));
  const float pw = lane < K ? expf(route_key_value(mine) - mx) : 0.f;
  // the sum of the K terms (lanes < K), by a butterfly over as few lanes as K needs
  float selsum = pw;
  selsum += __shfl_xor_sync(0xffffffffu, selsum, 1);
  selsum += __shfl_xor_sync(0xffffffffu, selsum, 2);
  selsum += __shfl_xor_sync(0xffffffffu, selsum, 4);
  if (K > 8) {  // warp-uniform
    selsum += __shfl_xor_sync(0xffffffffu, selsum, 8);
    selsum += __shfl_xor_sync(0xffffffffu, selsum, 16);
  }
  *e_out = route_key_expert(mine);
  *score_out = pw / selsum;
  return n_exact;
}

// Out-of-line form for kernels where code size matters less than one copy.
static __device__ __noinline__ int warp_route_token(const uint32_t* ivl, int Et, int K, const uint16_t* xrow,
                                                     const RouterSrc rs, int H, int lane, bool exact_all,
                                                     float* logits_row, int* e_out, float* score_out) {
  return warp_route_token_body(ivl, Et, K, xrow, rs, H, lane, exact_all, logits_row, e_out, score_out);
}

}  // namespace rnb
