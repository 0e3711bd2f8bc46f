// rnb_decode.cu -- sparse-MoE block for small token counts (decode, T <= 64).
//
// Three kernels per call, chained with programmatic dependent launch so each
// one is resident (and streaming its weights) before its producer finishes:
//
//   k_route    router logits on the tensor cores (bf16 mma; one CTA per 16
//              router rows, hidden dimension split over 16 warps and reduced
//              in shared memory), activation prep (per-token power-of-two scale
//              into fp16 range, per-group sums, MMA pair order), and -- in the
//              last CTA to arrive -- top-k, softmax weights, shared-expert gate,
//              and the per-expert token records (a counting sort).
//   k_gateup   one CTA per (8 channels, active expert): 16 rows (8 up + 8
//              gate) x the full hidden size, split over H/512 warps, dequantised
//              in registers from 16-byte streaming loads into fp16 mma; SwiGLU
//              in the epilogue.  Expert slot 0 of the grid is the shared expert.
//   k_down     one CTA per (16 output rows, active expert): down projection
//              from the fp32 SwiGLU activations, then -- in the last CTA to
//              finish a row tile -- the weighted combine with the sigmoid-gated
//              shared expert, written as bf16.
//
// Reference semantics: src/runnel/mlx.py:57-82 (packed gate/up, SwiGLU, down),
// bench/mlx_lm_adapter.py:82-94 (shared expert), mlx-lm Qwen3.5 block router.
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <unordered_map>

#include "rnb_common.cuh"
#include "rnb_route.cuh"
#include "rnb_umma.cuh"
#include "rnb_internal.h"
#include "rnb_moe.h"

namespace rnb {

constexpr int kMaxDecodeT = 64;
constexpr int kMaxEpRanks = 8;
constexpr int kEpMaxT = 64;  // tokens per exchange (receive buffers [2][world][kEpMaxT][H])
constexpr int kMaxE = 512;
constexpr int kMaxK = 16;
constexpr int kRecWords = 12;
constexpr int kRouterWarps = 16;  // hidden-dimension split of one router tile
constexpr int kGateUpGroupsPerWarp = 8;
constexpr int kDownGroupsPerWarp = 4;

enum Mode { kModeBlock = 0, kModeSwitchGLU = 1, kModeRouter = 2 };

struct Ws {
  uint32_t* xperm;  // [T][G][4][8] fp16 pairs (as u32)
  float* xsum;      // [T][G]
  float* xinv;      // [T]
  float* logit;     // [T][E_total + 1] fp32 router logits (last = shared gate)
  uint32_t* inds;   // [T][k]
  float* scores;    // [T][k]
  float* sgate;     // [T]
  uint32_t* nact;   // [1]
  uint32_t* rec;    // [E][kRecWords]: local expert, entry count, entry offset, 0,
                    // then the first 8 entry ids (repeating the first past the count)
  uint32_t* entries;  // [T*k]   entry id = t*(k+1) + slot
  float* h;           // [T][k+1][I]
  float* hmaxp;       // [T][k+1][I/8]: max |h| of each 8-channel gate/up tile
  float* yws;         // [T][k+1][H]
  uint32_t* ctr;      // [1 + H/16]
  uint32_t* status;   // [1]
  uint32_t* seq;      // [0] call sequence word, [1] exit counter (persistent kernel)
  uint2* lw;          // [2][E_total + 1] logit exchange words (persistent kernel)
  uint2* hw;          // [2][k + 1][I] SwiGLU exchange words (persistent kernel)
  uint2* yw;          // [16 (k + 1)][H] split-K partial words (persistent kernel, one token)
};

struct Params {
  int T, H, I, E, E_total, off, k, has_shared, mode, y_f32;
  int ncmax;  // columns (token slots) per MMA tile and staging buffer: min(8, T)
  int router_ctas;
  const uint16_t* x;
  const uint32_t* inds_in;
  const uint16_t* router_w;  // bf16 [E_total][H], or (router_q8) uint32 codes [E_total][H/4]
  const uint16_t* sgate_w;   // bf16 [H], or (router_q8) uint32 codes [H/4]
  int router_q8;             // 8-bit affine router and shared gate
  const uint16_t *router_s, *router_b, *sgate_s, *sgate_b;  // [E_total][H/64], [H/64] bf16
  const uint32_t *gu_w, *dn_w, *sgu_w, *sdn_w;
  const uint16_t *gu_s, *gu_b, *dn_s, *dn_b, *sgu_s, *sgu_b, *sdn_s, *sdn_b;
  void* out;  // bf16 [T][H] (block) or [T][k][H] (switchglu)
  uint32_t* inds_out;
  float* scores_out;
  float* logits_out;
  Ws ws;
  // Shared-expert quarters (128 intermediate channels each) this call
  // computes: all of them, or this rank's share under expert parallelism.
  uint32_t shared_qmask;
  // Expert-parallel exchange (ep_world > 1): every rank's fp32 partial
  // output goes into each rank's receive buffer [2 parities][world]
  // [kEpMaxT][H] as 8-byte words {value, epoch}; the epoch is this rank's
  // sequence word + 1 (device memory, so graph replays advance it; the
  // kernel's last CTA increments it).
  int ep_world, ep_rank;
  uint64_t ep_limit_ns;  // bounded wait for the peers' words
  uint2* ep_recv[kMaxEpRanks];
  uint32_t* ep_seq;  // [0] sequence word, [1] exit counter of k_ep_reduce
  // Fused layer glue (persistent kernel, norm_w non-null): the block input
  // is xn = bf16(rms_norm(r) * norm_w) with r = bf16(resid + y_prev) (y_prev
  // may be null); r goes to resid_out and xn to xn_out.  resid_out must not
  // alias resid or y_prev (other CTAs are still reading them).
  const uint16_t* resid;
  const uint16_t* y_prev;
  const uint16_t* norm_w;
  float norm_eps;
  uint16_t* resid_out;
  uint16_t* xn_out;
};

// The router rows for the exact fp64 recompute of uncertain logits.
__device__ __forceinline__ RouterSrc router_src(const Params& p) {
  RouterSrc r;
  r.w = p.router_q8 ? nullptr : p.router_w;
  r.q = p.router_q8 ? reinterpret_cast<const uint32_t*>(p.router_w) : nullptr;
  r.s = p.router_s;
  r.b = p.router_b;
  return r;
}

// Dequantised 8-bit router weights, exactly: w = s * code + b for the four
// codes of `word` (inputs 4j .. 4j+3 of a 64-group with scale s, bias b).
__device__ __forceinline__ void q8_router_quad(uint32_t word, double s, double b, double (&w)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) w[j] = fma(s, static_cast<double>((word >> (8 * j)) & 0xFFu), b);
}

// The four router weights (as doubles, exact) held by a lane of the
// persistent decode kernel: 4 bf16 in w, or (8-bit router) the word of 4
// codes in w.x and the group's bf16 scale | bias << 16 in w.y.
__device__ __forceinline__ void router_quad(const uint2 w, bool q8, double (&wd)[4]) {
  if (q8) {
    q8_router_quad(w.x, static_cast<double>(__uint_as_float(w.y << 16)),
                   static_cast<double>(__uint_as_float(w.y & 0xFFFF0000u)), wd);
  } else {
    wd[0] = __uint_as_float(w.x << 16);
    wd[1] = __uint_as_float(w.x & 0xFFFF0000u);
    wd[2] = __uint_as_float(w.y << 16);
    wd[3] = __uint_as_float(w.y & 0xFFFF0000u);
  }
}

// Reduce-scatter of four per-lane values over the warp: afterwards lane l
// holds the warp total of value 2 * bit4(l) + bit3(l).  Three shuffles fewer
// per value than four full butterflies; values 2 and 3 are reduced with max
// when max23 is set, every other value with +.
template <typename V>
__device__ __forceinline__ V warp_reduce_scatter4(const V (&v)[4], int lane, bool max23) {
  const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0;
  const bool mx = max23 && b4;  // the values this lane ends up with are 2, 3
  auto op = [&](V a, V b) { return mx ? static_cast<V>(fmax(a, b)) : a + b; };
  V k0 = b4 ? v[2] : v[0], k1 = b4 ? v[3] : v[1];
  const V s0 = b4 ? v[0] : v[2], s1 = b4 ? v[1] : v[3];
  k0 = op(k0, __shfl_xor_sync(0xffffffffu, s0, 16));
  k1 = op(k1, __shfl_xor_sync(0xffffffffu, s1, 16));
  V k = b3 ? k1 : k0;
  k = op(k, __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8));
  k = op(k, __shfl_xor_sync(0xffffffffu, k, 4));
  k = op(k, __shfl_xor_sync(0xffffffffu, k, 2));
  k = op(k, __shfl_xor_sync(0xffffffffu, k, 1));
  return k;
}

// Optional phase timeline (compile with -DRNB_TRACE): thread 0 of each CTA
// records %globaltimer at phase boundaries into the per-slot output area of
// the workspace, which the persistent kernel does not otherwise use.
#ifdef RNB_TRACE
__device__ __forceinline__ void trace_mark(const Params& p, int i) {
  if (threadIdx.x == 0) {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    reinterpret_cast<uint64_t*>(p.ws.yws)[blockIdx.x * 64 + i] = t;
    reinterpret_cast<uint64_t*>(p.ws.yws)[blockIdx.x * 64 + 32 + i] = clock64();
  }
}
__device__ __forceinline__ void trace_value(const Params& p, int i, int v) {
  reinterpret_cast<uint64_t*>(p.ws.yws)[blockIdx.x * 64 + i] = static_cast<uint64_t>(v);
}
#define RNB_TRACE_MARK(p, i) trace_mark(p, i)
#else
#define RNB_TRACE_MARK(p, i) ((void)0)
#endif

// ----------------------------------------------------------- k_route

// Router rows of one CTA: virtual rows [16*tile, 16*tile+16) of the
// (E_total+1)-row matrix whose last row is the shared-expert gate.  Warp w
// owns hidden range [w*H/16, (w+1)*H/16) in 32-wide chunks.
struct RouterRegs {
  uint4 a[4][2];  // up to 4 chunks (H <= 2048) x rows g, g+8: bf16 rows, or (8-bit
                  // router) .x,.y the 8 codes and .z the packed bf16 scale | bias << 16
};

__device__ __forceinline__ const uint16_t* router_row(const Params& p, int r) {
  if (r < p.E_total) return p.router_w + static_cast<size_t>(r) * p.H;
  if (r == p.E_total && p.has_shared) return p.sgate_w;
  return nullptr;
}

__device__ __forceinline__ void router_load(const Params& p, int tile, int warp, int lane, RouterRegs& rr) {
  const int g = lane >> 2, c = lane & 3;
  const int nch = p.H / (kRouterWarps * 32);
  const uint4 z = make_uint4(0, 0, 0, 0);
  if (p.router_q8) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = tile * 16 + g + 8 * h;
      const bool sh = r == p.E_total && p.has_shared;
      const bool ok = r < p.E_total || sh;
      const uint32_t* q = sh ? reinterpret_cast<const uint32_t*>(p.sgate_w)
                             : reinterpret_cast<const uint32_t*>(p.router_w) + static_cast<size_t>(r) * (p.H / 4);
      const uint16_t* sc = sh ? p.sgate_s : p.router_s + static_cast<size_t>(r) * (p.H / 64);
      const uint16_t* bi = sh ? p.sgate_b : p.router_b + static_cast<size_t>(r) * (p.H / 64);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        const int k0 = (warp * nch + ch) * 32 + 8 * c;
        if (ch < nch && ok) {
          const uint2 w = __ldg(reinterpret_cast<const uint2*>(q + k0 / 4));
          rr.a[ch][h] = make_uint4(w.x, w.y, static_cast<uint32_t>(__ldg(sc + k0 / 64)) |
                                                 (static_cast<uint32_t>(__ldg(bi + k0 / 64)) << 16), 0u);
        } else {
          rr.a[ch][h] = z;
        }
      }
    }
    return;
  }
  const uint16_t* pa = router_row(p, tile * 16 + g);
  const uint16_t* pb = router_row(p, tile * 16 + g + 8);
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const int k0 = (warp * nch + ch) * 32 + 8 * c;
    rr.a[ch][0] = (ch < nch && pa) ? ld_stream_v4(pa + k0) : z;
    rr.a[ch][1] = (ch < nch && pb) ? ld_stream_v4(pb + k0) : z;
  }
}

// The 8 dequantised weights of an 8-bit router chunk (RouterRegs form) as
// two bf16 parts, w = hi + lo + r with |r| <= 2^-16.9 |w|: s * code is exact
// in fp32 (a bf16 times an 8-bit integer), adding b rounds once (2^-24), and
// hi = bf16(w32), lo = bf16(w32 - hi) (the difference is exact).
__device__ __forceinline__ void q8_router_split(const uint4 v, uint4& hi, uint4& lo) {
  const float s = __uint_as_float(v.z << 16), b = __uint_as_float(v.z & 0xFFFF0000u);
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t word = j < 2 ? v.x : v.y;
    const int sh = 16 * (j & 1);
    const float w0 = fmaf(s, static_cast<float>((word >> sh) & 0xFFu), b);
    const float w1 = fmaf(s, static_cast<float>((word >> (sh + 8)) & 0xFFu), b);
    const __nv_bfloat162 hh = __floats2bfloat162_rn(w0, w1);
    const float2 hf = __bfloat1622float2(hh);
    const __nv_bfloat162 ll = __floats2bfloat162_rn(w0 - hf.x, w1 - hf.y);
    h[j] = *reinterpret_cast<const uint32_t*>(&hh);
    l[j] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ void router_cta(const Params& p, int tile, const RouterRegs& rr) {
  __shared__ float red[kRouterWarps][16][8];
  __shared__ float s_norm[kRouterWarps][48];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rows = p.E_total + 1;
  const int nch = p.H / (kRouterWarps * 32);
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int t0 = 0; t0 < p.T; t0 += 8) {
    const int tb = t0 + g;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    RouterNorms rn;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      if (ch < nch) {
        const int k0 = (warp * nch + ch) * 32 + 8 * c;
        const uint4 bx = tb < p.T ? __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(tb) * p.H + k0)) : z;
        uint4 a0 = rr.a[ch][0], a1 = rr.a[ch][1];
        if (p.router_q8) {
          uint4 l0, l1;
          q8_router_split(rr.a[ch][0], a0, l0);
          q8_router_split(rr.a[ch][1], a1, l1);
          mma_bf16(d, l0.x, l1.x, l0.y, l1.y, bx.x, bx.y);
          mma_bf16(d, l0.z, l1.z, l0.w, l1.w, bx.z, bx.w);
        }
        mma_bf16(d, a0.x, a1.x, a0.y, a1.y, bx.x, bx.y);
        mma_bf16(d, a0.z, a1.z, a0.w, a1.w, bx.z, bx.w);
        rn.add(bx, a0, a1);
      }
    }
    rn.reduce_quad();
    if (c == 0) rn.store(s_norm[warp], g);
    red[warp][g][2 * c] = d[0];
    red[warp][g][2 * c + 1] = d[1];
    red[warp][g + 8][2 * c] = d[2];
    red[warp][g + 8][2 * c + 1] = d[3];
    __syncthreads();
    if (threadIdx.x < 128) {
      const int r = threadIdx.x & 15, n = threadIdx.x >> 4;
      const int row = tile * 16 + r, t = t0 + n;
      if (row < rows && t < p.T) {
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < kRouterWarps; ++w) acc += red[w][r][n];
        // expert rows: candidate interval of the bf16 logit; last row: fp32 shared-gate logit
        // (8-bit router: twice the MMA steps, the hi + lo split's residual
        // and norms taken from hi -- a wider allowance)
        reinterpret_cast<uint32_t*>(p.ws.logit)[static_cast<size_t>(t) * rows + row] =
            row < p.E_total ? router_interval_from(&s_norm[0][0], kRouterWarps, r, n, acc,
                                                   p.router_q8 ? kRouteRelQ8 : kRouteRelDecode)
                            : __float_as_uint(acc);
      }
    }
    __syncthreads();
  }
}

// One warp: activation prep for token t.  Lane handles groups lane, lane+32..
template <int BITS>
__device__ void xprep_warp(const Params& p, int t, int lane) {
  const int G = p.H / kGroup;
  const uint16_t* xr = p.x + static_cast<size_t>(t) * p.H;
  float mx = 0.f;
  for (int gi = lane; gi < G; gi += 32) {
    const uint4* src = reinterpret_cast<const uint4*>(xr + gi * kGroup);
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const uint4 q = __ldg(src + v);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        mx = fmaxf(mx, fabsf(__uint_as_float(w[j] << 16)));
        mx = fmaxf(mx, fabsf(__uint_as_float(w[j] & 0xFFFF0000u)));
      }
    }
  }
  mx = warp_max(mx);
  float scale, inv;
  fp16_range_scale(mx, scale, inv);
  for (int gi = lane; gi < G; gi += 32) {
    const uint4* src = reinterpret_cast<const uint4*>(xr + gi * kGroup);
    float v[64];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 u = __ldg(src + q);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * q + 2 * j] = __half2float(__float2half_rn(__uint_as_float(w[j] << 16) * scale));
        v[8 * q + 2 * j + 1] = __half2float(__float2half_rn(__uint_as_float(w[j] & 0xFFFF0000u) * scale));
      }
    }
    float xs = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) xs += v[i];
    uint32_t* dst = p.ws.xperm + (static_cast<size_t>(t) * G + gi) * 32;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t pr[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // 4-bit pairs 1 and 3 of a word meet codes times 16 (subnormal form; exact)
        const float f = (BITS == 4 && (i & 1)) ? 0.0625f : 1.0f;
        const __half2 h2 = __floats2half2_rn(v[pair_pos<BITS>(cc, i, 0)] * f, v[pair_pos<BITS>(cc, i, 1)] * f);
        pr[i] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      reinterpret_cast<uint4*>(dst + cc * 8)[0] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
      reinterpret_cast<uint4*>(dst + cc * 8)[1] = make_uint4(pr[4], pr[5], pr[6], pr[7]);
    }
    p.ws.xsum[static_cast<size_t>(t) * G + gi] = xs;
  }
  if (lane == 0) p.ws.xinv[t] = inv;
}

// Last CTA of k_route: routing decisions and per-expert token records.
template <int BITS>
__device__ void route_finalize(const Params& p) {
  __shared__ uint32_t s_cnt[kMaxE], s_base[kMaxE], s_fill[kMaxE];
  __shared__ float s_lg[8][kMaxE + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.k, rows = p.E_total + 1;

  if (p.mode != kModeSwitchGLU) {
    for (int t0 = 0; t0 < p.T; t0 += 8) {
      const int nt = p.T - t0 < 8 ? p.T - t0 : 8;
      for (int q = tid; q < nt * rows; q += blockDim.x)
        reinterpret_cast<uint32_t*>(&s_lg[q / rows][0])[q % rows] =
            __ldcg(reinterpret_cast<const uint32_t*>(p.ws.logit) + static_cast<size_t>(t0) * rows + q);
      __syncthreads();
      if (warp < nt) {
        const int t = t0 + warp;
        int e;
        float sc;
        // a caller asking for the logits gets every one resolved exactly
        warp_route_token(reinterpret_cast<const uint32_t*>(s_lg[warp]), p.E_total, K,
                         p.x + static_cast<size_t>(t) * p.H, router_src(p), p.H, lane, p.logits_out != nullptr,
                         p.logits_out ? p.logits_out + static_cast<size_t>(t) * p.E_total : nullptr, &e, &sc);
        if (lane < K) {
          p.ws.inds[t * K + lane] = static_cast<uint32_t>(e);
          p.ws.scores[t * K + lane] = sc;
          if (p.inds_out) p.inds_out[t * K + lane] = static_cast<uint32_t>(e);
          if (p.scores_out) p.scores_out[t * K + lane] = sc;
        }
        if (lane == 0) p.ws.sgate[t] = p.has_shared ? 1.0f / (1.0f + expf(-s_lg[warp][p.E_total])) : 0.f;
      }
      __syncthreads();
    }
  } else {
    for (int i = tid; i < p.T * K; i += blockDim.x) p.ws.inds[i] = __ldg(p.inds_in + i);
  }
  if (p.mode == kModeRouter) return;
  __syncthreads();

  // Counting sort of (token, slot) entries by local expert.
  for (int i = tid; i < p.E; i += blockDim.x) {
    s_cnt[i] = 0;
    s_fill[i] = 0;
  }
  __syncthreads();
  for (int i = tid; i < p.T * K; i += blockDim.x) {
    const uint32_t e = p.ws.inds[i];
    if (e >= static_cast<uint32_t>(p.E_total)) {
      atomicOr(p.ws.status, RNB_STATUS_BAD_INDEX);
      continue;
    }
    const int le = static_cast<int>(e) - p.off;
    if (le >= 0 && le < p.E) atomicAdd(&s_cnt[le], 1u);
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t running = 0, nact = 0;
    for (int b0 = 0; b0 < p.E; b0 += 32) {
      const int e = b0 + lane;
      const uint32_t v = e < p.E ? s_cnt[e] : 0u;
      uint32_t incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const uint32_t base = running + incl - v;
      const uint32_t flags = __ballot_sync(0xffffffffu, v > 0);
      if (e < p.E) s_base[e] = base;
      if (v > 0) {
        const uint32_t pos = nact + __popc(flags & ((1u << lane) - 1u));
        s_fill[pos] = static_cast<uint32_t>(e);  // active expert list (s_fill reused below)
      }
      running += __shfl_sync(0xffffffffu, incl, 31);
      nact += __popc(flags);
    }
    if (lane == 0) *p.ws.nact = nact;
  }
  __syncthreads();
  const uint32_t nact = *p.ws.nact;  // written by warp 0 of this CTA before the barrier
  // active list -> records' first words; s_fill becomes the scatter cursor
  __shared__ uint32_t s_act[kMaxE];
  for (uint32_t a = tid; a < nact; a += blockDim.x) s_act[a] = s_fill[a];
  __syncthreads();
  for (int i = tid; i < p.E; i += blockDim.x) s_fill[i] = 0;
  __syncthreads();
  for (int i = tid; i < p.T * K; i += blockDim.x) {
    const uint32_t e = p.ws.inds[i];
    if (e >= static_cast<uint32_t>(p.E_total)) continue;
    const int le = static_cast<int>(e) - p.off;
    if (le < 0 || le >= p.E) continue;
    const uint32_t pos = s_base[le] + atomicAdd(&s_fill[le], 1u);
    p.ws.entries[pos] = static_cast<uint32_t>((i / K) * (K + 1) + (i % K));
  }
  __syncthreads();
  for (uint32_t a = tid; a < nact; a += blockDim.x) {
    const uint32_t le = s_act[a], cnt = s_cnt[le], off = s_base[le];
    uint32_t* r = p.ws.rec + a * kRecWords;
    r[0] = le;
    r[1] = cnt;
    r[2] = off;
    r[3] = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) r[4 + i] = p.ws.entries[off + (static_cast<uint32_t>(i) < cnt ? i : 0)];
  }
}

template <int BITS>
__global__ void __launch_bounds__(512) k_route(Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  // Router weights are constant inputs: stream them in before waiting for the
  // previous kernel on the stream (which may still be producing x).
  RouterRegs rr;
  if (b < p.router_ctas) router_load(p, b, warp, lane, rr);
  griddep_wait();
  griddep_launch_dependents();
  if (b < p.router_ctas) {
    router_cta(p, b, rr);
  } else if (p.mode != kModeRouter) {
    const int t = (b - p.router_ctas) * 16 + warp;
    if (t < p.T) xprep_warp<BITS>(p, t, lane);
  }
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.ws.ctr, 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  route_finalize<BITS>(p);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicExch(p.ws.ctr, 0u);
  }
}

// ---------------------------------------------------- quantized tiles

// One warp's weight tile in shared memory: 16 rows (MMA rows g and g+8) x NG
// quantization groups of the warp's K range, codes plus bf16 scales/biases.
// Rows are padded so the per-group fragment reads hit distinct banks: an
// 8-bit group is 64 B read as 16 B per lane (8 lanes = 2 rows per phase,
// rows 64 B apart mod 128); a 4-bit group is 32 B read as 8 B per lane
// (16 lanes = 4 rows per phase, rows 32 B apart mod 128).
template <int BITS, int NG>
struct Tile {
  static constexpr int kRowBytes = NG * 8 * BITS;
  static constexpr int kStride = kRowBytes + (BITS == 8 ? 64 : 32);
  static constexpr int kCodeBytes = 16 * kStride;
  static constexpr int kParBytes = 16 * NG * 2;
  static constexpr int kBytes = kCodeBytes + 2 * kParBytes;
  static constexpr int kPieces = kRowBytes / 16;  // 16-byte copies per row
};

// Issues the asynchronous copies of a tile.  row(i) is the global row index
// of tile row i; g0 the first group of the warp's K range.
template <int BITS, int NG, typename RowOf>
__device__ __forceinline__ void tile_issue(char* sm, const uint32_t* wbase, const uint16_t* sbase,
                                           const uint16_t* bbase, size_t wrow, size_t srow, int g0,
                                           RowOf row, int lane) {
  using TL = Tile<BITS, NG>;
  const size_t kw0 = static_cast<size_t>(g0) * kGroup * BITS / 32;  // first word of the range
#pragma unroll 4
  for (int q = lane; q < 16 * TL::kPieces; q += 32) {
    const int i = q / TL::kPieces, piece = q % TL::kPieces;
    cp_async16(sm + i * TL::kStride + piece * 16, wbase + row(i) * wrow + kw0 + piece * 4);
  }
  if (lane < 16) {
    const size_t r = row(lane);
    char* sd = sm + TL::kCodeBytes + lane * NG * 2;
    char* bd = sd + TL::kParBytes;
    if (NG == 8) {
      cp_async16(sd, sbase + r * srow + g0);
      cp_async16(bd, bbase + r * srow + g0);
    } else {
      cp_async8(sd, sbase + r * srow + g0);
      cp_async8(bd, bbase + r * srow + g0);
    }
  }
}

// acc[0..3] (rows g/g+8 x columns 2c/2c+1) += affine(tile . B) over NG groups.
// bfrag(gi, hi, lo) fills the 8 activation pairs of group gi for this lane's
// column (lo only when SPLIT: a second fp16 operand added in the same
// accumulator); gsum(gi, col) returns the group sum of column col
// (0 -> 2c, 1 -> 2c+1).
template <int BITS, int NG, bool SPLIT, typename BFrag, typename GSum>
__device__ __forceinline__ void tile_mma(const char* sm, int g, int c, BFrag bfrag, GSum gsum,
                                         float (&acc)[4]) {
  using TL = Tile<BITS, NG>;
  const uint16_t* S = reinterpret_cast<const uint16_t*>(sm + TL::kCodeBytes);
  const uint16_t* B = reinterpret_cast<const uint16_t*>(sm + TL::kCodeBytes + TL::kParBytes);
  const int q = (c == 1) ? 2 : (c == 2) ? 1 : c;
#pragma unroll
  for (int gi = 0; gi < NG; ++gi) {
    RowPairs pa, pb;
    if (BITS == 8) {
      pa = q8_group_pairs_sub(*reinterpret_cast<const uint4*>(sm + g * TL::kStride + gi * 64 + 16 * c));
      pb = q8_group_pairs_sub(*reinterpret_cast<const uint4*>(sm + (g + 8) * TL::kStride + gi * 64 + 16 * c));
    } else {
      pa = q4_group_pairs_sub(*reinterpret_cast<const uint2*>(sm + g * TL::kStride + gi * 32 + 8 * q));
      pb = q4_group_pairs_sub(*reinterpret_cast<const uint2*>(sm + (g + 8) * TL::kStride + gi * 32 + 8 * q));
    }
    uint32_t xh[8], xl[8];
    bfrag(gi, xh, xl);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      mma_f16(d, pa.p[2 * m], pb.p[2 * m], pa.p[2 * m + 1], pb.p[2 * m + 1], xh[2 * m], xh[2 * m + 1]);
      if (SPLIT)
        mma_f16(d, pa.p[2 * m], pb.p[2 * m], pa.p[2 * m + 1], pb.p[2 * m + 1], xl[2 * m], xl[2 * m + 1]);
    }
    // subnormal code form (rnb_common.cuh): the scales carry the 2^24 back
    const float sa = bf16_bits_to_f32(S[g * NG + gi]) * 0x1p24f, ba = bf16_bits_to_f32(B[g * NG + gi]);
    const float sb = bf16_bits_to_f32(S[(g + 8) * NG + gi]) * 0x1p24f, bb = bf16_bits_to_f32(B[(g + 8) * NG + gi]);
    const float xs0 = gsum(gi, 0), xs1 = gsum(gi, 1);
    acc[0] = fmaf(sa, d[0], fmaf(ba, xs0, acc[0]));
    acc[1] = fmaf(sa, d[1], fmaf(ba, xs1, acc[1]));
    acc[2] = fmaf(sb, d[2], fmaf(bb, xs0, acc[2]));
    acc[3] = fmaf(sb, d[3], fmaf(bb, xs1, acc[3]));
  }
}

// Work item of one grid row: expert slot j (0 = shared expert, j >= 1 =
// j-th active routed expert).  One round trip reads the active count and the
// expert's record (local id, entry count, entry offset, first 8 entries).
struct Item {
  bool active;
  uint32_t le;   // local expert (routed)
  int n_ent;     // (token, slot) entries
  const uint32_t* ents;  // all entries (routed) or nullptr (shared: token t -> t*(K+1)+K)
  uint32_t first[8];     // entries of the first column tile
};

__device__ __forceinline__ Item load_item(const Params& p, int j) {
  Item it;
  const int K = p.k;
  if (j == 0) {
    it.active = p.has_shared != 0;
    it.le = 0;
    it.n_ent = p.T;
    it.ents = nullptr;
#pragma unroll
    for (int i = 0; i < 8; ++i) it.first[i] = static_cast<uint32_t>((i < p.T ? i : 0) * (K + 1) + K);
    return it;
  }
  const uint32_t nact = __ldcg(p.ws.nact);
  const uint4* r = reinterpret_cast<const uint4*>(p.ws.rec + static_cast<size_t>(j - 1) * kRecWords);
  const uint4 r0 = __ldcg(r), r1 = __ldcg(r + 1), r2 = __ldcg(r + 2);
  it.active = static_cast<uint32_t>(j - 1) < nact;
  it.le = r0.x;
  it.n_ent = static_cast<int>(r0.y);
  it.ents = p.ws.entries + r0.z;
  it.first[0] = r1.x; it.first[1] = r1.y; it.first[2] = r1.z; it.first[3] = r1.w;
  it.first[4] = r2.x; it.first[5] = r2.y; it.first[6] = r2.z; it.first[7] = r2.w;
  return it;
}

// Entry id of column `lane` (lanes 0..7) of the column tile at nt; columns
// past n_ent repeat the tile's first entry.
__device__ __forceinline__ uint32_t lane_entry(const Item& it, int K, int nt, int lane) {
  if (lane >= 8) return 0;
  const int i = nt + lane < it.n_ent ? nt + lane : nt;
  if (!it.ents) return static_cast<uint32_t>(i * (K + 1) + K);
  if (nt == 0) {
    uint32_t v = it.first[0];
#pragma unroll
    for (int q = 1; q < 8; ++q) v = (i == q) ? it.first[q] : v;
    return v;
  }
  return __ldcg(it.ents + i);
}

// Max |h| of column `lane` (lanes < ncols; others get 0) from the per-tile
// partial maxima; the warp reads all columns' partials at once.
__device__ __forceinline__ float column_hmax(const Params& p, uint32_t ent_l, int ncols, int lane) {
  const int nt = p.I / 8;
  float mine = 0.f;
#pragma unroll
  for (int col = 0; col < 8; ++col) {
    if (col < ncols) {
      const uint32_t id = __shfl_sync(0xffffffffu, ent_l, col);
      const float* src = p.ws.hmaxp + static_cast<size_t>(id) * nt;
      float m = 0.f;
      for (int j = lane; j < nt; j += 32) m = fmaxf(m, __ldcg(src + j));
      m = warp_max(m);
      if (lane == col) mine = m;
    }
  }
  return mine;
}

// ---------------------------------------------------------- k_gateup

constexpr int kGateUpMaxWarps = 4;  // H / 512, H <= 2048

template <int BITS>
__host__ __device__ constexpr size_t gateup_smem(int nw, int ncmax) {
  using TL = Tile<BITS, kGateUpGroupsPerWarp>;
  return static_cast<size_t>(nw) *
             (TL::kBytes + ncmax * kGateUpGroupsPerWarp * 128 + ncmax * kGateUpGroupsPerWarp * 4) +
         nw * 16 * 8 * 4;
}

template <int BITS>
__global__ void __launch_bounds__(32 * kGateUpMaxWarps) k_gateup(Params p) {
  constexpr int NG = kGateUpGroupsPerWarp;
  using TL = Tile<BITS, NG>;
  extern __shared__ __align__(16) char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int j = blockIdx.y;
  const int ch0 = blockIdx.x * 8;
  const int K = p.k, G = p.H / kGroup, ncmax = p.ncmax;
  const size_t wrow = static_cast<size_t>(p.H) * BITS / 32, srow = p.H / kGroup;
  const int g0 = warp * NG;
  char* tile = smem + warp * TL::kBytes;
  uint32_t* sx = reinterpret_cast<uint32_t*>(smem + nw * TL::kBytes) + warp * ncmax * NG * 32;
  float* sxs = reinterpret_cast<float*>(smem + nw * (TL::kBytes + ncmax * NG * 128)) + warp * ncmax * NG;
  float* red = reinterpret_cast<float*>(smem + nw * (TL::kBytes + ncmax * NG * 128 + ncmax * NG * 4));
  // tile row i: up rows ch0..ch0+7, then gate rows I+ch0..I+ch0+7
  auto row_of = [&](int i) -> size_t { return i < 8 ? ch0 + i : p.I + ch0 + i - 8; };

  __shared__ uint32_t s_ent[8];
  __shared__ float s_inv[8];
  // The shared expert (grid row 0) does not depend on routing: start its
  // copies before waiting for k_route.
  if (j == 0) {
    if (!p.has_shared) return;
    tile_issue<BITS, NG>(tile, p.sgu_w, p.sgu_s, p.sgu_b, wrow, srow, g0, row_of, lane);
  }
  griddep_wait();
  griddep_launch_dependents();
  const Item it = load_item(p, j);
  if (!it.active) return;
  if (j != 0) {
    const size_t ew = static_cast<size_t>(2) * p.I * wrow, es = static_cast<size_t>(2) * p.I * srow;
    tile_issue<BITS, NG>(tile, p.gu_w + it.le * ew, p.gu_s + it.le * es, p.gu_b + it.le * es, wrow, srow,
                         g0, row_of, lane);
  }
  const int n_ent = it.n_ent;

  for (int nt = 0; nt < n_ent; nt += ncmax) {
    const int ncols = n_ent - nt < ncmax ? n_ent - nt : ncmax;
    const uint32_t ent_l = lane_entry(it, K, nt, lane);
    if (warp == 0 && lane < 8) {
      s_ent[lane] = ent_l;
      s_inv[lane] = __ldcg(p.ws.xinv + ent_l / (K + 1));
    }
    // stage this warp's activation fragments (128 B per column and group)
    for (int q0 = 0; q0 < ncols * NG * 8; q0 += 32) {
      const int q = q0 + lane;
      const int col = q / (NG * 8), rem = q % (NG * 8), gi = rem >> 3, part = rem & 7;
      const uint32_t id = __shfl_sync(0xffffffffu, ent_l, col < 8 ? col : 0);
      if (q < ncols * NG * 8)
        cp_async16(sx + (col * NG + gi) * 32 + part * 4,
                   p.ws.xperm + (static_cast<size_t>(id / (K + 1)) * G + g0 + gi) * 32 + part * 4);
    }
    for (int q0 = 0; q0 < ncols * NG; q0 += 32) {
      const int q = q0 + lane;
      const int col = q / NG, gi = q % NG;
      const uint32_t id = __shfl_sync(0xffffffffu, ent_l, col < 8 ? col : 0);
      if (q < ncols * NG) sxs[col * NG + gi] = __ldcg(p.ws.xsum + static_cast<size_t>(id / (K + 1)) * G + g0 + gi);
    }
    cp_async_wait_all();
    __syncwarp();
    const int colB = g < ncols ? g : 0;
    const int cl0 = 2 * c < ncols ? 2 * c : 0, cl1 = 2 * c + 1 < ncols ? 2 * c + 1 : 0;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma<BITS, NG, false>(
        tile, g, c,
        [&](int gi, uint32_t(&xb)[8], uint32_t(&)[8]) {
          const uint4 u0 = *reinterpret_cast<const uint4*>(sx + (colB * NG + gi) * 32 + c * 8);
          const uint4 u1 = *reinterpret_cast<const uint4*>(sx + (colB * NG + gi) * 32 + c * 8 + 4);
          xb[0] = u0.x; xb[1] = u0.y; xb[2] = u0.z; xb[3] = u0.w;
          xb[4] = u1.x; xb[5] = u1.y; xb[6] = u1.z; xb[7] = u1.w;
        },
        [&](int gi, int col) { return sxs[(col ? cl1 : cl0) * NG + gi]; }, acc);
    float* rw = red + warp * 128;
    rw[g * 8 + 2 * c] = acc[0];
    rw[g * 8 + 2 * c + 1] = acc[1];
    rw[(g + 8) * 8 + 2 * c] = acc[2];
    rw[(g + 8) * 8 + 2 * c + 1] = acc[3];
    __syncthreads();
    // SwiGLU; each 8-channel tile also records its column maxima (one plain
    // store per column: no atomics on shared addresses)
    for (int q0 = 0; q0 < 64; q0 += blockDim.x) {
      const int q = q0 + threadIdx.x;
      const int r = q & 7, n = q >> 3;
      const bool ok = q < 64 && n < ncols;
      float hv = 0.f;
      uint32_t id = 0;
      if (ok) {
        float up = 0.f, gate = 0.f;
        for (int w = 0; w < nw; ++w) {
          up += red[w * 128 + r * 8 + n];
          gate += red[w * 128 + (8 + r) * 8 + n];
        }
        id = s_ent[n];
        const float inv = s_inv[n];
        up *= inv;
        gate *= inv;
        hv = (gate / (1.0f + expf(-gate))) * up;
        p.ws.h[static_cast<size_t>(id) * p.I + ch0 + r] = hv;
      }
      float m = fabsf(hv);
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      if (ok && r == 0) p.ws.hmaxp[static_cast<size_t>(id) * (p.I / 8) + ch0 / 8] = m;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ k_down

constexpr int kDownMaxWarps = 4;  // I <= 1024

template <int BITS>
__host__ __device__ constexpr size_t down_smem(int nw, int ncmax) {
  using TL = Tile<BITS, kDownGroupsPerWarp>;
  return static_cast<size_t>(nw) * (TL::kBytes + ncmax * kDownGroupsPerWarp * kGroup * 4) + nw * 16 * 8 * 4;
}

template <int BITS>
__global__ void __launch_bounds__(32 * kDownMaxWarps) k_down(Params p) {
  constexpr int NG = kDownGroupsPerWarp;
  using TL = Tile<BITS, NG>;
  extern __shared__ __align__(16) char smem[];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int j = blockIdx.y;
  const int n0 = blockIdx.x * 16;
  const int K = p.k, ncmax = p.ncmax;
  const size_t wrow = static_cast<size_t>(p.I) * BITS / 32, srow = p.I / kGroup;
  const int g0 = warp * NG;
  char* tile = smem + warp * TL::kBytes;
  float* sh = reinterpret_cast<float*>(smem + nw * TL::kBytes) + warp * ncmax * NG * kGroup;
  float* red = reinterpret_cast<float*>(smem + nw * (TL::kBytes + ncmax * NG * kGroup * 4));
  auto row_of = [&](int i) -> size_t { return n0 + i; };

  __shared__ uint32_t s_ent[8];
  __shared__ float s_inv[8];
  // k_gateup launches this grid only after k_route has completed, so the
  // routing is readable here; the SwiGLU activations are not until the wait.
  const Item it = load_item(p, j);
  if (it.active && !(p.mode == kModeSwitchGLU && j == 0)) {
    if (j == 0) {
      tile_issue<BITS, NG>(tile, p.sdn_w, p.sdn_s, p.sdn_b, wrow, srow, g0, row_of, lane);
    } else {
      const size_t ew = static_cast<size_t>(p.H) * wrow, es = static_cast<size_t>(p.H) * srow;
      tile_issue<BITS, NG>(tile, p.dn_w + it.le * ew, p.dn_s + it.le * es, p.dn_b + it.le * es, wrow, srow,
                           g0, row_of, lane);
    }
  }
  // The next call's k_route may start now: it only streams router weights
  // until it waits for this grid to complete.
  griddep_launch_dependents();
  if (p.mode == kModeSwitchGLU && j == 0) {
    // Slots routed to experts outside this bank produce zeros.
    griddep_wait();
    for (int i = threadIdx.x; i < p.T * K * 16; i += blockDim.x) {
      const int slot = i / 16, r = i % 16;
      const uint32_t e = __ldcg(p.ws.inds + slot);
      const int le = static_cast<int>(e) - p.off;
      if (e >= static_cast<uint32_t>(p.E_total) || le < 0 || le >= p.E) {
        const size_t at = static_cast<size_t>(slot) * p.H + n0 + r;
        if (p.y_f32)
          static_cast<float*>(p.out)[at] = 0.f;
        else
          static_cast<__nv_bfloat16*>(p.out)[at] = __float2bfloat16_rn(0.f);
      }
    }
    return;
  }
  if (!it.active) return;
  griddep_wait();
  const int n_ent = it.n_ent;

  const int pbase = BITS == 8 ? 16 * c : 16 * ((c == 1) ? 2 : (c == 2) ? 1 : c);
  for (int nt = 0; nt < n_ent; nt += ncmax) {
    const int ncols = n_ent - nt < ncmax ? n_ent - nt : ncmax;
    const uint32_t ent_l = lane_entry(it, K, nt, lane);
    // stage this warp's hidden range of each column's fp32 SwiGLU output
    constexpr int kPieces = NG * kGroup / 4;  // 16-byte pieces per column
    for (int q0 = 0; q0 < ncols * kPieces; q0 += 32) {
      const int q = q0 + lane;
      const int col = q / kPieces, piece = q % kPieces;
      const uint32_t id = __shfl_sync(0xffffffffu, ent_l, col < 8 ? col : 0);
      if (q < ncols * kPieces)
        cp_async16(sh + col * NG * kGroup + piece * 4, p.ws.h + static_cast<size_t>(id) * p.I + g0 * kGroup + piece * 4);
    }
    // per-column fp16 range scale from the column's max |h|
    float hscale_l = 1.f, hinv_l = 1.f;
    fp16_range_scale(column_hmax(p, ent_l, ncols, lane), hscale_l, hinv_l);
    if (warp == 0 && lane < 8) {
      s_ent[lane] = ent_l;
      s_inv[lane] = hinv_l;
    }
    const float hscale = __shfl_sync(0xffffffffu, hscale_l, g < ncols ? g : 0);
    cp_async_wait_all();
    __syncwarp();
    const int colB = g < ncols ? g : 0;
    float gcur = 0.f;  // group sum of this lane's column g for the group just built
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // Activation pairs from fp32 h: scaled into fp16 range and split into a
    // high fp16 part and the fp16 remainder, so hi + lo carries ~22 bits; the
    // group sums use hi + lo so the affine bias term matches the products.
    auto bfrag = [&](int gi, uint32_t(&xh)[8], uint32_t(&xl)[8]) {
      const float* src = sh + colB * NG * kGroup + gi * kGroup + pbase;
      float f[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = reinterpret_cast<const float4*>(src)[q];
        f[4 * q] = v.x; f[4 * q + 1] = v.y; f[4 * q + 2] = v.z; f[4 * q + 3] = v.w;
      }
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float a = f[pair_rel<BITS>(i, 0)] * hscale, b = f[pair_rel<BITS>(i, 1)] * hscale;
        const __half2 hi = __floats2half2_rn(a, b);
        const float2 hf = __half22float2(hi);
        const __half2 lo = __floats2half2_rn(a - hf.x, b - hf.y);
        const float2 lf = __half22float2(lo);
        // 4-bit pairs 1 and 3 of a word meet codes times 16 (subnormal form)
        const __half2 q16 = __float2half2_rn((BITS == 4 && (i & 1)) ? 0.0625f : 1.0f);
        const __half2 his = __hmul2(hi, q16), los = __hmul2(lo, q16);
        xh[i] = *reinterpret_cast<const uint32_t*>(&his);
        xl[i] = *reinterpret_cast<const uint32_t*>(&los);
        part += (hf.x + lf.x) + (hf.y + lf.y);
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      gcur = part;
    };
    auto gsum = [&](int, int col) { return __shfl_sync(0xffffffffu, gcur, (2 * c + col) * 4); };
    tile_mma<BITS, NG, true>(tile, g, c, bfrag, gsum, acc);
    float* rw = red + warp * 128;
    rw[g * 8 + 2 * c] = acc[0];
    rw[g * 8 + 2 * c + 1] = acc[1];
    rw[(g + 8) * 8 + 2 * c] = acc[2];
    rw[(g + 8) * 8 + 2 * c + 1] = acc[3];
    __syncthreads();
    for (int q = threadIdx.x; q < 128; q += blockDim.x) {
      const int r = q & 15, n = q >> 4;
      if (n < ncols) {
        float y = 0.f;
        for (int w = 0; w < nw; ++w) y += red[w * 128 + r * 8 + n];
        const uint32_t id = s_ent[n];
        y *= s_inv[n];
        if (p.mode == kModeSwitchGLU) {
          const uint32_t t = id / (K + 1), slot = id % (K + 1);
          const size_t at = (static_cast<size_t>(t) * K + slot) * p.H + n0 + r;
          if (p.y_f32)
            static_cast<float*>(p.out)[at] = y;
          else
            static_cast<__nv_bfloat16*>(p.out)[at] = __float2bfloat16_rn(y);
        } else {
          p.ws.yws[static_cast<size_t>(id) * p.H + n0 + r] = y;
        }
      }
    }
    __syncthreads();
  }
  if (p.mode == kModeSwitchGLU) return;

  // Weighted combine by the last CTA to finish this 16-row tile.
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t expected = __ldcg(p.ws.nact) + (p.has_shared ? 1u : 0u);
    const uint32_t prev = atomicAdd(p.ws.ctr + 1 + blockIdx.x, 1u);
    s_last = prev == expected - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
  for (int i = threadIdx.x; i < p.T * 16; i += blockDim.x) {
    const int t = i / 16, r = i % 16, n = n0 + r;
    // issue every slot's loads before the ordered accumulation
    uint32_t e[kMaxK];
    float sc[kMaxK], y[kMaxK];
#pragma unroll
    for (int s = 0; s < kMaxK; ++s) {
      if (s < K) {
        e[s] = __ldcg(p.ws.inds + t * K + s);
        sc[s] = __ldcg(p.ws.scores + t * K + s);
        y[s] = __ldcg(p.ws.yws + (static_cast<size_t>(t) * (K + 1) + s) * p.H + n);
      }
    }
    const float ysh = p.has_shared ? __ldcg(p.ws.yws + (static_cast<size_t>(t) * (K + 1) + K) * p.H + n) : 0.f;
    const float sg = p.has_shared ? __ldcg(p.ws.sgate + t) : 0.f;
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxK; ++s) {
      if (s < K) {
        const int le = static_cast<int>(e[s]) - p.off;
        acc += (le >= 0 && le < p.E) ? sc[s] * y[s] : 0.f;
      }
    }
    if (p.has_shared) acc += sg * ysh;
    if (p.y_f32)
      static_cast<float*>(p.out)[static_cast<size_t>(t) * p.H + n] = acc;
    else
      out[static_cast<size_t>(t) * p.H + n] = __float2bfloat16_rn(acc);
  }
  __syncthreads();
  if (threadIdx.x == 0) atomicExch(p.ws.ctr + 1 + blockIdx.x, 0u);
}

// ------------------------------------------------- k_decode (persistent)
//
// One launch for one or two tokens, one CTA of 16 warps per SM, launched
// with programmatic stream serialisation so that its prologue (weights
// only) overlaps the previous kernel's tail.  CTAs hand data to each other
// through 8-byte {value, epoch} words in the workspace header's exchange
// region: the epoch is the workspace's call sequence word + 1, so a word
// carrying it was written by this call.  A reader polls the words it needs
// (bounded in time); there are no arrival counters, fences or grid
// barriers on the data path.
//   prologue  this CTA's router rows into registers; its shared-expert
//             gate/up slice (ring slot 0) and shared-expert down tiles into
//             shared memory.
//   router    two router rows (of E_total + 1; the last is the shared gate)
//             against the tokens -> logit words (bf16 candidate intervals,
//             rnb_route.cuh); activation prep; the shared-expert gate/up task
//             -> h words.
//   routing   every CTA polls the logit words, selects the top k exactly and
//             derives the same task lists.
//   gate/up   routed tasks (expert x 8 channels, hidden dimension split over
//             the 16 warps) round-robin over CTAs.  Each warp streams its
//             slices of the CTA's tasks, then its down slices, through its
//             own ring of shared-memory slots (cp.async groups; no CTA
//             barrier in the stream).  Epilogue: SwiGLU -> h words.
//   down      CTAs owning 16 output rows: per source (routed experts, shared
//             expert) and 128-channel quarter, a warp polls that quarter's
//             h words, converts them to fp16 with one power-of-two scale per
//             64-group and runs the MMAs; then the ordered weighted combine
//             (or, expert parallel, the cross-rank exchange).
//   exit      the last CTA out advances the sequence word.

constexpr int kPWarps = 16;
constexpr int kPMaxT = 2;
constexpr int kPMaxK = 8;
constexpr int kPMaxAct = kPMaxT * kPMaxK;  // distinct local experts of one call
constexpr int kPMaxMine = 8;               // routed gate/up tasks of one CTA
constexpr uint64_t kSpinLimitNs = 200ull * 1000 * 1000;  // a wait gives up after 200 ms
// Waits on other GPUs: ranks launch independently, so allow host-side skew
// (the default of an EP context; rnb_ep_set_wait_limit_ms changes it).
constexpr uint64_t kEpSpinLimitNs = 2000ull * 1000 * 1000;

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

// Wait until at most n of this thread's committed groups are pending; an n
// above 7 waits for all but the newest 7 (more than asked: still correct).
__device__ __forceinline__ void cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;\n" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;\n" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;\n" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;\n" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;\n" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;\n" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;\n" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;\n" ::: "memory"); break;
  }
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One 8-byte {value, epoch} exchange word, written and read as a single
// 64-bit access (single-copy atomic): a reader that sees the epoch sees the
// value stored with it.  .gpu scope within one device; .sys across devices.
__device__ __forceinline__ void xw_store(uint2* p, uint32_t v, uint32_t epoch) {
  const uint64_t w = (static_cast<uint64_t>(epoch) << 32) | v;
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;\n" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t xw_load(const uint2* p) {
  uint64_t w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];\n" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Two neighbouring exchange words (16-byte aligned) in one access; each word
// is read single-copy atomically on its own.
__device__ __forceinline__ void xw_load2(const uint2* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];\n" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t xw_load_acquire(const uint2* p) {
  uint64_t w;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];\n" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ void xw_store_sys(uint2* p, uint32_t v, uint32_t epoch) {
  const uint64_t w = (static_cast<uint64_t>(epoch) << 32) | v;
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;\n" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t xw_load_sys(const uint2* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];\n" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// The value of word p once it carries `epoch`.  Polls until then or until
// `deadline` (globaltimer ns); on timeout sets RNB_STATUS_TIMEOUT in *status
// and returns 0 (the call's results are void).  Each lane polls its own word.
__device__ __forceinline__ uint32_t xw_wait(const uint2* p, uint32_t epoch, uint64_t deadline, uint32_t* status) {
  uint64_t w = xw_load(p);
  while (static_cast<uint32_t>(w >> 32) != epoch) {
    if (gtimer() > deadline) {
      atomicOr(status, RNB_STATUS_TIMEOUT);
      return 0u;
    }
    __nanosleep(40);
    w = xw_load(p);
  }
  return static_cast<uint32_t>(w);
}

// Expert-parallel all-reduce of one 16-column output tile for T tokens.
// Every rank's fp32 partial part(t, r) (t < T, r < 16) goes to each rank as
// one 8-byte {value, epoch} word (a single 64-bit store, single-copy atomic),
// so a word that carries this call's epoch carries this call's value: the
// receiver polls the words themselves, with no separate flag and no fence,
// and sums the ranks' values in rank order (the same order on every rank)
// before handing them to emit(t, r, sum).  Polls are bounded; on timeout the
// status word gets RNB_STATUS_TIMEOUT and that value is not emitted.  Buffers
// alternate by epoch parity: a rank cannot start epoch e+2 before every rank
// has sent epoch e+1, which each rank does only after reading epoch e.
template <typename Part, typename Emit>
__device__ void ep_exchange_tile(const Params& p, int n0, int T, Part part, Emit emit) {
  const int tid = threadIdx.x, W = p.ep_world;
  __shared__ uint32_t s_epoch;
  if (tid == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(p.ep_seq) + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const size_t par = static_cast<size_t>(epoch & 1u) * W * kEpMaxT * p.H;
  for (int i = tid; i < T * 16; i += blockDim.x) {
    const int t = i >> 4, r = i & 15;
    const uint32_t v = __float_as_uint(part(t, r));
    const size_t o = par + (static_cast<size_t>(p.ep_rank) * kEpMaxT + t) * p.H + n0 + r;
    for (int q = 0; q < W; ++q) xw_store_sys(p.ep_recv[q] + o, v, epoch);
  }
  const uint64_t deadline = gtimer() + p.ep_limit_ns;
  for (int i = tid; i < T * 16; i += blockDim.x) {
    const int t = i >> 4, r = i & 15;
    const uint2* own = p.ep_recv[p.ep_rank] + par + static_cast<size_t>(t) * p.H + n0 + r;
    float sum = 0.f;
    bool ok = true;
    for (int q = 0; q < W && ok; ++q) {
      const uint2* src = own + static_cast<size_t>(q) * kEpMaxT * p.H;
      uint64_t w = xw_load_sys(src);
      while (static_cast<uint32_t>(w >> 32) != epoch) {
        if (gtimer() > deadline) {
          atomicOr(p.ws.status, RNB_STATUS_TIMEOUT);
          ok = false;
          break;
        }
        w = xw_load_sys(src);
      }
      sum += __uint_as_float(static_cast<uint32_t>(w));
    }
    if (ok) emit(t, r, sum);
  }
}

// Expert-parallel reduction after the decode chain: CTA b owns output
// columns [16b, 16b+16) of the fp32 partial (p.ws.yws reused as [T][H]).
// Cooperative launch, so every CTA is resident while it waits for peers.
__global__ void __launch_bounds__(256) k_ep_reduce(Params p, const float* partial) {
  const int n0 = blockIdx.x * 16;
  ep_exchange_tile(
      p, n0, p.T, [&](int t, int r) { return __ldcg(partial + static_cast<size_t>(t) * p.H + n0 + r); },
      [&](int t, int r, float v) {
        const size_t o = static_cast<size_t>(t) * p.H + n0 + r;
        if (p.y_f32)
          static_cast<float*>(p.out)[o] = v;
        else
          static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
      });
  // the last CTA out advances the sequence word for the next exchange
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.ep_seq + 1, 1u) == gridDim.x - 1) {
      p.ep_seq[1] = 0;
      p.ep_seq[0] += 1;
      __threadfence();
    }
  }
}

// Shared-memory plan of k_decode (host-computed).
struct PPlan {
  int S;   // ring slots per warp
  int sk;  // the split-K form (one token, one GPU)
  uint32_t off_tma;  // (split-K) the TMA destinations start at the next 1024-byte boundary from here
  uint32_t off_ring, off_sdn, off_x, off_xs, off_xn, off_ivl, off_red, off_hf, off_redc, off_misc;
};

// ---- split-K form of k_decode (one token, one GPU)
//
// Task i < 16 (k + 1) of CTA i: source s = i / 16 (routed slot s < k, the
// shared expert at s = k) and channel slice j = i % 16, channels
// [32 j, 32 j + 32).  The CTA computes the slice's gate/up (64 weight rows,
// its 16 warps splitting the hidden dimension), SwiGLU, and the slice's
// share of the down projection, y_i = W_down[:, slice] h[slice] over all H
// rows, weighted by the slot's routing weight (or the shared gate).  So h
// never leaves the CTA.  The weighted partials go out as {value, epoch}
// words; CTA r < H / 16 polls and sums the 16 (k + 1) partials of rows
// [16 r, 16 r + 16) in task order.
// The shared expert's CTAs know their weights at launch and load them in the
// prologue.
constexpr int kSkC = 32;                 // channels per task
constexpr int kSkUnits = kSkC / 8;       // gate/up tiles (8 up + 8 gate rows) per task
constexpr int kSkTasksPerSource = 512 / kSkC;

// TMA descriptors of the split-K loads (host-encoded, cached per tensor).
// Gate/up codes: 4-D {a warp's K slice (Tile2 row bytes, as u32), 2I rows,
// 16 slices, experts}, box {slice, 8 rows, 16 slices, 1}: one request puts
// one tile's 8 up (or gate) rows in shared memory as [slice][8 rows][slice
// bytes], swizzled (64 B or 128 B) so that the MMA reads are conflict-free.
// Gate/up scales and biases: 3-D {H/64 groups, 2I rows, experts}, box
// {H/64, 32, 1}.  Down codes: 4-D {row words, 256 rows, H/256 blocks,
// experts}, box {the slice's words, 256, H/256, 1}: the slice's codes of all
// H rows, [H][slice bytes].
struct SkMaps {
  CUtensorMap gu_w, gu_s, gu_b, dn_w;      // the routed bank
  CUtensorMap sgu_w, sgu_s, sgu_b, sdn_w;  // the shared expert
};

// The down slice's codes, [H rows][slice bytes] in shared memory (warp w
// takes rows [128 w, 128 w + 128)); each warp's rows' group scales and
// biases go to registers (lane l: rows l, l + 32, l + 64, l + 96; each a
// 4-byte word with the neighbouring group's value), as coalesced loads.
template <int BITS>
struct SkDown {
  static constexpr int kRow = kSkC * BITS / 8;  // code bytes per row (16 or 32)
  static constexpr int kCodeBytes = 128 * kRow;
  static constexpr int kBytes = kCodeBytes;
};

__device__ __forceinline__ void sk_down_sb(const uint16_t* sc, const uint16_t* bi, int I, int row0, int j, int lane,
                                           uint32_t (&sw)[4], uint32_t (&bw)[4]) {
  const size_t srow = I / kGroup;
  const int grp2 = (j * kSkC / kGroup) & ~1;  // the word of groups (grp2, grp2 + 1)
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const size_t o = static_cast<size_t>(row0 + lane + 32 * k) * srow + grp2;
    sw[k] = __ldg(reinterpret_cast<const uint32_t*>(sc + o));
    bw[k] = __ldg(reinterpret_cast<const uint32_t*>(bi + o));
  }
}

// The slice's down MMAs for one warp: 8 tiles of 16 rows x 32 channels.
// bt: the B pairs [lane c][pair 4] of the fp16 h slice; hs: its sum; hinv:
// its inverse scale; emit(row, value) for the rows this lane finishes
// (c == 0: rows g and g + 8 of each tile).
template <int BITS, typename Emit>
__device__ __forceinline__ void sk_down_mma(const char* sm, const uint32_t (&sw)[4], const uint32_t (&bw)[4],
                                            const uint32_t* bt, float hs, float hinv, int j, int g, int c,
                                            Emit emit) {
  using SD = SkDown<BITS>;
  const uint32_t b0 = bt[c * 4 + 0], b1 = bt[c * 4 + 1], b2 = bt[c * 4 + 2], b3 = bt[c * 4 + 3];
  const int half = (j * kSkC / kGroup) & 1;
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    const int ra = 16 * v + g, rb = ra + 8;
    uint32_t pa[4], pb[4];
    if (BITS == 8) {
      const uint2 wa = *reinterpret_cast<const uint2*>(sm + ra * SD::kRow + 8 * c);
      const uint2 wb = *reinterpret_cast<const uint2*>(sm + rb * SD::kRow + 8 * c);
      q8_word_to_pairs_sub(wa.x, pa[0], pa[1]);
      q8_word_to_pairs_sub(wa.y, pa[2], pa[3]);
      q8_word_to_pairs_sub(wb.x, pb[0], pb[1]);
      q8_word_to_pairs_sub(wb.y, pb[2], pb[3]);
    } else {
      const uint32_t wa = *reinterpret_cast<const uint32_t*>(sm + ra * SD::kRow + 4 * c);
      const uint32_t wb = *reinterpret_cast<const uint32_t*>(sm + rb * SD::kRow + 4 * c);
      q4_word_to_pairs_sub(wa, pa[0], pa[1], pa[2], pa[3]);
      q4_word_to_pairs_sub(wb, pb[0], pb[1], pb[2], pb[3]);
    }
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_f16(d, pa[0], pb[0], pa[1], pb[1], b0, b1);
    mma_f16(d, pa[2], pb[2], pa[3], pb[3], b2, b3);
    // rows ra and rb are held by lanes ra % 32 and rb % 32 in register v / 2
    const uint32_t sa2 = __shfl_sync(0xffffffffu, sw[v >> 1], ra & 31);
    const uint32_t ba2 = __shfl_sync(0xffffffffu, bw[v >> 1], ra & 31);
    const uint32_t sb2 = __shfl_sync(0xffffffffu, sw[v >> 1], rb & 31);
    const uint32_t bb2 = __shfl_sync(0xffffffffu, bw[v >> 1], rb & 31);
    if (c == 0) {
      auto pick = [&](uint32_t w2) { return __uint_as_float(half ? (w2 & 0xFFFF0000u) : (w2 << 16)); };
      // the codes entered the MMAs as fp16 subnormals q * 2^-24: the scale carries 2^24 back
      emit(ra, hinv * fmaf(pick(sa2) * 0x1p24f, d[0], pick(ba2) * hs));
      emit(rb, hinv * fmaf(pick(sb2) * 0x1p24f, d[2], pick(bb2) * hs));
    }
  }
}

struct PMisc {
  uint32_t inds[kPMaxT][kPMaxK];
  float scores[kPMaxT][kPMaxK];
  float sg[kPMaxT];
  float xinv[kPMaxT];
  float red[kPWarps];
  uint32_t epoch;
  uint32_t n_act;
  uint32_t act_e[kPMaxAct];        // local expert of active expert a
  uint32_t act_cnt[kPMaxAct];      // its columns (tokens that selected it)
  uint32_t act_ent[kPMaxAct][kPMaxT];  // entry id t*(K+1)+slot of each column
  double rdot[kPWarps][4];   // router partials: dot (row i, token t) at 2i+t, fp64
  float rnorm[kPWarps][8];   // [0,2) sum w^2; [2,4) sum |w|; [4,6) sum x^2; [6,8) max |x|
  uint32_t skbt[16];         // split-K: B pairs [lane c][pair] of the fp16 h slice
  float skhs, skhinv;        // split-K: sum of the fp16 h slice, its inverse scale
  int sk_slot;               // split-K: this CTA's routed slot (-1: none)
  uint32_t sk_lmask;         // split-K: the slots whose expert is on this GPU
};

// Activation prep of T tokens (H = 2048) by the whole CTA (512 threads, 4
// consecutive values each): power-of-two scale into fp16 range, per-group
// sums, then the MMA pair order [T][G][4][8] of the gate/up B operand.
// xh: 2048-half scratch.
template <int BITS>
__device__ void xprep_cta(const uint16_t* x, int T, uint32_t* sX, float* sXs, float* xinv, __half* xh,
                          float* red, bool from_regs = false, uint2 xr0 = make_uint2(0, 0),
                          uint2 xr1 = make_uint2(0, 0)) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int H = 2048, G = H / kGroup;
#pragma unroll 1
  for (int t = 0; t < T; ++t) {
    // this thread's 4 values of token t: given (the router's registers), or
    // from global or shared memory
    const uint2 u = from_regs ? (t == 0 ? xr0 : xr1)
                              : reinterpret_cast<const uint2*>(x + static_cast<size_t>(t) * H)[tid];
    const float v[4] = {__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                        __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u)};
    const float m4 = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    const uint32_t mw = __reduce_max_sync(0xffffffffu, __float_as_uint(m4));  // |v| >= 0: bit order = value order
    if (lane == 0) red[warp] = __uint_as_float(mw);
    __syncthreads();
    float mx = red[0];
#pragma unroll
    for (int q = 1; q < kPWarps; ++q) mx = fmaxf(mx, red[q]);
    float scale, inv;
    fp16_range_scale(mx, scale, inv);
    const __half2 h0 = __floats2half2_rn(v[0] * scale, v[1] * scale);
    const __half2 h1 = __floats2half2_rn(v[2] * scale, v[3] * scale);
    reinterpret_cast<__half2*>(xh)[tid * 2] = h0;
    reinterpret_cast<__half2*>(xh)[tid * 2 + 1] = h1;
    const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
    float sum = (f0.x + f0.y) + (f1.x + f1.y);
    // a 64-group is 16 consecutive threads
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    sum += __shfl_xor_sync(0xffffffffu, sum, 8);
    if ((tid & 15) == 0) sXs[t * G + (tid >> 4)] = sum;
    if (tid == 0) xinv[t] = inv;
    __syncthreads();
    // pair order: 32 groups x 4 lanes x 8 pairs = 1024 pairs, 2 per thread
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int q = tid + k * 512;
      const int grp = q >> 5, cc = (q >> 3) & 3, i = q & 7;
      const __half a = xh[grp * kGroup + pair_pos<BITS>(cc, i, 0)];
      const __half b = xh[grp * kGroup + pair_pos<BITS>(cc, i, 1)];
      __half2 h2 = __halves2half2(a, b);
      // 4-bit pairs 1 and 3 of a word meet codes times 16 (subnormal form)
      if (BITS == 4 && (i & 1)) h2 = __hmul2(h2, __float2half2_rn(0.0625f));
      sX[(static_cast<size_t>(t) * G + grp) * 32 + cc * 8 + i] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    __syncthreads();
  }
}

// Where position r (0..63) of a 64-group sits in the MMA pair order of the
// activation operand: quad (lane c) and u32 pair index i, half h.
template <int BITS>
__device__ __forceinline__ void pair_slot(int r, int& cq, int& i, int& h) {
  if (BITS == 8) {
    cq = r >> 4;
    const int rr = r & 15;
    i = 2 * (rr >> 2) + ((rr & 3) >> 1);
    h = rr & 1;
  } else {
    const int qq = r >> 4;  // 16q + 8(i>>2) + (i&3) + 4h with q = {0,2,1,3}[c]
    cq = (qq == 1) ? 2 : (qq == 2) ? 1 : qq;
    const int rr = r & 15;
    i = 4 * (rr >> 3) + (rr & 3);
    h = (rr >> 2) & 1;
  }
}

// Gate/up epilogue of up to nt tasks (threads q < nt*16: task q/16, channel
// (q/2)%8, column q%2): sum the 16 warps' partials, SwiGLU, publish the h word
// of the column's (token, slot) entry.  red: [task][warp][16 rows][2 columns].
__device__ __forceinline__ void p_gateup_epilogue(const Params& p, const float* red, int nt, const uint32_t* ent_of,
                                                  const int* ncols_of, const int* ch0_of, const float* xinv,
                                                  uint2* hw, uint32_t epoch) {
  const int q = threadIdx.x;
  if (q >= nt * 16) return;
  const int m = q >> 4, r = (q >> 1) & 7, n = q & 1;
  if (n >= ncols_of[m]) return;
  const float* rt = red + m * kPWarps * 32;
  float up = 0.f, gate = 0.f;
#pragma unroll
  for (int w = 0; w < kPWarps; ++w) {
    up += rt[w * 32 + r * 2 + n];
    gate += rt[w * 32 + (8 + r) * 2 + n];
  }
  const uint32_t id = ent_of[m * kPMaxT + n];
  const float inv = xinv[id / (p.k + 1)];
  up *= inv;
  gate *= inv;
  const float hv = (gate / (1.0f + expf(-gate))) * up;
  xw_store(hw + static_cast<size_t>(id) * p.I + ch0_of[m] + r, __float_as_uint(hv), epoch);
}

// Two-group weight tile of one warp (16 rows x 128 inputs): codes with a
// 16-byte-chunk XOR swizzle instead of padding, then bf16 scales and biases.
// 8-bit rows are 128 B: chunk ^= (row & 1) << 2, so the 8 lanes of a 16-byte
// read phase (rows g, g+1) hit disjoint banks; 4-bit rows are 64 B: chunk ^=
// ((row >> 1) & 1) << 1, so the 16 lanes of an 8-byte phase (rows g..g+3) do.
template <int BITS>
struct Tile2 {
  static constexpr int kRowBytes = 2 * 8 * BITS;
  static constexpr int kCodeBytes = 16 * kRowBytes;
  static constexpr int kParBytes = 16 * 2 * 2;
  static constexpr int kBytes = kCodeBytes + 2 * kParBytes;
  static constexpr int kChunks = kRowBytes / 16;
  __device__ static __forceinline__ int swz(int row) {
    return BITS == 8 ? ((row & 1) << 2) : (((row >> 1) & 1) << 1);
  }
};

template <int BITS, typename RowOf>
__device__ __forceinline__ void tile2_issue(char* sm, const uint32_t* wbase, const uint16_t* sbase,
                                            const uint16_t* bbase, size_t wrow, size_t srow, int g0,
                                            RowOf row, int lane) {
  using TL = Tile2<BITS>;
  const size_t kw0 = static_cast<size_t>(g0) * kGroup * BITS / 32;
#pragma unroll
  for (int q = lane; q < 16 * TL::kChunks; q += 32) {
    const int i = q / TL::kChunks, j = q % TL::kChunks;
    cp_async16(sm + i * TL::kRowBytes + ((j ^ TL::swz(i)) * 16), wbase + row(i) * wrow + kw0 + j * 4);
  }
  if (lane < 16) {
    const size_t r = row(lane);
    cp_async4(sm + TL::kCodeBytes + lane * 4, sbase + r * srow + g0);
    cp_async4(sm + TL::kCodeBytes + TL::kParBytes + lane * 4, bbase + r * srow + g0);
  }
}

// acc[0..3] (rows g, g+8 x columns 2c, 2c+1) += affine(tile . B) over the
// tile's two groups.  bfrag(gi, xb) fills the 8 activation pairs of group gi
// for this lane's column g; gsum(gi, col) is the group sum of column col
// (0 -> 2c, 1 -> 2c+1) of the values the MMAs see; ginv(gi, col) multiplies
// the group's contribution (an activation scale undone per group).
template <int BITS, typename BFrag, typename GSum, typename GInv>
__device__ __forceinline__ void tile2_mma(const char* sm, int g, int c, BFrag bfrag, GSum gsum, GInv ginv,
                                          float (&acc)[4]) {
  using TL = Tile2<BITS>;
  const uint16_t* S = reinterpret_cast<const uint16_t*>(sm + TL::kCodeBytes);
  const uint16_t* B = reinterpret_cast<const uint16_t*>(sm + TL::kCodeBytes + TL::kParBytes);
  const int q = (c == 1) ? 2 : (c == 2) ? 1 : c;
#pragma unroll
  for (int gi = 0; gi < 2; ++gi) {
    RowPairs pa, pb;
    if (BITS == 8) {
      const int ch = gi * 4 + c;
      pa = q8_group_pairs_sub(*reinterpret_cast<const uint4*>(sm + g * TL::kRowBytes + (ch ^ TL::swz(g)) * 16));
      pb = q8_group_pairs_sub(*reinterpret_cast<const uint4*>(sm + (g + 8) * TL::kRowBytes + (ch ^ TL::swz(g + 8)) * 16));
    } else {
      const int ch = gi * 2 + (q >> 1), off = 8 * (q & 1);
      pa = q4_group_pairs_sub(*reinterpret_cast<const uint2*>(sm + g * TL::kRowBytes + (ch ^ TL::swz(g)) * 16 + off));
      pb = q4_group_pairs_sub(*reinterpret_cast<const uint2*>(sm + (g + 8) * TL::kRowBytes + (ch ^ TL::swz(g + 8)) * 16 + off));
    }
    uint32_t xb[8];
    bfrag(gi, xb);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 4; ++m)
      mma_f16(d, pa.p[2 * m], pb.p[2 * m], pa.p[2 * m + 1], pb.p[2 * m + 1], xb[2 * m], xb[2 * m + 1]);
    // the codes entered the MMAs as fp16 subnormals q * 2^-24 (rnb_common.cuh):
    // the scales carry the 2^24 back (exact)
    const float sa = bf16_bits_to_f32(S[g * 2 + gi]) * 0x1p24f, ba = bf16_bits_to_f32(B[g * 2 + gi]);
    const float sb = bf16_bits_to_f32(S[(g + 8) * 2 + gi]) * 0x1p24f, bb = bf16_bits_to_f32(B[(g + 8) * 2 + gi]);
    const float xs0 = gsum(gi, 0), xs1 = gsum(gi, 1);
    const float i0 = ginv(gi, 0), i1 = ginv(gi, 1);
    acc[0] = fmaf(i0, fmaf(sa, d[0], ba * xs0), acc[0]);
    acc[1] = fmaf(i1, fmaf(sa, d[1], ba * xs1), acc[1]);
    acc[2] = fmaf(i0, fmaf(sb, d[2], bb * xs0), acc[2]);
    acc[3] = fmaf(i1, fmaf(sb, d[3], bb * xs1), acc[3]);
  }
}

// Physical byte offset of 16-byte chunk ch of row r in a TMA-swizzled block
// whose rows are kRowBytes long (64: 64-byte swizzle, 128: 128-byte).
template <int BITS>
__device__ __forceinline__ int sk_swz_chunk(int r, int ch) {
  return BITS == 8 ? ((ch ^ (r & 7)) << 4) : ((ch ^ ((r >> 1) & 3)) << 4);
}

// acc (rows g: up channel 8u + g, g + 8: gate channel 8u + g; columns 2c,
// 2c + 1) += affine(tile . B) over this warp's two groups, from the
// TMA-loaded blocks: up / gate codes [4 tiles][16 slices][8 rows][Tile2 row bytes],
// sb = [up scales | gate scales | up biases | gate biases], each [32 rows][H/64].
template <int BITS, typename BFrag, typename GSum, typename GInv>
__device__ __forceinline__ void sk_gu_mma(const char* up, const char* gate, const uint16_t* sb, int G, int u, int w,
                                          int g, int c, BFrag bfrag, GSum gsum, GInv ginv, float (&acc)[4]) {
  using TL = Tile2<BITS>;
  const int r = 8 * u + g;
  const char* ua = up + (u * 128 + w * 8 + g) * TL::kRowBytes;
  const char* ga = gate + (u * 128 + w * 8 + g) * TL::kRowBytes;
  const int q = (c == 1) ? 2 : (c == 2) ? 1 : c;
#pragma unroll
  for (int gi = 0; gi < 2; ++gi) {
    RowPairs pa, pb;
    if (BITS == 8) {
      const int ch = gi * 4 + c;
      pa = q8_group_pairs_sub(*reinterpret_cast<const uint4*>(ua + sk_swz_chunk<BITS>(r, ch)));
      pb = q8_group_pairs_sub(*reinterpret_cast<const uint4*>(ga + sk_swz_chunk<BITS>(r, ch)));
    } else {
      const int ch = gi * 2 + (q >> 1), off = 8 * (q & 1);
      pa = q4_group_pairs_sub(*reinterpret_cast<const uint2*>(ua + sk_swz_chunk<BITS>(r, ch) + off));
      pb = q4_group_pairs_sub(*reinterpret_cast<const uint2*>(ga + sk_swz_chunk<BITS>(r, ch) + off));
    }
    uint32_t xb[8];
    bfrag(gi, xb);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 4; ++m)
      mma_f16(d, pa.p[2 * m], pb.p[2 * m], pa.p[2 * m + 1], pb.p[2 * m + 1], xb[2 * m], xb[2 * m + 1]);
    const int gcol = 2 * w + gi, n = 32 * G;
    const float sa = bf16_bits_to_f32(sb[r * G + gcol]) * 0x1p24f, ba = bf16_bits_to_f32(sb[2 * n + r * G + gcol]);
    const float sg = bf16_bits_to_f32(sb[n + r * G + gcol]) * 0x1p24f, bg = bf16_bits_to_f32(sb[3 * n + r * G + gcol]);
    const float xs0 = gsum(gi, 0), xs1 = gsum(gi, 1);
    const float i0 = ginv(gi, 0), i1 = ginv(gi, 1);
    acc[0] = fmaf(i0, fmaf(sa, d[0], ba * xs0), acc[0]);
    acc[1] = fmaf(i1, fmaf(sa, d[1], ba * xs1), acc[1]);
    acc[2] = fmaf(i0, fmaf(sg, d[2], bg * xs0), acc[2]);
    acc[3] = fmaf(i1, fmaf(sg, d[3], bg * xs1), acc[3]);
  }
}

// EP: compiled with the expert-parallel exchange (ep_world > 1); the
// single-GPU instance carries no exchange code.
// SK: the split-K form for one token on one GPU (see kSkC); otherwise the
// h-exchange form (one or two tokens, expert parallel included).
template <int BITS, bool EP, bool SK>
__global__ void __launch_bounds__(32 * kPWarps, 1) k_decode(Params p_arg, PPlan pl, const __grid_constant__ SkMaps skm) {
  extern __shared__ __align__(16) char sm[];
  // (split-K) TMA phases: gate/up tiles 0..3 (tile 0 with the scales and
  // biases), then the down codes
  __shared__ __align__(8) uint64_t sk_bar[kSkUnits + 1];
  if (SK && threadIdx.x == 0) {
    for (int i = 0; i <= kSkUnits; ++i) mbar_init(&sk_bar[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  // The parameters are read from a shared-memory copy: a kernel parameter
  // is an operand in the constant bank, and on this single-pass kernel each
  // of its scattered reads would otherwise risk a constant-cache miss (an L2
  // round trip) on the critical path.
  __shared__ __align__(16) Params s_params;
  for (int i = threadIdx.x; i < static_cast<int>(sizeof(Params) / 4); i += blockDim.x)
    reinterpret_cast<uint32_t*>(&s_params)[i] = reinterpret_cast<const uint32_t*>(&p_arg)[i];
  using TL = Tile2<BITS>;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int cta = blockIdx.x, NC = gridDim.x;
  const int S = pl.S;  // ring slots per warp
  char* ring = sm + pl.off_ring + static_cast<size_t>(warp) * S * TL::kBytes;  // this warp's slots
  char* sSdn = sm + pl.off_sdn;
  uint32_t* sX = reinterpret_cast<uint32_t*>(sm + pl.off_x);
  float* sXs = reinterpret_cast<float*>(sm + pl.off_xs);
  uint32_t* sIvl = reinterpret_cast<uint32_t*>(sm + pl.off_ivl);
  float* sRed = reinterpret_cast<float*>(sm + pl.off_red);
  float* sRedC = reinterpret_cast<float*>(sm + pl.off_redc);
  PMisc* ms = reinterpret_cast<PMisc*>(sm + pl.off_misc);
  const uint32_t off_xn = pl.off_xn, off_hf = pl.off_hf;
  __syncthreads();
  const Params& p = s_params;
  const int T = p.T, K = p.k, Et = p.E_total, I = p.I, H = p.H;
  const int G = H / kGroup;
  const size_t gwrow = static_cast<size_t>(H) * BITS / 32, gsrow = H / kGroup;
  const size_t dwrow = static_cast<size_t>(I) * BITS / 32, dsrow = I / kGroup;
  const int n_ch = I / 8;  // gate/up tasks per expert
  const int nq = I / 128;  // down K quarters
  uint2* lw = p.ws.lw;     // [T][Et + 1] logit words, one per 128-byte line
  uint2* hw = p.ws.hw;     // [T][K + 1][I] h words
  const uint32_t e_off = static_cast<uint32_t>(p.off), e_cnt = static_cast<uint32_t>(p.E);
  auto is_local = [&](uint32_t e) { return e - e_off < e_cnt; };
  // roles
  const int row_cta0 = NC - H / 16;  // CTAs [row_cta0, NC) own 16 output rows each
  const bool owns_rows = cta >= row_cta0;
  const int n0 = (cta - row_cta0) * 16;
  const uint32_t qmask = p.shared_qmask & ((1u << nq) - 1u);
  const bool has_shared = p.has_shared != 0;
  // the shared-expert gate/up tasks go to the last I/8 CTAs: routed tasks are
  // dealt round-robin from CTA 0, so the last CTAs have one fewer
  const int sg_task = cta - (NC - n_ch);
  const bool owns_sgu = !SK && has_shared && sg_task >= 0 && ((qmask >> ((sg_task * 8) / 128)) & 1u);
  const bool sh_down = !SK && owns_rows && has_shared && qmask != 0u;
  // split-K task of this CTA: a 32-channel slice j of a source.  One GPU:
  // CTAs [0, 16k) the routed slots' slices, then the shared expert's 16.
  // Expert parallel: first this rank's shared slices (j = rank, rank +
  // world, ...), then 16 per local routed slot (the m-th local slot for CTA
  // sk_rbase + 16 m + j; known after routing).  CTAs past the last task only
  // route (and combine).
  const int sk_nsh = (SK && has_shared) ? (EP ? kSkTasksPerSource / p.ep_world : kSkTasksPerSource) : 0;
  const int sk_rbase = EP ? sk_nsh : 0, sk_sbase = EP ? 0 : kSkTasksPerSource * K;
  const bool sk_shared = SK && cta >= sk_sbase && cta < sk_sbase + sk_nsh;
  const int sk_j = sk_shared ? (EP ? p.ep_rank + p.ep_world * (cta - sk_sbase) : cta - sk_sbase)
                             : (cta - sk_rbase) % kSkTasksPerSource;
  const int sk_m = (cta - sk_rbase) / kSkTasksPerSource;  // (routed) which local slot
  // one GPU: every slot is local, so CTA i < 16k takes slot i / 16 (static)
  const int sk_slot0 = (SK && !EP && cta < kSkTasksPerSource * K) ? sk_m : -1;
  using SD = SkDown<BITS>;
  // (split-K) TMA destinations, from the first 1024-byte boundary at or after
  // off_tma: up and gate codes, [tile 4][16 slices][8 rows][Tile2 row bytes]
  // each, their scales and biases, the down codes [H][slice bytes]
  constexpr uint32_t kSkGuBox = 16u * 32u * TL::kRowBytes;
  constexpr uint32_t kSkGuTile = kSkGuBox / kSkUnits;
  constexpr uint32_t kSkSbBox = 32u * 32u * 2u;  // 32 rows x H/64 groups (H = 2048)
  char* skb = sm + pl.off_tma + (1024u - (smem_u32(sm) + pl.off_tma) % 1024u) % 1024u;
  char* sGu = skb;
  const uint16_t* sGsb = reinterpret_cast<const uint16_t*>(skb + 2 * kSkGuBox);
  char* sDnA = skb + 2 * kSkGuBox + 4 * kSkSbBox;
  char* sDn = sDnA + static_cast<size_t>(warp) * SD::kBytes;  // (split-K) this warp's down rows
  uint32_t sk_sw[4], sk_bw[4];  // (split-K) this lane's down rows' scale and bias words
  // (split-K) the task's TMA requests, by lanes 0 .. kSkUnits of one warp,
  // each the sole arrival on its barrier: lane u < kSkUnits the codes of
  // gate/up tile u (lane 0 also the scales and biases), lane kSkUnits the
  // down codes
  auto sk_issue_tma = [&](bool shared, int e, int ln) {
    const int r0 = sk_j * kSkC;
    if (ln < kSkUnits) {
      const CUtensorMap* mw = shared ? &skm.sgu_w : &skm.gu_w;
      const uint32_t bu = smem_u32(&sk_bar[ln]);
      mbar_arrive_expect_tx(&sk_bar[ln], 2 * kSkGuTile + (ln == 0 ? 4 * kSkSbBox : 0u));
      tma_load_4d(smem_u32(sGu + ln * kSkGuTile), mw, 0, r0 + 8 * ln, 0, e, bu);
      tma_load_4d(smem_u32(sGu + kSkGuBox + ln * kSkGuTile), mw, 0, I + r0 + 8 * ln, 0, e, bu);
      if (ln == 0) {
        const CUtensorMap* msc = shared ? &skm.sgu_s : &skm.gu_s;
        const CUtensorMap* mbi = shared ? &skm.sgu_b : &skm.gu_b;
        tma_load_3d(smem_u32(sGsb), msc, 0, r0, e, bu);
        tma_load_3d(smem_u32(sGsb + 1 * kSkSbBox / 2), msc, 0, I + r0, e, bu);
        tma_load_3d(smem_u32(sGsb + 2 * kSkSbBox / 2), mbi, 0, r0, e, bu);
        tma_load_3d(smem_u32(sGsb + 3 * kSkSbBox / 2), mbi, 0, I + r0, e, bu);
      }
    } else if (ln == kSkUnits) {
      const CUtensorMap* md = shared ? &skm.sdn_w : &skm.dn_w;
      mbar_arrive_expect_tx(&sk_bar[kSkUnits], static_cast<uint32_t>(H) * SD::kRow);
      tma_load_4d(smem_u32(sDnA), md, sk_j * BITS, 0, 0, e, smem_u32(&sk_bar[kSkUnits]));
    }
  };
  const int j0 = owns_sgu ? 1 : 0;  // ring unit 0: this warp's slice of the shared-expert gate/up task
  auto gu_row = [&](int ch0) { return [=](int i) -> size_t { return i < 8 ? ch0 + i : I + ch0 + i - 8; }; };
  auto dn_row = [=](int i) -> size_t { return static_cast<size_t>(n0 + i); };

  // ---- prologue: weights only (before the programmatic-launch wait)
  RNB_TRACE_MARK(p, 0);
  // Router rows of this CTA: cta and cta + NC of the Et + 1 rows (the last is
  // the shared gate); warp w covers hidden [128 w, 128 w + 128), 4 values per
  // lane: 4 bf16, or (8-bit router) the word of 4 codes in .x and the group's
  // bf16 scale | bias << 16 in .y.
  const int k0r = warp * 128 + lane * 4;
  uint2 wr[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int row = cta + i * NC;
    const bool sh = row == Et && has_shared;
    if (p.router_q8) {
      const uint32_t* q = sh ? reinterpret_cast<const uint32_t*>(p.sgate_w)
                             : reinterpret_cast<const uint32_t*>(p.router_w) + static_cast<size_t>(row) * (H / 4);
      const uint16_t* sc = sh ? p.sgate_s : p.router_s + static_cast<size_t>(row) * (H / 64);
      const uint16_t* bi = sh ? p.sgate_b : p.router_b + static_cast<size_t>(row) * (H / 64);
      wr[i] = row < Et || sh ? make_uint2(__ldg(q + k0r / 4), static_cast<uint32_t>(__ldg(sc + k0r / 64)) |
                                                                 (static_cast<uint32_t>(__ldg(bi + k0r / 64)) << 16))
                             : make_uint2(0, 0);
    } else {
      const uint16_t* pr = row < Et ? p.router_w + static_cast<size_t>(row) * H : (sh ? p.sgate_w : nullptr);
      wr[i] = pr ? __ldg(reinterpret_cast<const uint2*>(pr + k0r)) : make_uint2(0, 0);
    }
  }
  if (owns_sgu)
    tile2_issue<BITS>(ring, p.sgu_w, p.sgu_s, p.sgu_b, gwrow, gsrow, warp * 2, gu_row(sg_task * 8), lane);
  cp_async_commit();  // group: shared gate/up slice (ring unit 0; may be empty)
  {
    // the router rows' norms (weights only): sum w^2 and sum |w| of rows
    // cta, cta + NC, per warp into ms->rnorm[warp][0..3]
    float v[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      double wd[4];
      router_quad(wr[i], p.router_q8 != 0, wd);
      const float wf[4] = {static_cast<float>(wd[0]), static_cast<float>(wd[1]), static_cast<float>(wd[2]),
                           static_cast<float>(wd[3])};
      v[i] = fmaf(wf[0], wf[0], fmaf(wf[1], wf[1], fmaf(wf[2], wf[2], wf[3] * wf[3])));
      v[2 + i] = (fabsf(wf[0]) + fabsf(wf[1])) + (fabsf(wf[2]) + fabsf(wf[3]));
    }
    const float r = warp_reduce_scatter4(v, lane, false);
    if ((lane & 7) == 0) ms->rnorm[warp][lane >> 3] = r;
  }
  if (sh_down && warp < nq && ((qmask >> warp) & 1u))
    tile2_issue<BITS>(sSdn + warp * TL::kBytes, p.sdn_w, p.sdn_s, p.sdn_b, dwrow, dsrow, warp * 2, dn_row, lane);
  cp_async_commit();  // group: this warp's shared-down quarter
  RNB_TRACE_MARK(p, 1);
  griddep_launch_dependents();
  griddep_wait();  // x (and the workspace) may come from the previous kernel on the stream
  RNB_TRACE_MARK(p, 2);
  if (tid == 0) ms->epoch = *reinterpret_cast<volatile uint32_t*>(p.ws.seq) + 1u;
  // this lane's router activations (tokens 0, 1), loaded together with the
  // sequence word: one round trip (the fused layer glue reads them below)
  uint2 xr[2] = {make_uint2(0, 0), make_uint2(0, 0)};
  if (!p.norm_w) {
#pragma unroll
    for (int t = 0; t < 2; ++t)
      if (t < T) xr[t] = *reinterpret_cast<const uint2*>(p.x + static_cast<size_t>(t) * H + k0r);
  }
  // Fused layer glue: this CTA's own copy of the normalised tokens.  The sum
  // of squares runs exactly as in rnb_add_rmsnorm (threads 0..255 striding by
  // 256, a shuffle tree, the 8 warp sums in order), so both paths give the
  // same bits.  CTA 0 also writes the residual sum and the normalised tokens.
  const uint16_t* xin = p.x;
  if (p.norm_w) {
    uint16_t* sXn = reinterpret_cast<uint16_t*>(sm + off_xn);
    for (int t = 0; t < T; ++t) {
      const size_t b = static_cast<size_t>(t) * H;
      if (tid < 256) {
        float ss = 0.f;
        for (int i = tid; i < H; i += 256) {
          float v = bf16_bits_to_f32(p.resid[b + i]);
          if (p.y_prev) v = bf16_round(v + bf16_bits_to_f32(p.y_prev[b + i]));
          sXn[b + i] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
          ss = fmaf(v, v, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((tid & 31) == 0) ms->red[tid >> 5] = ss;
      }
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) tot += ms->red[i];
      const float r = rsqrtf(tot / static_cast<float>(H) + p.norm_eps);
      for (int i = tid; i < H; i += blockDim.x) {
        const uint16_t rv = sXn[b + i];
        const uint16_t xn = __bfloat16_as_ushort(__float2bfloat16_rn(bf16_bits_to_f32(rv) * r * bf16_bits_to_f32(p.norm_w[i])));
        if (cta == 0) {
          p.resid_out[b + i] = rv;
          if (p.xn_out) p.xn_out[b + i] = xn;
        }
        sXn[b + i] = xn;
      }
      __syncthreads();
    }
    xin = sXn;
  }
  __syncthreads();
  const uint32_t epoch = ms->epoch;

  // ---- router: rows cta, cta + NC against tokens 0, 1
  {
    // Dots in fp64: bf16 products (and 8-bit dequantised weights s * code + b
    // and their products) are exact or within 2^-53, and the fp64 partial sums
    // err by at most ~2^-49 of sum |x_i w_i|, so the bf16 rounding of each
    // logit is certified (route_interval_f64) without an fp64 recompute in
    // routing.  Norms (for the certificate's bound) in fp32.
    float xf[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const uint2 xv = p.norm_w && t < T ? *reinterpret_cast<const uint2*>(xin + static_cast<size_t>(t) * H + k0r) : xr[t];
      xf[t][0] = __uint_as_float(xv.x << 16);
      xf[t][1] = __uint_as_float(xv.x & 0xFFFF0000u);
      xf[t][2] = __uint_as_float(xv.y << 16);
      xf[t][3] = __uint_as_float(xv.y & 0xFFFF0000u);
    }
    double dv[4];
    float v[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      double wd[4];
      router_quad(wr[i], p.router_q8 != 0, wd);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        double d = wd[0] * static_cast<double>(xf[t][0]);
        d = fma(wd[1], static_cast<double>(xf[t][1]), d);
        d = fma(wd[2], static_cast<double>(xf[t][2]), d);
        d = fma(wd[3], static_cast<double>(xf[t][3]), d);
        dv[2 * i + t] = d;
      }
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      v[t] = fmaf(xf[t][0], xf[t][0], fmaf(xf[t][1], xf[t][1], fmaf(xf[t][2], xf[t][2], xf[t][3] * xf[t][3])));
      v[2 + t] = fmaxf(fmaxf(fabsf(xf[t][0]), fabsf(xf[t][1])), fmaxf(fabsf(xf[t][2]), fabsf(xf[t][3])));
    }
    // lane 8q holds the warp's dot q = 2 * row + token and token statistic
    // q (sum x^2 of tokens 0, 1, then max |x| of tokens 0, 1)
    const double dq = warp_reduce_scatter4(dv, lane, false);
    const float xq = warp_reduce_scatter4(v, lane, true);
    if ((lane & 7) == 0) {
      ms->rdot[warp][lane >> 3] = dq;
      ms->rnorm[warp][4 + (lane >> 3)] = xq;
    }
    __syncthreads();
    // warp w < 4 finishes (row cta + (w >> 1) * NC, token w & 1): lanes 0..15
    // hold the 16 warps' partials, added by a fixed shuffle tree
    if (warp < 4) {
      const int i = warp >> 1, t = warp & 1, row = cta + i * NC;
      if (row <= Et && t < T) {
        const int w = lane & 15;
        double a0 = ms->rdot[w][2 * i + t];
        float a1 = ms->rnorm[w][i], a2 = ms->rnorm[w][2 + i], a3 = ms->rnorm[w][4 + t], a4 = ms->rnorm[w][6 + t];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
          a0 += __shfl_xor_sync(0xffffffffu, a0, o);
          a1 += __shfl_xor_sync(0xffffffffu, a1, o);
          a2 += __shfl_xor_sync(0xffffffffu, a2, o);
          a3 += __shfl_xor_sync(0xffffffffu, a3, o);
          a4 = fmaxf(a4, __shfl_xor_sync(0xffffffffu, a4, o));
        }
        // expert rows: candidate interval of the bf16 logit; last row: fp32 shared-gate logit
        if (lane == 0) {
          const uint32_t val = row < Et ? route_interval_f64(a0, a3, a4, a1, a2) : __float_as_uint(static_cast<float>(a0));
          xw_store(lw + (static_cast<size_t>(t) * (Et + 1) + row) * kLwStride, val, epoch);
        }
      }
    }
  }
  RNB_TRACE_MARK(p, 3);
  // (split-K) the shared expert's tasks know their weights: load them now,
  // once this CTA's router rows are out (they are on every CTA's path)
  if (sk_shared) {
    if (warp == 0) sk_issue_tma(true, 0, lane);
    sk_down_sb(p.sdn_s, p.sdn_b, I, warp * 128, sk_j, lane, sk_sw, sk_bw);
  }
  // (the B-fragment area is free until the down phase: 4 KB of it are xprep's scratch)
  xprep_cta<BITS>(xin, T, sX, sXs, ms->xinv, reinterpret_cast<__half*>(sm + off_hf), ms->red, !p.norm_w, xr[0],
                  xr[1]);
  RNB_TRACE_MARK(p, 4);

  // B operand of the gate/up MMAs: this lane's column g is entry ent[g].
  auto gateup_mma = [&](const char* slot, const uint32_t* ent, int ncols, float (&acc)[4]) {
    const int colB = g < ncols ? g : 0;
    const int tB = static_cast<int>(ent[colB] / (K + 1));
    const int t0 = static_cast<int>(ent[2 * c < ncols ? 2 * c : 0] / (K + 1));
    const int t1 = static_cast<int>(ent[2 * c + 1 < ncols ? 2 * c + 1 : 0] / (K + 1));
    const int g0 = warp * 2;
    tile2_mma<BITS>(
        slot, g, c,
        [&](int gi, uint32_t(&xb)[8]) {
          const uint32_t* src = sX + (static_cast<size_t>(tB) * G + g0 + gi) * 32 + c * 8;
          const uint4 u0 = reinterpret_cast<const uint4*>(src)[0];
          const uint4 u1 = reinterpret_cast<const uint4*>(src)[1];
          xb[0] = u0.x; xb[1] = u0.y; xb[2] = u0.z; xb[3] = u0.w;
          xb[4] = u1.x; xb[5] = u1.y; xb[6] = u1.z; xb[7] = u1.w;
        },
        [&](int gi, int col) { return sXs[(col ? t1 : t0) * G + g0 + gi]; }, [](int, int) { return 1.0f; }, acc);
  };
  // partials of this warp for task m: lanes c == 0 hold columns 0, 1
  auto store_partials = [&](int m, const float (&acc)[4]) {
    if (c == 0) {
      float* rw = sRed + (m * kPWarps + warp) * 32;
      rw[g * 2] = acc[0];
      rw[g * 2 + 1] = acc[1];
      rw[(g + 8) * 2] = acc[2];
      rw[(g + 8) * 2 + 1] = acc[3];
    }
  };

  __shared__ uint32_t s_ent[kPMaxMine + 1][kPMaxT];
  __shared__ int s_ncols[kPMaxMine + 1], s_ch0[kPMaxMine + 1];

  // ---- routing (every CTA, redundantly): poll the logit words
  {
    const uint64_t deadline = gtimer() + kSpinLimitNs;
    for (int i = tid; i < T * (Et + 1); i += blockDim.x)
      sIvl[i] = xw_wait(lw + static_cast<size_t>(i) * kLwStride, epoch, deadline, p.ws.status);
  }
  __syncthreads();
  RNB_TRACE_MARK(p, 6);
  if (warp < T) {
    const int t = warp;
    int e;
    float sc;
    const int nre = warp_route_token_body(sIvl + t * (Et + 1), Et, K, xin + static_cast<size_t>(t) * H, router_src(p), H,
                                          lane, false, nullptr, &e, &sc);
#ifdef RNB_TRACE
    if (t == 0 && lane == 0) trace_value(p, 31, nre);
#else
    (void)nre;
#endif
    RNB_TRACE_MARK(p, 18);
    if (lane < K) {
      ms->inds[t][lane] = static_cast<uint32_t>(e);
      ms->scores[t][lane] = sc;
    }
    if (lane == 0) ms->sg[t] = p.has_shared ? 1.0f / (1.0f + expf(-__uint_as_float(sIvl[t * (Et + 1) + Et]))) : 0.f;
    if (SK) {
      // (split-K, one token) the routing warp issues this CTA's loads; expert
      // parallel, it first finds the CTA's routed slot (the sk_m-th slot
      // whose expert is on this GPU)
      int slot = sk_slot0;
      if (EP) {
        const uint32_t lmask = __ballot_sync(0xffffffffu, lane < K && is_local(static_cast<uint32_t>(e)));
        uint32_t mm = lmask;
        for (int i = 0; i < sk_m; ++i) mm &= mm - 1u;
        slot = (!sk_shared && cta >= sk_rbase && sk_m < kPMaxK && mm) ? __ffs(mm) - 1 : -1;
        if (lane == 0) {
          ms->sk_slot = slot;
          ms->sk_lmask = lmask;
        }
      }
      const int es = __shfl_sync(0xffffffffu, e, slot >= 0 ? slot : 0);
      RNB_TRACE_MARK(p, 21);
      if (slot >= 0) sk_issue_tma(false, es - p.off, lane);
      RNB_TRACE_MARK(p, 22);
    }
    // the routing warps meet (warp 0 reads every token's selection); the
    // rest of the CTA waits at the one CTA barrier below
    if (T > 1)
      asm volatile("bar.sync 1, %0;\n" ::"r"(32 * T) : "memory");
    else
      __syncwarp();
  }
  RNB_TRACE_MARK(p, 7);
  // Warp 0: the active local experts in (token, slot) order of first use,
  // with their columns (lane i < T*K holds entry i; lanes holding the same
  // expert find each other with one match, the expert's index is the number
  // of first occurrences before its first lane), then the CTA's task list
  // (the h-exchange form only).
  if (!SK && warp == 0) {
    const bool act = lane < T * K;
    const uint32_t e = act ? ms->inds[lane / K][lane % K] : 0xFFFFFFFFu;
    const bool loc = act && is_local(e);
    const uint32_t same = __match_any_sync(0xffffffffu, e);
    const uint32_t below = (1u << lane) - 1u;
    const bool first = loc && (same & below) == 0u;
    const uint32_t firsts = __ballot_sync(0xffffffffu, first);
    const int lead = __ffs(same) - 1;
    const int a = __popc(firsts & ((1u << lead) - 1u));
    if (loc) {
      ms->act_ent[a][__popc(same & below)] = static_cast<uint32_t>((lane / K) * (K + 1) + lane % K);
      if (first) {
        ms->act_e[a] = e - static_cast<uint32_t>(p.off);
        ms->act_cnt[a] = static_cast<uint32_t>(__popc(same));
      }
    }
    if (lane == 0) ms->n_act = static_cast<uint32_t>(__popc(firsts));
    __syncwarp();
    // this CTA's routed gate/up tasks m < mine: task i = cta + m NC
    const int nb = __popc(firsts) * n_ch;
    const int mn = nb > cta ? (nb - cta + NC - 1) / NC : 0;
    if (lane < mn) {
      const int i = cta + lane * NC, a2 = i / n_ch;
      const int cnt = static_cast<int>(ms->act_cnt[a2]);
      s_ncols[lane] = cnt;
      s_ch0[lane] = (i % n_ch) * 8;
      for (int n = 0; n < kPMaxT; ++n) s_ent[lane][n] = ms->act_ent[a2][n < cnt ? n : 0];
    }
    if (lane < kPMaxT) s_ent[kPMaxMine][lane] = static_cast<uint32_t>((lane < T ? lane : 0) * (K + 1) + K);
  }
  __syncthreads();
  RNB_TRACE_MARK(p, 20);
  const int n_act = static_cast<int>(ms->n_act);
  if (cta == 0 && tid < T * K) {
    const int t = tid / K, s = tid % K;
    if (p.inds_out) p.inds_out[tid] = ms->inds[t][s];
    if (p.scores_out) p.scores_out[tid] = ms->scores[t][s];
  }

  bool timed_out = false;
  if constexpr (SK) {
    // ---- split-K (one token): this CTA's task, then the combine of its rows
    const int ntask = kSkTasksPerSource * (K + (has_shared ? 1 : 0));
    uint2* yw = p.ws.yw;  // [task][H] weighted partial words (task g: slot g / 16, slice g % 16)
    const int sk_slot = EP ? ms->sk_slot : sk_slot0;
    const uint32_t sk_lmask = EP ? ms->sk_lmask : 0u;
    const bool sk_task = sk_shared || sk_slot >= 0;
    // the tasks on this GPU: its routed slots' slices, and its shared slices
    // (one GPU: all of them)
    auto task_here = [&](int t) {
      if (!EP) return true;
      if (t < kSkTasksPerSource * K) return ((sk_lmask >> (t / kSkTasksPerSource)) & 1u) != 0u;
      const int j = t - kSkTasksPerSource * K;
      return has_shared && j < kSkTasksPerSource && (!EP || j % p.ep_world == p.ep_rank);
    };
    if (sk_task) {
      float wgt = ms->sg[0];
      if (!sk_shared) {
        // (the TMA requests went out from the routing warp)
        const uint32_t le = ms->inds[0][sk_slot] - static_cast<uint32_t>(p.off);
        const size_t dse = static_cast<size_t>(H) * dsrow;
        wgt = ms->scores[0][sk_slot];
        sk_down_sb(p.dn_s + le * dse, p.dn_b + le * dse, I, warp * 128, sk_j, lane, sk_sw, sk_bw);
      }
      // gate/up: the four 8-channel tiles, each once its TMA loads are in
      RNB_TRACE_MARK(p, 9);
      // the token's B fragments and group sums of this warp's two groups,
      // the same for every tile
      const int g0 = warp * 2;
      uint32_t xbr[2][8];
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const uint4* src = reinterpret_cast<const uint4*>(sX + static_cast<size_t>(g0 + gi) * 32 + c * 8);
        const uint4 u0 = src[0], u1 = src[1];
        xbr[gi][0] = u0.x; xbr[gi][1] = u0.y; xbr[gi][2] = u0.z; xbr[gi][3] = u0.w;
        xbr[gi][4] = u1.x; xbr[gi][5] = u1.y; xbr[gi][6] = u1.z; xbr[gi][7] = u1.w;
      }
      const float xs0 = sXs[g0], xs1 = sXs[g0 + 1];
#pragma unroll
      for (int u = 0; u < kSkUnits; ++u) {
        if (!mbar_wait(&sk_bar[u], 0, kSpinLimitNs)) timed_out = true;
        if (u == 0) RNB_TRACE_MARK(p, 10);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        sk_gu_mma<BITS>(
            sGu, sGu + kSkGuBox, sGsb, G, u, warp, g, c,
            [&](int gi, uint32_t(&xb)[8]) {
#pragma unroll
              for (int i = 0; i < 8; ++i) xb[i] = gi ? xbr[1][i] : xbr[0][i];
            },
            [&](int gi, int) { return gi ? xs1 : xs0; }, [](int, int) { return 1.0f; }, acc);
        store_partials(u, acc);
      }
      RNB_TRACE_MARK(p, 11);
      __syncthreads();
      // SwiGLU of the slice's 32 channels (warp 0, lane = channel), its fp16
      // form with one power-of-two scale, and the down MMAs' B pairs
      if (warp == 0) {
        const int u = lane >> 3, r = lane & 7;
        float up = 0.f, gate = 0.f;
#pragma unroll
        for (int w = 0; w < kPWarps; ++w) {
          up += sRed[(u * kPWarps + w) * 32 + r * 2];
          gate += sRed[(u * kPWarps + w) * 32 + (8 + r) * 2];
        }
        up *= ms->xinv[0];
        gate *= ms->xinv[0];
        const float h = (gate / (1.0f + expf(-gate))) * up;
        float sc, inv;
        fp16_range_scale(warp_max(fabsf(h)), sc, inv);
        const __half hh = __float2half_rn(h * sc);
        const float hs = warp_sum(__half2float(hh));
        const uint32_t hb = __half_as_ushort(hh);
        // lane t < 16: pair (c = t / 4, i = t % 4) of the positions a lane c
        // of a quad holds (its codes 8c .. 8c + 7): (8c + i, 8c + i + 4) at 4
        // bits, odd pairs times 1/16 (they meet codes times 16); (8c + 2i,
        // 8c + 2i + 1) at 8 bits
        const int cq = (lane >> 2) & 3, ip = lane & 3;
        const int plo = BITS == 8 ? 8 * cq + 2 * ip : 8 * cq + ip, phi = BITS == 8 ? plo + 1 : plo + 4;
        __half lo = __ushort_as_half(static_cast<uint16_t>(__shfl_sync(0xffffffffu, hb, plo)));
        __half hi = __ushort_as_half(static_cast<uint16_t>(__shfl_sync(0xffffffffu, hb, phi)));
        if (BITS == 4 && (ip & 1)) {
          lo = __hmul(lo, __float2half_rn(0.0625f));
          hi = __hmul(hi, __float2half_rn(0.0625f));
        }
        if (lane < 16)
          ms->skbt[lane] = static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
        if (lane == 0) {
          ms->skhs = hs;
          ms->skhinv = inv;
        }
      }
      if (!mbar_wait(&sk_bar[kSkUnits], 0, kSpinLimitNs)) timed_out = true;  // the down codes
      __syncthreads();
      RNB_TRACE_MARK(p, 12);
      const int gtask = sk_shared ? kSkTasksPerSource * K + sk_j : kSkTasksPerSource * sk_slot + sk_j;
      uint2* ydst = yw + static_cast<size_t>(gtask) * H + warp * 128;
      sk_down_mma<BITS>(sDn, sk_sw, sk_bw, ms->skbt, ms->skhs, ms->skhinv, sk_j, g, c,
                        [&](int r, float v) { xw_store(ydst + r, __float_as_uint(v * wgt), epoch); });
      RNB_TRACE_MARK(p, 14);
    }
    if (cta < H / 16) {
      // rows [16 cta, 16 cta + 16): warp w takes tasks [tpw w, tpw w + tpw),
      // whose 16-row words are one 128-byte line each: lanes 0-15 read rows
      // 0-15 of one task, lanes 16-31 of the next (all polled together,
      // bounded); each warp's row sums (its tasks in order) then add up
      // over the warps in order
      constexpr int kMaxPer = (kSkTasksPerSource * (kPMaxK + 1) + 31) / 32;
      const int tpw = (ntask + kPWarps - 1) / kPWarps;
      const int rr = lane & 15;
      uint64_t wv[kMaxPer];
      auto word_of = [&](int k2) {
        const int q = lane + 32 * k2, t = warp * tpw + (q >> 4);
        return (q >> 4) < tpw && t < ntask && task_here(t) ? yw + static_cast<size_t>(t) * H + 16 * cta + rr
                                                             : nullptr;
      };
#pragma unroll
      for (int k2 = 0; k2 < kMaxPer; ++k2) {
        const uint2* w = word_of(k2);
        wv[k2] = w ? xw_load(w) : (static_cast<uint64_t>(epoch) << 32);
      }
      const uint64_t deadline = gtimer() + kSpinLimitNs;
      for (;;) {
        bool all = true;
#pragma unroll
        for (int k2 = 0; k2 < kMaxPer; ++k2) {
          if (static_cast<uint32_t>(wv[k2] >> 32) != epoch) {
            all = false;
            wv[k2] = xw_load(word_of(k2));
          }
        }
        const bool late = !all && gtimer() > deadline;
        if (late) timed_out = true;
        if (__all_sync(0xffffffffu, all || late)) break;
        __nanosleep(32);
      }
      RNB_TRACE_MARK(p, 23);
      float acc = 0.f;
#pragma unroll
      for (int k2 = 0; k2 < kMaxPer; ++k2)
        if (word_of(k2)) acc += __uint_as_float(static_cast<uint32_t>(wv[k2]));
      acc += __shfl_xor_sync(0xffffffffu, acc, 16);  // lanes r and r + 16 hold the same row
      if (lane < 16) sRed[warp * 16 + lane] = acc;
      __syncthreads();
      auto emit = [&](int, int r, float v) {
        const size_t o = static_cast<size_t>(16 * cta + r);
        if (p.y_f32)
          static_cast<float*>(p.out)[o] = v;
        else
          static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
      };
      if (tid < 16) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kPWarps; ++w) sum += sRed[w * 16 + tid];
        if (EP)
          sRed[kPWarps * 16 + tid] = sum;  // this rank's part of the rows
        else
          emit(0, tid, sum);
      }
      if (EP) {
        // expert parallel: the ranks' parts of the 16 rows over NVLink,
        // added in rank order
        __syncthreads();
        ep_exchange_tile(p, 16 * cta, 1, [&](int, int r) { return sRed[kPWarps * 16 + r]; }, emit);
      }
      RNB_TRACE_MARK(p, 19);
    }
  } else {

  // ---- this CTA's work.  Every warp streams, in this order, its units
  // through its own ring of S shared-memory slots (unit j in slot j % S,
  // issued once unit j - S has been consumed; one cp.async group each):
  //   [its slice of the shared-expert gate/up task (CTAs < I/8)], its slices
  //   of the routed gate/up tasks m < mine (task i = cta + m NC: expert
  //   i / (I/8), channels 8 (i % (I/8))), then its down pairs (routed source,
  //   quarter) k = warp, warp + 16, ... of this CTA's rows.  The gate/up
  //   slices go out first (the down weights are needed only after every
  //   CTA's gate/up is done); the shared expert's down quarters were loaded
  //   in the prologue.
  const int n_btask = n_act * n_ch;
  const int mine = n_btask > cta ? (n_btask - cta + NC - 1) / NC : 0;  // <= kPMaxMine (host-checked)
  const int n_rpair = owns_rows ? n_act * nq : 0;  // routed down pairs of the CTA
  const int my_down = n_rpair > warp ? (n_rpair - warp + kPWarps - 1) / kPWarps : 0;
  const int n_units = j0 + mine + my_down;
  auto issue = [&](int j) {  // unit j of this warp (j >= j0)
    char* slot = ring + (j % S) * TL::kBytes;
    const int u = j - j0;
    if (u < mine) {
      const int i = cta + u * NC, a = i / n_ch;
      const uint32_t le = ms->act_e[a];
      const size_t ew = static_cast<size_t>(2) * I * gwrow, es = static_cast<size_t>(2) * I * gsrow;
      tile2_issue<BITS>(slot, p.gu_w + le * ew, p.gu_s + le * es, p.gu_b + le * es, gwrow, gsrow, warp * 2,
                        gu_row((i % n_ch) * 8), lane);
    } else {
      const int q = warp + (u - mine) * kPWarps, a = q / nq, qq = q % nq;
      const uint32_t le = ms->act_e[a];
      const size_t ew = static_cast<size_t>(H) * dwrow, es = static_cast<size_t>(H) * dsrow;
      tile2_issue<BITS>(slot, p.dn_w + le * ew, p.dn_s + le * es, p.dn_b + le * es, dwrow, dsrow, qq * 2, dn_row,
                        lane);
    }
  };
  RNB_TRACE_MARK(p, 21);
  int issued = j0;  // next unit to issue (unit 0, the shared slice, went out in the prologue)
  for (; issued < j0 + mine && issued < S; ++issued) {
    issue(issued);
    cp_async_commit();
  }
  RNB_TRACE_MARK(p, 22);
  // unit j: at most (issued - 1 - j) younger groups may stay pending
  auto wait_unit = [&](int j) {
    cp_async_wait_pending(issued - 1 - j);
    __syncwarp();
  };
  auto refill = [&]() {  // the slot of the unit just consumed is free again
    __syncwarp();
    if (issued < n_units) issue(issued);
    cp_async_commit();  // (an empty group keeps the pending count exact)
    ++issued;
  };

  // ---- the shared-expert gate/up task (unit 0), loaded since the prologue
  if (owns_sgu) {
    cp_async_wait_pending(issued - j0 + 1);  // its group is older than the shared-down group and the ring's
    __syncwarp();
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    gateup_mma(ring, s_ent[kPMaxMine], T, acc);
    store_partials(0, acc);  // red slot 0; the routed tasks use 1 .. mine
  }
  RNB_TRACE_MARK(p, 5);

  // ---- routed gate/up: each slice as it arrives; its slot takes the
  // warp's next unit at once
  RNB_TRACE_MARK(p, 8);
  for (int m = 0; m < mine; ++m) {
    const int j = j0 + m;
    wait_unit(j);
    if (m == 0) RNB_TRACE_MARK(p, 9);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    gateup_mma(ring + (j % S) * TL::kBytes, s_ent[m], s_ncols[m], acc);
    store_partials(m + 1, acc);
    refill();
    if (m == 0) RNB_TRACE_MARK(p, 10);
  }
  // the remaining down units, into the slots still free (unit j takes slot
  // j % S once unit j - S has been consumed: every unit below j0 + mine has
  // been; the plan gives S >= 1 + the warp's down units, so all fit)
  for (; issued < n_units && issued < j0 + mine + S; ++issued) {
    issue(issued);
    cp_async_commit();
  }
  RNB_TRACE_MARK(p, 11);
  __syncthreads();
  p_gateup_epilogue(p, sRed + kPWarps * 32, mine, &s_ent[0][0], s_ncols, s_ch0, ms->xinv, hw, epoch);
  if (owns_sgu && tid >= 256 && tid < 256 + 16 * T) {
    // threads of the upper half publish the shared task (red slot 0)
    const int q = tid - 256;
    const float* rt = sRed;
    const int r = (q >> 1) & 7, n = q & 1;
    float up = 0.f, gate = 0.f;
#pragma unroll
    for (int w = 0; w < kPWarps; ++w) {
      up += rt[w * 32 + r * 2 + n];
      gate += rt[w * 32 + (8 + r) * 2 + n];
    }
    const uint32_t id = static_cast<uint32_t>(n * (K + 1) + K);
    up *= ms->xinv[n];
    gate *= ms->xinv[n];
    xw_store(hw + static_cast<size_t>(id) * I + sg_task * 8 + r, __float_as_uint((gate / (1.0f + expf(-gate))) * up),
             epoch);
  }
  RNB_TRACE_MARK(p, 12);

  if (!owns_rows) {
    cp_async_wait_pending(0);
  } else {
    // ---- down projection of rows [n0, n0 + 16).  First the whole CTA polls
    // every h word it needs (each warp until its own words are in) and
    // converts it once: thread c takes 8-channel
    // chunks c, c + 512, ... of the T (K + 1) entries (an entry's channels
    // are 64 chunks; a 64-group is 8 chunks on 8 neighbouring lanes), with
    // one power-of-two fp16 scale per (entry, group) (fp16_range_scale) and
    // the group's sum, into the B fragments sHE[entry][group][32].  Entries
    // whose expert is not on this rank, and shared-expert quarters outside
    // this rank's share, are never produced and are skipped.  Then each warp
    // runs its pairs (source, quarter): the shared expert's quarter `warp`
    // (tile in sSdn) and the routed pairs of its ring units.
    const uint64_t deadline = gtimer() + kSpinLimitNs;
    const bool sh_unit = sh_down && warp < nq && ((qmask >> warp) & 1u);
    const int n_du = (sh_unit ? 1 : 0) + my_down;
    const int n_ent = T * (K + 1), cpe = I / 8;  // entries, chunks per entry
    uint32_t* sHE = reinterpret_cast<uint32_t*>(sm + off_hf);
    float* sHs = reinterpret_cast<float*>(sHE + static_cast<size_t>(n_ent) * (I / 64) * 32);
    float* sHi = sHs + n_ent * (I / 64);
    RNB_TRACE_MARK(p, 13);
    {
      constexpr int kMaxRounds = (kPMaxT * (kPMaxK + 1) * 64 + 32 * kPWarps - 1) / (32 * kPWarps);
      uint64_t wv[kMaxRounds][8];
      bool need[kMaxRounds];
#pragma unroll
      for (int r = 0; r < kMaxRounds; ++r) {
        const int ch = tid + r * 32 * kPWarps, en = ch / cpe, k8 = ch % cpe;
        bool nd = ch < n_ent * cpe;
        if (nd) {
          const int t = en / (K + 1), sl = en % (K + 1);
          nd = sl < K ? is_local(ms->inds[t][sl]) : (sh_down && ((qmask >> (k8 / 16)) & 1u));
        }
        need[r] = nd;
#pragma unroll
        for (int j = 0; j < 8; ++j) wv[r][j] = static_cast<uint64_t>(epoch) << 32;  // (never polled)
        if (nd) {
          const uint2* src = hw + static_cast<size_t>(en) * I + k8 * 8;
#pragma unroll
          for (int j = 0; j < 8; j += 2) xw_load2(src + j, wv[r][j], wv[r][j + 1]);
        }
      }
      // words that did not yet carry this call's epoch are polled again, all
      // of them per round trip, until they do (bounded)
#ifdef RNB_TRACE
      int polls = 0;
#endif
      for (;;) {
#ifdef RNB_TRACE
        ++polls;
#endif
        bool all = true;
#pragma unroll
        for (int r = 0; r < kMaxRounds; ++r) {
          const int ch = tid + r * 32 * kPWarps;
          const uint2* src = hw + static_cast<size_t>(ch / cpe) * I + (ch % cpe) * 8;
#pragma unroll
          for (int j = 0; j < 8; j += 2)
            if (need[r] && (static_cast<uint32_t>(wv[r][j] >> 32) != epoch ||
                            static_cast<uint32_t>(wv[r][j + 1] >> 32) != epoch)) {
              all = false;
              xw_load2(src + j, wv[r][j], wv[r][j + 1]);
            }
        }
        // the warp leaves together (its lanes share 64-groups): once every
        // lane has its words or is past the deadline (then the results are
        // void; stale words are used as they are)
        const bool late = !all && gtimer() > deadline;
        if (late) timed_out = true;
        if (__all_sync(0xffffffffu, all || late)) break;
        __nanosleep(32);
      }
#ifdef RNB_TRACE
      RNB_TRACE_MARK(p, 23);
      if (tid == 0) trace_value(p, 30, polls);
#endif
      // convert: the 8 lanes of a 64-group share its scale and sum
#pragma unroll
      for (int r = 0; r < kMaxRounds; ++r) {
        const int ch = tid + r * 32 * kPWarps;
        if (r * 32 * kPWarps >= n_ent * cpe) break;  // CTA-uniform
        float hv[8];
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          hv[j] = need[r] ? __uint_as_float(static_cast<uint32_t>(wv[r][j])) : 0.f;
          m = fmaxf(m, fabsf(hv[j]));
        }
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        float sc, inv;
        fp16_range_scale(m, sc, inv);
        const int en = ch / cpe, k8 = ch % cpe, grp = k8 >> 3;
        float part = 0.f;
        __half hh[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          hh[j] = __float2half_rn(hv[j] * sc);
          part += __half2float(hh[j]);
        }
        // The chunk's 8 values fill 4 consecutive fragment words (pair_slot
        // of positions 8 (k8 % 8) + j): word cq 8 + 4 (k8 % 2) + w holds
        // values (w, w + 4) at 4 bits, (2w, 2w + 1) at 8 bits.  4-bit pairs
        // 1 and 3 of a word (odd w) meet codes times 16 (subnormal form).
        const int qk = (k8 & 7) >> 1;
        const int cq = BITS == 8 ? qk : ((qk == 1) ? 2 : (qk == 2) ? 1 : qk);
        uint32_t wd[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          __half lo = BITS == 8 ? hh[2 * w] : hh[w], hi = BITS == 8 ? hh[2 * w + 1] : hh[w + 4];
          if (BITS == 4 && (w & 1)) {
            lo = __hmul(lo, __float2half_rn(0.0625f));
            hi = __hmul(hi, __float2half_rn(0.0625f));
          }
          wd[w] = static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
        }
        if (ch < n_ent * cpe)
          *reinterpret_cast<uint4*>(sHE + (static_cast<size_t>(en) * (I / 64) + grp) * 32 + cq * 8 + 4 * (k8 & 1)) =
              make_uint4(wd[0], wd[1], wd[2], wd[3]);
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        part += __shfl_xor_sync(0xffffffffu, part, 4);
        if ((k8 & 7) == 0 && ch < n_ent * cpe) {
          sHs[en * (I / 64) + grp] = part;
          sHi[en * (I / 64) + grp] = inv;
        }
      }
    }
    cp_async_wait_pending(0);  // every tile of this warp (the shared-down group and the ring units)
    __syncthreads();
    RNB_TRACE_MARK(p, 14);
    // unit b of this warp: tile, quarter, columns
    auto unit_of = [&](int b, const char*& tile, int& qq, uint32_t (&ent)[kPMaxT], int& ncols) {
      if (sh_unit && b == 0) {
        tile = sSdn + warp * TL::kBytes;
        qq = warp;
        ncols = T;
#pragma unroll
        for (int n = 0; n < kPMaxT; ++n) ent[n] = static_cast<uint32_t>((n < T ? n : 0) * (K + 1) + K);
      } else {
        const int u = b - (sh_unit ? 1 : 0);
        const int jj = j0 + mine + u, q = warp + u * kPWarps, a = q / nq;
        tile = ring + (jj % S) * TL::kBytes;
        qq = q % nq;
        ncols = static_cast<int>(ms->act_cnt[a]);
#pragma unroll
        for (int n = 0; n < kPMaxT; ++n) ent[n] = ms->act_ent[a][n < ncols ? n : 0];
      }
    };
#pragma unroll 1
    for (int b = 0; b < n_du; ++b) {
      const char* tile;
      int qq, nc;
      uint32_t ent[kPMaxT];
      unit_of(b, tile, qq, ent, nc);
      const int colB = g < nc ? g : 0;
      const uint32_t* fB = sHE + (static_cast<size_t>(ent[colB]) * (I / 64) + 2 * qq) * 32 + c * 8;
      const int h0 = static_cast<int>(ent[0]) * (I / 64) + 2 * qq;
      const int h1 = static_cast<int>(ent[nc > 1 ? 1 : 0]) * (I / 64) + 2 * qq;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      tile2_mma<BITS>(
          tile, g, c,
          [&](int gi, uint32_t(&xb)[8]) {
            const uint4 u0 = reinterpret_cast<const uint4*>(fB + gi * 32)[0];
            const uint4 u1 = reinterpret_cast<const uint4*>(fB + gi * 32)[1];
            xb[0] = u0.x; xb[1] = u0.y; xb[2] = u0.z; xb[3] = u0.w;
            xb[4] = u1.x; xb[5] = u1.y; xb[6] = u1.z; xb[7] = u1.w;
          },
          [&](int gi, int col) { return (c == 0 && col < nc) ? sHs[(col ? h1 : h0) + gi] : 0.f; },
          [&](int gi, int col) { return (c == 0 && col < nc) ? sHi[(col ? h1 : h0) + gi] : 0.f; }, acc);
      if (c == 0) {
#pragma unroll
        for (int n = 0; n < kPMaxT; ++n) {
          if (n < nc) {
            float* dst = sRedC + (static_cast<size_t>(ent[n]) * nq + qq) * 16;
            dst[g] = n == 0 ? acc[0] : acc[1];
            dst[g + 8] = n == 0 ? acc[2] : acc[3];
          }
        }
      }
    }
    RNB_TRACE_MARK(p, 15);
    __syncthreads();
    RNB_TRACE_MARK(p, 16);
    // Ordered weighted sum per (token, row), four lanes per output: lane j
    // of the four takes sources s = j, j + 4, ... (slot order; source K is the
    // shared expert), each the sum of its quarters in order; then the four
    // partial sums are added in a fixed tree.
    float acc = 0.f;
    if (tid < 64 * T) {
      const int o = tid >> 2, jl = tid & 3, t = o >> 4, r = o & 15;
      for (int s3 = jl; s3 <= K; s3 += 4) {
        float wgt;
        uint32_t qm;
        if (s3 < K) {
          if (!is_local(ms->inds[t][s3])) continue;
          wgt = ms->scores[t][s3];
          qm = (1u << nq) - 1u;
        } else {
          if (!sh_down) continue;
          wgt = ms->sg[t];
          qm = qmask;
        }
        const float* y = sRedC + static_cast<size_t>(t * (K + 1) + s3) * nq * 16 + r;
        float ys = 0.f;
        for (int q2 = 0; q2 < nq; ++q2)
          if ((qm >> q2) & 1u) ys += y[q2 * 16];
        acc = fmaf(wgt, ys, acc);
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    RNB_TRACE_MARK(p, 19);
    void* const out = p.out;
    const bool y_f32 = p.y_f32 != 0;
    auto emit = [&](int t, int r, float v) {
      const size_t o = static_cast<size_t>(t) * H + n0 + r;
      if (y_f32)
        static_cast<float*>(out)[o] = v;
      else
        static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(v);
    };
    if (EP) {
      float* stage = sRed;  // this tile's partials, [t][r]
      __syncthreads();
      if (tid < 64 * T && (tid & 3) == 0) stage[tid >> 2] = acc;
      __syncthreads();
      ep_exchange_tile(p, n0, T, [&](int t, int r) { return stage[t * 16 + r]; }, emit);
    } else if (tid < 64 * T && (tid & 3) == 0) {
      emit(tid >> 6, (tid >> 2) & 15, acc);
    }
  }
  }  // h-exchange form
  RNB_TRACE_MARK(p, 17);
  if (timed_out) atomicOr(p.ws.status, RNB_STATUS_TIMEOUT);

  // ---- exit: the last CTA out advances the sequence word
  __syncthreads();
  if (tid == 0) {
    uint32_t* seq = p.ws.seq;
    if (atomicAdd(seq + 1, 1u) == static_cast<uint32_t>(NC - 1)) {
      seq[1] = 0u;
      seq[0] = epoch;
      if (EP) p.ep_seq[0] += 1;  // every CTA's exchange is done
      __threadfence();
    }
  }
}

// ------------------------------------------------------------- host

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct Layout {
  size_t xperm, xsum, xinv, logit, inds, scores, sgate, nact, rec, entries, h,
      hmax, yws, ctr, status, xchg, total;
};

Layout make_layout(const rnb_moe_desc& d) {
  const size_t T = kMaxDecodeT, H = d.H, I = d.I, E = d.E, K = d.k, G = H / kGroup;
  Layout L;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align256(o + bytes);
    return at;
  };
  L.status = take(4);                // offset 0: rnb_moe_status reads it without a descriptor
  L.ctr = take(ws_counter_bytes(d));  // arrival counters, back to zero after every call
  L.xchg = take(kXchgBytes);          // persistent kernel's exchange words (same offset in every layout)
  L.xperm = take(T * H * 2);
  L.xsum = take(T * G * 4);
  L.xinv = take(T * 4);
  L.logit = take(T * (d.E_total + 1) * 4);
  L.inds = take(T * K * 4);
  L.scores = take(T * K * 4);
  L.sgate = take(T * 4);
  L.nact = take(4);
  L.rec = take(E * kRecWords * 4);
  L.entries = take(T * K * 4);
  L.h = take(T * (K + 1) * I * 4);
  L.hmax = take(T * (K + 1) * (I / 8) * 4);
  L.yws = take(T * (K + 1) * H * 4);
  L.total = o;
  static_assert(kWsCountersOffset == 256, "status word takes the first 256-byte slot");
  return L;
}

Ws bind(const Layout& L, void* ws) {
  char* b = static_cast<char*>(ws);
  Ws w;
  w.xperm = reinterpret_cast<uint32_t*>(b + L.xperm);
  w.xsum = reinterpret_cast<float*>(b + L.xsum);
  w.xinv = reinterpret_cast<float*>(b + L.xinv);
  w.logit = reinterpret_cast<float*>(b + L.logit);
  w.inds = reinterpret_cast<uint32_t*>(b + L.inds);
  w.scores = reinterpret_cast<float*>(b + L.scores);
  w.sgate = reinterpret_cast<float*>(b + L.sgate);
  w.nact = reinterpret_cast<uint32_t*>(b + L.nact);
  w.rec = reinterpret_cast<uint32_t*>(b + L.rec);
  w.entries = reinterpret_cast<uint32_t*>(b + L.entries);
  w.h = reinterpret_cast<float*>(b + L.h);
  w.hmaxp = reinterpret_cast<float*>(b + L.hmax);
  w.yws = reinterpret_cast<float*>(b + L.yws);
  w.ctr = reinterpret_cast<uint32_t*>(b + L.ctr);
  w.status = reinterpret_cast<uint32_t*>(b + L.status);
  w.seq = reinterpret_cast<uint32_t*>(b + L.status + kWsSeqOffset);
  w.lw = reinterpret_cast<uint2*>(b + L.xchg);
  w.hw = w.lw + kXchgLogitWords;
  w.yw = w.hw + kXchgHWords;
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int validate(const rnb_moe_desc* d, bool need_router, bool need_bank) {
  if (!d) return fail(RNB_ERR_INVALID, "descriptor is NULL");
  if (d->bits != 4 && d->bits != 8) return fail(RNB_ERR_INVALID, "bits must be 4 or 8");
  if (d->group != kGroup) return fail(RNB_ERR_INVALID, "group size must be 64");
  if (d->T < 0) return fail(RNB_ERR_INVALID, "T must be >= 0");
  if (d->H <= 0 || d->H % 512 || d->H > 2048)
    return fail(RNB_ERR_INVALID, "H must be 512, 1024, 1536 or 2048");
  if (d->I <= 0 || d->I % 256 || d->I > 1024)
    return fail(RNB_ERR_INVALID, "I must be 256, 512, 768 or 1024");
  if (d->k <= 0 || d->k > kMaxK) return fail(RNB_ERR_INVALID, "k must be in [1, 16]");
  if (d->E_total <= 0 || d->E_total > kMaxE || d->k > d->E_total)
    return fail(RNB_ERR_INVALID, "E_total must be in [k, 512]");
  if (d->E <= 0 || d->expert_offset < 0 || d->expert_offset + d->E > d->E_total)
    return fail(RNB_ERR_INVALID, "expert shard [expert_offset, expert_offset+E) must lie in [0, E_total)");
  if (need_bank) {
    const void* ptrs[] = {d->gu_w, d->gu_s, d->gu_b, d->dn_w, d->dn_s, d->dn_b};
    for (const void* q : ptrs) {
      if (!q) return fail(RNB_ERR_INVALID, "routed expert weights must be non-NULL");
      if (!aligned16(q)) return fail(RNB_ERR_ALIGN, "routed expert tensors must be 16-byte aligned");
    }
  }
  if (d->router_bits != 0 && d->router_bits != 16 && d->router_bits != 8)
    return fail(RNB_ERR_INVALID, "router_bits must be 0, 16 or 8");
  if (need_router) {
    if (!d->router_w) return fail(RNB_ERR_INVALID, "router_w must be non-NULL");
    if (!aligned16(d->router_w)) return fail(RNB_ERR_ALIGN, "router_w must be 16-byte aligned");
    if (d->router_bits == 8) {
      if (!d->router_s || !d->router_b)
        return fail(RNB_ERR_INVALID, "an 8-bit router needs router_s and router_b");
      if (d->shared_gate_w && !(d->flags & RNB_FLAG_NO_SHARED) && (!d->sgate_s || !d->sgate_b))
        return fail(RNB_ERR_INVALID, "an 8-bit shared gate needs sgate_s and sgate_b");
      if (d->shared_gate_w && !aligned16(d->shared_gate_w))
        return fail(RNB_ERR_ALIGN, "shared_gate_w must be 16-byte aligned");
    }
  }
  return RNB_OK;
}

bool has_shared(const rnb_moe_desc* d) {
  if (d->flags & RNB_FLAG_NO_SHARED) return false;
  return d->shared_gate_w && d->sgu_w && d->sdn_w;
}

int check_device() {
  static std::once_flag once;
  static int major = -1;
  std::call_once(once, [] {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  });
  if (major != 10) return fail(RNB_ERR_DEVICE, "an sm_100 (B200) device is required");
  return RNB_OK;
}

template <typename Kern>
cudaError_t launch(Kern kern, dim3 grid, dim3 block, cudaStream_t st, bool pdl, const Params& p,
                   size_t smem = 0) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

DevInfo dev_info() {
  static std::mutex mu;
  static DevInfo cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  DevInfo& di = cache[dev & 63];
  if (di.sms == 0) {
    cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&di.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  }
  return di;
}

// Static shared memory of k_decode (counts against the per-block limit).
template <int BITS>
size_t persistent_static_smem() {
  static size_t bytes = [] {
    cudaFuncAttributes fa;
    cudaFuncAttributes fb;
    cudaFuncAttributes fc, fd;
    const bool ok = cudaFuncGetAttributes(&fa, k_decode<BITS, false, false>) == cudaSuccess &&
                    cudaFuncGetAttributes(&fb, k_decode<BITS, true, false>) == cudaSuccess &&
                    cudaFuncGetAttributes(&fc, k_decode<BITS, false, true>) == cudaSuccess &&
                    cudaFuncGetAttributes(&fd, k_decode<BITS, true, true>) == cudaSuccess;
    size_t m = fa.sharedSizeBytes > fb.sharedSizeBytes ? fa.sharedSizeBytes : fb.sharedSizeBytes;
    m = m > fc.sharedSizeBytes ? m : fc.sharedSizeBytes;
    m = m > fd.sharedSizeBytes ? m : fd.sharedSizeBytes;
    return ok ? m : size_t(2048);
  }();
  return bytes;
}

// Tensor maps of the split-K loads (SkMaps), encoded once per weight tensor
// and shape and then served from a process-wide cache (encoding costs a few
// microseconds of host time; decode calls repeat with the same weights).
struct SkMapKey {
  const void* base;
  int kind, bits, E, H, I;
  bool operator==(const SkMapKey& o) const {
    return base == o.base && kind == o.kind && bits == o.bits && E == o.E && H == o.H && I == o.I;
  }
};
struct SkMapKeyHash {
  size_t operator()(const SkMapKey& k) const {
    size_t h = reinterpret_cast<size_t>(k.base);
    for (int v : {k.kind, k.bits, k.E, k.H, k.I}) h = h * 1000003u ^ static_cast<size_t>(v);
    return h;
  }
};

// kind 0: gate/up codes, 1: gate/up scales or biases, 2: down codes.
bool sk_map(CUtensorMap* m, int kind, const void* base, int bits, int E, int H, int I) {
  static std::mutex mu;
  static std::unordered_map<SkMapKey, CUtensorMap, SkMapKeyHash> cache;
  const SkMapKey key{base, kind, bits, E, H, I};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *m = it->second;
      return true;
    }
  }
  const uint64_t rowb = static_cast<uint64_t>(H) * bits / 8, I2 = 2ull * I, G = H / kGroup;
  const uint64_t slice = 16ull * bits;  // a warp's K slice of a gate/up row (Tile2 row bytes)
  bool ok = false;
  if (kind == 0) {
    const uint64_t dims[4] = {slice / 4, I2, static_cast<uint64_t>(H) * bits / 8 / slice, static_cast<uint64_t>(E)};
    const uint64_t str[3] = {rowb, slice, I2 * rowb};
    const uint32_t box[4] = {static_cast<uint32_t>(slice / 4), 8, static_cast<uint32_t>(dims[2]), 1};
    ok = encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, base, dims, str, box,
                      bits == 8 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  } else if (kind == 1) {
    const uint64_t dims[3] = {G, I2, static_cast<uint64_t>(E)};
    const uint64_t str[2] = {G * 2, I2 * G * 2};
    const uint32_t box[3] = {static_cast<uint32_t>(G), 32, 1};
    ok = encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, base, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    const uint64_t rw = static_cast<uint64_t>(I) * bits / 32;  // words per down row
    const uint64_t dims[4] = {rw, 256, static_cast<uint64_t>(H) / 256, static_cast<uint64_t>(E)};
    const uint64_t str[3] = {rw * 4, 256 * rw * 4, static_cast<uint64_t>(H) * rw * 4};
    const uint32_t box[4] = {static_cast<uint32_t>(kSkC * bits / 32), 256, static_cast<uint32_t>(H / 256), 1};
    ok = encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, base, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (!ok) return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *m);
  return true;
}

bool sk_maps(const Params& p, int bits, SkMaps& m) {
  bool ok = sk_map(&m.gu_w, 0, p.gu_w, bits, p.E, p.H, p.I) && sk_map(&m.gu_s, 1, p.gu_s, bits, p.E, p.H, p.I) &&
            sk_map(&m.gu_b, 1, p.gu_b, bits, p.E, p.H, p.I) && sk_map(&m.dn_w, 2, p.dn_w, bits, p.E, p.H, p.I);
  if (ok && p.has_shared) {
    ok = sk_map(&m.sgu_w, 0, p.sgu_w, bits, 1, p.H, p.I) && sk_map(&m.sgu_s, 1, p.sgu_s, bits, 1, p.H, p.I) &&
         sk_map(&m.sgu_b, 1, p.sgu_b, bits, 1, p.H, p.I) && sk_map(&m.sdn_w, 2, p.sdn_w, bits, 1, p.H, p.I);
  } else if (ok) {
    m.sgu_w = m.gu_w;  // (never read without a shared expert)
    m.sgu_s = m.gu_s;
    m.sgu_b = m.gu_b;
    m.sdn_w = m.dn_w;
  }
  return ok;
}

// Shared-memory plan of the split-K form: one token, the whole expert bank
// on this GPU (no expert parallelism, the whole shared expert), and a CTA for
// each of the 16 (k + 1) tasks.
template <int BITS>
bool persistent_plan_sk(const Params& p, const DevInfo& di, PPlan& pl, size_t& smem) {
  const int nq = p.I / 128;
  if (p.mode != kModeBlock || p.T != 1 || p.H != 2048 || p.I != 512 || p.E_total > 256 || p.k > kPMaxK)
    return false;
  if (p.ep_world > 1) {
    // expert parallel: even expert shards, the shared expert's 16 slices
    // split evenly over the ranks
    if (kSkTasksPerSource % p.ep_world || p.E * p.ep_world != p.E_total || p.off != p.ep_rank * p.E) return false;
  } else if (p.off != 0 || p.E != p.E_total || p.shared_qmask != (1u << nq) - 1u) {
    return false;
  }
  const int NC = di.sms;
  if (NC < p.H / 16 || 2 * NC < p.E_total + 1) return false;
  if (kSkTasksPerSource * (p.k + (p.has_shared ? 1 : 0)) > NC) return false;
  using TL = Tile2<BITS>;
  using SD = SkDown<BITS>;
  const int G = p.H / kGroup;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = (o + bytes + 127) & ~static_cast<size_t>(127);
    return static_cast<uint32_t>(at);
  };
  pl.sk = 1;
  pl.S = 1;
  pl.off_ring = 0;
  pl.off_sdn = 0;
  pl.off_x = take(static_cast<size_t>(G) * 32 * 4);
  pl.off_xs = take(static_cast<size_t>(G) * 4);
  pl.off_xn = p.norm_w ? take(static_cast<size_t>(p.H) * 2) : 0u;
  pl.off_ivl = take(static_cast<size_t>(p.E_total + 1) * 4);
  pl.off_red = take(static_cast<size_t>(kSkUnits) * kPWarps * 32 * 4);
  pl.off_hf = pl.off_red;  // xprep's scratch (done before the partials are written)
  pl.off_redc = 0;
  pl.off_misc = take(sizeof(PMisc));
  // the TMA destinations: up and gate codes, 4 scale / bias blocks, down codes
  pl.off_tma = static_cast<uint32_t>(o);
  o += 1023 + 2 * 16 * 32 * TL::kRowBytes + 4 * 32 * (p.H / kGroup) * 2 + static_cast<size_t>(p.H) * SD::kRow;
  const size_t limit = static_cast<size_t>(di.smem_optin) - persistent_static_smem<BITS>();
  smem = o;
  if (smem > limit) return false;
  SkMaps probe;  // (cached: the launch reuses them)
  return sk_maps(p, BITS, probe);
}

// Shared-memory plan of k_decode; false when the call does not fit it.
template <int BITS>
bool persistent_plan(const Params& p, const DevInfo& di, PPlan& pl, size_t& smem) {
  if (persistent_plan_sk<BITS>(p, di, pl, smem)) return true;
  pl.sk = 0;
  if (p.mode != kModeBlock || p.T < 1 || p.T > kPMaxT || p.H != 2048 || p.I != 512 || p.E_total > 256 ||
      p.k > kPMaxK || p.off < 0 || p.off + p.E > p.E_total)
    return false;
  const int NC = di.sms;
  // roles: H/16 CTAs own 16 output rows, the first I/8 CTAs a shared-expert
  // gate/up task, every CTA at most two router rows, and no CTA more than
  // kPMaxMine routed gate/up tasks
  if (NC < p.H / 16 || NC < p.I / 8 || 2 * NC < p.E_total + 1) return false;
  const int n_act_max = p.T * p.k < p.E ? p.T * p.k : p.E;
  const int mine_max = (n_act_max * (p.I / 8) + NC - 1) / NC;
  if (mine_max > kPMaxMine) return false;
  using TL = Tile2<BITS>;
  const int T = p.T, G = p.H / kGroup, nq = p.I / 128;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = (o + bytes + 127) & ~static_cast<size_t>(127);
    return static_cast<uint32_t>(at);
  };
  pl.off_sdn = take(static_cast<size_t>(nq) * TL::kBytes);
  pl.off_x = take(static_cast<size_t>(T) * G * 32 * 4);
  pl.off_xs = take(static_cast<size_t>(T) * G * 4);
  pl.off_xn = p.norm_w ? take(static_cast<size_t>(T) * p.H * 2) : 0u;
  pl.off_ivl = take(static_cast<size_t>(T) * (p.E_total + 1) * 4);
  pl.off_red = take(static_cast<size_t>(1 + mine_max) * kPWarps * 32 * 4);
  // the down MMAs' B fragments of every entry (fp16, [T(k+1)][I/64][32] words)
  // with a sum and an inverse scale per (entry, group); also xprep's scratch
  pl.off_hf = take(std::max<size_t>(static_cast<size_t>(T) * (p.k + 1) * (p.I / 64) * (32 + 2) * 4, 4096));
  pl.off_redc = take(static_cast<size_t>(T) * (p.k + 1) * nq * 16 * 4);
  pl.off_misc = take(sizeof(PMisc));
  const size_t limit = static_cast<size_t>(di.smem_optin) - persistent_static_smem<BITS>();
  if (o + 256 > limit) return false;
  const size_t per_slot = static_cast<size_t>(kPWarps) * TL::kBytes;
  pl.S = static_cast<int>((limit - o - 256) / per_slot);
  if (pl.S > 8) pl.S = 8;
  // every warp's down units must all be in flight once its gate/up units are
  // consumed: a slot each, plus the shared gate/up slice's
  const int max_down = (nq * n_act_max + kPWarps - 1) / kPWarps;
  if (pl.S < 2 || pl.S < 1 + max_down) return false;
  pl.off_ring = take(pl.S * per_slot);
  smem = o;
  return smem <= limit;
}

// One launch with programmatic stream serialisation: the kernel's prologue
// (weights only) may start while the previous kernel on the stream drains;
// its griddepcontrol.wait holds everything else back.
template <int BITS>
int run_persistent(Params& p, const PPlan& pl, size_t smem, int nc, cudaStream_t st) {
  auto kern = p.ep_world > 1 ? (pl.sk ? k_decode<BITS, true, true> : k_decode<BITS, true, false>)
                             : (pl.sk ? k_decode<BITS, false, true> : k_decode<BITS, false, false>);
  SkMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (pl.sk && !sk_maps(p, BITS, maps)) return fail(RNB_ERR_CUDA, "k_decode: tensor map encoding failed");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("k_decode smem attribute: ") + cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nc);
  cfg.blockDim = dim3(32 * kPWarps);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  stage_begin(st);
  e = cudaLaunchKernelEx(&cfg, kern, p, pl, maps);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("k_decode launch: ") + cudaGetErrorString(e));
  stage_end(st, RNB_STAGE_DECODE);
  return RNB_OK;
}

template <int BITS>
int run_decode(const rnb_moe_desc* d, Params& p, cudaStream_t st) {
  if (p.mode == kModeBlock && !(d->flags & RNB_FLAG_CHAIN)) {
    const DevInfo di = dev_info();
    PPlan pl;
    size_t smem = 0;
    if (persistent_plan<BITS>(p, di, pl, smem)) return run_persistent<BITS>(p, pl, smem, di.sms, st);
  }
  const int tiles = (p.E_total + 1 + 15) / 16;
  p.router_ctas = p.mode == kModeSwitchGLU ? 0 : tiles;
  const int prep_ctas = p.mode == kModeRouter ? 0 : (p.T + 15) / 16;
  // Programmatic launch: k_route streams its router weights in while the
  // previous kernel on the stream finishes, and waits before touching x.
  stage_begin(st);
  cudaError_t e = launch(k_route<BITS>, dim3(p.router_ctas + prep_ctas), dim3(32 * kRouterWarps), st, true, p);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("k_route launch: ") + cudaGetErrorString(e));
  stage_end(st, RNB_STAGE_ROUTE);
  if (p.mode == kModeRouter) return RNB_OK;
  const int slots = 1 + (p.T * p.k < p.E ? p.T * p.k : p.E);
  p.ncmax = p.T < 8 ? p.T : 8;
  const int gnw = p.H / (kGroup * kGateUpGroupsPerWarp);
  const size_t gsm = gateup_smem<BITS>(gnw, p.ncmax);
  const int dnw = p.I / (kGroup * kDownGroupsPerWarp);
  const size_t dsm = down_smem<BITS>(dnw, p.ncmax);
  static bool attr_set = false;  // per template instance
  if (!attr_set) {
    e = cudaFuncSetAttribute(k_gateup<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(gateup_smem<BITS>(kGateUpMaxWarps, 8)));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_down<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(down_smem<BITS>(kDownMaxWarps, 8)));
    if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("smem attribute: ") + cudaGetErrorString(e));
    attr_set = true;
  }
  e = launch(k_gateup<BITS>, dim3(p.I / 8, slots), dim3(32 * gnw), st, true, p, gsm);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("k_gateup launch: ") + cudaGetErrorString(e));
  stage_end(st, RNB_STAGE_GATEUP);
  e = launch(k_down<BITS>, dim3(p.H / 16, slots), dim3(32 * dnw), st, true, p, dsm);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("k_down launch: ") + cudaGetErrorString(e));
  stage_end(st, RNB_STAGE_DOWN);
  return RNB_OK;
}

Params base_params(const rnb_moe_desc* d, const void* x, void* ws, int mode) {
  Params p;
  memset(&p, 0, sizeof(p));
  p.T = d->T;
  p.H = d->H;
  p.I = d->I;
  p.E = d->E;
  p.E_total = d->E_total;
  p.off = d->expert_offset;
  p.k = d->k;
  p.mode = mode;
  p.has_shared = (mode == kModeSwitchGLU) ? 0 : (has_shared(d) ? 1 : 0);
  p.x = static_cast<const uint16_t*>(x);
  p.router_w = d->router_w;
  p.sgate_w = d->shared_gate_w;
  p.router_q8 = d->router_bits == 8 ? 1 : 0;
  p.router_s = d->router_s;
  p.router_b = d->router_b;
  p.sgate_s = d->sgate_s;
  p.sgate_b = d->sgate_b;
  p.gu_w = d->gu_w;
  p.gu_s = d->gu_s;
  p.gu_b = d->gu_b;
  p.dn_w = d->dn_w;
  p.dn_s = d->dn_s;
  p.dn_b = d->dn_b;
  p.sgu_w = d->sgu_w;
  p.sgu_s = d->sgu_s;
  p.sgu_b = d->sgu_b;
  p.sdn_w = d->sdn_w;
  p.sdn_s = d->sdn_s;
  p.sdn_b = d->sdn_b;
  p.ws = bind(make_layout(*d), ws);
  p.shared_qmask = (1u << (d->I / 128)) - 1u;
  p.ep_world = 1;
  p.ep_limit_ns = kEpSpinLimitNs;
  p.y_f32 = (mode == kModeBlock && (d->flags & RNB_FLAG_Y_F32)) ? 1 : 0;
  return p;
}

int check_ws(const rnb_moe_desc* d, void* ws, size_t ws_bytes) {
  if (!ws) return fail(RNB_ERR_WORKSPACE, "workspace is NULL");
  if (!aligned16(ws)) return fail(RNB_ERR_ALIGN, "workspace must be 16-byte aligned");
  if (ws_bytes < make_layout(*d).total) return fail(RNB_ERR_WORKSPACE, "workspace too small");
  return RNB_OK;
}

// Runs [0, T) in chunks of kMaxDecodeT tokens.
template <typename F>
int for_chunks(const rnb_moe_desc* d, F f) {
  for (int t0 = 0; t0 < d->T; t0 += kMaxDecodeT) {
    rnb_moe_desc c = *d;
    c.T = d->T - t0 < kMaxDecodeT ? d->T - t0 : kMaxDecodeT;
    const int rc = f(c, t0);
    if (rc != RNB_OK) return rc;
  }
  return RNB_OK;
}

int dispatch_bits(const rnb_moe_desc* d, Params& p, cudaStream_t st) {
  return d->bits == 8 ? run_decode<8>(d, p, st) : run_decode<4>(d, p, st);
}

}  // namespace rnb

namespace rnb {

// Scratch for rnb_moe_block_fwd_noalloc: a file-scope device array, so a
// caller that cannot allocate device memory still gets the workspace the
// kernels need.  Every GPU that loads this library holds it until exit.
constexpr size_t kNoAllocScratchBytes = 12u << 20;  // 12 MiB; Ornith shapes need 9.6 MB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  The host-side
// name is only a stand-in, so the address is looked up once per device with
// that device current and cached.
int noalloc_scratch(void** out) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(RNB_ERR_DEVICE, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(RNB_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return RNB_OK;
}

// Copy streams and events of rnb_moe_block_fwd_host's chunked form, made once
// per device.  g_host_pipe_mu is held while a call queues its work, so two
// host threads never interleave records and waits on the shared events.
constexpr int kHostMaxChunks = 4;
constexpr int kHostChunkMin = 2048;  // tokens per chunk when a call is split
struct HostPipe {
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t start = nullptr, done = nullptr;
  cudaEvent_t ready[kHostMaxChunks] = {}, computed[kHostMaxChunks] = {};
};
std::mutex g_host_pipe_mu;

int host_pipe(HostPipe** out) {
  constexpr int kMaxDevices = 64;
  static HostPipe pipes[kMaxDevices];
  static bool made[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(RNB_ERR_DEVICE, "device index out of range");
  HostPipe& hp = pipes[dev];
  if (!made[dev]) {
    e = cudaStreamCreateWithFlags(&hp.in, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&hp.out, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&hp.start, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&hp.done, cudaEventDisableTiming);
    for (int j = 0; j < kHostMaxChunks && e == cudaSuccess; ++j) {
      e = cudaEventCreateWithFlags(&hp.ready[j], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&hp.computed[j], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) {
      // release what was made, so a later attempt starts from nothing
      for (cudaStream_t* s : {&hp.in, &hp.out})
        if (*s) (void)cudaStreamDestroy(*s);
      for (cudaEvent_t* v : {&hp.start, &hp.done})
        if (*v) (void)cudaEventDestroy(*v);
      for (int j = 0; j < kHostMaxChunks; ++j) {
        if (hp.ready[j]) (void)cudaEventDestroy(hp.ready[j]);
        if (hp.computed[j]) (void)cudaEventDestroy(hp.computed[j]);
      }
      hp = HostPipe{};
      return fail(RNB_ERR_CUDA, std::string("creating copy streams: ") + cudaGetErrorString(e));
    }
    made[dev] = true;
  }
  *out = &hp;
  return RNB_OK;
}

}  // namespace rnb

using namespace rnb;

extern "C" {

int rnb_version(void) { return 100; }

const char* rnb_last_error(void) { return g_last_error.c_str(); }

int rnb_moe_workspace_size(const rnb_moe_desc* d, size_t* bytes) {
  int rc = validate(d, false, false);
  if (rc) return rc;
  if (!bytes) return fail(RNB_ERR_INVALID, "bytes is NULL");
  size_t n = make_layout(*d).total;
  if (d->T > kMaxDecodeT && prefill_supported(*d)) {
    const size_t pn = prefill_workspace_bytes(*d);
    n = pn > n ? pn : n;
  }
  *bytes = n;
  return RNB_OK;
}

int rnb_moe_workspace_init(void* ws, size_t ws_bytes, void* stream) {
  if (!ws) return fail(RNB_ERR_WORKSPACE, "workspace is NULL");
  const cudaError_t e = cudaMemsetAsync(ws, 0, ws_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, cudaGetErrorString(e));
  return RNB_OK;
}

int rnb_router_topk(const rnb_moe_desc* d, const void* x, uint32_t* inds, float* scores,
                    float* logits, void* ws, size_t ws_bytes, void* stream) {
  int rc = validate(d, true, false);
  if (!rc) rc = check_device();
  if (!rc) rc = check_ws(d, ws, ws_bytes);
  if (rc) return rc;
  if (!x || !inds || !scores) return fail(RNB_ERR_INVALID, "x, inds and scores must be non-NULL");
  if (!aligned16(x)) return fail(RNB_ERR_ALIGN, "x must be 16-byte aligned");
  return for_chunks(d, [&](const rnb_moe_desc& c, int t0) {
    Params p = base_params(&c, static_cast<const uint16_t*>(x) + static_cast<size_t>(t0) * c.H, ws, kModeRouter);
    p.has_shared = has_shared(d) ? 1 : 0;
    p.inds_out = inds + static_cast<size_t>(t0) * c.k;
    p.scores_out = scores + static_cast<size_t>(t0) * c.k;
    p.logits_out = logits ? logits + static_cast<size_t>(t0) * c.E_total : nullptr;
    return dispatch_bits(&c, p, static_cast<cudaStream_t>(stream));
  });
}

int rnb_moe_experts_workspace_size(const rnb_moe_desc* d, size_t* bytes) {
  using namespace rnb;
  if (!bytes) return fail(RNB_ERR_INVALID, "bytes must be non-NULL");
  int rc = validate(d, false, false);
  if (rc) return rc;
  if (!prefill_supported(*d)) return fail(RNB_ERR_INVALID, "rnb_moe_experts_fwd does not support these shapes");
  *bytes = prefill_workspace_bytes(*d);
  return RNB_OK;
}

int rnb_moe_experts_fwd(const rnb_moe_desc* d, const void* x, const uint32_t* inds, const float* scores, void* out,
                        void* ws, size_t ws_bytes, void* stream) {
  using namespace rnb;
  int rc = validate(d, false, true);
  if (!rc) rc = check_device();
  if (rc) return rc;
  if (!x || !inds || !scores || !out || !ws) return fail(RNB_ERR_INVALID, "x, inds, scores, out and ws must be non-NULL");
  if (!aligned16(x) || !aligned16(out) || !aligned16(ws)) return fail(RNB_ERR_ALIGN, "x, out and ws must be 16-byte aligned");
  if (!prefill_supported(*d)) return fail(RNB_ERR_INVALID, "rnb_moe_experts_fwd does not support these shapes");
  if (ws_bytes < prefill_workspace_bytes(*d)) return fail(RNB_ERR_WORKSPACE, "workspace too small (rnb_moe_experts_workspace_size)");
  if (d->T == 0) return RNB_OK;
  return run_prefill(d, x, out, nullptr, nullptr, ws, ws_bytes, static_cast<cudaStream_t>(stream), inds, scores);
}

int rnb_switchglu_fwd(const rnb_moe_desc* d, const void* x, const uint32_t* inds, void* y, void* ws,
                      size_t ws_bytes, void* stream) {
  int rc = validate(d, false, true);
  if (!rc) rc = check_device();
  if (!rc) rc = check_ws(d, ws, ws_bytes);
  if (rc) return rc;
  if (!x || !inds || !y) return fail(RNB_ERR_INVALID, "x, inds and y must be non-NULL");
  if (!aligned16(x) || !aligned16(y)) return fail(RNB_ERR_ALIGN, "x and y must be 16-byte aligned");
  return for_chunks(d, [&](const rnb_moe_desc& c, int t0) {
    Params p = base_params(&c, static_cast<const uint16_t*>(x) + static_cast<size_t>(t0) * c.H, ws, kModeSwitchGLU);
    p.inds_in = inds + static_cast<size_t>(t0) * c.k;
    p.y_f32 = (d->flags & RNB_FLAG_Y_F32) ? 1 : 0;
    p.out = p.y_f32 ? static_cast<void*>(static_cast<float*>(y) + static_cast<size_t>(t0) * c.k * c.H)
                    : static_cast<void*>(static_cast<uint16_t*>(y) + static_cast<size_t>(t0) * c.k * c.H);
    return dispatch_bits(&c, p, static_cast<cudaStream_t>(stream));
  });
}

int rnb_moe_block_fwd(const rnb_moe_desc* d, const void* x, void* out, uint32_t* inds_out,
                      float* scores_out, void* ws, size_t ws_bytes, void* stream) {
  int rc = validate(d, true, true);
  if (!rc) rc = check_device();
  if (!rc) rc = check_ws(d, ws, ws_bytes);
  if (rc) return rc;
  if (!x || !out) return fail(RNB_ERR_INVALID, "x and out must be non-NULL");
  if (!aligned16(x) || !aligned16(out)) return fail(RNB_ERR_ALIGN, "x and out must be 16-byte aligned");
  if (has_shared(d)) {
    const void* sp[] = {d->shared_gate_w, d->sgu_w, d->sgu_s, d->sgu_b, d->sdn_w, d->sdn_s, d->sdn_b};
    for (const void* q : sp)
      if (!q || !aligned16(q)) return fail(RNB_ERR_ALIGN, "shared-expert tensors must be non-NULL and 16-byte aligned");
  }
  // Many tokens: the sorted grouped-GEMM (tcgen05) path, when the workspace
  // was sized for it; otherwise the decode kernels in 64-token chunks.
  if (d->T > kMaxDecodeT && !(d->flags & RNB_FLAG_CHAIN) && prefill_supported(*d) &&
      ws_bytes >= prefill_workspace_bytes(*d))
    return run_prefill(d, x, out, inds_out, scores_out, ws, ws_bytes, static_cast<cudaStream_t>(stream));
  return for_chunks(d, [&](const rnb_moe_desc& c, int t0) {
    Params p = base_params(&c, static_cast<const uint16_t*>(x) + static_cast<size_t>(t0) * c.H, ws, kModeBlock);
    p.out = static_cast<uint16_t*>(out) + static_cast<size_t>(t0) * c.H;
    p.inds_out = inds_out ? inds_out + static_cast<size_t>(t0) * c.k : nullptr;
    p.scores_out = scores_out ? scores_out + static_cast<size_t>(t0) * c.k : nullptr;
    return dispatch_bits(&c, p, static_cast<cudaStream_t>(stream));
  });
}

#ifdef RNB_TRACE
// Byte offset of the trace area in the workspace (trace builds only).
RNB_API size_t rnb_trace_offset(const rnb_moe_desc* d) { return make_layout(*d).yws; }
#endif

int rnb_moe_block_fwd_host(const rnb_moe_desc* d, const void* x_host, void* out_host, void* x_dev,
                           void* out_dev, void* ws, size_t ws_bytes, void* stream) {
  // everything the block call checks is checked before the first copy is queued
  int rc = validate(d, true, true);
  if (!rc) rc = check_device();
  if (!rc) rc = check_ws(d, ws, ws_bytes);
  if (rc) return rc;
  if (!x_host || !out_host || !x_dev || !out_dev)
    return fail(RNB_ERR_INVALID, "x_host, out_host, x_dev and out_dev must be non-NULL");
  if (!aligned16(x_dev) || !aligned16(out_dev)) return fail(RNB_ERR_ALIGN, "x_dev and out_dev must be 16-byte aligned");
  const size_t n = static_cast<size_t>(d->T) * static_cast<size_t>(d->H);
  const size_t out_bytes = n * ((d->flags & RNB_FLAG_Y_F32) ? 4 : 2);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // For decode-sized calls, page-locked host memory mapped into this device's
  // address space takes the kernels' stores directly (every path only stores
  // to out), which saves the copy-out and its wait.  Larger outputs cross PCIe
  // faster as one copy.  Pageable or unmapped memory is never handed to a
  // kernel: it gets the device-to-host copy.
  void* direct = nullptr;
  cudaPointerAttributes pa{};
  if (d->T > kMaxDecodeT) {
    // copy-out below
  } else if (cudaPointerGetAttributes(&pa, out_host) == cudaSuccess) {
    if (pa.type == cudaMemoryTypeHost && pa.devicePointer && aligned16(pa.devicePointer)) direct = pa.devicePointer;
  } else {
    (void)cudaGetLastError();  // an unknown (pageable) pointer is not an error here
  }
  // Chunked copies only between page-locked host buffers: a copy from or to
  // pageable memory blocks the host thread, which would serialise the chunks
  // while the pipe's lock is held.
  auto pinned = [](const void* ptr) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    return a.type == cudaMemoryTypeHost;
  };
  int nchunk = std::min(kHostMaxChunks, d->T / kHostChunkMin);
  if (nchunk >= 2 && !(pinned(x_host) && pinned(out_host))) nchunk = 1;
  if (nchunk < 2) {
    cudaError_t e = cudaMemcpyAsync(x_dev, x_host, n * 2, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("copying x to the device: ") + cudaGetErrorString(e));
    rc = rnb_moe_block_fwd(d, x_dev, direct ? direct : out_dev, nullptr, nullptr, ws, ws_bytes, stream);
    if (rc || direct) return rc;
    e = cudaMemcpyAsync(out_host, out_dev, out_bytes, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("copying out to the host: ") + cudaGetErrorString(e));
    return RNB_OK;
  }
  // Many tokens: the call is split into chunks of whole tokens.  All
  // copies-in run back to back on one copy stream; chunk j's block waits for
  // its copy-in, and its copy-out on a second copy stream waits for the block,
  // so the copies overlap the other chunks' compute.  The caller's stream
  // waits for the last copy-out before the call's work counts as done.
  std::lock_guard<std::mutex> lock(g_host_pipe_mu);
  HostPipe* hp = nullptr;
  rc = host_pipe(&hp);
  if (rc) return rc;
  const size_t osz = (d->flags & RNB_FLAG_Y_F32) ? 4 : 2, row_in = static_cast<size_t>(d->H) * 2,
               row_out = static_cast<size_t>(d->H) * osz;
  int t0s[kHostMaxChunks + 1];
  for (int j = 0; j <= nchunk; ++j)
    t0s[j] = static_cast<int>(static_cast<long long>(d->T) * j / nchunk);
  // on an error the caller's stream still waits for whatever was queued on
  // the copy streams (best effort), so out_host is not written after it
  auto join = [&]() {
    for (cudaStream_t cs : {hp->in, hp->out})
      if (cudaEventRecord(hp->done, cs) == cudaSuccess) (void)cudaStreamWaitEvent(st, hp->done, 0);
  };
  auto cuda_fail = [&](const char* what, cudaError_t e) {
    const int r = fail(RNB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    join();
    return r;
  };
  // the staging buffers and out_host are reused: start after earlier work on the caller's stream
  cudaError_t e = cudaEventRecord(hp->start, st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(hp->in, hp->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(hp->out, hp->start, 0);
  if (e != cudaSuccess) return cuda_fail("ordering the copy streams", e);
  for (int j = 0; j < nchunk; ++j) {
    const size_t off = static_cast<size_t>(t0s[j]), rows = static_cast<size_t>(t0s[j + 1] - t0s[j]);
    e = cudaMemcpyAsync(static_cast<char*>(x_dev) + off * row_in, static_cast<const char*>(x_host) + off * row_in,
                        rows * row_in, cudaMemcpyHostToDevice, hp->in);
    if (e == cudaSuccess) e = cudaEventRecord(hp->ready[j], hp->in);
    if (e != cudaSuccess) return cuda_fail("copying x to the device", e);
  }
  for (int j = 0; j < nchunk; ++j) {
    const size_t off = static_cast<size_t>(t0s[j]), rows = static_cast<size_t>(t0s[j + 1] - t0s[j]);
    rnb_moe_desc c = *d;
    c.T = t0s[j + 1] - t0s[j];
    e = cudaStreamWaitEvent(st, hp->ready[j], 0);
    if (e != cudaSuccess) return cuda_fail("waiting for the copy-in", e);
    rc = rnb_moe_block_fwd(&c, static_cast<char*>(x_dev) + off * row_in, static_cast<char*>(out_dev) + off * row_out,
                           nullptr, nullptr, ws, ws_bytes, stream);
    if (rc) {
      join();
      return rc;
    }
    e = cudaEventRecord(hp->computed[j], st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(hp->out, hp->computed[j], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(static_cast<char*>(out_host) + off * row_out, static_cast<char*>(out_dev) + off * row_out,
                          rows * row_out, cudaMemcpyDeviceToHost, hp->out);
    if (e != cudaSuccess) return cuda_fail("copying out to the host", e);
  }
  e = cudaEventRecord(hp->done, hp->out);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st, hp->done, 0);
  if (e != cudaSuccess) return cuda_fail("joining the copy streams", e);
  return RNB_OK;
}

int rnb_moe_status(void* ws, size_t ws_bytes, uint32_t* status, void* stream) {
  if (!ws || !status) return fail(RNB_ERR_INVALID, "ws and status must be non-NULL");
  if (ws_bytes < 4) return fail(RNB_ERR_WORKSPACE, "workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status, ws, 4, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(ws, 0, 4, st);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, cudaGetErrorString(e));
  return RNB_OK;
}

int rnb_moe_block_fwd_noalloc(const rnb_moe_desc* d, const void* x, void* out, uint32_t* inds_out,
                              float* scores_out, void* stream) {
  int rc = validate(d, true, true);
  if (rc) return rc;
  const Layout L = make_layout(*d);
  if (L.total > kNoAllocScratchBytes)
    return fail(RNB_ERR_WORKSPACE, "rnb_moe_block_fwd_noalloc: these shapes need " + std::to_string(L.total) +
                                       " bytes of scratch; the static scratch holds " +
                                       std::to_string(kNoAllocScratchBytes) + " bytes");
  rc = check_device();
  if (rc) return rc;
  void* ws = nullptr;
  rc = noalloc_scratch(&ws);
  if (rc) return rc;
  // The arrival counters must start at zero; a call leaves them at zero, but
  // clear them so a call never depends on earlier ones.  The status word (the
  // first 256-byte slot) is left alone: its bits add up over calls until
  // rnb_moe_noalloc_status reads and clears them.
  const cudaError_t e = cudaMemsetAsync(static_cast<char*>(ws) + L.ctr, 0, L.xperm - L.ctr,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("clearing scratch counters: ") + cudaGetErrorString(e));
  return rnb_moe_block_fwd(d, x, out, inds_out, scores_out, ws, kNoAllocScratchBytes, stream);
}

int rnb_moe_noalloc_status(uint32_t* status, void* stream) {
  if (!status) return fail(RNB_ERR_INVALID, "status must be non-NULL");
  int rc = check_device();
  if (rc) return rc;
  void* ws = nullptr;
  rc = noalloc_scratch(&ws);
  if (rc) return rc;
  return rnb_moe_status(ws, kNoAllocScratchBytes, status, stream);
}

}  // extern "C"

// ------------------------------------------------------------ expert parallel

struct rnb_ep {
  int rank = 0, world = 1, H = 0, dev = 0;
  uint64_t wait_ns = rnb::kEpSpinLimitNs;
  size_t recv_bytes = 0, bytes = 0;
  void* local = nullptr;
  uint2* recv[rnb::kMaxEpRanks] = {};
  void* opened[rnb::kMaxEpRanks] = {};
  float* partial = nullptr;  // [kEpMaxT][H] fp32: the chain's partial before the exchange
  uint32_t* seq = nullptr;   // this rank's sequence word and exit counter (after the flags)
  bool connected = false;
};

namespace rnb {
namespace {

size_t ep_recv_bytes(int world, int H) { return static_cast<size_t>(2) * world * kEpMaxT * H * sizeof(uint2); }
constexpr size_t kEpSeqBytes = 256;  // sequence word and exit counter after the receive buffer

}  // namespace
}  // namespace rnb

extern "C" {

int rnb_ep_create(int rank, int world, int H, rnb_ep** ep_out, void* handle_out) {
  using namespace rnb;
  if (!ep_out || !handle_out) return fail(RNB_ERR_INVALID, "rnb_ep_create: NULL output pointer");
  *ep_out = nullptr;
  if (world < 1 || world > kMaxEpRanks || rank < 0 || rank >= world)
    return fail(RNB_ERR_INVALID, "rnb_ep_create: need 0 <= rank < world <= 8");
  if (H <= 0 || H % 16) return fail(RNB_ERR_INVALID, "rnb_ep_create: H must be a positive multiple of 16");
  int rc = check_device();
  if (rc) return rc;
  rnb_ep* ep = new rnb_ep();
  ep->rank = rank;
  ep->world = world;
  ep->H = H;
  cudaGetDevice(&ep->dev);
  ep->recv_bytes = ep_recv_bytes(world, H);
  ep->bytes = ep->recv_bytes + kEpSeqBytes;
  cudaError_t e = cudaMalloc(&ep->local, ep->bytes);
  if (e == cudaSuccess) e = cudaMemset(ep->local, 0, ep->bytes);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&ep->partial), static_cast<size_t>(kEpMaxT) * H * 4);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ep->local);
  if (e != cudaSuccess) {
    if (ep->local) cudaFree(ep->local);
    if (ep->partial) cudaFree(ep->partial);
    delete ep;
    return fail(RNB_ERR_CUDA, std::string("rnb_ep_create: ") + cudaGetErrorString(e));
  }
  memcpy(handle_out, &h, sizeof(h));
  ep->recv[rank] = static_cast<uint2*>(ep->local);
  ep->seq = reinterpret_cast<uint32_t*>(static_cast<char*>(ep->local) + ep->recv_bytes);
  *ep_out = ep;
  return RNB_OK;
}

int rnb_ep_connect(rnb_ep* ep, const void* handles) {
  using namespace rnb;
  if (!ep || !handles) return fail(RNB_ERR_INVALID, "rnb_ep_connect: NULL argument");
  if (ep->connected) return fail(RNB_ERR_INVALID, "rnb_ep_connect: already connected");
  for (int q = 0; q < ep->world; ++q) {
    if (q == ep->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + static_cast<size_t>(q) * RNB_EP_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int j = 0; j < q; ++j)
        if (ep->opened[j]) {
          cudaIpcCloseMemHandle(ep->opened[j]);
          ep->opened[j] = nullptr;
        }
      return fail(RNB_ERR_CUDA, std::string("rnb_ep_connect: peer ") + std::to_string(q) + ": " +
                                    cudaGetErrorString(e));
    }
    ep->opened[q] = ptr;
    ep->recv[q] = static_cast<uint2*>(ptr);
  }
  ep->connected = true;
  return RNB_OK;
}

int rnb_ep_set_wait_limit_ms(rnb_ep* ep, int ms) {
  using namespace rnb;
  if (!ep) return fail(RNB_ERR_INVALID, "rnb_ep_set_wait_limit_ms: ep is NULL");
  if (ms < 1 || ms > 600000) return fail(RNB_ERR_INVALID, "rnb_ep_set_wait_limit_ms: ms must be in [1, 600000]");
  ep->wait_ns = static_cast<uint64_t>(ms) * 1000000ull;
  return RNB_OK;
}

int rnb_ep_destroy(rnb_ep* ep) {
  if (!ep) return RNB_OK;
  for (int q = 0; q < ep->world; ++q)
    if (ep->opened[q]) cudaIpcCloseMemHandle(ep->opened[q]);
  if (ep->local) cudaFree(ep->local);
  if (ep->partial) cudaFree(ep->partial);
  delete ep;
  return RNB_OK;
}

int rnb_moe_block_ep_fwd(const rnb_moe_desc* d, rnb_ep* ep, const void* x, void* out, uint32_t* inds_out,
                         float* scores_out, void* ws, size_t ws_bytes, void* stream) {
  using namespace rnb;
  if (!ep) return fail(RNB_ERR_INVALID, "rnb_moe_block_ep_fwd: ep is NULL");
  if (ep->world > 1 && !ep->connected) return fail(RNB_ERR_INVALID, "rnb_moe_block_ep_fwd: call rnb_ep_connect first");
  int rc = validate(d, true, true);
  if (!rc) rc = check_device();
  if (!rc) rc = check_ws(d, ws, ws_bytes);
  if (rc) return rc;
  if (!x || !out) return fail(RNB_ERR_INVALID, "x and out must be non-NULL");
  if (!aligned16(x) || !aligned16(out)) return fail(RNB_ERR_ALIGN, "x and out must be 16-byte aligned");
  if (d->H != ep->H) return fail(RNB_ERR_INVALID, "rnb_moe_block_ep_fwd: H differs from the EP context's");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != ep->dev) return fail(RNB_ERR_INVALID, "rnb_moe_block_ep_fwd: current device is not the EP context's");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto set_ep = [&](Params& p) {
    p.ep_world = ep->world;
    p.ep_rank = ep->rank;
    p.ep_limit_ns = ep->wait_ns;
    for (int q = 0; q < ep->world; ++q) {
      p.ep_recv[q] = ep->recv[q];
    }
    p.ep_seq = ep->seq;
  };
  // Few tokens: one persistent launch; the shared expert's 128-channel
  // quarters are split round-robin over the ranks and the partial tiles are
  // exchanged inside the kernel.
  {
    Params p = base_params(d, x, ws, kModeBlock);
    p.out = out;
    p.inds_out = inds_out;
    p.scores_out = scores_out;
    const int nq = d->I / 128;
    p.shared_qmask = 0;
    for (int q = ep->rank; q < nq; q += ep->world) p.shared_qmask |= 1u << q;
    const DevInfo di = dev_info();
    PPlan pl;
    size_t smem = 0;
    set_ep(p);  // (before the plan: the split-K form is for one GPU only)
    const bool ok = d->bits == 8 ? persistent_plan<8>(p, di, pl, smem) : persistent_plan<4>(p, di, pl, smem);
    if (ok) return d->bits == 8 ? run_persistent<8>(p, pl, smem, di.sms, st) : run_persistent<4>(p, pl, smem, di.sms, st);
  }
  // Otherwise per 64-token chunk: the decode chain writes this rank's fp32
  // partial (shared expert on rank 0), then k_ep_reduce exchanges and sums.
  rnb_moe_desc dc = *d;
  dc.flags |= RNB_FLAG_CHAIN | RNB_FLAG_Y_F32;
  if (ep->rank != 0) dc.flags |= RNB_FLAG_NO_SHARED;
  const bool f32_out = (d->flags & RNB_FLAG_Y_F32) != 0;
  return for_chunks(&dc, [&](const rnb_moe_desc& c, int t0) {
    Params p = base_params(&c, static_cast<const uint16_t*>(x) + static_cast<size_t>(t0) * c.H, ws, kModeBlock);
    p.out = ep->partial;
    p.inds_out = inds_out ? inds_out + static_cast<size_t>(t0) * c.k : nullptr;
    p.scores_out = scores_out ? scores_out + static_cast<size_t>(t0) * c.k : nullptr;
    int rc2 = dispatch_bits(&c, p, st);
    if (rc2) return rc2;
    Params r = p;
    r.y_f32 = f32_out ? 1 : 0;
    r.out = f32_out ? static_cast<void*>(static_cast<float*>(out) + static_cast<size_t>(t0) * c.H)
                    : static_cast<void*>(static_cast<uint16_t*>(out) + static_cast<size_t>(t0) * c.H);
    set_ep(r);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c.H / 16);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_ep_reduce, r, static_cast<const float*>(ep->partial));
    if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("k_ep_reduce launch: ") + cudaGetErrorString(e));
    return RNB_OK;
  });
}

}  // extern "C"

int rnb_moe_block_norm_fwd(const rnb_moe_desc* d, rnb_ep* ep, const void* resid, const void* y_prev,
                           const void* norm_w, float eps, void* resid_out, void* xn_out, void* out, void* ws,
                           size_t ws_bytes, void* stream) {
  using namespace rnb;
  int rc = validate(d, true, true);
  if (!rc) rc = check_device();
  if (!rc) rc = check_ws(d, ws, ws_bytes);
  if (rc) return rc;
  if (!resid || !norm_w || !resid_out || !xn_out || !out)
    return fail(RNB_ERR_INVALID, "resid, norm_w, resid_out, xn_out and out must be non-NULL");
  if (!aligned16(resid) || !aligned16(resid_out) || !aligned16(xn_out) || !aligned16(out) ||
      (y_prev && !aligned16(y_prev)))
    return fail(RNB_ERR_ALIGN, "resid, y_prev, resid_out, xn_out and out must be 16-byte aligned");
  if (resid_out == resid || resid_out == y_prev || xn_out == resid || xn_out == y_prev)
    return fail(RNB_ERR_INVALID, "resid_out and xn_out must not alias resid or y_prev");
  if (ep && ep->world > 1 && !ep->connected) return fail(RNB_ERR_INVALID, "call rnb_ep_connect first");
  if (ep && d->H != ep->H) return fail(RNB_ERR_INVALID, "H differs from the EP context's");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // One persistent launch when the plan fits: the glue runs in its prologue.
  if (!(d->flags & RNB_FLAG_CHAIN)) {
    Params p = base_params(d, resid, ws, kModeBlock);
    p.out = out;
    p.resid = static_cast<const uint16_t*>(resid);
    p.y_prev = static_cast<const uint16_t*>(y_prev);
    p.norm_w = static_cast<const uint16_t*>(norm_w);
    p.norm_eps = eps;
    p.resid_out = static_cast<uint16_t*>(resid_out);
    p.xn_out = static_cast<uint16_t*>(xn_out);
    if (ep) {
      const int nq = d->I / 128;
      p.shared_qmask = 0;
      for (int q = ep->rank; q < nq; q += ep->world) p.shared_qmask |= 1u << q;
      p.ep_world = ep->world;
      p.ep_rank = ep->rank;
      p.ep_limit_ns = ep->wait_ns;
      for (int q = 0; q < ep->world; ++q) p.ep_recv[q] = ep->recv[q];
      p.ep_seq = ep->seq;
    }
    const DevInfo di = dev_info();
    PPlan pl;
    size_t smem = 0;
    const bool ok = d->bits == 8 ? persistent_plan<8>(p, di, pl, smem) : persistent_plan<4>(p, di, pl, smem);
    if (ok) return d->bits == 8 ? run_persistent<8>(p, pl, smem, di.sms, st) : run_persistent<4>(p, pl, smem, di.sms, st);
  }
  // Otherwise the glue kernel, then the block on its output.
  rc = rnb_add_rmsnorm(resid, y_prev, norm_w, resid_out, xn_out, d->T, d->H, eps, stream);
  if (rc) return rc;
  return ep ? rnb_moe_block_ep_fwd(d, ep, xn_out, out, nullptr, nullptr, ws, ws_bytes, stream)
            : rnb_moe_block_fwd(d, xn_out, out, nullptr, nullptr, ws, ws_bytes, stream);
}
