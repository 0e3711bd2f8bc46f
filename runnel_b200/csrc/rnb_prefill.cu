// rnb_prefill.cu -- sparse-MoE block for many tokens (prefill) on tcgen05.
//
//   k_route_gemm   router logits of 128 tokens x 128 experts per CTA on
//                  tcgen05 (bf16, fp32 TMEM accumulation in four K quarters
//                  added in fp64) and the router rows' norms.
//   k_pre_select   a warp per token: candidate intervals of the bf16 logits
//                  (rnb_route.cuh), exact top-k, softmax weights,
//                  shared-expert gate, power-of-two fp16 scale and fp16 copy
//                  of the token, per-expert token histogram.
//   k_pre_sort     one CTA: per-expert row bases padded to 128 rows and the
//                  list of 256-row work tiles (the shared expert is expert E,
//                  all tokens).
//   k_pre_scatter  (token, slot) entries -> expert-sorted rows (counting sort).
//   k_pre_gather   the sorted rows' fp16 tokens (the gate/up A operand).
//   k_pre_gemm<0>  grouped gate/up GEMM + SwiGLU: 256 rows x (64 up + 64 gate)
//                  channels per work item, K = H in 64-wide stages.
//   k_pre_hrow     one power-of-two scale per SwiGLU row.
//   k_pre_gemm<1>  grouped down GEMM: 256 rows x 128 outputs, K = I; writes
//                  score * y of every sorted row as fp16 with one power-of-two
//                  scale per (row, 128-column n-tile) -- no atomics.
//   k_pre_final    per token, the sum of its rows (routed slots, then the
//                  shared expert) in slot order -> bf16 (or fp32) output;
//                  results do not depend on the schedule.
//
// The weights stay in MLX's affine layout; k_pre_gemm's converter warps
// dequantise them in shared memory to fp16 (w = s*q + b with one rounding)
// right before the tensor cores read them; see k_pre_gemm for the pipeline.
//
// Reference semantics: src/runnel/mlx.py:57-82 (sorted gather_qmm when
// indices.size >= 64), bench/mlx_lm_adapter.py:82-94 (shared expert).
#include <cuda.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <string>

#include "rnb_common.cuh"
#include "rnb_route.cuh"
#include "rnb_internal.h"
#include "rnb_moe.h"
#include "rnb_umma.cuh"

namespace rnb {
namespace pre {

constexpr int kTileM = 128;  // MMA M; expert rows are padded to multiples of it
constexpr int kItemM = 256;  // rows of a GEMM work item: two M tiles sharing one dequantised B tile
constexpr int kProducerWarps = 8;
constexpr int kMmaWarp = 8;
// warps 9..12: epilogue, one per TMEM lane quadrant (warp % 4); warp 13: TMA loader
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;
constexpr int kMaxE = 256;
constexpr int kMaxK = 8;

struct Ws {
  uint32_t* status;
  uint32_t* counts;  // [E+1] rows per local expert (index E: shared expert)
  uint32_t* fill;    // [E+1]
  uint32_t* base;    // [E+1] first sorted row
  uint32_t* n_mt;    // [1] number of 256-row item tiles
  uint4* tiles;      // [max_mt] (expert, row0, nrows <= 256, 0)
  uint32_t* perm;    // [rows_cap] entry id t*(K+1)+slot, 0xFFFFFFFF for padding
  uint32_t* inds;    // [T][K]
  float* scores;     // [T][K]
  float* sg;         // [T]
  float* xscale;     // [T] power of two bringing max|x_t| into [2^14, 2^15)
  __half* x16;       // [T][H] activations times xscale, fp16
  __half* xs16;      // [rows_cap][H] x16 rows in expert order (gate/up A operand)
  __half* h16;       // [rows_cap][I] SwiGLU activations, one scale per row after k_pre_hrow
  float* hinv;       // [rows_cap][I/64] inverse scale of each 64-channel chunk
  float* hrow;       // [rows_cap] inverse scale of the row (largest chunk inverse scale)
  uint32_t* lg;      // [T][E_total+1] fp32 router logits (tcgen05 router; the last column unused)
  float* wn;         // [2][E_total] router rows' sums of squares and of absolute values
  __half* y16;       // [rows_cap][H] down outputs times their weight, fp16, one scale per (row, n-tile)
  float* yinv;       // [rows_cap][H/128] inverse of that scale
  uint32_t* rowpos;  // [T][K+1] sorted row of entry t*(K+1)+slot, 0xFFFFFFFF if none
  uint16_t* rhi;     // 8-bit router: [E_total+1][H] bf16 high parts of the dequantised rows
  uint16_t* rlo;     //   (the last row the shared gate) and [E_total+1][H] low parts
};

struct Params {
  int T, H, I, E, E_total, off, k, has_shared, y_f32;
  int rows_cap, max_mt;
  const uint16_t* x;
  const uint16_t* router_w;  // bf16 router rows (8-bit router: ws.rhi)
  const uint16_t* sgate_w;   // bf16 shared-gate row (8-bit router: row E_total of ws.rhi)
  int router_q8;             // 8-bit affine router: codes, scales and biases below
  const uint32_t *router_q, *sgate_q;
  const uint16_t *router_s, *router_b, *sgate_s, *sgate_b;
  const uint32_t *gu_w, *dn_w, *sgu_w, *sdn_w;
  const uint16_t *gu_s, *gu_b, *dn_s, *dn_b, *sgu_s, *sgu_b, *sdn_s, *sdn_b;
  void* out;  // bf16 [T][H], or fp32 with y_f32
  uint32_t* inds_out;
  float* scores_out;
  // given routing (rnb_moe_experts_fwd): [T][k] global expert ids and weights
  const uint32_t* inds_in;
  const float* scores_in;
  Ws ws;
};

// fp16 pair helpers
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b),
                            *reinterpret_cast<const __half2*>(&c));
  return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t half2_bits(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 16 bytes of 8-bit codes (16 consecutive K) -> two 16-byte fp16 chunks, w = s*q + b.
__device__ __forceinline__ void deq_q8_16(const uint4 v, uint32_t s2, uint32_t b2, uint4& o0, uint4& o1) {
  uint32_t p[8];
  q8_word_to_pairs(v.x, p[0], p[1]);
  q8_word_to_pairs(v.y, p[2], p[3]);
  q8_word_to_pairs(v.z, p[4], p[5]);
  q8_word_to_pairs(v.w, p[6], p[7]);
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = hfma2_u32(p[i], s2, b2);
  o0 = make_uint4(p[0], p[1], p[2], p[3]);
  o1 = make_uint4(p[4], p[5], p[6], p[7]);
}


// one word of 4-bit codes (8 consecutive K) -> one 16-byte fp16 chunk in
// natural K order, pairs (0,1),(2,3),(4,5),(6,7): even nibbles sit in the
// low nibbles of x's bytes, odd ones in y's; a byte permute puts nibbles 2j
// and 2j+1 into the two halves, the AND/OR makes 1024 + q of each.
__device__ __forceinline__ uint4 deq_q4_word_nat(uint32_t w, uint32_t s2, uint32_t b2) {
  const uint32_t x = w & 0x0F0F0F0Fu, y = (w >> 4) & 0x0F0F0F0Fu;
  const uint32_t p0 = hsub_1024(lop3_and_or(__byte_perm(x, y, 0x0400), 0x000F000Fu, 0x64006400u));
  const uint32_t p1 = hsub_1024(lop3_and_or(__byte_perm(x, y, 0x0501), 0x000F000Fu, 0x64006400u));
  const uint32_t p2 = hsub_1024(lop3_and_or(__byte_perm(x, y, 0x0602), 0x000F000Fu, 0x64006400u));
  const uint32_t p3 = hsub_1024(lop3_and_or(__byte_perm(x, y, 0x0703), 0x000F000Fu, 0x64006400u));
  return make_uint4(hfma2_u32(p0, s2, b2), hfma2_u32(p1, s2, b2), hfma2_u32(p2, s2, b2), hfma2_u32(p3, s2, b2));
}


__device__ __forceinline__ uint32_t bf16_to_half2_dup(uint16_t b) {
  const float f = __uint_as_float(static_cast<uint32_t>(b) << 16);
  return half2_bits(f, f);
}

// ------------------------------------------------------------ router

// Given routing (no router): a warp per token copies its k expert ids and
// weights, computes the power-of-two fp16 scale and the fp16 token copy, and
// counts local experts.  Ids outside [0, E_total) are skipped and flagged.
__global__ void __launch_bounds__(512) k_pre_given(Params p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * 16 + warp;
  if (t >= p.T) return;
  const int K = p.k, H = p.H;
  if (lane < K) {
    const uint32_t e = __ldg(p.inds_in + static_cast<size_t>(t) * K + lane);
    const float w = __ldg(p.scores_in + static_cast<size_t>(t) * K + lane);
    const bool bad = e >= static_cast<uint32_t>(p.E_total);
    if (bad) atomicOr(p.ws.status, RNB_STATUS_BAD_INDEX);
    const uint32_t eo = bad ? 0xFFFFFFFFu : e;
    p.ws.inds[static_cast<size_t>(t) * K + lane] = eo;
    p.ws.scores[static_cast<size_t>(t) * K + lane] = w;
    const int le = static_cast<int>(eo) - p.off;
    if (!bad && le >= 0 && le < p.E) atomicAdd(&p.ws.counts[le], 1u);
  }
  const uint4* xr = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * H);
  float m = 0.f;
  for (int q = lane; q < H / 8; q += 32) {
    const uint4 v = __ldg(xr + q);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[j] << 16)), fabsf(__uint_as_float(w[j] & 0xFFFF0000u))));
  }
  m = warp_max(m);
  float sc, inv;
  fp16_range_scale(m, sc, inv);
  if (lane == 0) {
    p.ws.xscale[t] = sc;
    p.ws.sg[t] = 0.f;
  }
  uint4* xo = reinterpret_cast<uint4*>(p.ws.x16 + static_cast<size_t>(t) * H);
  for (int q = lane; q < H / 8; q += 32) {
    const uint4 v = __ldg(xr + q);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = half2_bits(__uint_as_float(w[j] << 16) * sc, __uint_as_float(w[j] & 0xFFFF0000u) * sc);
    xo[q] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Standalone quantized matmul (rnb_qmm) through the down GEMM: one expert (the
// whole W, H = N outputs, I = K), every token one row with weight 1.  A warp
// per token: the fp16 row with a power-of-two scale (h16, hrow = its inverse)
// and the row's entry; thread 0 of block 0 writes the 256-row item tiles.
__global__ void __launch_bounds__(512) k_qmm_prep(Params p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const uint32_t n = static_cast<uint32_t>((p.T + kItemM - 1) / kItemM);
    for (uint32_t j = 0; j < n; ++j) {
      const uint32_t left = static_cast<uint32_t>(p.T) - j * kItemM;
      p.ws.tiles[j] = make_uint4(0u, j * kItemM, left < static_cast<uint32_t>(kItemM) ? left : kItemM, 0u);
    }
    *p.ws.n_mt = n;
  }
  const int t = blockIdx.x * 16 + warp;
  if (t >= p.T) return;
  const int K = p.I;
  const uint4* xr = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * K);
  float m = 0.f;
  for (int q = lane; q < K / 8; q += 32) {
    const uint4 v = __ldg(xr + q);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[j] << 16)), fabsf(__uint_as_float(w[j] & 0xFFFF0000u))));
  }
  m = warp_max(m);
  float sc, inv;
  fp16_range_scale(m, sc, inv);
  uint4* ho = reinterpret_cast<uint4*>(p.ws.h16 + static_cast<size_t>(t) * K);
  for (int q = lane; q < K / 8; q += 32) {
    const uint4 v = __ldg(xr + q);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = half2_bits(__uint_as_float(w[j] << 16) * sc, __uint_as_float(w[j] & 0xFFFF0000u) * sc);
    ho[q] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (lane == 0) {
    p.ws.hrow[t] = inv;
    p.ws.perm[t] = static_cast<uint32_t>(t) * 2u;  // entry t * (k + 1) + 0 with k = 1
    p.ws.rowpos[static_cast<size_t>(t) * 2] = static_cast<uint32_t>(t);
    p.ws.scores[t] = 1.0f;
  }
}

// ------------------------------------------------ router on tcgen05

// k_route_gemm: router logits of 128 tokens x 128 experts per CTA on the
// tensor cores (kind::f16 with bf16 x and bf16 router rows, fp32 TMEM
// accumulation).  The K range is split into four quarters accumulated
// separately (4 x 128 TMEM columns) and added in fp64, so each fp32
// accumulation spans 32 MMA steps: the error allowance is kRouteRelTc
// (rnb_route.cuh).  Roles (8 warps):
//   warp 0    TMA: per 64-wide K stage the 128 x rows and the 128 router rows
//             (128-byte swizzle; boxes reaching past T or E_total read zeros);
//   warp 1    one thread issues the MMAs (M=128, N=128, K=16) into the
//             stage's K quarter;
//   warps 2-3 a share of the router rows' norms (sum of squares, sum of
//             absolute values; rows spread over the token tiles);
//   warps 4-7 one token per thread (one TMEM lane each): the 128 fp32 logits.
// k_pre_select turns the logits into candidate intervals and routes.
// 8-bit router: a warp per row of the router (and the shared gate) writes the
// dequantised weights w = fp32(s * code + b) as two bf16 parts, hi = bf16(w)
// and lo = bf16(w - hi), so the router GEMM runs on bf16 tensor cores over
// hi and then lo (|w - hi - lo| <= 2^-17.9 |w|; kRouteRelQ8 covers it).
__global__ void __launch_bounds__(512) k_router_split(Params p) {
  const int lane = threadIdx.x & 31, row = blockIdx.x * 16 + (threadIdx.x >> 5);
  const int H = p.H, Et = p.E_total;
  if (row > Et || (row == Et && !p.has_shared)) return;
  const uint32_t* q = row < Et ? p.router_q + static_cast<size_t>(row) * (H / 4) : p.sgate_q;
  const uint16_t* sc = row < Et ? p.router_s + static_cast<size_t>(row) * (H / 64) : p.sgate_s;
  const uint16_t* bi = row < Et ? p.router_b + static_cast<size_t>(row) * (H / 64) : p.sgate_b;
  uint4* hi = reinterpret_cast<uint4*>(p.ws.rhi + static_cast<size_t>(row) * H);
  uint4* lo = reinterpret_cast<uint4*>(p.ws.rlo + static_cast<size_t>(row) * H);
  for (int c = lane; c < H / 8; c += 32) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(q) + c);
    const float s = bf16_bits_to_f32(__ldg(sc + c / 8)), b = bf16_bits_to_f32(__ldg(bi + c / 8));
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t word = j < 2 ? w.x : w.y;
      const int sh = 16 * (j & 1);
      const float w0 = fmaf(s, static_cast<float>((word >> sh) & 0xFFu), b);
      const float w1 = fmaf(s, static_cast<float>((word >> (sh + 8)) & 0xFFu), b);
      const __nv_bfloat162 hh = __floats2bfloat162_rn(w0, w1);
      const float2 hf = __bfloat1622float2(hh);
      const __nv_bfloat162 ll = __floats2bfloat162_rn(w0 - hf.x, w1 - hf.y);
      h[j] = *reinterpret_cast<const uint32_t*>(&hh);
      l[j] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    hi[c] = make_uint4(h[0], h[1], h[2], h[3]);
    lo[c] = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

constexpr int kRgStages = 6;
constexpr int kRgTile = 128 * 128;                    // 128 rows x 64 bf16
constexpr int kRgStage = 2 * kRgTile;                 // x tile + router tile
constexpr size_t kRgSmem = static_cast<size_t>(kRgStages) * kRgStage + 1024;
static_assert(kRgStage % 1024 == 0, "stages keep the 1024-byte swizzle alignment");

struct RouteMaps {
  CUtensorMap x, w, wl;  // wl: the low parts of an 8-bit router (unused otherwise)
};

__global__ void __launch_bounds__(256, 1) k_route_gemm(Params p, const __grid_constant__ RouteMaps tm) {
  extern __shared__ char rgraw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(rgraw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[kRgStages], empty[kRgStages], mdone;
  __shared__ uint32_t tslot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * 128, e0 = blockIdx.y * 128;
  const int H = p.H, Et = p.E_total, nks = H / 64, qk = nks / 4;
  // an 8-bit router runs the K range twice: high parts, then low parts
  const int nsteps = p.router_q8 ? 2 * nks : nks;
  if (tid == 0) {
    for (int s = 0; s < kRgStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&mdone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = tslot;
  bool timed_out = false;
  if (warp == 0) {
    if (lane == 0) {
      for (int ks = 0; ks < nsteps; ++ks) {
        const int s = ks % kRgStages, n = ks / kRgStages, kk = ks % nks;
        if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, kWaitNs)) {
          timed_out = true;
          break;
        }
        const uint32_t bar = smem_u32(&full[s]);
        mbar_arrive_expect_tx(&full[s], kRgStage);
        tma_load_2d(smem_u32(sm + s * kRgStage), &tm.x, kk * 64, t0, bar);
        tma_load_2d(smem_u32(sm + s * kRgStage + kRgTile), ks < nks ? &tm.w : &tm.wl, kk * 64, e0, bar);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(128, 128, true);
      for (int ks = 0; ks < nsteps; ++ks) {
        const int s = ks % kRgStages, n = ks / kRgStages, kk = ks % nks;
        if (!mbar_wait(&full[s], n & 1, kWaitNs)) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sm + s * kRgStage), b0 = a0 + kRgTile;
        const uint32_t d = taddr + static_cast<uint32_t>(kk / qk) * 128u;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(d, umma_desc_sw128(a0 + k * 32), umma_desc_sw128(b0 + k * 32), idesc,
                   (ks < nks && kk % qk == 0 && k == 0) ? 0u : 1u);
        umma_commit(smem_u32(&empty[s]));
      }
      umma_commit(smem_u32(&mdone));  // also when the loop ended early: every issued MMA done
      // every MMA this thread issued has completed before TMEM is released
      if (!mbar_wait(&mdone, 0, kWaitNs)) timed_out = true;
    }
  } else if (warp < 4) {
    // router-row norms, a warp per row: rows e0 + r with r / 8 = blockIdx.x
    // (mod gridDim.x); every CTA column covers its 128 rows once
    for (int r = blockIdx.x * 8 + (warp - 2); r < 128; r += gridDim.x * 8) {
      for (int rr = r; rr < r + 8 && rr < 128; rr += 2) {
        const int e = e0 + rr;
        if (e >= Et) break;
        const uint4* wr = reinterpret_cast<const uint4*>(p.router_w + static_cast<size_t>(e) * H);
        float n2 = 0.f, n1 = 0.f;
        for (int q = lane; q < H / 8; q += 32) {
          const uint4 v = __ldg(wr + q);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xFFFF0000u);
            n2 = fmaf(lo, lo, fmaf(hi, hi, n2));
            n1 += fabsf(lo) + fabsf(hi);
          }
        }
        n2 = warp_sum(n2);
        n1 = warp_sum(n1);
        if (lane == 0) {
          p.ws.wn[e] = n2;
          p.ws.wn[Et + e] = n1;
        }
      }
    }
  } else {
    // one token per thread: TMEM lane 32 (warp % 4) + lane
    const int q4 = warp & 3, t = t0 + 32 * q4 + lane;
    const bool ok = mbar_wait(&mdone, 0, kWaitNs);
    // the whole warp leaves together: tcgen05.ld below is warp-collective
    if (__any_sync(0xffffffffu, !ok)) {
      timed_out = true;
    } else {
      tc_fence_after();
      uint32_t* lg = p.ws.lg + static_cast<size_t>(t < p.T ? t : 0) * (Et + 1);
      const uint32_t tl = taddr + (static_cast<uint32_t>(q4 * 32) << 16);
      for (int c0 = 0; c0 < 128; c0 += 16) {
        uint32_t v[4][16];
#pragma unroll
        for (int kq = 0; kq < 4; ++kq) tmem_ld16(tl + kq * 128 + c0, v[kq]);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int e = e0 + c0 + j;
          const double L = (static_cast<double>(__uint_as_float(v[0][j])) + __uint_as_float(v[1][j])) +
                           (static_cast<double>(__uint_as_float(v[2][j])) + __uint_as_float(v[3][j]));
          if (t < p.T && e < Et) lg[e] = __float_as_uint(static_cast<float>(L));
        }
      }
    }
  }
  if (timed_out) atomicOr(p.ws.status, RNB_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    tmem_dealloc(taddr, 512);
    tmem_relinquish();
  }
}

// One warp per token, after k_route_gemm: the token's norms, the candidate
// intervals of its bf16 logits (rnb_route.cuh), top-k selection with the
// exact recompute of uncertain candidates, the weights, the shared-expert
// gate (fp32 dot), the power-of-two fp16 scale and fp16 copy of the token,
// and the local-expert histogram.
constexpr int kSelMaxH = 2048;
__global__ void __launch_bounds__(512, 2) k_pre_select(Params p) {
  __shared__ uint32_t hist[kMaxE];
  __shared__ uint32_t s_ivl[16][kMaxE + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < kMaxE; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int t = blockIdx.x * 16 + warp;
  const int K = p.k, H = p.H, Et = p.E_total, nq = H / 256;  // 16-byte pieces per lane
  if (t < p.T) {
    const size_t tg = static_cast<size_t>(t);
    const uint4* xr = reinterpret_cast<const uint4*>(p.x + tg * H);
    const uint4* gr = reinterpret_cast<const uint4*>(p.sgate_w);
    // 8-bit shared gate: the high parts above, the low parts here
    const uint4* grl = p.router_q8 ? reinterpret_cast<const uint4*>(p.ws.rlo + static_cast<size_t>(Et) * H) : nullptr;
    uint4 xv[kSelMaxH / 256];
    float xn2 = 0.f, xinf = 0.f, sgl = 0.f;
#pragma unroll
    for (int q = 0; q < kSelMaxH / 256; ++q) {
      if (q < nq) {
        xv[q] = __ldg(xr + q * 32 + lane);
        uint4 gw = make_uint4(0u, 0u, 0u, 0u), gl = gw;
        if (p.has_shared) gw = __ldcg(gr + q * 32 + lane);
        if (p.has_shared && grl) gl = __ldcg(grl + q * 32 + lane);
        const uint32_t w[4] = {xv[q].x, xv[q].y, xv[q].z, xv[q].w}, g[4] = {gw.x, gw.y, gw.z, gw.w},
                       gq[4] = {gl.x, gl.y, gl.z, gl.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xFFFF0000u);
          xn2 = fmaf(lo, lo, fmaf(hi, hi, xn2));
          xinf = fmaxf(xinf, fmaxf(fabsf(lo), fabsf(hi)));
          const float g0 = __uint_as_float(g[j] << 16) + __uint_as_float(gq[j] << 16);
          const float g1 = __uint_as_float(g[j] & 0xFFFF0000u) + __uint_as_float(gq[j] & 0xFFFF0000u);
          sgl = fmaf(lo, g0, fmaf(hi, g1, sgl));
        }
      }
    }
    xn2 = warp_sum(xn2);
    sgl = warp_sum(sgl);
    xinf = warp_max(xinf);
    // the fp16 copy first, so the token's registers are free before routing
    float xsc, xinv;
    fp16_range_scale(xinf, xsc, xinv);
    if (lane == 0) {
      p.ws.sg[tg] = p.has_shared ? 1.0f / (1.0f + expf(-sgl)) : 0.f;
      p.ws.xscale[tg] = xsc;
    }
    uint4* xo = reinterpret_cast<uint4*>(p.ws.x16 + tg * H);
#pragma unroll
    for (int q = 0; q < kSelMaxH / 256; ++q) {
      if (q < nq) {
        const uint32_t w[4] = {xv[q].x, xv[q].y, xv[q].z, xv[q].w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = half2_bits(__uint_as_float(w[j] << 16) * xsc, __uint_as_float(w[j] & 0xFFFF0000u) * xsc);
        xo[q * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    // every load of the token's logits and the router-row norms is issued
    // before the intervals are formed (E_total <= kMaxE = 256: 8 per lane)
    const uint32_t* lgt = p.ws.lg + tg * (Et + 1);
    float lv[kMaxE / 32], w2[kMaxE / 32], w1[kMaxE / 32];
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
      const int e = lane + 32 * i;
      lv[i] = e < Et ? __uint_as_float(__ldcg(lgt + e)) : 0.f;
      w2[i] = e < Et ? __ldcg(p.ws.wn + e) : 0.f;
      w1[i] = e < Et ? __ldcg(p.ws.wn + Et + e) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
      const int e = lane + 32 * i;
      if (e < Et)
        s_ivl[warp][e] = route_interval(lv[i], xn2, xinf, w2[i], w1[i], p.router_q8 ? kRouteRelQ8 : kRouteRelTc);
    }
    __syncwarp();
    int e;
    float sc;
    RouterSrc rs;
    rs.w = p.router_q8 ? nullptr : p.router_w;
    rs.q = p.router_q8 ? p.router_q : nullptr;
    rs.s = p.router_s;
    rs.b = p.router_b;
    warp_route_token(s_ivl[warp], Et, K, p.x + tg * H, rs, H, lane, false, nullptr, &e, &sc);
    if (lane < K) {
      p.ws.inds[tg * K + lane] = static_cast<uint32_t>(e);
      p.ws.scores[tg * K + lane] = sc;
      if (p.inds_out) p.inds_out[tg * K + lane] = static_cast<uint32_t>(e);
      if (p.scores_out) p.scores_out[tg * K + lane] = sc;
      const int le = e - p.off;
      if (le >= 0 && le < p.E) atomicAdd(&hist[le], 1u);
    }
  }
  __syncthreads();
  for (int e = tid; e < p.E; e += blockDim.x)
    if (hist[e]) atomicAdd(&p.ws.counts[e], hist[e]);
}

// ------------------------------------------------------ sort / scatter

__global__ void __launch_bounds__(512) k_pre_sort(Params p) {
  __shared__ uint32_t s_rows[kMaxE + 1], s_tiles[kMaxE + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E1 = p.E + (p.has_shared ? 1 : 0);
  for (int e = tid; e < E1; e += blockDim.x) {
    const uint32_t cnt = e < p.E ? p.ws.counts[e] : static_cast<uint32_t>(p.T);
    s_rows[e] = cnt;
    p.ws.fill[e] = 0;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t run_rows = 0, run_tiles = 0;
    for (int b0 = 0; b0 < E1; b0 += 32) {
      const int e = b0 + lane;
      const uint32_t cnt = e < E1 ? s_rows[e] : 0u;
      const uint32_t nt = (cnt + kTileM - 1) / kTileM, nst = (cnt + kItemM - 1) / kItemM;
      uint32_t ir = nt * kTileM, it = nst;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t a = __shfl_up_sync(0xffffffffu, ir, o), b = __shfl_up_sync(0xffffffffu, it, o);
        if (lane >= o) {
          ir += a;
          it += b;
        }
      }
      if (e < E1) {
        p.ws.base[e] = run_rows + ir - nt * kTileM;
        s_tiles[e] = run_tiles + it - nst;
      }
      run_rows += __shfl_sync(0xffffffffu, ir, 31);
      run_tiles += __shfl_sync(0xffffffffu, it, 31);
    }
    if (lane == 0) *p.ws.n_mt = run_tiles;
  }
  __syncthreads();
  for (int e = tid; e < E1; e += blockDim.x) {
    const uint32_t cnt = s_rows[e], nst = (cnt + kItemM - 1) / kItemM, b = p.ws.base[e];
    for (uint32_t j = 0; j < nst; ++j) {
      const uint32_t rows = cnt - j * kItemM < static_cast<uint32_t>(kItemM) ? cnt - j * kItemM : kItemM;
      p.ws.tiles[s_tiles[e] + j] = make_uint4(static_cast<uint32_t>(e), b + j * kItemM, rows, 0);
    }
  }
}

__global__ void k_pre_scatter(Params p) {
  const int K = p.k;
  const size_t n_routed = static_cast<size_t>(p.T) * K;
  const size_t total = n_routed + (p.has_shared ? p.T : 0);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    if (i < n_routed) {
      if (p.ws.inds[i] == 0xFFFFFFFFu) continue;
      const int le = static_cast<int>(p.ws.inds[i]) - p.off;
      if (le < 0 || le >= p.E) continue;
      const uint32_t pos = p.ws.base[le] + atomicAdd(&p.ws.fill[le], 1u);
      const uint32_t ent = static_cast<uint32_t>((i / K) * (K + 1) + (i % K));
      p.ws.perm[pos] = ent;
      p.ws.rowpos[ent] = pos;
    } else {
      const size_t t = i - n_routed;
      p.ws.perm[p.ws.base[p.E] + t] = static_cast<uint32_t>(t * (K + 1) + K);
      p.ws.rowpos[t * (K + 1) + K] = p.ws.base[p.E] + static_cast<uint32_t>(t);
    }
  }
}

// ------------------------------------------------------ grouped GEMM

// k_pre_gemm: persistent, one CTA per SM; work item = 256 rows of one
// expert (two M=128 tiles) x one 128-column n-tile (64 up + 64 gate
// channels, or 128 down outputs).  All global -> shared traffic is TMA,
// issued by one thread, so the SMs keep few requests of their own in flight:
//   warp 13    loader: per stage one 256-row A box (128-byte swizzle, the
//              tensor-core operand layout), the n-tile's raw MLX codes and
//              its scales and biases, all counted on one transaction barrier;
//              runs up to S stages ahead of the tensor core.
//   warps 0-7  converters: raw codes -> fp16 s*q + b into the swizzled B tile.
//   warp 8     one thread issues tcgen05.mma (M=128, N=128, K=16) for both
//              M halves into one of two TMEM accumulators (256 columns each).
//   warps 9-12 epilogue, one TMEM lane quadrant each; drains accumulator j&1
//              while the MMA fills the other.
// The gate/up A operand is the tokens' fp16 copy gathered into expert order
// (k_pre_gather); the down A operand is the SwiGLU rows, already in order.
template <int BITS>
struct GemmCfg {
  static constexpr int N = 128;
  static constexpr int S = 3;                          // shared-memory stages
  static constexpr int kA = kItemM * 128;              // two M=128 operands, 16 KB apart
  static constexpr int kB = N * 128;                   // fp16 B tile (swizzled)
  static constexpr int kRawRow = 64 * BITS / 8;        // raw code bytes of a B row per stage
  static constexpr int kRaw = N * kRawRow;
  static constexpr int kScl = N * 16;                  // 8 groups of bf16 scales per B row
  static constexpr int kStage = kA + kB + kRaw + 2 * kScl;
  static constexpr uint32_t kTx = kA + kRaw + 2 * kScl;  // TMA bytes per stage
  static constexpr uint32_t kTmemCols = 512;
  // down epilogue: per epilogue warp a 32 x 32 fp32 tile (rows padded to 36
  // floats) to turn row-per-lane results into row-contiguous atomics
  static constexpr int kTpPitch = 36;
  static constexpr int kTp = 4 * 32 * kTpPitch * 4;
  static constexpr size_t kSmem = static_cast<size_t>(S) * kStage + kTp + 1024;
  static_assert(kStage % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
};

// TMA descriptors of one grouped GEMM: the A operand and the routed and
// shared experts' codes, scales and biases.
struct TmaMaps {
  CUtensorMap a, bw, bs, bb, sbw, sbs, sbb;
};

constexpr int kGemmThreads = 14 * 32;
constexpr int kLoaderWarp = 13;

template <int BITS, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1) k_pre_gemm(Params p, const __grid_constant__ TmaMaps tm) {
  using C = GemmCfg<BITS>;
  extern __shared__ char smraw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t tld[C::S], full[C::S], empty[C::S], tfull[2], tempty[2], mdone;
  __shared__ uint32_t tslot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.k, H = p.H, I = p.I;
  const int kdim = MODE == 0 ? H : I;
  const int nks = kdim / 64;
  const int n_nt = MODE == 0 ? (2 * I) / C::N : H / C::N;  // n-tiles: 64 up + 64 gate channels, or 128 outputs
  const uint32_t n_items = __ldcg(p.ws.n_mt) * static_cast<uint32_t>(n_nt);
  const uint32_t G = gridDim.x;
  const uint32_t n_local = n_items > blockIdx.x ? (n_items - blockIdx.x + G - 1) / G : 0u;
  const uint32_t n_stages = n_local * static_cast<uint32_t>(nks);

  if (tid == 0) {
    for (int s = 0; s < C::S; ++s) {
      mbar_init(&tld[s], 1);
      mbar_init(&full[s], kProducerWarps * 32);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4 * 32);
    }
    mbar_init(&mdone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == kMmaWarp) tmem_alloc(&tslot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = tslot;
  bool timed_out = false;

  if (warp == kLoaderWarp) {
    // ------------------------------------------------ TMA loader (one thread)
    if (lane == 0) {
      uint32_t cur_li = 0xFFFFFFFFu;
      int ya = 0, yb = 0;
      bool se = false;
      for (uint32_t st = 0; st < n_stages; ++st) {
        const int slot = static_cast<int>(st % C::S);
        const uint32_t n = st / C::S;
        if (n > 0 && !mbar_wait(&empty[slot], (n - 1) & 1, kWaitNs)) {
          timed_out = true;
          break;
        }
        const uint32_t li = st / nks;
        const int ks = static_cast<int>(st % nks);
        if (li != cur_li) {
          cur_li = li;
          const uint32_t item = blockIdx.x + li * G;
          const uint4 tile = __ldg(p.ws.tiles + item / n_nt);
          const int e = static_cast<int>(tile.x), nt = static_cast<int>(item % n_nt);
          se = e == p.E;
          ya = static_cast<int>(tile.y);
          // first B row of the n-tile in the expert bank (or the shared expert)
          yb = MODE == 0 ? (se ? 0 : e * 2 * I) + nt * 64 : (se ? 0 : e * H) + nt * C::N;
        }
        char* sA = sm + slot * C::kStage;
        char* sRaw = sA + C::kA + C::kB;
        char* sScl = sRaw + C::kRaw;
        const uint32_t bar = smem_u32(&tld[slot]);
        mbar_arrive_expect_tx(&tld[slot], C::kTx);
        tma_load_2d(smem_u32(sA), &tm.a, ks * 64, ya, bar);
        const CUtensorMap* mw = se ? &tm.sbw : &tm.bw;
        const CUtensorMap* ms = se ? &tm.sbs : &tm.bs;
        const CUtensorMap* mb = se ? &tm.sbb : &tm.bb;
        const int xs = (ks >> 3) * 8;  // 8-group block of the scales holding group ks
        if (MODE == 0) {
          // up rows then gate rows, 64 each
          for (int h = 0; h < 2; ++h) {
            const int y = yb + h * I;
            tma_load_2d(smem_u32(sRaw + h * 64 * C::kRawRow), mw, ks * C::kRawRow, y, bar);
            tma_load_2d(smem_u32(sScl + h * 64 * 16), ms, xs, y, bar);
            tma_load_2d(smem_u32(sScl + C::kScl + h * 64 * 16), mb, xs, y, bar);
          }
        } else {
          tma_load_2d(smem_u32(sRaw), mw, ks * C::kRawRow, yb, bar);
          tma_load_2d(smem_u32(sScl), ms, xs, yb, bar);
          tma_load_2d(smem_u32(sScl + C::kScl), mb, xs, yb, bar);
        }
      }
    }
  } else if (warp < kProducerWarps) {
    // ------------------------------------------------ converters
    const int pt = tid;  // 0..255
    for (uint32_t st = 0; st < n_stages; ++st) {
      const int slot = static_cast<int>(st % C::S);
      const uint32_t n = st / C::S;
      const bool ok = mbar_wait(&tld[slot], n & 1, kWaitNs);
      if (!ok) {
        timed_out = true;
        break;
      }
      const int ks = static_cast<int>(st % nks);
      char* sA = sm + slot * C::kStage;
      char* sB = sA + C::kA;
      const char* sRaw = sB + C::kB;
      const uint16_t* sSc = reinterpret_cast<const uint16_t*>(sRaw + C::kRaw);
      const uint16_t* sBi = sSc + C::kScl / 2;
      const int g = ks & 7;
      if (BITS == 8) {
        // 128 rows x 4 16-byte chunks: thread -> chunk pt % 4 of rows pt / 4 and pt / 4 + 64
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int tr = (pt >> 2) + 64 * i, c = pt & 3;
          const uint4 v = *reinterpret_cast<const uint4*>(sRaw + tr * C::kRawRow + c * 16);
          const uint32_t s2 = bf16_to_half2_dup(sSc[tr * 8 + g]);
          const uint32_t b2 = bf16_to_half2_dup(sBi[tr * 8 + g]);
          uint4 o0, o1;
          deq_q8_16(v, s2, b2, o0, o1);
          *reinterpret_cast<uint4*>(sB + sw128_offset(tr, c * 16)) = o0;
          *reinterpret_cast<uint4*>(sB + sw128_offset(tr, c * 16 + 8)) = o1;
        }
      } else {
        // 128 rows x 2 16-byte chunks (32 codes each): thread -> chunk pt % 2 of row pt / 2
        const int tr = pt >> 1, c = pt & 1;
        const uint4 v = *reinterpret_cast<const uint4*>(sRaw + tr * C::kRawRow + c * 16);
        const uint32_t s2 = bf16_to_half2_dup(sSc[tr * 8 + g]);
        const uint32_t b2 = bf16_to_half2_dup(sBi[tr * 8 + g]);
        *reinterpret_cast<uint4*>(sB + sw128_offset(tr, c * 32)) = deq_q4_word_nat(v.x, s2, b2);
        *reinterpret_cast<uint4*>(sB + sw128_offset(tr, c * 32 + 8)) = deq_q4_word_nat(v.y, s2, b2);
        *reinterpret_cast<uint4*>(sB + sw128_offset(tr, c * 32 + 16)) = deq_q4_word_nat(v.z, s2, b2);
        *reinterpret_cast<uint4*>(sB + sw128_offset(tr, c * 32 + 24)) = deq_q4_word_nat(v.w, s2, b2);
      }
      fence_proxy_async_smem();
      mbar_arrive(&full[slot]);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------ MMA issue (one thread)
    // item j accumulates in TMEM columns [256 (j & 1), +256): M half h in
    // [+128 h, +128); a second half with no rows is skipped
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(kTileM, C::N, false);
      uint32_t st = 0;
      for (uint32_t j = 0; j < n_local && !timed_out; ++j) {
        const uint32_t buf = j & 1;
        const uint32_t nrows = __ldcg(p.ws.tiles + (blockIdx.x + j * G) / n_nt).z;
        const int nh = nrows > static_cast<uint32_t>(kTileM) ? 2 : 1;
        if (j >= 2 && !mbar_wait(&tempty[buf], ((j >> 1) - 1) & 1, kWaitNs)) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        for (int ks = 0; ks < nks; ++ks, ++st) {
          const int s = static_cast<int>(st % C::S);
          if (!mbar_wait(&full[s], (st / C::S) & 1, kWaitNs)) {
            timed_out = true;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sm + s * C::kStage), b0 = a0 + C::kA;
          for (int h = 0; h < nh; ++h) {
            const uint32_t d = taddr + buf * 256 + h * 128;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(d, umma_desc_sw128(a0 + h * (C::kA / 2) + k * 32), umma_desc_sw128(b0 + k * 32), idesc,
                       (ks == 0 && k == 0) ? 0u : 1u);
          }
          umma_commit(smem_u32(&empty[s]));
        }
        if (timed_out) break;
        umma_commit(smem_u32(&tfull[buf]));
      }
      // every MMA this thread issued has completed before TMEM is released
      umma_commit(smem_u32(&mdone));
      if (!mbar_wait(&mdone, 0, kWaitNs)) timed_out = true;
    }
  } else {
    // ------------------------------------------------ epilogue (warps 9..12)
    // thread (quad, lane) owns TMEM lane r = 32 quad + lane: item row r of
    // M half 0 and row 128 + r of M half 1
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    for (uint32_t j = 0; j < n_local; ++j) {
      const uint32_t item = blockIdx.x + j * G;
      const uint32_t mt = item / n_nt, nt = item % n_nt;
      const uint32_t buf = j & 1;
      const uint4 tile = __ldcg(p.ws.tiles + mt);
      const int row0 = static_cast<int>(tile.y), nrows = static_cast<int>(tile.z);
      const int nh = nrows > kTileM ? 2 : 1;
      uint32_t ent[2];
      for (int h = 0; h < 2; ++h) {
        const int rr = h * kTileM + r;
        ent[h] = (h < nh && rr < nrows) ? __ldcg(p.ws.perm + row0 + rr) : 0xFFFFFFFFu;
      }
      // the whole warp leaves together: tcgen05.ld below is warp-collective
      const bool ok = mbar_wait(&tfull[buf], (j >> 1) & 1, kWaitNs);
      if (__any_sync(0xffffffffu, !ok)) {
        timed_out = true;
        break;
      }
      tc_fence_after();
      for (int h = 0; h < nh; ++h) {
        const uint32_t tl = taddr + buf * 256 + h * 128 + (static_cast<uint32_t>(quad * 32) << 16);
        const bool valid = ent[h] != 0xFFFFFFFFu;
        const uint32_t e_id = valid ? ent[h] : 0u;
        const size_t row = static_cast<size_t>(row0 + h * kTileM + r);
        if (MODE == 0) {
          // up in columns [0, 64), gate in [64, 128): 64 SwiGLU channels nt*64..,
          // computed once into registers, then scaled into fp16 and stored
          const uint32_t t = e_id / (K + 1);
          const float xinv = valid ? 1.0f / __ldcg(p.ws.xscale + t) : 1.f;
          float hv[64];
          float mx = 0.f;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t u[16], gt[16];
            tmem_ld16(tl + cc * 16, u);
            tmem_ld16(tl + 64 + cc * 16, gt);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const float up = __uint_as_float(u[q]) * xinv, ga = __uint_as_float(gt[q]) * xinv;
              // silu(g) = g / (1 + e^-g); the clamp keeps the denominator finite
              const float hq = __fdividef(ga, 1.0f + __expf(fminf(-ga, 80.0f))) * up;
              hv[cc * 16 + q] = hq;
              mx = fmaxf(mx, fabsf(hq));
            }
          }
          float hs, hi;
          fp16_range_scale(mx, hs, hi);
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(p.ws.h16 + row * I + nt * 64);
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8)
              dst[c8] = make_uint4(half2_bits(hv[c8 * 8] * hs, hv[c8 * 8 + 1] * hs),
                                   half2_bits(hv[c8 * 8 + 2] * hs, hv[c8 * 8 + 3] * hs),
                                   half2_bits(hv[c8 * 8 + 4] * hs, hv[c8 * 8 + 5] * hs),
                                   half2_bits(hv[c8 * 8 + 6] * hs, hv[c8 * 8 + 7] * hs));
            p.ws.hinv[row * (I / 64) + nt] = hi;
          }
        } else {
          const uint32_t t = e_id / (K + 1), slot = e_id % (K + 1);
          float w = 0.f;
          if (valid) {
            w = slot < static_cast<uint32_t>(K) ? __ldcg(p.ws.scores + static_cast<size_t>(t) * K + slot)
                                                : __ldcg(p.ws.sg + t);
            w *= __ldcg(p.ws.hrow + row);
          }
          // The n-tile of this row, times its weight, goes to y16 as fp16
          // with one power-of-two scale (the largest |value| of the 128
          // columns into fp16 range; read from TMEM twice) -- no atomics:
          // k_pre_final adds a token's rows in slot order.  The rows are
          // written through a shared-memory transpose so that four lanes
          // cover one row's 64 contiguous bytes.
          float mx = 0.f;
          for (int cc = 0; cc < C::N / 16; cc += 2) {
            uint32_t v[2][16];
            tmem_ld16(tl + cc * 16, v[0]);
            tmem_ld16(tl + (cc + 1) * 16, v[1]);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 16; ++q)
              mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(v[0][q])), fabsf(__uint_as_float(v[1][q]))));
          }
          float ysc, yiv;
          fp16_range_scale(mx * fabsf(w), ysc, yiv);
          const float m = w * ysc;
          uint32_t* tp = reinterpret_cast<uint32_t*>(sm + C::S * C::kStage) + quad * 32 * C::kTpPitch;
          const size_t grow0 = static_cast<size_t>(row0 + h * kTileM + quad * 32);
          for (int cc = 0; cc < C::N / 16; cc += 2) {
            uint32_t v[2][16];
            tmem_ld16(tl + cc * 16, v[0]);
            tmem_ld16(tl + (cc + 1) * 16, v[1]);
            tmem_wait_ld();
            __syncwarp();  // the previous chunk's reads are done
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t* vq = v[q >> 1] + (q & 1) * 8;
              *reinterpret_cast<uint4*>(tp + lane * C::kTpPitch + q * 4) =
                  make_uint4(half2_bits(__uint_as_float(vq[0]) * m, __uint_as_float(vq[1]) * m),
                             half2_bits(__uint_as_float(vq[2]) * m, __uint_as_float(vq[3]) * m),
                             half2_bits(__uint_as_float(vq[4]) * m, __uint_as_float(vq[5]) * m),
                             half2_bits(__uint_as_float(vq[6]) * m, __uint_as_float(vq[7]) * m));
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rr = (lane >> 2) + 8 * i, pc = lane & 3;
              const bool vr = __shfl_sync(0xffffffffu, valid ? 1 : 0, rr) != 0;
              const uint4 d = *reinterpret_cast<const uint4*>(tp + rr * C::kTpPitch + pc * 4);
              if (vr)
                *reinterpret_cast<uint4*>(p.ws.y16 + (grow0 + rr) * H + nt * C::N + cc * 16 + pc * 8) = d;
            }
          }
          if (valid) p.ws.yinv[row * (H / C::N) + nt] = yiv;
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }
  if (timed_out) atomicOr(p.ws.status, RNB_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    tmem_dealloc(taddr, C::kTmemCols);
    tmem_relinquish();
  }
}

// Gate/up A operand: each routed row's fp16 token copy, in expert order
// (a warp per row; padding rows stay unwritten and are never stored from).
__global__ void k_pre_gather(Params p) {
  const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const int n16 = p.H / 8;
  for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < p.rows_cap; row += gridDim.x * wpb) {
    const uint32_t ent = __ldcg(p.ws.perm + row);
    if (ent == 0xFFFFFFFFu) continue;
    const uint4* src = reinterpret_cast<const uint4*>(p.ws.x16 + static_cast<size_t>(ent / (p.k + 1)) * p.H);
    uint4* dst = reinterpret_cast<uint4*>(p.ws.xs16 + static_cast<size_t>(row) * p.H);
    // the whole row's loads in flight before its stores (H <= 2048: 8 per lane)
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane + 32 * j < n16) v[j] = __ldcg(src + lane + 32 * j);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane + 32 * j < n16) dst[lane + 32 * j] = v[j];
  }
}

// Between the GEMMs: give all 64-channel chunks of a SwiGLU row one scale,
// the smallest of the chunks' (the chunk with the largest values keeps its
// scale; the others are multiplied by a power of two <= 1, exact unless a
// value falls below fp16's normal range).  hrow = that scale's inverse.
// One warp per row; lane l handles 8-value pieces l, l+32.
__global__ void k_pre_hrow(Params p) {
  const int nq = p.I / 64, lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < p.rows_cap; row += gridDim.x * wpb) {
    if (__ldcg(p.ws.perm + row) == 0xFFFFFFFFu) continue;
    const float* h = p.ws.hinv + static_cast<size_t>(row) * nq;
    float m = 0.f;
    for (int c = 0; c < nq; ++c) m = fmaxf(m, __ldcg(h + c));
    uint4* hv = reinterpret_cast<uint4*>(p.ws.h16 + static_cast<size_t>(row) * p.I);
    for (int q = lane; q < p.I / 8; q += 32) {
      const float f = __ldcg(h + q / 8) / m;
      if (f != 1.0f) {
        const uint32_t f2 = half2_bits(f, f);
        uint4 v = hv[q];
        v.x = hmul2_u32(v.x, f2);
        v.y = hmul2_u32(v.y, f2);
        v.z = hmul2_u32(v.z, f2);
        v.w = hmul2_u32(v.w, f2);
        hv[q] = v;
      }
    }
    if (lane == 0) p.ws.hrow[row] = m;
  }
}

// out[t] = sum over slots s = 0..k (routed slots, then the shared expert) of
// yinv * y16 of the entry's sorted row, in slot order; 8 columns a thread.
__global__ void k_pre_final(Params p) {
  const int K = p.k, H = p.H, per_t = H / 8, ntile = H / 128;
  const size_t n = static_cast<size_t>(p.T) * per_t;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t t = i / per_t;
    const int c8 = static_cast<int>(i % per_t);
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // all rows first, then all their loads, then the ordered sum
    uint32_t row[kMaxK + 1];
#pragma unroll
    for (int s = 0; s <= kMaxK; ++s) row[s] = s <= K ? __ldcg(p.ws.rowpos + t * (K + 1) + s) : 0xFFFFFFFFu;
    float inv[kMaxK + 1];
    uint4 v[kMaxK + 1];
#pragma unroll
    for (int s = 0; s <= kMaxK; ++s) {
      const bool ok = row[s] != 0xFFFFFFFFu;
      inv[s] = ok ? __ldcg(p.ws.yinv + static_cast<size_t>(row[s]) * ntile + c8 / 16) : 0.f;
      v[s] = ok ? __ldcg(reinterpret_cast<const uint4*>(p.ws.y16 + static_cast<size_t>(row[s]) * H) + c8)
                : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int s = 0; s <= kMaxK; ++s) {
      const uint32_t w[4] = {v[s].x, v[s].y, v[s].z, v[s].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
        a[2 * j] = fmaf(f.x, inv[s], a[2 * j]);
        a[2 * j + 1] = fmaf(f.y, inv[s], a[2 * j + 1]);
      }
    }
    if (p.y_f32) {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(p.out) + t * H + c8 * 8);
      o[0] = make_float4(a[0], a[1], a[2], a[3]);
      o[1] = make_float4(a[4], a[5], a[6], a[7]);
    } else {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(a[2 * j], a[2 * j + 1]);
        o[j] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + t * H)[c8] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ----------------------------------------------------------- host side

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct Layout {
  size_t status, counts, fill, base, n_mt, tiles, perm, inds, scores, sg, xscale, x16, xs16, h16, hinv, hrow, lg, wn, y16, yinv,
      rowpos, rhi, rlo, total;
  int rows_cap, max_mt;
};

Layout make_layout(const rnb_moe_desc& d) {
  Layout L;
  const size_t T = d.T, K = d.k, E1 = d.E + 1;
  // sorted rows: every entry plus each non-empty expert's padding to 128
  // rows (at most T*(K+1) experts can be non-empty)
  const size_t nonempty = E1 < T * (K + 1) ? E1 : T * (K + 1);
  L.rows_cap = static_cast<int>(T * K + T + nonempty * (kTileM - 1) + kTileM);
  L.max_mt = L.rows_cap / kTileM + static_cast<int>(E1) + 1;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align256(o + bytes);
    return at;
  };
  L.status = take(4);
  take(ws_counter_bytes(d));  // the decode kernels' arrival counters: never touched here
  take(kXchgBytes);           // the persistent decode kernel's exchange words: never touched here
  L.counts = take(E1 * 4);
  L.fill = take(E1 * 4);
  L.base = take(E1 * 4);
  L.n_mt = take(4);
  L.tiles = take(static_cast<size_t>(L.max_mt) * 16);
  L.perm = take(static_cast<size_t>(L.rows_cap) * 4);
  L.inds = take(T * K * 4);
  L.scores = take(T * K * 4);
  L.sg = take(T * 4);
  L.xscale = take(T * 4);
  L.x16 = take(T * d.H * 2);
  L.xs16 = take(static_cast<size_t>(L.rows_cap) * d.H * 2);
  L.h16 = take(static_cast<size_t>(L.rows_cap) * d.I * 2);
  L.hinv = take(static_cast<size_t>(L.rows_cap) * (d.I / 64) * 4);
  L.hrow = take(static_cast<size_t>(L.rows_cap) * 4);
  L.lg = take(T * (d.E_total + 1) * 4);
  L.wn = take(static_cast<size_t>(d.E_total) * 2 * 4);
  L.y16 = take(static_cast<size_t>(L.rows_cap) * d.H * 2);
  L.yinv = take(static_cast<size_t>(L.rows_cap) * (d.H / 128) * 4);
  L.rowpos = take(T * (K + 1) * 4);
  const size_t rsplit = d.router_bits == 8 ? static_cast<size_t>(d.E_total + 1) * d.H * 2 : 0;
  L.rhi = take(rsplit);
  L.rlo = take(rsplit);
  L.total = o;
  return L;
}

}  // namespace pre

size_t prefill_workspace_bytes(const rnb_moe_desc& d) { return pre::make_layout(d).total; }

bool prefill_supported(const rnb_moe_desc& d) {
  return d.H % 128 == 0 && d.I % 128 == 0 && d.I <= 512 && d.E_total <= pre::kMaxE && d.E <= pre::kMaxE &&
         d.k <= pre::kMaxK && (d.bits == 4 || d.bits == 8) && d.group == 64;
}

namespace pre {

// The driver's tensor-map encoder, looked up through the runtime so the
// library does not link against the driver (it loads on hosts without one).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

}  // namespace pre

bool encode_tiled(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle sw) {
  const pre::EncodeTiledFn enc = pre::encode_fn();
  if (!enc || rank < 1 || rank > 5) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  return enc(m, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace pre {

// 2-D tensor map over a row-major [rows][inner] array (inner in elements).
bool encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
  const EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t es[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Descriptors of one GEMM: A (rows of xs16 or h16, 256-row boxes, 128-byte
// swizzle) and the codes / scales / biases of the routed and shared experts
// (boxes of one stage's 64 K for the n-tile's rows).
template <int BITS>
bool make_maps(const Params& p, int mode, int rows_cap, TmaMaps& tm) {
  using C = GemmCfg<BITS>;
  const int K = mode == 0 ? p.H : p.I;              // contraction length
  const uint64_t rows_e = mode == 0 ? 2ull * p.I : static_cast<uint64_t>(p.H);  // weight rows per expert
  const uint32_t box_rows = mode == 0 ? 64 : 128;   // gate/up: up and gate halves separately
  const uint64_t wbytes = static_cast<uint64_t>(K) * BITS / 8, groups = K / 64;
  bool ok = encode_2d(&tm.a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, mode == 0 ? static_cast<const void*>(p.ws.xs16) : p.ws.h16,
                      K, rows_cap, static_cast<uint64_t>(K) * 2, 64, kItemM, CU_TENSOR_MAP_SWIZZLE_128B);
  const void* w = mode == 0 ? static_cast<const void*>(p.gu_w) : p.dn_w;
  const void* sc = mode == 0 ? static_cast<const void*>(p.gu_s) : p.dn_s;
  const void* bi = mode == 0 ? static_cast<const void*>(p.gu_b) : p.dn_b;
  ok = ok && encode_2d(&tm.bw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, wbytes, rows_e * p.E, wbytes, C::kRawRow, box_rows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  ok = ok && encode_2d(&tm.bs, CU_TENSOR_MAP_DATA_TYPE_UINT16, sc, groups, rows_e * p.E, groups * 2, 8, box_rows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  ok = ok && encode_2d(&tm.bb, CU_TENSOR_MAP_DATA_TYPE_UINT16, bi, groups, rows_e * p.E, groups * 2, 8, box_rows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  // shared expert (the routed bank again when there is none: never read)
  const void* sw = p.has_shared ? (mode == 0 ? static_cast<const void*>(p.sgu_w) : p.sdn_w) : w;
  const void* ss = p.has_shared ? (mode == 0 ? static_cast<const void*>(p.sgu_s) : p.sdn_s) : sc;
  const void* sb = p.has_shared ? (mode == 0 ? static_cast<const void*>(p.sgu_b) : p.sdn_b) : bi;
  ok = ok && encode_2d(&tm.sbw, CU_TENSOR_MAP_DATA_TYPE_UINT8, sw, wbytes, rows_e, wbytes, C::kRawRow, box_rows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  ok = ok && encode_2d(&tm.sbs, CU_TENSOR_MAP_DATA_TYPE_UINT16, ss, groups, rows_e, groups * 2, 8, box_rows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  ok = ok && encode_2d(&tm.sbb, CU_TENSOR_MAP_DATA_TYPE_UINT16, sb, groups, rows_e, groups * 2, 8, box_rows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  return ok;
}

}  // namespace pre

namespace {
thread_local cudaEvent_t g_route_event = nullptr;
thread_local bool* g_route_fired = nullptr;
}  // namespace

void set_prefill_route_event(cudaEvent_t ev, bool* fired) {
  g_route_event = ev;
  g_route_fired = fired;
}

template <int BITS>
static int launch_prefill(pre::Params& p, const pre::Layout& L, cudaStream_t st) {
  using namespace pre;
  using C = GemmCfg<BITS>;
  cudaError_t e;
  TmaMaps tm0, tm1;
  if (!make_maps<BITS>(p, 0, L.rows_cap, tm0) || !make_maps<BITS>(p, 1, L.rows_cap, tm1))
    return fail(RNB_ERR_CUDA, "prefill: tensor map encoding failed");
  stage_begin(st);
  // zero the histogram and the fp32 accumulator; padding rows of perm = ~0
  e = cudaMemsetAsync(p.ws.counts, 0, (p.E + 1) * 4, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.ws.perm, 0xFF, static_cast<size_t>(L.rows_cap) * 4, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.ws.rowpos, 0xFF, static_cast<size_t>(p.T) * (p.k + 1) * 4, st);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("prefill memset: ") + cudaGetErrorString(e));
  static bool attr = false;
  if (!attr) {
    e = cudaFuncSetAttribute(k_route_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kRgSmem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_pre_gemm<BITS, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(C::kSmem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_pre_gemm<BITS, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(C::kSmem));
    if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("prefill smem attribute: ") + cudaGetErrorString(e));
    attr = true;
  }
  if (p.inds_in) {
    k_pre_given<<<(p.T + 15) / 16, 512, 0, st>>>(p);
  } else {
    RouteMaps rm;
    if (!encode_2d(&rm.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.x, p.H, static_cast<uint64_t>(p.T),
                   static_cast<uint64_t>(p.H) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&rm.w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.router_w, p.H, static_cast<uint64_t>(p.E_total),
                   static_cast<uint64_t>(p.H) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&rm.wl, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.router_q8 ? p.ws.rlo : p.router_w, p.H,
                   static_cast<uint64_t>(p.E_total), static_cast<uint64_t>(p.H) * 2, 64, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(RNB_ERR_CUDA, "prefill: router tensor map encoding failed");
    if (p.router_q8) k_router_split<<<(p.E_total + 1 + 15) / 16, 512, 0, st>>>(p);
    const dim3 rg((p.T + 127) / 128, (p.E_total + 127) / 128);
    k_route_gemm<<<rg, 256, kRgSmem, st>>>(p, rm);
    k_pre_select<<<(p.T + 15) / 16, 512, 0, st>>>(p);
  }
  stage_end(st, RNB_STAGE_ROUTE);
  if (g_route_event && cudaEventRecord(g_route_event, st) == cudaSuccess && g_route_fired) *g_route_fired = true;
  k_pre_sort<<<1, 512, 0, st>>>(p);
  stage_end(st, RNB_STAGE_SORT);
  const size_t n_scatter = static_cast<size_t>(p.T) * (p.k + 1);
  k_pre_scatter<<<static_cast<unsigned>((n_scatter + 255) / 256), 256, 0, st>>>(p);
  k_pre_gather<<<(L.rows_cap + 7) / 8, 256, 0, st>>>(p);
  stage_end(st, RNB_STAGE_SCATTER);
  const int nc = dev_info().sms;
  k_pre_gemm<BITS, 0><<<nc, kGemmThreads, C::kSmem, st>>>(p, tm0);
  stage_end(st, RNB_STAGE_GATEUP);
  k_pre_hrow<<<(L.rows_cap + 7) / 8, 256, 0, st>>>(p);
  k_pre_gemm<BITS, 1><<<nc, kGemmThreads, C::kSmem, st>>>(p, tm1);
  stage_end(st, RNB_STAGE_DOWN);
  const size_t n_final = static_cast<size_t>(p.T) * (p.H / 8);
  k_pre_final<<<static_cast<unsigned>((n_final + 255) / 256), 256, 0, st>>>(p);
  stage_end(st, RNB_STAGE_FINAL);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("prefill launch: ") + cudaGetErrorString(e));
  return RNB_OK;
}

int run_prefill(const rnb_moe_desc* d, const void* x, void* out, uint32_t* inds_out, float* scores_out, void* ws,
                size_t ws_bytes, cudaStream_t st, const uint32_t* inds_in, const float* scores_in) {
  using namespace pre;
  const Layout L = make_layout(*d);
  if (ws_bytes < L.total) return fail(RNB_ERR_WORKSPACE, "workspace too small for the prefill path");
  Params p;
  memset(&p, 0, sizeof(p));
  p.T = d->T;
  p.H = d->H;
  p.I = d->I;
  p.E = d->E;
  p.E_total = d->E_total;
  p.off = d->expert_offset;
  p.k = d->k;
  p.has_shared = (has_shared(d) && !inds_in) ? 1 : 0;
  p.inds_in = inds_in;
  p.scores_in = scores_in;
  p.rows_cap = L.rows_cap;
  p.max_mt = L.max_mt;
  p.x = static_cast<const uint16_t*>(x);
  p.router_w = d->router_w;
  p.sgate_w = d->shared_gate_w;
  if (d->router_bits == 8) {
    // the router GEMM, the norms and the shared gate read the split rows
    // (the workspace's rhi / rlo); the exact recompute reads the codes
    char* wsb = static_cast<char*>(ws);
    p.router_q8 = 1;
    p.router_q = reinterpret_cast<const uint32_t*>(d->router_w);
    p.sgate_q = reinterpret_cast<const uint32_t*>(d->shared_gate_w);
    p.router_s = d->router_s;
    p.router_b = d->router_b;
    p.sgate_s = d->sgate_s;
    p.sgate_b = d->sgate_b;
    p.router_w = reinterpret_cast<const uint16_t*>(wsb + L.rhi);
    p.sgate_w = p.router_w + static_cast<size_t>(d->E_total) * d->H;
  }
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
  p.out = out;
  p.y_f32 = (d->flags & RNB_FLAG_Y_F32) ? 1 : 0;
  p.inds_out = inds_out;
  p.scores_out = scores_out;
  char* b = static_cast<char*>(ws);
  p.ws.status = reinterpret_cast<uint32_t*>(b + L.status);
  p.ws.counts = reinterpret_cast<uint32_t*>(b + L.counts);
  p.ws.fill = reinterpret_cast<uint32_t*>(b + L.fill);
  p.ws.base = reinterpret_cast<uint32_t*>(b + L.base);
  p.ws.n_mt = reinterpret_cast<uint32_t*>(b + L.n_mt);
  p.ws.tiles = reinterpret_cast<uint4*>(b + L.tiles);
  p.ws.perm = reinterpret_cast<uint32_t*>(b + L.perm);
  p.ws.inds = reinterpret_cast<uint32_t*>(b + L.inds);
  p.ws.scores = reinterpret_cast<float*>(b + L.scores);
  p.ws.sg = reinterpret_cast<float*>(b + L.sg);
  p.ws.xscale = reinterpret_cast<float*>(b + L.xscale);
  p.ws.x16 = reinterpret_cast<__half*>(b + L.x16);
  p.ws.xs16 = reinterpret_cast<__half*>(b + L.xs16);
  p.ws.h16 = reinterpret_cast<__half*>(b + L.h16);
  p.ws.hinv = reinterpret_cast<float*>(b + L.hinv);
  p.ws.hrow = reinterpret_cast<float*>(b + L.hrow);
  p.ws.lg = reinterpret_cast<uint32_t*>(b + L.lg);
  p.ws.wn = reinterpret_cast<float*>(b + L.wn);
  p.ws.y16 = reinterpret_cast<__half*>(b + L.y16);
  p.ws.yinv = reinterpret_cast<float*>(b + L.yinv);
  p.ws.rowpos = reinterpret_cast<uint32_t*>(b + L.rowpos);
  p.ws.rhi = reinterpret_cast<uint16_t*>(b + L.rhi);
  p.ws.rlo = reinterpret_cast<uint16_t*>(b + L.rlo);
  return d->bits == 8 ? launch_prefill<8>(p, L, st) : launch_prefill<4>(p, L, st);
}

// ---------------------------------------------------------------- QMM probe

static rnb_moe_desc qmm_desc(int bits, int T, int N, int K) {
  rnb_moe_desc d;
  memset(&d, 0, sizeof(d));
  d.T = T;
  d.H = N;
  d.I = K;
  d.E = 1;
  d.E_total = 1;
  d.k = 1;
  d.bits = bits;
  d.group = 64;
  return d;
}

int qmm_workspace_bytes(int bits, int group, int T, int N, int K, size_t* bytes) {
  if (bits != 4 && bits != 8) return fail(RNB_ERR_INVALID, "bits must be 4 or 8");
  if (group != 64) return fail(RNB_ERR_INVALID, "group size must be 64");
  if (T < 0 || N <= 0 || N % 128 || K <= 0 || K % 512 || K > 16384)
    return fail(RNB_ERR_INVALID, "qmm: T >= 0, N a multiple of 128, K a multiple of 512 up to 16384");
  *bytes = pre::make_layout(qmm_desc(bits, T, N, K)).total;
  return RNB_OK;
}

template <int BITS>
static int launch_qmm(pre::Params& p, const pre::Layout& L, cudaStream_t st) {
  using namespace pre;
  using C = GemmCfg<BITS>;
  TmaMaps tm;
  if (!make_maps<BITS>(p, 1, L.rows_cap, tm)) return fail(RNB_ERR_CUDA, "qmm: tensor map encoding failed");
  cudaError_t e = cudaFuncSetAttribute(k_pre_gemm<BITS, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(C::kSmem));
  if (e == cudaSuccess) e = cudaMemsetAsync(p.ws.perm, 0xFF, static_cast<size_t>(L.rows_cap) * 4, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.ws.rowpos, 0xFF, static_cast<size_t>(p.T) * 2 * 4, st);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("qmm setup: ") + cudaGetErrorString(e));
  k_qmm_prep<<<(p.T + 15) / 16, 512, 0, st>>>(p);
  const int nc = dev_info().sms;
  k_pre_gemm<BITS, 1><<<nc, kGemmThreads, C::kSmem, st>>>(p, tm);
  const size_t n_final = static_cast<size_t>(p.T) * (p.H / 8);
  k_pre_final<<<static_cast<unsigned>((n_final + 255) / 256), 256, 0, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("qmm launch: ") + cudaGetErrorString(e));
  return RNB_OK;
}

int run_qmm(int bits, int T, int N, int K, const uint32_t* w, const uint16_t* s, const uint16_t* b, const void* x,
            void* y, bool y_f32, void* ws, size_t ws_bytes, cudaStream_t st) {
  using namespace pre;
  const rnb_moe_desc d = qmm_desc(bits, T, N, K);
  const Layout L = make_layout(d);
  if (ws_bytes < L.total) return fail(RNB_ERR_WORKSPACE, "workspace too small for qmm");
  Params p;
  memset(&p, 0, sizeof(p));
  p.T = T;
  p.H = N;
  p.I = K;
  p.E = 1;
  p.E_total = 1;
  p.k = 1;
  p.rows_cap = L.rows_cap;
  p.max_mt = L.max_mt;
  p.x = static_cast<const uint16_t*>(x);
  p.dn_w = w;
  p.dn_s = s;
  p.dn_b = b;
  p.out = y;
  p.y_f32 = y_f32 ? 1 : 0;
  char* base = static_cast<char*>(ws);
  p.ws.status = reinterpret_cast<uint32_t*>(base + L.status);
  p.ws.counts = reinterpret_cast<uint32_t*>(base + L.counts);
  p.ws.fill = reinterpret_cast<uint32_t*>(base + L.fill);
  p.ws.base = reinterpret_cast<uint32_t*>(base + L.base);
  p.ws.n_mt = reinterpret_cast<uint32_t*>(base + L.n_mt);
  p.ws.tiles = reinterpret_cast<uint4*>(base + L.tiles);
  p.ws.perm = reinterpret_cast<uint32_t*>(base + L.perm);
  p.ws.inds = reinterpret_cast<uint32_t*>(base + L.inds);
  p.ws.scores = reinterpret_cast<float*>(base + L.scores);
  p.ws.sg = reinterpret_cast<float*>(base + L.sg);
  p.ws.xscale = reinterpret_cast<float*>(base + L.xscale);
  p.ws.x16 = reinterpret_cast<__half*>(base + L.x16);
  p.ws.xs16 = reinterpret_cast<__half*>(base + L.xs16);
  p.ws.h16 = reinterpret_cast<__half*>(base + L.h16);
  p.ws.hinv = reinterpret_cast<float*>(base + L.hinv);
  p.ws.hrow = reinterpret_cast<float*>(base + L.hrow);
  p.ws.lg = reinterpret_cast<uint32_t*>(base + L.lg);
  p.ws.wn = reinterpret_cast<float*>(base + L.wn);
  p.ws.y16 = reinterpret_cast<__half*>(base + L.y16);
  p.ws.yinv = reinterpret_cast<float*>(base + L.yinv);
  p.ws.rowpos = reinterpret_cast<uint32_t*>(base + L.rowpos);
  return bits == 8 ? launch_qmm<8>(p, L, st) : launch_qmm<4>(p, L, st);
}

}  // namespace rnb
