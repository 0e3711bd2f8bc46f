// rnb_probe.cu -- standalone quantized matvec (QMV) and matmul (QMM).
//
// B200 counterparts of the reference's probe CLIs runnel-metal-qmv and
// runnel-metal-qmm (native/bench/quantized_qmv.cpp, quantized_qmm.cpp; their
// Metal kernels and CPU checks in native/src/quantized_qmv_probe.mm and
// quantized_qmm_probe.mm).  Both contract MLX affine rows (uint32 words,
// LSB-first 4/8-bit codes, bf16 scale and bias per 64-group) with bf16
// activations and return fp32:
//
//   rnb_qmv  y[r] = W[row(r)] . x, a dense weight matrix or, in expert mode,
//            the rows of the selected experts of a bank (the gather QMV of
//            quantized_qmv_probe.mm).  One streaming kernel, k_qmv: each warp
//            owns 16 output rows, loads their codes with 16-byte streaming
//            loads straight into registers (no shared-memory staging, nothing
//            re-read), turns them into exact fp16 integers and contracts them
//            with the activations on the tensor cores (mma.sync m16n8k16,
//            fp32 accumulation); the per-group affine terms are applied in
//            fp32 with the group sums of x (see rnb_common.cuh).  The codes
//            enter the MMA as fp16 subnormals q * 2^-24 (one mask or byte
//            permute per two codes); the group sums carry the same 2^-24 and
//            the result is rescaled once.  HBM-bound: its roofline is the
//            weight bytes over the copy bandwidth.
//   rnb_qmm  y[t][n] = W[n] . x[t] through the prefill path's tcgen05 grouped
//            GEMM (rnb_prefill.cu, run_qmm): one expert, every token one row.
#include <stdio.h>
#include <string.h>

#include <string>

#include "rnb_common.cuh"
#include "rnb_internal.h"
#include "rnb_moe.h"

namespace rnb {
namespace probe {

constexpr int kQmvThreads = 256;
constexpr int kQmvWarps = kQmvThreads / 32;
constexpr int kQmvMaxK = 16384;

struct QmvParams {
  int K, G;             // reduction length and its 64-groups
  long long blocks;     // 16-row output blocks
  long long rpe;        // rows per expert (expert mode)
  int nsel;             // selected experts (0: dense)
  uint32_t sel[RNB_QMV_MAX_EXPERTS];
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  const uint16_t* x;
  float* y;
};

// One 64-group of 16 rows (g and g+8 of this lane) against the activations:
// four MMAs over the group's 64 positions, then the affine terms in fp32.
__device__ __forceinline__ void qmv_group(const RowPairs& pa, const RowPairs& pb, const uint32_t* sX,
                                          const float* sXs, int grp, int c, float sa, float ba, float sb,
                                          float bb, float& acc0, float& acc1) {
  const uint4* xq = reinterpret_cast<const uint4*>(sX + grp * 32 + c * 8);
  const uint4 x0 = xq[0], x1 = xq[1];
  const uint32_t xh[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int m = 0; m < 4; ++m)
    mma_f16(d, pa.p[2 * m], pb.p[2 * m], pa.p[2 * m + 1], pb.p[2 * m + 1], xh[2 * m], xh[2 * m + 1]);
  const float xs = sXs[grp];
  acc0 = fmaf(sa, d[0], fmaf(ba, xs, acc0));
  acc1 = fmaf(sb, d[2], fmaf(bb, xs, acc1));
}

// bf16 j (0..7) of a 16-byte vector as fp32
__device__ __forceinline__ float bf16_at(const uint4& v, int j) {
  const uint32_t w = (j >> 1) == 0 ? v.x : (j >> 1) == 1 ? v.y : (j >> 1) == 2 ? v.z : v.w;
  return __uint_as_float((j & 1) ? (w & 0xFFFF0000u) : (w << 16));
}

// K slices per 16-row block: 4, 2 or 1, keeping a slice a multiple of 8
// groups (whole 16-byte scale loads, aligned L2 prefetches).
// 4-bit rows stay whole per warp (measured faster than sliced: the 4-bit
// chunk holds only 4 KB per warp in flight, and whole rows keep four of them
// back to back).
__host__ __device__ __forceinline__ int qmv_slices(int bits, int G) {
  return bits == 8 ? (G % 32 == 0 ? 4 : (G % 16 == 0 ? 2 : 1)) : 1;
}

// One chunk of 2*NJ 4-bit groups [g0, g0 + 2 NJ) of rows g, g + 8: all loads first.
// (NJ = 4: 8 groups, 4 KB of a warp's codes in flight.)
template <int NJ>
__device__ __forceinline__ void qmv_q4_chunk(const uint32_t* wa, const uint32_t* wb, const uint16_t* spa,
                                             const uint16_t* bpa, size_t srow, int g0, const uint32_t* sX,
                                             const float* sXs, int c, float& acc0, float& acc1) {
  constexpr int NS = NJ / 4;  // 16-byte scale vectors (8 groups each) per row
  uint4 s8a[NS], s8b[NS], b8a[NS], b8b[NS], va[NJ], vb[NJ];
#pragma unroll
  for (int k = 0; k < NS; ++k) {
    s8a[k] = ld_stream_v4(spa + g0 + 8 * k);
    s8b[k] = ld_stream_v4(spa + 8 * srow + g0 + 8 * k);
    b8a[k] = ld_stream_v4(bpa + g0 + 8 * k);
    b8b[k] = ld_stream_v4(bpa + 8 * srow + g0 + 8 * k);
  }
  // a 64-byte chunk holds two groups; lane c loads bytes [16c, 16c + 16)
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    va[j] = ld_stream_v4(wa + (g0 / 2 + j) * 16 + c * 4);
    vb[j] = ld_stream_v4(wb + (g0 / 2 + j) * 16 + c * 4);
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    uint2 ea, oa, eb, ob;
    q4_exchange(va[j], c, ea, oa);
    q4_exchange(vb[j], c, eb, ob);
    const int e = 2 * (j & 3), k = j >> 2;
    qmv_group(q4_group_pairs_sub(ea), q4_group_pairs_sub(eb), sX, sXs, g0 + 2 * j, c, bf16_at(s8a[k], e),
              bf16_at(b8a[k], e), bf16_at(s8b[k], e), bf16_at(b8b[k], e), acc0, acc1);
    qmv_group(q4_group_pairs_sub(oa), q4_group_pairs_sub(ob), sX, sXs, g0 + 2 * j + 1, c, bf16_at(s8a[k], e + 1),
              bf16_at(b8a[k], e + 1), bf16_at(s8b[k], e + 1), bf16_at(b8b[k], e + 1), acc0, acc1);
  }
}

// Work split: a round of a CTA covers 8/S 16-row blocks, each split over S
// warps by K (S slices of K/S, see qmv_slices); the slices' partial sums meet
// in shared memory and are added in slice order, so results do not depend on
// the schedule.  Small units keep the last round short.
template <int BITS>
__global__ void __launch_bounds__(kQmvThreads, 2) k_qmv(const __grid_constant__ QmvParams p) {
  extern __shared__ __align__(16) uint32_t qsm[];
  __shared__ float red[kQmvWarps];
  __shared__ float part[2][kQmvWarps][16];
  uint32_t* sX = qsm;                                      // [G][32] fp16 pairs in MMA order
  float* sXs = reinterpret_cast<float*>(qsm + p.G * 32);   // [G] group sums
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, c = lane & 3;
  const int S = qmv_slices(BITS, p.G);                     // K slices per block
  const int bpr = kQmvWarps / S;                           // blocks per round
  const int mb = warp / S, ms = warp % S;
  const int Gs = p.G / S, gb = ms * Gs;                    // this warp's groups [gb, gb + Gs)
  const size_t wrow = static_cast<size_t>(p.K) * BITS / 32, srow = static_cast<size_t>(p.G);
  auto block_row = [&](long long blk) -> long long {
    const long long r0 = blk * 16;
    return p.nsel ? static_cast<long long>(p.sel[r0 / p.rpe]) * p.rpe + r0 % p.rpe : r0;
  };
  const long long first = static_cast<long long>(blockIdx.x) * bpr;

  // ---- warm L2 with this warp's first slice while the activations are staged
  if (first + mb < p.blocks && lane < 16) {
    const long long row = block_row(first + mb) + lane;
    prefetch_l2_bulk(p.w + static_cast<size_t>(row) * wrow + static_cast<size_t>(gb) * 2 * BITS,
                     static_cast<uint32_t>(Gs) * 8 * BITS);
    prefetch_l2_bulk(p.s + static_cast<size_t>(row) * srow + gb, static_cast<uint32_t>(Gs) * 2);
    prefetch_l2_bulk(p.b + static_cast<size_t>(row) * srow + gb, static_cast<uint32_t>(Gs) * 2);
  }

  // ---- activations: one power-of-two scale into fp16 range, then the pairs
  float m = 0.f;
  for (int k = tid; k < p.K; k += kQmvThreads) m = fmaxf(m, fabsf(bf16_bits_to_f32(p.x[k])));
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int q = 1; q < kQmvWarps; ++q) m = fmaxf(m, red[q]);
  float sc, inv;
  fp16_range_scale(m, sc, inv);
  // entry q = (group, lane c, pair i); a warp covers exactly one group
  for (int q = tid; q < p.G * 32; q += kQmvThreads) {
    const int grp = q >> 5, cc = (q >> 3) & 3, i = q & 7;
    const uint16_t* xg = p.x + grp * kGroup;
    const float a = bf16_bits_to_f32(xg[pair_pos<BITS>(cc, i, 0)]) * sc;
    const float b = bf16_bits_to_f32(xg[pair_pos<BITS>(cc, i, 1)]) * sc;
    const __half2 h = __floats2half2_rn(a, b);
    // 4-bit pairs 1 and 3 of a word meet codes times 16: their x times 2^-4
    const float f16 = (BITS == 4 && (i & 1)) ? 0.0625f : 1.0f;
    const __half2 hs = __floats2half2_rn(__low2float(h) * f16, __high2float(h) * f16);
    sX[q] = *reinterpret_cast<const uint32_t*>(&hs);
    const float2 f = __half22float2(h);
    float sum = f.x + f.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) sXs[grp] = sum * 0x1p-24f;  // the MMA results carry 2^-24
  }
  __syncthreads();

  int buf = 0;
  for (long long base = first; base < p.blocks; base += static_cast<long long>(gridDim.x) * bpr, buf ^= 1) {
    const long long blk = base + mb;
    if (blk < p.blocks) {
      const long long row0 = block_row(blk);
      const uint32_t* wa = p.w + static_cast<size_t>(row0 + g) * wrow;
      const uint32_t* wb = wa + 8 * wrow;
      const uint16_t* spa = p.s + static_cast<size_t>(row0 + g) * srow;
      const uint16_t* bpa = p.b + static_cast<size_t>(row0 + g) * srow;
      float acc0 = 0.f, acc1 = 0.f;
      if (BITS == 8) {
        for (int g0 = gb; g0 < gb + Gs; g0 += 8) {
          // 8 groups: scales and biases of rows g and g + 8
          const uint4 s8a = ld_stream_v4(spa + g0), s8b = ld_stream_v4(spa + 8 * srow + g0);
          const uint4 b8a = ld_stream_v4(bpa + g0), b8b = ld_stream_v4(bpa + 8 * srow + g0);
          // a group is 64 bytes; lane c holds bytes [16c, 16c + 16)
          uint4 va[8], vb[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            va[j] = ld_stream_v4(wa + (g0 + j) * 16 + c * 4);
            vb[j] = ld_stream_v4(wb + (g0 + j) * 16 + c * 4);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            qmv_group(q8_group_pairs_sub(va[j]), q8_group_pairs_sub(vb[j]), sX, sXs, g0 + j, c, bf16_at(s8a, j),
                      bf16_at(b8a, j), bf16_at(s8b, j), bf16_at(b8b, j), acc0, acc1);
        }
      } else {
        for (int g0 = gb; g0 < gb + Gs; g0 += 8) qmv_q4_chunk<4>(wa, wb, spa, bpa, srow, g0, sX, sXs, c, acc0, acc1);
      }
      if (c == 0) {
        part[buf][warp][g] = acc0;
        part[buf][warp][g + 8] = acc1;
      }
    }
    __syncthreads();
    // slice sums in slice order; part[buf] is rewritten two rounds later,
    // after the next round's barrier
    if (tid < bpr * 16) {
      const int b = tid >> 4, r = tid & 15;
      if (base + b < p.blocks) {
        float v = part[buf][b * S][r];
        for (int q = 1; q < S; ++q) v += part[buf][b * S + q][r];
        p.y[(base + b) * 16 + r] = v * inv * 0x1p24f;
      }
    }
  }
}

}  // namespace probe
}  // namespace rnb

using namespace rnb;

int rnb_qmv(int bits, int group, int64_t rows, int64_t K, const uint32_t* w, const uint16_t* scales,
            const uint16_t* biases, const void* x, const uint32_t* selected, int n_selected,
            int64_t rows_per_expert, int64_t bank_rows, float* y, void* stream) {
  using namespace probe;
  if (bits != 4 && bits != 8) return fail(RNB_ERR_INVALID, "bits must be 4 or 8");
  if (group != kGroup) return fail(RNB_ERR_INVALID, "group size must be 64");
  if (K <= 0 || K % 512 || K > kQmvMaxK) return fail(RNB_ERR_INVALID, "K must be a multiple of 512 in [512, 16384]");
  if (rows < 0 || rows % 16) return fail(RNB_ERR_INVALID, "rows must be a non-negative multiple of 16");
  if (!w || !scales || !biases || !x || !y) return fail(RNB_ERR_INVALID, "w, scales, biases, x and y must be non-NULL");
  if (!aligned16(w) || !aligned16(scales) || !aligned16(biases) || !aligned16(x))
    return fail(RNB_ERR_ALIGN, "w, scales, biases and x must be 16-byte aligned");
  QmvParams p;
  memset(&p, 0, sizeof(p));
  if (n_selected > 0 || selected) {
    if (!selected || n_selected <= 0 || n_selected > RNB_QMV_MAX_EXPERTS)
      return fail(RNB_ERR_INVALID, "expert mode needs 1..64 selected experts");
    if (rows_per_expert <= 0 || rows_per_expert % 16 || rows != n_selected * rows_per_expert)
      return fail(RNB_ERR_INVALID, "expert mode: rows must be n_selected * rows_per_expert, a multiple of 16");
    if (bank_rows < rows_per_expert || bank_rows % rows_per_expert)
      return fail(RNB_ERR_INVALID, "expert mode: bank_rows must be a multiple of rows_per_expert");
    for (int i = 0; i < n_selected; ++i) {
      if (static_cast<int64_t>(selected[i]) >= bank_rows / rows_per_expert)
        return fail(RNB_ERR_INVALID, "selected expert outside the bank");
      p.sel[i] = selected[i];
    }
    p.nsel = n_selected;
    p.rpe = rows_per_expert;
  } else if (bank_rows != 0 && bank_rows < rows) {
    return fail(RNB_ERR_INVALID, "bank_rows is smaller than rows");
  }
  if (check_device()) return RNB_ERR_DEVICE;
  if (rows == 0) return RNB_OK;
  p.K = static_cast<int>(K);
  p.G = static_cast<int>(K / kGroup);
  p.blocks = rows / 16;
  p.w = w;
  p.s = scales;
  p.b = biases;
  p.x = static_cast<const uint16_t*>(x);
  p.y = y;
  const size_t smem = static_cast<size_t>(p.G) * 32 * 4 + static_cast<size_t>(p.G) * 4;
  const int S = qmv_slices(bits, p.G);
  const long long want = (p.blocks + kQmvWarps / S - 1) / (kQmvWarps / S);
  const long long cap = 2ll * dev_info().sms;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bits == 8)
    k_qmv<8><<<grid, kQmvThreads, smem, st>>>(p);
  else
    k_qmv<4><<<grid, kQmvThreads, smem, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("rnb_qmv launch: ") + cudaGetErrorString(e));
  return RNB_OK;
}

int rnb_qmm_workspace_size(int bits, int group, int T, int N, int K, size_t* bytes) {
  if (!bytes) return fail(RNB_ERR_INVALID, "bytes must be non-NULL");
  return qmm_workspace_bytes(bits, group, T, N, K, bytes);
}

int rnb_qmm(int bits, int group, int T, int N, int K, const uint32_t* w, const uint16_t* scales,
            const uint16_t* biases, const void* x, void* y, int y_f32, void* ws, size_t ws_bytes, void* stream) {
  if (!w || !scales || !biases || !x || !y || !ws)
    return fail(RNB_ERR_INVALID, "w, scales, biases, x, y and ws must be non-NULL");
  if (!aligned16(w) || !aligned16(scales) || !aligned16(biases) || !aligned16(x) || !aligned16(y) || !aligned16(ws))
    return fail(RNB_ERR_ALIGN, "w, scales, biases, x, y and ws must be 16-byte aligned");
  size_t need = 0;
  const int rc = qmm_workspace_bytes(bits, group, T, N, K, &need);
  if (rc) return rc;
  if (ws_bytes < need) return fail(RNB_ERR_WORKSPACE, "workspace too small (rnb_qmm_workspace_size)");
  if (check_device()) return RNB_ERR_DEVICE;
  if (T == 0) return RNB_OK;
  return run_qmm(bits, T, N, K, w, scales, biases, x, y, y_f32 != 0, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}
