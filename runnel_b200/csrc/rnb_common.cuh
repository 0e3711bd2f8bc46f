// rnb_common.cuh -- device helpers shared by the MoE kernels (sm_100a).
//
// Quantized rows are contracted on the tensor cores with mma.sync m16n8k16
// (fp16 x fp16 -> fp32).  MLX affine codes (4 or 8 bit) enter the MMAs as
// exact fp16 subnormals q * 2^-24 (the code in the low mantissa bits of a
// zero-exponent fp16: one mask or byte permute per two codes), so every
// product q * x is exact and the per-group affine
//     sum_k (s q_k + b) x_k = s * sum_k q_k x_k + b * sum_k x_k
// is applied in fp32 once per 64-group (the scale carrying the 2^24 back),
// with sum_k x_k precomputed.  The prefill converters, which write real fp16
// weights s * q + b, use the magic-number form (0x6400 | q == 1024 + q, then
// subtract 1024).
//
// Lane layout of one 64-wide group for one weight row (lane = 4*g + c):
// lane c owns 16 of the 64 positions and hands them to the MMA as 8 fp16
// pairs; MMA m (0..3) of the group takes pairs 2m (logical k 2c,2c+1) and
// 2m+1 (logical k 2c+8,2c+9).  The activation operand is stored in exactly the
// same pair order (see pair_pos), so logical k matches physical k on both sides.
//   8-bit: lane c holds bytes [16c, 16c+16) of the group's 64 bytes;
//          pair 2j+h = positions (16c+4j+2h, 16c+4j+2h+1).
//   4-bit: a 16-byte load covers two groups; after one shuffle exchange lane
//          c holds bytes [8q, 8q+8) of each group with q = {0,2,1,3}[c];
//          pair 4j+i = positions (16q+8j+i, 16q+8j+i+4).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rnb {

constexpr int kGroup = 64;

// ------------------------------------------------------------------ PTX

// (not volatile: a pure function of its operands, so the compiler may
// interleave independent MMAs)
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t a0, const uint32_t a1,
                                        const uint32_t a2, const uint32_t a3, const uint32_t b0,
                                        const uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t a0, const uint32_t a1,
                                         const uint32_t a2, const uint32_t a3, const uint32_t b0,
                                         const uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 16-byte load of weights that are read once: skip L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 16-byte load of data another kernel of this call wrote (L2-coherent).
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  // bytes must be a multiple of 16 and p 16-byte aligned
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// 16-byte asynchronous global -> shared copy through L2 (no registers held).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}

// Programmatic dependent launch (sm_90+).
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
  return d;
}

// ------------------------------------------------- code -> fp16 pairs

__device__ __forceinline__ uint32_t hsub_1024(uint32_t v) {
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&v), __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400)));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// 8-bit word (codes b0..b3) -> pairs (b0,b1), (b2,b3) as exact fp16.
__device__ __forceinline__ void q8_word_to_pairs(uint32_t w, uint32_t& p0, uint32_t& p1) {
  p0 = hsub_1024(__byte_perm(w, 0x64646464u, 0x4140));
  p1 = hsub_1024(__byte_perm(w, 0x64646464u, 0x4342));
}

// 4-bit word (codes n0..n7) -> pairs (n0,n4), (n1,n5), (n2,n6), (n3,n7).
__device__ __forceinline__ void q4_word_to_pairs(uint32_t w, uint32_t& p0, uint32_t& p1,
                                                 uint32_t& p2, uint32_t& p3) {
  p0 = hsub_1024(lop3_and_or(w, 0x000F000Fu, 0x64006400u));
  p1 = hsub_1024(lop3_and_or(w >> 4, 0x000F000Fu, 0x64006400u));
  p2 = hsub_1024(lop3_and_or(w >> 8, 0x000F000Fu, 0x64006400u));
  p3 = hsub_1024(lop3_and_or(w >> 12, 0x000F000Fu, 0x64006400u));
}

// Subnormal form (no magic-number subtraction): a code placed in the low
// mantissa bits of an fp16 with a zero exponent IS the fp16 subnormal
// q * 2^-24, exactly, so one mask (4-bit) or one byte permute (8-bit) makes
// two operands.  The tensor cores take fp16 subnormals at full precision, so
// products with x stay exact in fp32 and a contraction's result is
// 2^-24 * sum q x.  4-bit: pairs 1 and 3 of a word keep their nibbles at bits
// 4-7 (value 16 q 2^-24); their activations are staged times 2^-4 instead.
__device__ __forceinline__ void q8_word_to_pairs_sub(uint32_t w, uint32_t& p0, uint32_t& p1) {
  p0 = __byte_perm(w, 0u, 0x4140);
  p1 = __byte_perm(w, 0u, 0x4342);
}

__device__ __forceinline__ void q4_word_to_pairs_sub(uint32_t w, uint32_t& p0, uint32_t& p1, uint32_t& p2,
                                                     uint32_t& p3) {
  const uint32_t h = w >> 8;
  p0 = w & 0x000F000Fu;
  p1 = w & 0x00F000F0u;  // 16 x
  p2 = h & 0x000F000Fu;
  p3 = h & 0x00F000F0u;  // 16 x
}

// Position (within a 64-group) of the two halves of pair i held by lane c.
template <int BITS>
__host__ __device__ __forceinline__ int pair_pos(int c, int i, int half) {
  if (BITS == 8) {
    return 16 * c + 4 * (i >> 1) + 2 * (i & 1) + half;
  } else {
    const int q = (c == 1) ? 2 : (c == 2) ? 1 : c;
    return 16 * q + 8 * (i >> 2) + (i & 3) + 4 * half;
  }
}

// The same positions relative to the lane's first position (16c for 8-bit,
// 16q for 4-bit); independent of the lane, so usable as a register index.
template <int BITS>
__host__ __device__ __forceinline__ constexpr int pair_rel(int i, int half) {
  return BITS == 8 ? 4 * (i >> 1) + 2 * (i & 1) + half : 8 * (i >> 2) + (i & 3) + 4 * half;
}

// 4-bit exchange: a lane's 16-byte load (v.x,v.y | v.z,v.w) covers bytes
// [16c,16c+16) of a 64-byte two-group chunk; afterwards ev = its 8 bytes of
// the even group, od = its 8 bytes of the odd group.
__device__ __forceinline__ void q4_exchange(const uint4 v, int c, uint2& ev, uint2& od) {
  const bool lo = c < 2;
  const uint32_t s0 = lo ? v.z : v.x, s1 = lo ? v.w : v.y;
  const uint32_t r0 = __shfl_xor_sync(0xffffffffu, s0, 2);
  const uint32_t r1 = __shfl_xor_sync(0xffffffffu, s1, 2);
  if (lo) {
    ev = make_uint2(v.x, v.y);
    od = make_uint2(r0, r1);
  } else {
    ev = make_uint2(r0, r1);
    od = make_uint2(v.z, v.w);
  }
}

// Eight fp16 pairs of one row for one group, in MMA pair order.
struct RowPairs {
  uint32_t p[8];
};

__device__ __forceinline__ RowPairs q8_group_pairs_sub(const uint4 v) {
  RowPairs r;
  q8_word_to_pairs_sub(v.x, r.p[0], r.p[1]);
  q8_word_to_pairs_sub(v.y, r.p[2], r.p[3]);
  q8_word_to_pairs_sub(v.z, r.p[4], r.p[5]);
  q8_word_to_pairs_sub(v.w, r.p[6], r.p[7]);
  return r;
}

// Pairs i with i & 1 set come out times 16 (see q4_word_to_pairs_sub).
__device__ __forceinline__ RowPairs q4_group_pairs_sub(const uint2 v) {
  RowPairs r;
  q4_word_to_pairs_sub(v.x, r.p[0], r.p[1], r.p[2], r.p[3]);
  q4_word_to_pairs_sub(v.y, r.p[4], r.p[5], r.p[6], r.p[7]);
  return r;
}

// ------------------------------------------------------------ scalar

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t v) {
  return __uint_as_float(static_cast<uint32_t>(v) << 16);
}

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// Power-of-two scale 2^e that maps max|v| into [2^14, 2^15) (fp16
// headroom), e clamped to [-100, 100], and its inverse; both exact.  With
// maxabs = m 2^p, m in [0.5, 1), e = 15 - p; for a normal maxabs with biased
// exponent field E, p = E - 126, so e = 141 - E (a subnormal maxabs, E = 0,
// clamps to 100 as its true p would).  Built from exponent bits: no branches
// beyond the zero / non-finite case.
__device__ __forceinline__ void fp16_range_scale(float maxabs, float& scale, float& inv) {
  const int E = static_cast<int>((__float_as_uint(maxabs) >> 23) & 0xFFu);
  int e = 141 - E;
  e = e > 100 ? 100 : (e < -100 ? -100 : e);
  const bool ok = maxabs > 0.0f && E != 255;
  scale = ok ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23) : 1.0f;
  inv = ok ? __uint_as_float(static_cast<uint32_t>(127 - e) << 23) : 1.0f;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace rnb
