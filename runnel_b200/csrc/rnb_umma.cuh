// rnb_umma.cuh -- 5th-generation tensor core (tcgen05) primitives for sm_100a.
//
// Operands live in shared memory in the canonical K-major SWIZZLE_128B layout:
// a tile of R rows x 64 16-bit elements (128 bytes per row) is stored as 8-row
// atoms of 1024 bytes; element (r, k) sits at byte
//     (r / 8) * 1024 + (r % 8) * 128 + (((k / 8) ^ (r % 8)) * 16) + (k % 8) * 2
// from a 1024-byte-aligned tile base.  A shared-memory matrix descriptor for
// such a tile has start address = base >> 4, leading byte offset field 1,
// stride byte offset = 1024 >> 4 (distance between 8-row atoms), descriptor
// version 1 and layout type 2 (128-byte swizzle); stepping K by 16 elements
// advances the start address by 32 bytes.  Accumulators are fp32 in tensor
// memory: row i of an M=128 tile is TMEM lane i, column j is TMEM column j.
#pragma once

#include <stdint.h>

namespace rnb {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of element (r, k) of a K-major SWIZZLE_128B tile (16-bit elements).
__host__ __device__ __forceinline__ uint32_t sw128_offset(int r, int k) {
  return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 3) ^ (r & 7))) << 4) + (k & 7) * 2);
}

// Shared-memory matrix descriptor of a K-major SWIZZLE_128B tile at byte
// address `saddr` (shared window, 1024-byte aligned tile base; K-steps add 32).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address [0,14)
  d |= static_cast<uint64_t>(1u) << 16;                 // leading byte offset [16,30)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;         // stride byte offset [32,46)
  d |= static_cast<uint64_t>(1u) << 46;                 // version [46,48)
  d |= static_cast<uint64_t>(2u) << 61;                 // layout: 128-byte swizzle [61,64)
  return d;
}

// Instruction descriptor, kind::f16: A, B fp16 (or bf16), D fp32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N, bool bf16 = false) {
  return (1u << 4)                                             // D format: F32 [4,6)
         | (static_cast<uint32_t>(bf16 ? 1 : 0) << 7)          // A format [7,10)
         | (static_cast<uint32_t>(bf16 ? 1 : 0) << 10)         // B format [10,13)
         | (static_cast<uint32_t>(N >> 3) << 17)               // N >> 3 [17,23)
         | (static_cast<uint32_t>(M >> 4) << 24);              // M >> 4 [24,29)
}

// D[tmem] (+)= A[smem] * B[smem]^T; issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// Arrive on an mbarrier once all previously issued MMAs of this thread complete.
__device__ __forceinline__ void umma_commit(uint32_t mbar_saddr) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar_saddr)
               : "memory");
}

// Tensor-memory allocation (one warp, all lanes).  The address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// Writes by this thread to shared memory become visible to the tensor core.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive once and raise the barrier's expected transaction count by `bytes`
// (the TMA loads of the phase complete them).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 2-D tiled TMA load (no multicast): box at element coordinates (x, y) of
// the tensor map into shared memory at dst; completes `box bytes` on mbar.
// x times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}

// 3-D and 4-D tiled TMA loads (no multicast), as tma_load_2d.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int x, int y, int z, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(mbar)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, int x, int y, int z, int w,
                                            uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(mbar)
      : "memory");
}

// Bounded wait for phase `parity` of an mbarrier: true on completion, false
// after `limit_ns` of waiting.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  uint64_t t0, now;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (now - t0 > limit_ns) return false;
  }
}

}  // namespace rnb
