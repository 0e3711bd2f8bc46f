/*
 * rnb_oracle.h -- the block descriptor shared by the CPU oracle
 * (rnb_oracle.c, exact order) and the vectorised CPU baseline
 * (rnb_cpu_fast.c).  TEST AND BENCHMARK INFRASTRUCTURE ONLY: the product
 * path (runnel_b200) never includes, links or calls either.
 */
#ifndef RNB_ORACLE_H
#define RNB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define RNBO_OK 0
#define RNBO_EINVAL -1

typedef struct rnbo_block {
  int T, H, I, E, k, bits, group;
  const uint16_t* x;             /* [T,H] bf16 */
  const uint16_t* router_w;      /* [E,H] bf16 */
  const uint16_t* shared_gate_w; /* [H] bf16, NULL = no shared expert */
  const uint32_t* gu_w;          /* [E,2I,H*bits/32] packed up||gate */
  const uint16_t* gu_s;          /* [E,2I,H/group] */
  const uint16_t* gu_b;
  const uint32_t* dn_w; /* [E,H,I*bits/32] */
  const uint16_t* dn_s; /* [E,H,I/group] */
  const uint16_t* dn_b;
  const uint32_t* sgu_w; /* [2I,H*bits/32] shared up||gate */
  const uint16_t* sgu_s;
  const uint16_t* sgu_b;
  const uint32_t* sdn_w; /* [H,I*bits/32] */
  const uint16_t* sdn_s;
  const uint16_t* sdn_b;
  /* 8-bit affine router and shared gate (router_bits == 8; real Ornith
   * checkpoints store mlp.gate and mlp.shared_expert_gate so): codes
   * [E,H/4] / [H/4] in router_q / sgate_q, bf16 scales and biases per 64
   * inputs.  router_bits 0 or 16: the bf16 router_w / shared_gate_w above. */
  int router_bits;
  const uint32_t* router_q;
  const uint16_t* router_s; /* [E,H/64] */
  const uint16_t* router_b;
  const uint32_t* sgate_q; /* [H/4] */
  const uint16_t* sgate_s; /* [H/64] */
  const uint16_t* sgate_b;
} rnbo_block;

float rnbo_bf16_to_f32(uint16_t value);
float rnbo_f64_to_bf16_f32(double v);
int rnbo_router(const rnbo_block* d, float* logits, int32_t* inds, float* scores, float* shared_gate,
                int nthreads);

/* Vectorised CPU baseline (rnb_cpu_fast.c): the same block and the same
 * routing as rnbo_moe_block, computed with wide fp32 arithmetic in another
 * order.  simd: 1 when the AVX2/FMA kernels run on this host, else 0. */
int rnbc_moe_block(const rnbo_block* d, float* out, int32_t* inds, float* scores, int nthreads);
int rnbc_simd(void);

#endif
