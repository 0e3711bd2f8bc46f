/*
 * rnb_moe.h -- C ABI of runnel-b200's sparse-MoE block for NVIDIA B200 (sm_100a).
 *
 * Plain C: device pointers, sizes and a CUDA stream passed as void*.  No
 * allocation happens inside any entry point: the caller owns the weights,
 * the activations, the outputs and one workspace sized by
 * rnb_moe_workspace_size().  Every call is stream-ordered and asynchronous;
 * it returns RNB_OK or a negative error code, and rnb_last_error() gives a
 * thread-local message for the last failure on the calling thread.
 *
 * Weight layout is MLX affine quantization, exactly as Runnel stores it:
 *   codes  uint32 words, 32/bits codes per word, code j of a word in bits
 *          [bits*j, bits*(j+1)) (LSB first); bits = 4 or 8
 *   scales, biases  bf16, one per 64 consecutive inputs of a row (group 64)
 *   w = scale * code + bias
 * Routed gate/up is Runnel's packed tensor: per expert 2*I rows, rows
 * [0, I) = up_proj, rows [I, 2I) = gate_proj (src/runnel/mlx.py:38-48).
 *
 * Reference interfaces replaced (paths inside the waylake/runnel project;
 * MLX / mlx-lm are third-party and not vendored there):
 *   rnb_switchglu_fwd  <- FusedQuantizedSwitchGLU.__call__(x, indices)
 *                         src/runnel/mlx.py:57-82 (one mx.gather_qmm over the
 *                         packed gate/up, SwiGLU, down_proj gather_qmm)
 *   rnb_moe_block_fwd  <- layer.mlp(x): mlx-lm Qwen3.5 sparse-MoE block as
 *                         timed by bench/mlx_component_profile.py:130 (router
 *                         Linear, softmax, argpartition top-k, renormalise,
 *                         switch_mlp, weighted sum, sigmoid-gated shared
 *                         expert bench/mlx_lm_adapter.py:82-94)
 *   rnb_router_topk    <- the router half of the same block (gate Linear,
 *                         softmax, top-k, renormalise)
 */
#ifndef RNB_MOE_H_
#define RNB_MOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RNB_API __attribute__((visibility("default")))
#else
#define RNB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define RNB_OK 0
#define RNB_ERR_INVALID -1     /* bad shape, null pointer, unsupported format */
#define RNB_ERR_ALIGN -2       /* a pointer is not 16-byte aligned */
#define RNB_ERR_WORKSPACE -3   /* workspace missing or smaller than required */
#define RNB_ERR_CUDA -4        /* a CUDA runtime call failed */
#define RNB_ERR_DEVICE -5      /* sm_100 device required */
#define RNB_ERR_TIMEOUT -6     /* a bounded device-side wait gave up */

/* Device status bits, accumulated in the workspace by the kernels and read
 * with rnb_moe_status(). */
#define RNB_STATUS_BAD_INDEX 0x1u  /* an expert index >= E was skipped */
#define RNB_STATUS_TIMEOUT 0x2u    /* a bounded device wait expired */

typedef struct rnb_moe_desc {
  int32_t T;             /* tokens in this call (rows of x) */
  int32_t H;             /* hidden size (2048 for Ornith) */
  int32_t I;             /* expert intermediate size (512) */
  int32_t E;             /* experts held in gu_w/dn_w (256, or a shard) */
  int32_t E_total;       /* router width (256); E_total == E without sharding */
  int32_t expert_offset; /* global id of gu_w[0] (expert-parallel shard) */
  int32_t k;             /* experts per token (8) */
  int32_t bits;          /* 4 or 8 */
  int32_t group;         /* quantization group, must be 64 */
  int32_t flags;         /* RNB_FLAG_* */
  /* routed bank */
  const uint32_t* gu_w; /* [E, 2I, H*bits/32]  up rows then gate rows */
  const uint16_t* gu_s; /* [E, 2I, H/64] bf16 */
  const uint16_t* gu_b; /* [E, 2I, H/64] bf16 */
  const uint32_t* dn_w; /* [E, H, I*bits/32] */
  const uint16_t* dn_s; /* [E, H, I/64] bf16 */
  const uint16_t* dn_b; /* [E, H, I/64] bf16 */
  /* router and shared expert (rnb_moe_block_fwd / rnb_router_topk only) */
  const uint16_t* router_w;      /* [E_total, H] bf16 */
  const uint16_t* shared_gate_w; /* [H] bf16; NULL = block without shared expert */
  const uint32_t* sgu_w;         /* [2I, H*bits/32]  up rows then gate rows */
  const uint16_t* sgu_s;         /* [2I, H/64] */
  const uint16_t* sgu_b;
  const uint32_t* sdn_w; /* [H, I*bits/32] */
  const uint16_t* sdn_s; /* [H, I/64] */
  const uint16_t* sdn_b;
  /* 8-bit router (real Ornith checkpoints keep mlp.gate and
   * mlp.shared_expert_gate as 8-bit MLX affine, group 64).  router_bits 0 or
   * 16: router_w [E_total, H] and shared_gate_w [H] are bf16.  router_bits 8:
   * router_w points at uint32 codes [E_total, H/4] and shared_gate_w at codes
   * [H/4], with bf16 scales and biases per 64 inputs in router_s / router_b
   * [E_total, H/64] and sgate_s / sgate_b [H/64]; a logit is then the
   * correctly rounded bf16 of the exact dot product with the dequantised row
   * s * code + b. */
  int32_t router_bits;
  int32_t reserved0;
  const uint16_t* router_s;
  const uint16_t* router_b;
  const uint16_t* sgate_s;
  const uint16_t* sgate_b;
} rnb_moe_desc;

/* rnb_moe_desc.flags */
#define RNB_FLAG_SHARED_ON_THIS_RANK 0x1 /* add the shared expert (set on one EP rank only
                                            when the shared expert is split off) */
#define RNB_FLAG_NO_SHARED 0x2           /* skip the shared expert even if pointers are set */
#define RNB_FLAG_Y_F32 0x4               /* rnb_switchglu_fwd / rnb_moe_block_fwd write fp32
                                            instead of bf16 (partial sums for a cross-rank reduce) */
#define RNB_FLAG_CHAIN 0x8               /* rnb_moe_block_fwd: use the three-kernel decode chain
                                            (in 64-token chunks) even where the persistent
                                            single-launch kernel or the prefill path applies */

/* Library version (major*10000 + minor*100 + patch). */
RNB_API int rnb_version(void);

/* Thread-local message describing the last error returned on this thread. */
RNB_API const char* rnb_last_error(void);

/* Bytes of workspace a call with this descriptor needs.  The workspace must
 * be zero-filled once when allocated (rnb_moe_workspace_init does it); every
 * call leaves its counters at zero again.  Calls that share one workspace
 * must be ordered on one stream. */
RNB_API int rnb_moe_workspace_size(const rnb_moe_desc* d, size_t* bytes);
RNB_API int rnb_moe_workspace_init(void* ws, size_t ws_bytes, void* stream);

/* Router half of the block: bf16 logits = x . router_w^T, top-k of those
 * logits (ties to the lower expert index), routing weights = fp32 softmax over
 * all E_total logits at the selected experts, renormalised to sum 1.
 *   x        [T, H] bf16 (device)
 *   inds     [T, k] uint32 out, slots ordered by descending logit
 *   scores   [T, k] fp32 out
 *   logits   [T, E_total] fp32 out (bf16-rounded values) or NULL */
RNB_API int rnb_router_topk(const rnb_moe_desc* d, const void* x, uint32_t* inds, float* scores,
                    float* logits, void* ws, size_t ws_bytes, void* stream);

/* SwitchGLU over caller-chosen experts: for every token t and slot s,
 *   y[t, s, :] = down_e(silu(gate_e . x_t) * (up_e . x_t)),  e = inds[t, s]
 * unweighted, in bf16 (fp32 with RNB_FLAG_Y_F32), like
 * FusedQuantizedSwitchGLU.__call__.
 *   x    [T, H] bf16;  inds [T, k] uint32 global expert ids;  y [T, k, H] bf16
 * With expert parallelism (E < E_total) slots whose expert is not in
 * [expert_offset, expert_offset + E) are written as zeros. */
RNB_API int rnb_switchglu_fwd(const rnb_moe_desc* d, const void* x, const uint32_t* inds, void* y,
                      void* ws, size_t ws_bytes, void* stream);

/* Whole sparse-MoE block:
 *   out[t] = sum_s scores[t,s] * y[t,s] + sigmoid(x_t . shared_gate_w) * shared(x_t)
 *   x [T, H] bf16 -> out [T, H] bf16; inds_out [T, k] / scores_out [T, k]
 * are optional copies of the routing (NULL to skip).  Up to 64 tokens run the
 * decode kernels; more tokens run the sorted grouped-GEMM path (tensor-core
 * tcgen05 GEMMs) when the workspace has rnb_moe_workspace_size() bytes for
 * this T, else the decode kernels in 64-token chunks.  Both paths add a
 * token's expert contributions in slot order, so repeated calls give the same
 * bits. */
RNB_API int rnb_moe_block_fwd(const rnb_moe_desc* d, const void* x, void* out, uint32_t* inds_out,
                      float* scores_out, void* ws, size_t ws_bytes, void* stream);

/* rnb_moe_block_fwd for callers that cannot allocate device memory -- for
 * example a host that may not call cudaMalloc while it captures a CUDA graph,
 * or an engine plugin that owns no allocator.  It takes no workspace: scratch
 * is a static 12 MiB device array inside this library, present on every GPU
 * that loads it (enough for the Ornith shapes; larger shapes are rejected
 * with RNB_ERR_WORKSPACE).  The first call on a device looks up that array's
 * address, so make it before any stream capture.  All calls share the one
 * array: calls that can overlap on the GPU (other streams, other threads)
 * race and must be serialised by the caller.  The device status bits of
 * these calls (RNB_STATUS_*) accumulate in the static array until
 * rnb_moe_noalloc_status reads them.  No counterpart in the reference. */
RNB_API int rnb_moe_block_fwd_noalloc(const rnb_moe_desc* d, const void* x, void* out,
                                      uint32_t* inds_out, float* scores_out, void* stream);
/* Status bits (RNB_STATUS_*) of the rnb_moe_block_fwd_noalloc calls on the
 * current device since the last read: copies them to *status and clears
 * them.  Synchronises the stream.  A call whose status has
 * RNB_STATUS_TIMEOUT produced void results.  No counterpart in the
 * reference. */
RNB_API int rnb_moe_noalloc_status(uint32_t* status, void* stream);

/* rnb_moe_block_fwd from host memory, one call for the whole round trip:
 * copies x_host ([T, H] bf16) into the device staging buffer x_dev, runs the
 * block into out_dev, and copies out_dev back to out_host ([T, H] bf16, or
 * fp32 with RNB_FLAG_Y_F32).  The three steps are queued on `stream` and the
 * call returns without waiting: out_host holds the result once the stream has
 * been synchronised.  Use page-locked (pinned) host buffers, since copies from
 * pageable memory are staged and partly synchronous.  Up to 64 tokens, when
 * out_host is page-locked, mapped for this device and 16-byte aligned, the
 * block's kernels store the result straight into it and out_dev is not used.  x_dev and out_dev
 * are caller-owned, 16-byte aligned and sized for T tokens.  From 4096 tokens
 * on, when both host buffers are page-locked, the call is split into 2-4
 * chunks of whole tokens whose copies run on two copy streams of the
 * library's own and overlap the other chunks' compute; the output bits are
 * those of one whole-batch call.  The first such call on a device creates
 * those streams (valid for that device's context only, like every cached
 * per-device object of this library), so make it before any stream capture.  No routing copies are
 * returned (use rnb_moe_block_fwd for those).  The reference's block call takes
 * unified-memory MLX arrays and needs no copies; on a discrete GPU this is the
 * closest call with host buffers. */
RNB_API int rnb_moe_block_fwd_host(const rnb_moe_desc* d, const void* x_host, void* out_host,
                                   void* x_dev, void* out_dev, void* ws, size_t ws_bytes,
                                   void* stream);

/* Copies the device status word (RNB_STATUS_* bits) to *status and clears it.
 * Synchronises the stream. */
RNB_API int rnb_moe_status(void* ws, size_t ws_bytes, uint32_t* status, void* stream);

/* Routed experts with given routing (the receive side of an expert-parallel
 * all-to-all; no reference counterpart).  T rows x, each with k global
 * expert ids inds[t][j] and weights scores[t][j]:
 *   out[t] = sum over j with inds[t][j] in this descriptor's shard of
 *            scores[t][j] * expert_{inds[t][j]}(x[t])
 * (bf16 out, or fp32 with RNB_FLAG_Y_F32).  No router and no shared expert;
 * ids >= E_total are skipped and set RNB_STATUS_BAD_INDEX.  Runs the grouped
 * GEMM pipeline for any T; its workspace size comes from
 * rnb_moe_experts_workspace_size. */
RNB_API int rnb_moe_experts_workspace_size(const rnb_moe_desc* d, size_t* bytes);
RNB_API int rnb_moe_experts_fwd(const rnb_moe_desc* d, const void* x, const uint32_t* inds, const float* scores,
                                void* out, void* ws, size_t ws_bytes, void* stream);

/* ---- Standalone quantized matvec / matmul probes ----
 * The reference's runnel-metal-qmv and runnel-metal-qmm CLIs
 * (native/bench/quantized_qmv.cpp:186-270, quantized_qmm.cpp:112-145; kernels
 * and CPU checks in native/src/quantized_qmv_probe.mm and
 * quantized_qmm_probe.mm).  W is MLX affine: [rows][K*bits/32] uint32 codes,
 * [rows][K/group] bf16 scales and biases; x is bf16.
 *
 * rnb_qmv: y[r] = W[row(r)] . x for r < rows (fp32).  Dense when selected is
 * NULL: row(r) = r.  Expert mode (the gather QMV): selected is a HOST array of
 * n_selected expert ids, rows = n_selected * rows_per_expert and
 * row(r) = selected[r / rows_per_expert] * rows_per_expert + r % rows_per_expert
 * within a bank of bank_rows rows.  K: multiple of 512 up to 16384; rows and
 * rows_per_expert: multiples of 16. */
#define RNB_QMV_MAX_EXPERTS 64
RNB_API int rnb_qmv(int bits, int group, int64_t rows, int64_t K, const uint32_t* w, const uint16_t* scales,
                    const uint16_t* biases, const void* x, const uint32_t* selected, int n_selected,
                    int64_t rows_per_expert, int64_t bank_rows, float* y, void* stream);
/* rnb_qmm: y[t][n] = W[n] . x[t] for t < T, n < N (bf16 out, fp32 with y_f32).
 * N: multiple of 128; K: multiple of 512.  Workspace from
 * rnb_qmm_workspace_size. */
RNB_API int rnb_qmm_workspace_size(int bits, int group, int T, int N, int K, size_t* bytes);
RNB_API int rnb_qmm(int bits, int group, int T, int N, int K, const uint32_t* w, const uint16_t* scales,
                    const uint16_t* biases, const void* x, void* y, int y_f32, void* ws, size_t ws_bytes,
                    void* stream);

/* ---- Expert parallelism (one process per GPU, ranks on one node) ----
 * Reference counterpart: none in waylake/runnel (single Apple GPU); this is
 * the rnb_ep_* surface of the B200 build.  Rank r holds experts
 * [expert_offset, expert_offset + E) of E_total (its rnb_moe_desc says so),
 * the router and the shared expert; the shared expert's 128-channel
 * intermediate quarters are split round-robin over the ranks.
 * rnb_ep_create allocates this rank's receive buffer and writes its CUDA IPC
 * handle (RNB_EP_HANDLE_BYTES) to handle_out; the caller gathers every rank's
 * handle (rank order) and passes them to rnb_ep_connect.  Every rank then
 * makes the same sequence of rnb_moe_block_ep_fwd calls with the same T; each
 * returns the full block output (the sum over ranks, in rank order) in bf16,
 * or fp32 with RNB_FLAG_Y_F32.  The ranks exchange partial outputs by NVLink
 * stores inside the kernel (no multicast); device waits are bounded and set
 * RNB_STATUS_TIMEOUT if a peer does not arrive.  Token counts the
 * persistent decode kernel takes (T <= 2) run as one launch with the shared
 * expert split by quarter; larger T runs in 64-token chunks of the decode
 * chain (shared expert on rank 0) followed by an exchange kernel.
 * Call rnb_ep_destroy on every rank after a host barrier. */
#define RNB_EP_HANDLE_BYTES 64
typedef struct rnb_ep rnb_ep;
RNB_API int rnb_ep_create(int rank, int world, int H, rnb_ep** ep, void* handle_out);
RNB_API int rnb_ep_connect(rnb_ep* ep, const void* handles);
RNB_API int rnb_ep_destroy(rnb_ep* ep);
/* How long a call of this context waits for the other ranks' partial words
 * before it gives up, sets RNB_STATUS_TIMEOUT and returns (its results are
 * then void); default 2000 ms (ranks launch independently).  ms in
 * [1, 600000]. */
RNB_API int rnb_ep_set_wait_limit_ms(rnb_ep* ep, int ms);
RNB_API int rnb_moe_block_ep_fwd(const rnb_moe_desc* d, rnb_ep* ep, const void* x, void* out,
                                 uint32_t* inds_out, float* scores_out, void* ws, size_t ws_bytes,
                                 void* stream);

/* ---- Expert parallelism for many tokens: device-side all-to-all ----
 * (No reference counterpart.)  Every rank holds its own T tokens (the same T
 * on every rank) and the expert shard [rank E, rank E + E) of E_total =
 * world E, with the router and the whole shared expert.  One
 * rnb_moe_block_a2a_fwd call computes the full block for this rank's tokens:
 * the home block on the shard (routing, its experts, the shared expert),
 * then each token's row goes by NVLink stores (CUDA IPC, no multicast) to
 * every other rank that owns one of its experts, those ranks run their
 * experts on the rows they received (the grouped GEMM pipeline), the fp32
 * sums come back the same way, and the partials are added in a fixed order.
 * There is no host synchronisation inside a call; cross-GPU waits are
 * bounded and set RNB_STATUS_TIMEOUT in the workspace status word.  The
 * exchange and the remote experts run on a stream of the context's own,
 * which forks from the caller's stream once the home routing is queued and
 * joins it before the combine.  Not for CUDA graph capture: the exchange
 * epoch is the context's host-side call count, which a replay would not
 * advance.
 * rnb_a2a_create allocates this rank's areas for up to max_tokens tokens and
 * writes its IPC handle (RNB_A2A_HANDLE_BYTES); gather every rank's handle
 * (rank order) and pass them to rnb_a2a_connect.  Every rank then makes the
 * same sequence of calls with the same T; the descriptor is this rank's
 * shard (E_total = world E, expert_offset = rank E).  The workspace size
 * comes from rnb_moe_block_a2a_workspace_size.  Call rnb_a2a_destroy on every
 * rank after a host barrier. */
#define RNB_A2A_HANDLE_BYTES 64
typedef struct rnb_a2a rnb_a2a;
RNB_API int rnb_a2a_create(int rank, int world, int H, int k, int max_tokens, rnb_a2a** a, void* handle_out);
RNB_API int rnb_a2a_connect(rnb_a2a* a, const void* handles);
RNB_API int rnb_a2a_destroy(rnb_a2a* a);
RNB_API int rnb_a2a_set_wait_limit_ms(rnb_a2a* a, int ms);
RNB_API int rnb_moe_block_a2a_workspace_size(const rnb_moe_desc* d, rnb_a2a* a, size_t* bytes);
RNB_API int rnb_moe_block_a2a_fwd(const rnb_moe_desc* d, rnb_a2a* a, const void* x, void* out, uint32_t* inds_out,
                                  float* scores_out, void* ws, size_t ws_bytes, void* stream);

/* Layer glue of a decoder stack, around the block (no reference counterpart in
 * runnel itself -- mlx-lm's Qwen3.5 decoder layer does `x + mlp(rms_norm(x))`).  For T tokens of H bf16 values:
 *   x_out = bf16(x + y)   (y may be NULL: x_out = x)
 *   xn_out = bf16(x_out * rsqrt(mean(x_out^2) + eps) * w)   (fp32 math, w bf16 [H])
 * x_out may alias x. */
RNB_API int rnb_add_rmsnorm(const void* x, const void* y, const void* w, void* x_out, void* xn_out, int T, int H,
                            float eps, void* stream);

/* One decoder layer's glue plus block (no reference counterpart; the layer
 * glue of the 40-layer configuration):
 *   resid_out = bf16(resid + y_prev)            (y_prev may be NULL: a copy)
 *   xn_out    = bf16(rms_norm(resid_out) * norm_w)   (as rnb_add_rmsnorm)
 *   out       = block(xn_out)                   (expert parallel when ep != NULL)
 * bit-identical to rnb_add_rmsnorm followed by the block call.  For 1-2 tokens
 * the glue runs inside the block's single persistent launch.  resid_out and
 * xn_out must not alias resid or y_prev; out may alias y_prev. */
RNB_API int rnb_moe_block_norm_fwd(const rnb_moe_desc* d, rnb_ep* ep, const void* resid, const void* y_prev,
                                   const void* norm_w, float eps, void* resid_out, void* xn_out, void* out,
                                   void* ws, size_t ws_bytes, void* stream);

/* Per-stage device timing (diagnostics; no reference counterpart -- the
 * reference profiles its block from the host, bench/mlx_component_profile.py).
 * While enabled, every block call records CUDA events on its stream between
 * its kernels: prefill stages route, sort, scatter, gateup, down, final;
 * decode stages decode (persistent kernel) or route, gateup, down (chain).
 * Do not enable it while a stream is being captured into a graph.
 * rnb_stage_times waits for the recorded calls, writes per stage the summed
 * milliseconds over them (ms[i], i < max_stages, stage ids below) and the
 * number of timed calls, and forgets them; returns the number of stage ids. */
#define RNB_STAGE_DECODE 0
#define RNB_STAGE_ROUTE 1
#define RNB_STAGE_SORT 2
#define RNB_STAGE_SCATTER 3
#define RNB_STAGE_GATEUP 4
#define RNB_STAGE_DOWN 5
#define RNB_STAGE_FINAL 6
#define RNB_NUM_STAGES 7
RNB_API int rnb_stage_timing(int enable);
RNB_API int rnb_stage_times(float* ms, int max_stages, int* calls);

#ifdef __cplusplus
}
#endif

#endif /* RNB_MOE_H_ */
