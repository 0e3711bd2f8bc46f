// rnb_internal.h -- host-side helpers shared by the decode and prefill units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "rnb_moe.h"

namespace rnb {

// Records the message for rnb_last_error() and returns code.
int fail(int code, const std::string& msg);
bool aligned16(const void* p);
bool has_shared(const rnb_moe_desc* d);

// A tiled TMA tensor map of `rank` dimensions (innermost first): dims in
// elements, strides in bytes for dimensions 1 .. rank-1, box in elements.
// Uses the driver's encoder through the runtime (no link against the
// driver).  False when the encoder is missing or rejects the description.
bool encode_tiled(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle sw);

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
};
DevInfo dev_info();

// Every workspace starts with the status word (offset 0) and, at offset 256,
// the decode kernels' arrival counters, which each decode call leaves at zero
// for the next; both layouts reserve this header so any call may follow any
// other on one workspace.
constexpr size_t kWsCountersOffset = 256;
inline size_t ws_counter_bytes(const rnb_moe_desc& d) { return 4u * (4u + static_cast<size_t>(d.H) / 16u); }

// The first 256-byte slot holds, besides the status word (offset 0), the
// persistent decode kernel's call sequence word (offset 64) and exit counter
// (offset 68); neither is ever cleared by a call or by rnb_moe_status.
constexpr size_t kWsSeqOffset = 64;

// After the counters, both layouts reserve the persistent decode kernel's
// exchange words: 8-byte {value, epoch} words that only that kernel writes
// (an epoch is a sequence number, so no other path may leave data there):
// router logits [2 tokens][257 rows], SwiGLU rows [2 tokens][9 slots][512]
// and the one-token split-K partials [16 tasks x 9 sources][2048 rows].
// Each logit word has a 128-byte line of its own: every CTA polls all of
// them, and packed into a few lines the polls would queue at a few L2 slices.
constexpr size_t kLwStride = 16;
constexpr size_t kXchgLogitWords = 2 * 257 * kLwStride;
constexpr size_t kXchgHWords = 2 * 9 * 512;
constexpr size_t kXchgYWords = 16 * 9 * 2048;
constexpr size_t kXchgBytes = 8 * (kXchgLogitWords + kXchgHWords + kXchgYWords);

// Stage timing (rnb_timing.cu): no-ops unless rnb_stage_timing(1) was called.
void stage_begin(cudaStream_t st);
void stage_end(cudaStream_t st, int stage);

// Prefill path (many tokens): workspace bytes it needs for d->T tokens, and
// whether it supports the descriptor's shapes.
size_t prefill_workspace_bytes(const rnb_moe_desc& d);
bool prefill_supported(const rnb_moe_desc& d);
// When set (per host thread), the prefill pipeline records this event on its
// stream as soon as the routing stage is queued, and sets *fired; the
// device-side all-to-all uses it to start its dispatch before the home
// experts run.  Null (the default) records nothing.
void set_prefill_route_event(cudaEvent_t ev, bool* fired);
// inds_in / scores_in ([T][k]): given routing (no router, no shared expert).
int run_prefill(const rnb_moe_desc* d, const void* x, void* out, uint32_t* inds_out, float* scores_out,
                void* ws, size_t ws_bytes, cudaStream_t st, const uint32_t* inds_in = nullptr,
                const float* scores_in = nullptr);

// RNB_ERR_DEVICE (with a message) unless the current device is an sm_100 part.
int check_device();

// Standalone quantized matmul through the prefill GEMM (rnb_prefill.cu).
int qmm_workspace_bytes(int bits, int group, int T, int N, int K, size_t* bytes);
int run_qmm(int bits, int T, int N, int K, const uint32_t* w, const uint16_t* s, const uint16_t* b, const void* x,
            void* y, bool y_f32, void* ws, size_t ws_bytes, cudaStream_t st);

}  // namespace rnb
