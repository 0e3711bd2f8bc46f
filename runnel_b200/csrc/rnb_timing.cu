// rnb_timing.cu -- optional per-stage device timing of block calls.
//
// A timed call records one CUDA event when it starts and one after each of
// its kernels, all on the caller's stream; the elapsed time between
// consecutive events is charged to the stage that ended.  Events come from a
// pool and go back to it when the times are read.
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "rnb_internal.h"
#include "rnb_moe.h"

namespace rnb {
namespace {

constexpr int kMaxMarks = 8;
constexpr size_t kMaxCalls = 4096;

struct CallRecord {
  cudaEvent_t ev[kMaxMarks];
  int stage[kMaxMarks];
  int n = 0;
};

struct Timing {
  std::mutex mu;
  bool enabled = false;
  std::vector<cudaEvent_t> pool;
  std::vector<CallRecord> calls;
  bool open = false;  // the last record still takes marks
};

Timing& timing() {
  static Timing t;
  return t;
}

cudaEvent_t take_event(Timing& t) {
  if (!t.pool.empty()) {
    cudaEvent_t e = t.pool.back();
    t.pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

}  // namespace

void stage_begin(cudaStream_t st) {
  Timing& t = timing();
  std::lock_guard<std::mutex> lk(t.mu);
  t.open = false;
  if (!t.enabled || t.calls.size() >= kMaxCalls) return;
  cudaEvent_t e = take_event(t);
  if (!e) return;
  CallRecord r;
  r.ev[0] = e;
  r.stage[0] = -1;
  r.n = 1;
  cudaEventRecord(e, st);
  t.calls.push_back(r);
  t.open = true;
}

void stage_end(cudaStream_t st, int stage) {
  Timing& t = timing();
  std::lock_guard<std::mutex> lk(t.mu);
  if (!t.enabled || !t.open || t.calls.empty()) return;
  CallRecord& r = t.calls.back();
  if (r.n >= kMaxMarks) return;
  cudaEvent_t e = take_event(t);
  if (!e) return;
  cudaEventRecord(e, st);
  r.ev[r.n] = e;
  r.stage[r.n] = stage;
  ++r.n;
}

}  // namespace rnb

extern "C" {

int rnb_stage_timing(int enable) {
  rnb::Timing& t = rnb::timing();
  std::lock_guard<std::mutex> lk(t.mu);
  t.enabled = enable != 0;
  t.open = false;
  return RNB_OK;
}

int rnb_stage_times(float* ms, int max_stages, int* calls) {
  rnb::Timing& t = rnb::timing();
  std::lock_guard<std::mutex> lk(t.mu);
  for (int i = 0; i < max_stages && ms; ++i) ms[i] = 0.f;
  int n = 0;
  int rc = RNB_OK;
  for (rnb::CallRecord& r : t.calls) {
    if (r.n > 1 && cudaEventSynchronize(r.ev[r.n - 1]) == cudaSuccess) {
      for (int i = 1; i < r.n; ++i) {
        float el = 0.f;
        if (cudaEventElapsedTime(&el, r.ev[i - 1], r.ev[i]) != cudaSuccess) {
          rc = rnb::fail(RNB_ERR_CUDA, "rnb_stage_times: event timing failed");
          continue;
        }
        if (ms && r.stage[i] >= 0 && r.stage[i] < max_stages) ms[r.stage[i]] += el;
      }
      ++n;
    }
    for (int i = 0; i < r.n; ++i) t.pool.push_back(r.ev[i]);
  }
  t.calls.clear();
  t.open = false;
  if (calls) *calls = n;
  return rc == RNB_OK ? RNB_NUM_STAGES : rc;
}

}  // extern "C"
