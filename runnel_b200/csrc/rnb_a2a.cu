// rnb_a2a.cu -- expert parallelism for many tokens with a device-side
// all-to-all over NVLink (no host synchronisation inside a call).
//
// Every rank holds its own T tokens and the expert shard [rank E, rank E + E)
// of E_total = world E (router and shared expert whole).  One call:
//   1. home block: rnb_moe_block_fwd on the shard -> fp32 partial (the
//      shard's experts and the shared expert) and the routing of every token;
//   2. dispatch (k_a2a_dispatch): for each token and each other rank, the
//      token's k expert ids and weights go into that rank's receive slot for
//      this rank, and its bf16 row too when one of its experts is there;
//      direct stores into the peer's memory (CUDA IPC), then, per CTA, one
//      {1, epoch} flag after a system-scope fence;
//   3. the flags of every peer are awaited (k_a2a_wait, bounded);
//   4. remote experts: rnb_moe_experts_fwd over the (world - 1) T received
//      rows (fp32 sums; rows with no expert here stay zero and their stale
//      x is never read);
//   5. return (k_a2a_return): each received row that had an expert here
//      goes back, fp32, into its home rank's return slot for this rank; flags
//      as in 2; k_a2a_wait again;
//   6. combine (k_a2a_combine): out[t] = bf16(home[t] + the returned rows of
//      t in rank order) -- only the rows its routing sent out are read.
// Steps 2-5 run on the context's own stream, which forks from the caller's
// as soon as the home block's routing is queued (prefill) or after the home
// block (decode sizes) and joins it before the combine: the NVLink traffic
// and the remote experts overlap the home block's gather and GEMMs.  The
// workspace is two regions, the home block's and the remote experts'; the
// combine folds the second region's status bits into the first's.
// Receive and return areas alternate by the call's parity: a rank cannot
// start call n + 2 before every peer has returned call n + 1's rows, which
// a peer does only after it has consumed call n.  The epoch is a per-context
// call count; every rank makes the same sequence of calls with the same T.
//
// Slot of source rank r at receiver q: (r - q - 1) mod world, so the
// (world - 1) slots of a receiver are contiguous rows for one experts call.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <string>

#include "rnb_internal.h"
#include "rnb_moe.h"

namespace rnb {
namespace {

constexpr int kA2aCtas = 128;     // CTAs of the dispatch and return kernels
constexpr int kA2aMaxRanks = 8;
constexpr uint64_t kA2aWaitNs = 2000ull * 1000 * 1000;  // default bound on a peer wait

__device__ __forceinline__ uint64_t a2a_timer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void a2a_flag_store(uint64_t* p, uint32_t epoch) {
  const uint64_t w = (static_cast<uint64_t>(epoch) << 32) | 1u;
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;\n" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t a2a_flag_load(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];\n" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Byte offsets of one parity's areas in a rank's shared (IPC) region.
struct A2aArea {
  size_t rx_x, rx_i, rx_s, back, rx_flags, back_flags, bytes;
};

size_t a2a_align(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

A2aArea a2a_area(int world, int H, int k, int Tmax) {
  A2aArea a;
  const size_t slots = static_cast<size_t>(world - 1) * Tmax;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = a2a_align(o + bytes);
    return at;
  };
  a.rx_x = take(slots * H * 2);
  a.rx_i = take(slots * k * 4);
  a.rx_s = take(slots * k * 4);
  a.back = take(slots * H * 4);
  a.rx_flags = take(static_cast<size_t>(kA2aMaxRanks) * kA2aCtas * 8);
  a.back_flags = take(static_cast<size_t>(kA2aMaxRanks) * kA2aCtas * 8);
  a.bytes = o;
  return a;
}

struct A2aParams {
  int rank, world, H, k, T, per;  // per: experts per rank
  uint32_t epoch;
  uint64_t wait_ns;
  uint32_t* status;
  uint32_t* status2;         // the remote experts' status word, folded in by the combine
  char* peer[kA2aMaxRanks];  // each rank's shared region, this call's parity
  A2aArea area;
  const uint16_t* x;       // [T][H] this rank's tokens
  const uint32_t* inds;    // [T][k] their routing
  const float* scores;     // [T][k]
  const float* part;       // [T][H] home partial (fp32)
  const float* y;          // [(world - 1) T][H] remote experts' sums (fp32)
  void* out;               // [T][H] bf16, or fp32 with y_f32
  int y_f32;
};

__device__ __forceinline__ int a2a_slot(int src, int dst, int world) { return (src - dst - 1 + world) % world; }

}  // namespace
}  // namespace rnb

namespace rnb {
namespace {

// Dispatch: a warp per token; to every other rank its k ids and weights,
// and its bf16 row when one of its experts is there.  Then one flag per CTA
// and peer after a system-scope fence.
__global__ void __launch_bounds__(256) k_a2a_dispatch(const __grid_constant__ A2aParams p) {
  const int lane = threadIdx.x & 31, gw = blockIdx.x * 8 + (threadIdx.x >> 5), nw = gridDim.x * 8;
  const int H8 = p.H / 8;  // 16-byte chunks of a bf16 row
  for (int t = gw; t < p.T; t += nw) {
    const uint32_t id = lane < p.k ? p.inds[static_cast<size_t>(t) * p.k + lane] : 0u;
    const float sc = lane < p.k ? p.scores[static_cast<size_t>(t) * p.k + lane] : 0.f;
    const uint32_t own = lane < p.k ? id / static_cast<uint32_t>(p.per) : 0xFFFFFFFFu;
    const uint32_t bit = own < static_cast<uint32_t>(p.world) ? (1u << own) : 0u;
    const uint32_t mask = __reduce_or_sync(0xffffffffu, bit) & ~(1u << p.rank);
    const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * p.H);
    for (int q = 0; q < p.world; ++q) {
      if (q == p.rank) continue;
      char* base = p.peer[q];
      const size_t row = static_cast<size_t>(a2a_slot(p.rank, q, p.world)) * p.T + t;
      if (lane < p.k) {
        reinterpret_cast<uint32_t*>(base + p.area.rx_i)[row * p.k + lane] = id;
        reinterpret_cast<float*>(base + p.area.rx_s)[row * p.k + lane] = sc;
      }
      if ((mask >> q) & 1u) {
        uint4* dst = reinterpret_cast<uint4*>(base + p.area.rx_x) + row * H8;
        for (int i = lane; i < H8; i += 32) dst[i] = __ldg(src + i);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // the CTA's stores before its flags
    for (int q = 0; q < p.world; ++q)
      if (q != p.rank)
        a2a_flag_store(reinterpret_cast<uint64_t*>(p.peer[q] + p.area.rx_flags) +
                           static_cast<size_t>(p.rank) * kA2aCtas + blockIdx.x,
                       p.epoch);
  }
}

// Every peer's flags in this rank's region at `off` for this call's epoch
// (bounded; on expiry RNB_STATUS_TIMEOUT and the call's results are void).
__global__ void __launch_bounds__(256) k_a2a_wait(const __grid_constant__ A2aParams p, size_t off) {
  const uint64_t* f = reinterpret_cast<const uint64_t*>(p.peer[p.rank] + off);
  const uint64_t deadline = a2a_timer() + p.wait_ns;
  for (int i = threadIdx.x; i < p.world * kA2aCtas; i += blockDim.x) {
    if (i / kA2aCtas == p.rank) continue;
    while (static_cast<uint32_t>(a2a_flag_load(f + i) >> 32) != p.epoch) {
      if (a2a_timer() > deadline) {
        atomicOr(p.status, RNB_STATUS_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
}

// Return: a warp per received row that had an expert here; its fp32 sum goes
// into the home rank's return slot for this rank.  Flags as in dispatch.
__global__ void __launch_bounds__(256) k_a2a_return(const __grid_constant__ A2aParams p) {
  const int lane = threadIdx.x & 31, gw = blockIdx.x * 8 + (threadIdx.x >> 5), nw = gridDim.x * 8;
  const int H4 = p.H / 4;  // 16-byte chunks of an fp32 row
  const char* own = p.peer[p.rank];
  const int rows = (p.world - 1) * p.T;
  for (int ri = gw; ri < rows; ri += nw) {
    const int j = ri / p.T, t = ri % p.T;
    const uint32_t id = lane < p.k ? reinterpret_cast<const uint32_t*>(own + p.area.rx_i)[static_cast<size_t>(ri) * p.k + lane]
                                   : 0xFFFFFFFFu;
    const bool here = lane < p.k && id / static_cast<uint32_t>(p.per) == static_cast<uint32_t>(p.rank);
    if (!__any_sync(0xffffffffu, here)) continue;
    const int r = (p.rank + 1 + j) % p.world;  // the row's home rank
    const size_t drow = static_cast<size_t>(a2a_slot(p.rank, r, p.world)) * p.T + t;
    const uint4* src = reinterpret_cast<const uint4*>(p.y + static_cast<size_t>(ri) * p.H);
    uint4* dst = reinterpret_cast<uint4*>(p.peer[r] + p.area.back) + drow * H4;
    for (int i = lane; i < H4; i += 32) dst[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < p.world; ++q)
      if (q != p.rank)
        a2a_flag_store(reinterpret_cast<uint64_t*>(p.peer[q] + p.area.back_flags) +
                           static_cast<size_t>(p.rank) * kA2aCtas + blockIdx.x,
                       p.epoch);
  }
}

// Combine: 8 values of one token per thread; the home partial plus, in slot
// order, the rows this token's routing sent out.
__global__ void __launch_bounds__(256) k_a2a_combine(const __grid_constant__ A2aParams p) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int H8 = p.H / 8;
  if (i == 0 && p.status2) {
    const uint32_t s2 = *p.status2;
    if (s2) {
      atomicOr(p.status, s2);
      *p.status2 = 0;
    }
  }
  if (i >= static_cast<size_t>(p.T) * H8) return;
  const int t = static_cast<int>(i / H8), h0 = static_cast<int>(i % H8) * 8;
  uint32_t mask = 0;
  for (int s = 0; s < p.k; ++s) {
    const uint32_t r = p.inds[static_cast<size_t>(t) * p.k + s] / static_cast<uint32_t>(p.per);
    if (r < static_cast<uint32_t>(p.world)) mask |= 1u << r;
  }
  const float4* hp = reinterpret_cast<const float4*>(p.part + static_cast<size_t>(t) * p.H + h0);
  float4 a = hp[0], b = hp[1];
  const char* own = p.peer[p.rank];
  for (int j = 0; j < p.world - 1; ++j) {
    const int r = (p.rank + 1 + j) % p.world;
    if (!((mask >> r) & 1u)) continue;
    const float4* bp = reinterpret_cast<const float4*>(own + p.area.back) +
                       ((static_cast<size_t>(j) * p.T + t) * p.H + h0) / 4;
    const float4 u = __ldcg(bp), v = __ldcg(bp + 1);
    a.x += u.x; a.y += u.y; a.z += u.z; a.w += u.w;
    b.x += v.x; b.y += v.y; b.z += v.z; b.w += v.w;
  }
  const size_t o = static_cast<size_t>(t) * p.H + h0;
  if (p.y_f32) {
    float4* d = reinterpret_cast<float4*>(static_cast<float*>(p.out) + o);
    d[0] = a;
    d[1] = b;
  } else {
    __nv_bfloat162 q[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                           __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + o) = *reinterpret_cast<const uint4*>(q);
  }
}

}  // namespace
}  // namespace rnb

// ------------------------------------------------------------- host

struct rnb_a2a {
  int rank = 0, world = 1, H = 0, k = 0, Tmax = 0, dev = 0;
  uint64_t wait_ns = rnb::kA2aWaitNs;
  uint32_t calls = 0;       // the epoch of the last call
  size_t par_bytes = 0;     // one parity's shared area
  void* local = nullptr;    // both parities, exported by CUDA IPC
  char* peer[rnb::kA2aMaxRanks] = {};
  void* opened[rnb::kA2aMaxRanks] = {};
  float* part = nullptr;    // [Tmax][H] home partial
  uint32_t* inds = nullptr; // [Tmax][k]
  float* scores = nullptr;  // [Tmax][k]
  float* y = nullptr;       // [(world - 1) Tmax][H] remote experts' sums
  cudaStream_t side = nullptr;     // dispatch, remote experts and return
  cudaEvent_t ev_route = nullptr;  // the home routing is in a->inds / a->scores
  cudaEvent_t ev_done = nullptr;   // the side stream's work of the call is queued
  bool connected = false;
};

namespace rnb {
namespace {

void a2a_free(rnb_a2a* a) {
  for (int q = 0; q < a->world; ++q)
    if (a->opened[q]) cudaIpcCloseMemHandle(a->opened[q]);
  for (void* p : {a->local, static_cast<void*>(a->part), static_cast<void*>(a->inds), static_cast<void*>(a->scores),
                  static_cast<void*>(a->y)})
    if (p) cudaFree(p);
  if (a->ev_route) cudaEventDestroy(a->ev_route);
  if (a->ev_done) cudaEventDestroy(a->ev_done);
  if (a->side) cudaStreamDestroy(a->side);
  delete a;
}

// The descriptor of this rank's shard, checked against the context.
int a2a_check(const rnb_moe_desc* d, const rnb_a2a* a) {
  using namespace rnb;
  if (!d || !a) return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a: NULL descriptor or context");
  if (!a->connected) return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a: context not connected");
  if (d->H != a->H || d->k != a->k) return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a: H or k differs from the context's");
  if (d->T < 0 || d->T > a->Tmax) return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a: T exceeds the context's max_tokens");
  if (d->E * a->world != d->E_total || d->expert_offset != a->rank * d->E)
    return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a: the descriptor is not this rank's shard (E_total = world E, "
                                 "expert_offset = rank E)");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != a->dev) return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a: current device is not the context's");
  return RNB_OK;
}

// The two workspace regions: the home block's [0, home) and the remote
// experts' [home, home + experts).  `home` is sized for the context's
// max_tokens, so the experts' region (its status word first) starts at the
// same offset in every call whatever its T: the home block's scratch of one
// call never lands under the experts' status word of another.
int a2a_ws_split(const rnb_moe_desc* d, const rnb_a2a* a, size_t* home, size_t* experts);

rnb_moe_desc a2a_experts_desc(const rnb_moe_desc* d, const rnb_a2a* a) {
  rnb_moe_desc e = *d;
  e.T = (a->world - 1) * d->T;
  e.flags |= RNB_FLAG_Y_F32;
  return e;
}

int a2a_ws_split(const rnb_moe_desc* d, const rnb_a2a* a, size_t* home, size_t* experts) {
  rnb_moe_desc h = *d;
  h.flags |= RNB_FLAG_Y_F32;
  h.T = a->Tmax;  // the block's workspace size grows with T
  size_t b0 = 0, b1 = 0;
  int rc = rnb_moe_workspace_size(&h, &b0);
  if (rc) return rc;
  if (a->world > 1) {
    const rnb_moe_desc e = a2a_experts_desc(d, a);
    rc = rnb_moe_experts_workspace_size(&e, &b1);
    if (rc) return rc;
    b0 = (b0 + 255) & ~static_cast<size_t>(255);
  }
  *home = b0;
  *experts = b1;
  return RNB_OK;
}

}  // namespace

}  // namespace rnb

using rnb::fail;

int rnb_a2a_create(int rank, int world, int H, int k, int max_tokens, rnb_a2a** out, void* handle_out) {
  using namespace rnb;
  if (!out || !handle_out) return fail(RNB_ERR_INVALID, "rnb_a2a_create: NULL output pointer");
  *out = nullptr;
  if (world < 1 || world > kA2aMaxRanks || rank < 0 || rank >= world)
    return fail(RNB_ERR_INVALID, "rnb_a2a_create: need 0 <= rank < world <= 8");
  if (H <= 0 || H % 64 || k < 1 || k > 32 || max_tokens < 1)
    return fail(RNB_ERR_INVALID, "rnb_a2a_create: need H a positive multiple of 64, 1 <= k <= 32, max_tokens >= 1");
  rnb_a2a* a = new rnb_a2a();
  a->rank = rank;
  a->world = world;
  a->H = H;
  a->k = k;
  a->Tmax = max_tokens;
  cudaGetDevice(&a->dev);
  a->par_bytes = a2a_area(world, H, k, max_tokens).bytes;
  const size_t T = max_tokens;
  cudaError_t e = cudaMalloc(&a->local, 2 * a->par_bytes);
  if (e == cudaSuccess) e = cudaMemset(a->local, 0, 2 * a->par_bytes);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&a->part), T * H * 4);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&a->inds), T * k * 4);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&a->scores), T * k * 4);
  if (e == cudaSuccess && world > 1)
    e = cudaMalloc(reinterpret_cast<void**>(&a->y), static_cast<size_t>(world - 1) * T * H * 4);
  if (e == cudaSuccess && world > 1) {
    int least = 0, greatest = 0;
    e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&a->side, cudaStreamNonBlocking, greatest);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a->ev_route, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a->ev_done, cudaEventDisableTiming);
  }
  cudaIpcMemHandle_t h;
  memset(&h, 0, sizeof(h));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, a->local);
  if (e != cudaSuccess) {
    a2a_free(a);
    return fail(RNB_ERR_CUDA, std::string("rnb_a2a_create: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) <= RNB_A2A_HANDLE_BYTES, "IPC handle fits the handle bytes");
  memset(handle_out, 0, RNB_A2A_HANDLE_BYTES);
  memcpy(handle_out, &h, sizeof(h));
  a->peer[rank] = static_cast<char*>(a->local);
  if (world == 1) a->connected = true;
  *out = a;
  return RNB_OK;
}

int rnb_a2a_connect(rnb_a2a* a, const void* handles) {
  using namespace rnb;
  if (!a || !handles) return fail(RNB_ERR_INVALID, "rnb_a2a_connect: NULL argument");
  if (a->connected && a->world > 1) return fail(RNB_ERR_INVALID, "rnb_a2a_connect: already connected");
  for (int q = 0; q < a->world; ++q) {
    if (q == a->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + static_cast<size_t>(q) * RNB_A2A_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int j = 0; j < q; ++j)
        if (a->opened[j]) {
          cudaIpcCloseMemHandle(a->opened[j]);
          a->opened[j] = nullptr;
          a->peer[j] = nullptr;
        }
      return fail(RNB_ERR_CUDA, std::string("rnb_a2a_connect: peer ") + std::to_string(q) + ": " +
                                    cudaGetErrorString(e));
    }
    a->opened[q] = ptr;
    a->peer[q] = static_cast<char*>(ptr);
  }
  a->connected = true;
  return RNB_OK;
}

int rnb_a2a_set_wait_limit_ms(rnb_a2a* a, int ms) {
  using namespace rnb;
  if (!a) return fail(RNB_ERR_INVALID, "rnb_a2a_set_wait_limit_ms: context is NULL");
  if (ms < 1 || ms > 600000) return fail(RNB_ERR_INVALID, "rnb_a2a_set_wait_limit_ms: ms must be in [1, 600000]");
  a->wait_ns = static_cast<uint64_t>(ms) * 1000000ull;
  return RNB_OK;
}

int rnb_a2a_destroy(rnb_a2a* a) {
  if (a) rnb::a2a_free(a);
  return RNB_OK;
}

int rnb_moe_block_a2a_workspace_size(const rnb_moe_desc* d, rnb_a2a* a, size_t* bytes) {
  using namespace rnb;
  if (!bytes) return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a_workspace_size: bytes is NULL");
  if (!d || !a) return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a_workspace_size: NULL descriptor or context");
  size_t b0 = 0, b1 = 0;
  const int rc = a2a_ws_split(d, a, &b0, &b1);
  if (rc) return rc;
  *bytes = b0 + b1;
  return RNB_OK;
}

int rnb_moe_block_a2a_fwd(const rnb_moe_desc* d, rnb_a2a* a, const void* x, void* out, uint32_t* inds_out,
                          float* scores_out, void* ws, size_t ws_bytes, void* stream) {
  using namespace rnb;
  int rc = a2a_check(d, a);
  if (rc) return rc;
  if (!x || !out || !ws) return fail(RNB_ERR_INVALID, "rnb_moe_block_a2a_fwd: x, out and ws must be non-NULL");
  if (!aligned16(x) || !aligned16(out)) return fail(RNB_ERR_ALIGN, "x and out must be 16-byte aligned");
  size_t need = 0;
  rc = rnb_moe_block_a2a_workspace_size(d, a, &need);
  if (rc) return rc;
  if (ws_bytes < need) return fail(RNB_ERR_WORKSPACE, "rnb_moe_block_a2a_fwd: workspace too small");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int T = d->T, H = d->H, k = d->k;
  if (T == 0) return RNB_OK;
  if (a->world == 1) return rnb_moe_block_fwd(d, x, out, inds_out, scores_out, ws, ws_bytes, stream);
  size_t b0 = 0, b1 = 0;
  rc = a2a_ws_split(d, a, &b0, &b1);
  if (rc) return rc;
  char* ws0 = static_cast<char*>(ws);
  char* ws1 = ws0 + b0;
  // 1. home block: the shard's experts and the shared expert, fp32, and the
  // routing; ev_route marks the routing (prefill) or the whole block (decode)
  rnb_moe_desc h = *d;
  h.flags |= RNB_FLAG_Y_F32;
  bool fired = false;
  set_prefill_route_event(a->ev_route, &fired);
  rc = rnb_moe_block_fwd(&h, x, a->part, a->inds, a->scores, ws0, b0, stream);
  set_prefill_route_event(nullptr, nullptr);
  if (rc) return rc;
  cudaError_t e = fired ? cudaSuccess : cudaEventRecord(a->ev_route, st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(a->side, a->ev_route, 0);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("rnb_moe_block_a2a_fwd fork: ") + cudaGetErrorString(e));
  const uint32_t epoch = ++a->calls;
  const size_t par = static_cast<size_t>(epoch & 1u) * a->par_bytes;
  A2aParams p;
  memset(&p, 0, sizeof(p));
  p.rank = a->rank;
  p.world = a->world;
  p.H = H;
  p.k = k;
  p.T = T;
  p.per = d->E;
  p.epoch = epoch;
  p.wait_ns = a->wait_ns;
  p.status = reinterpret_cast<uint32_t*>(ws0);   // the home region's status word (offset 0)
  p.status2 = reinterpret_cast<uint32_t*>(ws1);  // the remote experts' (offset 0 of theirs)
  for (int q = 0; q < a->world; ++q) p.peer[q] = a->peer[q] + par;
  p.area = a2a_area(a->world, H, k, a->Tmax);
  p.x = static_cast<const uint16_t*>(x);
  p.inds = a->inds;
  p.scores = a->scores;
  p.part = a->part;
  p.y = a->y;
  p.out = out;
  p.y_f32 = (d->flags & RNB_FLAG_Y_F32) ? 1 : 0;
  // 2-5 on the side stream, which always joins the caller's stream again
  // (also on an error), so later work on the caller's stream never runs
  // beside a half-finished exchange
  const cudaStream_t sd = a->side;
  k_a2a_dispatch<<<kA2aCtas, 256, 0, sd>>>(p);
  k_a2a_wait<<<1, 256, 0, sd>>>(p, p.area.rx_flags);
  e = cudaGetLastError();
  if (e != cudaSuccess) rc = fail(RNB_ERR_CUDA, std::string("rnb_moe_block_a2a_fwd dispatch: ") + cudaGetErrorString(e));
  if (!rc) {
    const char* own = p.peer[a->rank];
    const rnb_moe_desc ed = a2a_experts_desc(d, a);
    rc = rnb_moe_experts_fwd(&ed, own + p.area.rx_x, reinterpret_cast<const uint32_t*>(own + p.area.rx_i),
                             reinterpret_cast<const float*>(own + p.area.rx_s), a->y, ws1, b1, sd);
  }
  if (!rc) {
    k_a2a_return<<<kA2aCtas, 256, 0, sd>>>(p);
    k_a2a_wait<<<1, 256, 0, sd>>>(p, p.area.back_flags);
    e = cudaGetLastError();
    if (e != cudaSuccess) rc = fail(RNB_ERR_CUDA, std::string("rnb_moe_block_a2a_fwd return: ") + cudaGetErrorString(e));
  }
  e = cudaEventRecord(a->ev_done, sd);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st, a->ev_done, 0);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("rnb_moe_block_a2a_fwd join: ") + cudaGetErrorString(e));
  if (rc) return rc;
  // 6. the combine on the caller's stream
  const size_t n = static_cast<size_t>(T) * (H / 8);
  k_a2a_combine<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("rnb_moe_block_a2a_fwd: ") + cudaGetErrorString(e));
  if (inds_out) e = cudaMemcpyAsync(inds_out, a->inds, static_cast<size_t>(T) * k * 4, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && scores_out)
    e = cudaMemcpyAsync(scores_out, a->scores, static_cast<size_t>(T) * k * 4, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("rnb_moe_block_a2a_fwd routing copy: ") + cudaGetErrorString(e));
  return RNB_OK;
}
