// rnb_glue.cu -- the layer glue around the MoE block in a decoder stack:
// residual add and RMSNorm (x <- x + y; xn = x * rsqrt(mean(x^2) + eps) * w).
//
// Semantics follow MLX's bf16 decoder layers (mlx-lm Qwen3.5 block:
// `h = x + mlp(post_attention_layernorm(x))`, `mx.fast.rms_norm`): the sum is
// rounded to bf16, the norm is computed in fp32 and its output rounded to bf16.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "rnb_internal.h"
#include "rnb_moe.h"

namespace rnb {
namespace {

// One CTA per token; 256 threads, each with H/256 consecutive elements.
__global__ void __launch_bounds__(256) k_add_rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* y,
                                                      const __nv_bfloat16* w, __nv_bfloat16* x_out,
                                                      __nv_bfloat16* xn_out, int H, float eps) {
  __shared__ float red[8];
  const int t = blockIdx.x, tid = threadIdx.x;
  const size_t base = static_cast<size_t>(t) * H;
  float ss = 0.f;
  for (int i = tid; i < H; i += blockDim.x) {
    float v = __bfloat162float(x[base + i]);
    if (y) v = __bfloat162float(__float2bfloat16_rn(v + __bfloat162float(y[base + i])));
    x_out[base + i] = __float2bfloat16_rn(v);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(H) + eps);
  for (int i = tid; i < H; i += blockDim.x) {
    const float v = __bfloat162float(x_out[base + i]);
    xn_out[base + i] = __float2bfloat16_rn(v * r * __bfloat162float(w[i]));
  }
}

}  // namespace
}  // namespace rnb

extern "C" int rnb_add_rmsnorm(const void* x, const void* y, const void* w, void* x_out, void* xn_out, int T, int H,
                               float eps, void* stream) {
  using namespace rnb;
  if (T < 0 || H <= 0 || H % 8) return fail(RNB_ERR_INVALID, "rnb_add_rmsnorm: T >= 0 and H a positive multiple of 8");
  if (!x || !w || !x_out || !xn_out) return fail(RNB_ERR_INVALID, "rnb_add_rmsnorm: x, w, x_out, xn_out must be non-NULL");
  if (T == 0) return RNB_OK;
  k_add_rmsnorm<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(w),
      static_cast<__nv_bfloat16*>(x_out), static_cast<__nv_bfloat16*>(xn_out), H, eps);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RNB_ERR_CUDA, std::string("rnb_add_rmsnorm launch: ") + cudaGetErrorString(e));
  return RNB_OK;
}
