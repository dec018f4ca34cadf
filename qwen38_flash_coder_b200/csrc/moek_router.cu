// MoE router for sm_100a: softmax over the experts, top-k, optional renormalisation — the gating step in front of
// the routed-expert layer (vLLM's fused_topk with scoring "softmax", vllm/.../router/fused_topk_router.py:69-108,
// which the reference's model calls before its MoE layer, vllm/.../models/qwen3_next.py:158-165).
//
// One warp per token row: the row's E logits are read once (lane L reads experts L, L + 32, ...), the softmax is
// formed in fp32 (max, exp(x - max), sum, one IEEE division per value), then k rounds of a warp-wide argmax pick the
// experts: largest probability first, the lowest expert index among equal probabilities. The weights are the
// selected probabilities, divided by their sum when renormalising. Outputs per slot j of token t:
// ids[t*k + j], weights[t*k + j] and, when asked for, token_expert_indices[t*k + j] = j*M + t (the slot-major flat
// index vLLM returns beside them).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "moek_common.cuh"
#include "moek_kernels.cuh"
#include "moek_route.cuh"

namespace moek {

constexpr int RT_WARPS = 8;
constexpr int RT_MAXE = 1024;  // experts per row (32 per lane)

template <typename T>
__global__ void __launch_bounds__(RT_WARPS * 32) router_topk_kernel(const T* __restrict__ logits, int M, int E, int k,
                                                                    int renorm, int32_t* __restrict__ ids,
                                                                    float* __restrict__ weights,
                                                                    int32_t* __restrict__ tok_idx) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * RT_WARPS + (threadIdx.x >> 5);
  if (t >= M) return;
  int esel;
  float wsel;
  route_token<RT_MAXE / 32>(logits + (int64_t)t * E, E, k, renorm, esel, wsel);
  if (lane < k) {
    const int64_t o = (int64_t)t * k + lane;
    ids[o] = esel;
    weights[o] = wsel;
    if (tok_idx) tok_idx[o] = lane * M + t;
  }
}

cudaError_t launch_router_topk(const void* logits, int dtype, int M, int E, int k, int renorm, int32_t* ids,
                               float* weights, int32_t* tok_idx, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  const dim3 grid((M + RT_WARPS - 1) / RT_WARPS), block(RT_WARPS * 32);
  cudaError_t e;
  if (dtype == 0)
    e = launch_pdl(router_topk_kernel<float>, grid, block, 0, st, static_cast<const float*>(logits), M, E, k, renorm,
                   ids, weights, tok_idx);
  else
    e = launch_pdl(router_topk_kernel<__nv_bfloat16>, grid, block, 0, st,
                   static_cast<const __nv_bfloat16*>(logits), M, E, k, renorm, ids, weights, tok_idx);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace moek
