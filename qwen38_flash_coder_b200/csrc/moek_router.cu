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

namespace moek {

constexpr int RT_WARPS = 8;
constexpr int RT_MAXE = 1024;  // experts per row (32 per lane)

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

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
  const T* row = logits + (int64_t)t * E;
  // expert e = 32 j + lane in register v[j]
  constexpr int PER = RT_MAXE / 32;
  float v[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; j++) {
    const int e = 32 * j + lane;
    v[j] = e < E ? to_f32(row[e]) : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < PER; j++) {
    v[j] = 32 * j + lane < E ? expf(v[j] - mx) : 0.f;
    sum += v[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
  for (int j = 0; j < PER; j++) v[j] = 32 * j + lane < E ? v[j] / sum : -1.f;  // taken / absent: -1
  float wsel = 0.f, wsum = 0.f;
  int esel = 0;
  for (int s = 0; s < k; s++) {
    // the lane's best (largest value, lowest expert on ties: j ascending visits experts in ascending order)
    float bv = -1.f;
    int be = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; j++)
      if (v[j] > bv) {
        bv = v[j];
        be = 32 * j + lane;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if (lane == s) {  // lane s keeps slot s
      wsel = bv;
      esel = be;
    }
    wsum += bv;
#pragma unroll
    for (int j = 0; j < PER; j++)  // remove the winner (a constant-index select keeps v in registers)
      if (32 * j + lane == be) v[j] = -1.f;
  }
  if (lane < k) {
    const int64_t o = (int64_t)t * k + lane;
    ids[o] = esel;
    weights[o] = renorm ? wsel / wsum : wsel;
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
