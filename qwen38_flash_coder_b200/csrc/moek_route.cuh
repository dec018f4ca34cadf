// The router's per-token step, shared by the router kernel (moek_router.cu) and the whole-layer kernel's fused
// routing prologue (moek_layer.cu), so that both give the same bits: softmax over the experts in fp32, top-k with the
// largest probability first and the lowest expert index among equal probabilities, weights renormalised by their sum
// when asked (vLLM's fused_topk with scoring "softmax", vllm/.../router/fused_topk_router.py:69-108).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace moek {

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

// One warp routes one token row of E <= 32 * PER logits: lane L reads experts L, L + 32, ...; after the call lane
// s < k holds slot s's expert (esel) and weight (wsel).
template <int PER, typename T>
__device__ __forceinline__ void route_token(const T* __restrict__ row, int E, int k, int renorm, int& esel,
                                            float& wsel) {
  const int lane = threadIdx.x & 31;
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
  float wsum = 0.f;
  wsel = 0.f;
  esel = 0;
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
  if (renorm) wsel = wsel / wsum;
}

}  // namespace moek
