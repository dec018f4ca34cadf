// The peer-memory expert-parallel exchange's per-CTA steps, shared by its own kernels (moek_ep.cu) and the
// whole-layer kernel (moek_layer.cu), which can run the dispatch in its prologue and the unpack in its epilogue so
// that an expert-parallel decode layer is one launch. The protocol is described in moek_ep.cu.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "moek_common.cuh"
#include "moek_kernels.cuh"

namespace moek {

__device__ __forceinline__ int* p2p_flags(const P2PArgs& q, int r) {
  return reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(q.peer[r]) + q.lay.flags);
}
// This rank's completed-call count ([2 world] of its counters) and the unpack's arrival counter ([2 world + 1]).
__device__ __forceinline__ int* p2p_call(const P2PArgs& q) {
  return reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(q.peer[q.rank]) + q.lay.ctr) + 2 * q.world;
}
__device__ __forceinline__ int current_call(const P2PArgs& q) {
  return *reinterpret_cast<volatile int*>(p2p_call(q)) + 1;
}
// The last of `n` arrivals on a self-resetting counter (one thread per CTA calls it, after its writes and a fence).
__device__ __forceinline__ bool last_arrival(int* ctr, int n) {
  if (n == 1) return true;
  if (atomicAdd(ctr, 1) != n - 1) return false;
  *ctr = 0;
  return true;
}

// Dispatch, CTA g of the G that serve destination d (all NT threads of the CTA): place my tokens in d's segment for
// me (ascending token order), write pos[t * world + d] (CTA 0 of d), copy rows g, g + G, ... with their slot ids and
// router weights, mark the unused rows; the last of the G CTAs fences and sets d's receive flag for me to `call`.
// spos: int[M], wcnt: int[NT / 32] of shared memory. RB rows are loaded before they are stored; thread 0 stamps trace
// slots TR0 (fenced) and TR0 + 1 (flag raised).
template <int NT, int RB, int TR0>
__device__ __forceinline__ void ep_dispatch_cta(const P2PArgs& q, const uint4* __restrict__ x,
                                                const int32_t* __restrict__ ids, const float* __restrict__ topk_w,
                                                int M, int E, int d, int g, int G, int call,
                                                int32_t* __restrict__ pos, int* spos, int* wcnt) {
  const int per = E / q.world, k = q.k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int* d_flags = p2p_flags(q, d);
  int count = 0;  // rows of mine that go to d
  for (int t0 = 0; t0 < M; t0 += NT) {
    const int t = t0 + tid;
    bool has = false;
    if (t < M)
      for (int j = 0; j < k; j++) {
        const int e = ids[(int64_t)t * k + j];
        has |= e >= 0 && e < E && e / per == d;
      }
    const uint32_t b = __ballot_sync(0xffffffffu, has);
    if (lane == 0) wcnt[warp] = __popc(b);
    __syncthreads();
    int before = count, chunk = 0;
    for (int w = 0; w < NT / 32; w++) {
      if (w < warp) before += wcnt[w];
      chunk += wcnt[w];
    }
    if (t < M) spos[t] = has ? before + __popc(b & ((1u << lane) - 1u)) : -1;
    count += chunk;
    __syncthreads();  // wcnt is rewritten by the next chunk
  }
  __syncthreads();  // spos (also when M is 0)
  if (g == 0)
    for (int t = tid; t < M; t += NT) pos[(int64_t)t * q.world + d] = spos[t];
  uint8_t* blk = reinterpret_cast<uint8_t*>(q.peer[d]);
  const int64_t row0 = (int64_t)q.rank * q.mcap;  // my segment in d's receive buffers
  const int H16 = q.H / 8;
  uint4* seg_x = reinterpret_cast<uint4*>(blk + q.lay.x) + row0 * H16;
  int32_t* seg_ids = reinterpret_cast<int32_t*>(blk + q.lay.ids) + row0 * k;
  float* seg_w = reinterpret_cast<float*>(blk + q.lay.w) + row0 * k;
  // rows in batches of RB tokens: all of a batch's loads are issued before its stores to the peer, so the copy costs
  // one load latency per batch, not one per token
  constexpr int PT = (EP_P2P_MAXH / 8 + NT - 1) / NT;
  for (int t0 = g; t0 < M; t0 += RB * G) {
    uint4 v[RB][PT];
#pragma unroll
    for (int b = 0; b < RB; b++) {
      const int t = t0 + b * G;
      if (t >= M || spos[t] < 0) continue;
#pragma unroll
      for (int j = 0; j < PT; j++) {
        const int c = tid + j * NT;
        if (c < H16) v[b][j] = x[(int64_t)t * H16 + c];
      }
    }
#pragma unroll
    for (int b = 0; b < RB; b++) {
      const int t = t0 + b * G;
      if (t >= M || spos[t] < 0) continue;
      const int p = spos[t];
#pragma unroll
      for (int j = 0; j < PT; j++) {
        const int c = tid + j * NT;
        if (c < H16) seg_x[(int64_t)p * H16 + c] = v[b][j];
      }
      if (tid < k) {
        const int e = ids[(int64_t)t * k + tid];
        const bool mine = e >= 0 && e < E && e / per == d;
        seg_ids[(int64_t)p * k + tid] = mine ? e - d * per : -1;
        seg_w[(int64_t)p * k + tid] = mine ? topk_w[(int64_t)t * k + tid] : 0.f;
      }
    }
  }
  for (int i = g * NT + tid; i < (q.mcap - count) * k; i += G * NT) {  // rows no token uses
    seg_ids[(int64_t)count * k + i] = -1;
    seg_w[(int64_t)count * k + i] = 0.f;
  }
  __syncthreads();
  if (tid == 0) {  // one system-scope fence (the CTA's stores to the peer are complete), then the release store
    MOEK_TR(TR0);
    __threadfence_system();
    int* ctr = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(q.peer[q.rank]) + q.lay.ctr) + d;
    if (last_arrival(ctr, G)) {
      st_sys(d_flags + q.rank, call);
      MOEK_TR(TR0 + 1);
    }
  }
}

// Unpack, CTA `cta` of `ncta` (all NT threads), once every owner's back flag for this rank reads `call`: out[t] =
// bf16(sum over owners d in rank order of my segment of d's back buffer, row pos[t][d]), elements cta, cta + ncta, ...
// of [M, H/4] float4; the caller advances the completed-call count once every CTA is done.
template <int NT>
__device__ __forceinline__ void ep_unpack_slice(const P2PArgs& q, const int32_t* __restrict__ pos, int M,
                                                __nv_bfloat16* __restrict__ out, int cta, int ncta) {
  const int H4 = q.H / 4;
  for (int64_t i = (int64_t)cta * NT + threadIdx.x; i < (int64_t)M * H4; i += (int64_t)ncta * NT) {
    const int64_t t = i / H4;
    const int c = (int)(i - t * H4);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d < q.world; d++) {
      const int p = __ldcg(pos + t * q.world + d);  // written in the same kernel when the layer kernel runs this
      if (p < 0) continue;
      // owner d's partial of my row p: my segment of d's back buffer, read over NVLink
      const float4* back = reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(q.peer[d]) + q.lay.back);
      const float4 v = __ldcg(back + ((int64_t)q.rank * q.mcap + p) * H4 + c);
      o.x += v.x;
      o.y += v.y;
      o.z += v.z;
      o.w += v.w;
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(o.x, o.y), hi = __floats2bfloat162_rn(o.z, o.w);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&lo);
    w.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(out)[i] = w;
  }
}

}  // namespace moek
