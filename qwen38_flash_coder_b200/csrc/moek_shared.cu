// The decode-regime neighbours of the routed experts in the same MoE block, sm_100a: the router gate GEMM and the
// MXFP8 shared expert (vllm/model_executor/models/qwen3_next.py:125-204, the block the kit's model subclasses at
// files/v54/model.py:193-210; the shared expert is vllm/model_executor/models/qwen2_moe.py:114-122's MLP with its
// sigmoid expert gate, MXFP8 in the kit's checkpoint, README.md:38).
//
// Both are weight-streaming GEMMs at decode sizes (M <= 64 tokens): the gate reads E x H bf16 (2 MB at E = 512,
// H = 2048), the shared expert 3 x Is x H e4m3 bytes plus one E8M0 scale per 32 (3.1 MB at Is = 512). So each CTA owns
// 16 weight rows (the 16-row A operand of mma.sync m16n8k16, tokens as the 8-column B operand), its eight warps split
// K, and the warps' fp32 partials are added in warp order in shared memory, so every call gives the same bits.
//
// MXFP8 dequantisation is exact: the e4m3 byte's exponent and mantissa bits placed at bf16 bits 4-10 (sign at 15)
// are the bf16 value e4m3 x 2^-120 (normal and subnormal e4m3 alike), and one bf16 multiply by 2^(s - 7) (the E8M0
// scale s, bf16 exponent field s + 120) gives e4m3 x 2^(s - 127) with no rounding for scales 10 <= s <= 134 (every
// product a normal bf16).
//
// Kernels (one launch each, chained with programmatic dependent launch):
//   router_gate_kernel      logits fp32 [M, E] = x @ W_gate^T
//   shared_gate_up_kernel   act bf16 [M, Is] = bf16(silu(x @ Wg^T) * (x @ Wu^T)) for 16 act columns per CTA, and
//                           (CTA 0) the expert gate sg fp32 [M] = sigmoid(x @ w_sg)
//   shared_down_kernel      rows fp32 [M, H] = sg * (act @ Wd^T) for 16 output columns per CTA
// The routed layer adds the rows to each token's fp32 sum before its one bf16 rounding (moek_layer.cu).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "moek_common.cuh"
#include "moek_kernels.cuh"

namespace moek {
namespace sh {

constexpr int NW = 8;            // warps per CTA, each a K slice
constexpr int THREADS = NW * 32;
constexpr int MAXT = SHARED_MAXM / 8;  // token tiles of 8

__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two e4m3 bytes (low byte = lower k) -> bf16x2 of e4m3 x 2^-120 (see the file comment).
__device__ __forceinline__ uint32_t e4m3x2_pattern(uint32_t two) {
  uint32_t t;
  asm("prmt.b32 %0, %1, 0, 0x4140;" : "=r"(t) : "r"(two));  // bytes [b0, 0, b1, 0]
  return ((t & 0x007F007Fu) << 4) | ((t & 0x00800080u) << 8);
}
// bf16x2 of 2^(s - 7) for an E8M0 scale byte s in [10, 134]
__device__ __forceinline__ uint32_t e8m0_factor2(uint32_t s) {
  const uint32_t h = (s + 120u) << 7;
  return h | (h << 16);
}

// B fragment of token tile t (tokens 8t .. 8t+7 = column g of the tile) at k: two bf16 pairs of x row 8t + g, zero
// for rows past M.
__device__ __forceinline__ void b_frag(const __nv_bfloat16* x, int M, int ld, int row, int k, uint32_t& b0,
                                       uint32_t& b1) {
  if (row < M) {
    const __nv_bfloat16* p = x + (int64_t)row * ld + k;
    b0 = *reinterpret_cast<const uint32_t*>(p);
    b1 = *reinterpret_cast<const uint32_t*>(p + 8);
  } else {
    b0 = b1 = 0u;
  }
}

// The eight warps' accumulators of one 16-row tile, red[warp][16][SHARED_MAXM], are added in warp order; f(row, token,
// v) consumes each sum. acc[t][i]: i = 0, 1 row g, tokens 8t + 2c, + 1; i = 2, 3 row g + 8.
template <class F>
__device__ __forceinline__ void reduce_tile(float (*acc)[4], float* red, int ntile, int M, F f) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int t = 0; t < MAXT; t++)  // unrolled with a test, so that acc stays in registers
    if (t < ntile)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int row = g + 8 * (i >> 1), tok = 8 * t + 2 * c + (i & 1);
        red[(warp * 16 + row) * SHARED_MAXM + tok] = acc[t][i];
      }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 16 * M; idx += THREADS) {
    const int row = idx / M, tok = idx - row * M;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NW; w++) s += red[(w * 16 + row) * SHARED_MAXM + tok];
    f(row, tok, s);
  }
  __syncthreads();
}

// logits[t][e] = sum_h x[t][h] * Wg[e][h]: CTA = 16 experts, warp w = K slice [w H / 8, (w + 1) H / 8).
__global__ void __launch_bounds__(THREADS) router_gate_kernel(const __nv_bfloat16* x, int M, int H,
                                                              const __nv_bfloat16* wg, int E, float* logits) {
  __shared__ float red[NW * 16 * SHARED_MAXM];
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int e0 = blockIdx.x * 16, ntile = (M + 7) >> 3, ks = H / NW;
  float acc[MAXT][4];
#pragma unroll
  for (int t = 0; t < MAXT; t++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[t][i] = 0.f;
  const __nv_bfloat16* r0 = wg + (int64_t)(e0 + g) * H;
  const __nv_bfloat16* r1 = r0 + 8 * (int64_t)H;
  for (int k = warp * ks; k < (warp + 1) * ks; k += 16) {
    const int kk = k + 2 * c;
    const uint32_t a[4] = {*reinterpret_cast<const uint32_t*>(r0 + kk), *reinterpret_cast<const uint32_t*>(r1 + kk),
                           *reinterpret_cast<const uint32_t*>(r0 + kk + 8),
                           *reinterpret_cast<const uint32_t*>(r1 + kk + 8)};
#pragma unroll
    for (int t = 0; t < MAXT; t++) {
      if (t < ntile) {
        uint32_t b0, b1;
        b_frag(x, M, H, 8 * t + g, kk, b0, b1);
        mma_16816(acc[t], a, b0, b1);
      }
    }
  }
  reduce_tile(acc, red, ntile, M, [&](int row, int tok, float s) { logits[(int64_t)tok * E + e0 + row] = s; });
}

// A fragment of 16 MXFP8 rows (r0 = row g, r1 = row g + 8, each row H bytes) at k, scaled: the bf16 weights.
__device__ __forceinline__ void a_frag_mx(const uint8_t* r0, const uint8_t* r1, int kk, uint32_t f0, uint32_t f1,
                                          uint32_t* a) {
  const uint32_t q0 = *reinterpret_cast<const uint16_t*>(r0 + kk), q1 = *reinterpret_cast<const uint16_t*>(r1 + kk);
  const uint32_t q2 = *reinterpret_cast<const uint16_t*>(r0 + kk + 8);
  const uint32_t q3 = *reinterpret_cast<const uint16_t*>(r1 + kk + 8);
  a[0] = bf2_mul(e4m3x2_pattern(q0), f0);
  a[1] = bf2_mul(e4m3x2_pattern(q1), f1);
  a[2] = bf2_mul(e4m3x2_pattern(q2), f0);
  a[3] = bf2_mul(e4m3x2_pattern(q3), f1);
}

// act[t][16 b + j] = bf16(silu(gate) * up) for gate row 16 b + j and up row Is + 16 b + j; CTA 0 also sg[t].
__global__ void __launch_bounds__(THREADS) shared_gate_up_kernel(const __nv_bfloat16* x, int M, int H, int Is,
                                                                 const uint8_t* wgu, const uint8_t* sgu,
                                                                 const __nv_bfloat16* wsg, __nv_bfloat16* act,
                                                                 float* sg) {
  __shared__ float red[NW * 16 * SHARED_MAXM];
  __shared__ float gsum[16 * SHARED_MAXM];
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int b = blockIdx.x, ntile = (M + 7) >> 3, ks = H / NW, nsc = H / 32;
  float accg[MAXT][4], accu[MAXT][4];
#pragma unroll
  for (int t = 0; t < MAXT; t++)
#pragma unroll
    for (int i = 0; i < 4; i++) accg[t][i] = accu[t][i] = 0.f;
  const int rg = 16 * b + g, ru = Is + 16 * b + g;  // this lane's gate and up rows (and + 8)
  for (int k = warp * ks; k < (warp + 1) * ks; k += 16) {
    const int kk = k + 2 * c, sb = k >> 5;
    uint32_t ag[4], au[4];
    a_frag_mx(wgu + (int64_t)rg * H, wgu + (int64_t)(rg + 8) * H, kk, e8m0_factor2(sgu[(int64_t)rg * nsc + sb]),
              e8m0_factor2(sgu[(int64_t)(rg + 8) * nsc + sb]), ag);
    a_frag_mx(wgu + (int64_t)ru * H, wgu + (int64_t)(ru + 8) * H, kk, e8m0_factor2(sgu[(int64_t)ru * nsc + sb]),
              e8m0_factor2(sgu[(int64_t)(ru + 8) * nsc + sb]), au);
#pragma unroll
    for (int t = 0; t < MAXT; t++) {
      if (t < ntile) {
        uint32_t b0, b1;
        b_frag(x, M, H, 8 * t + g, kk, b0, b1);
        mma_16816(accg[t], ag, b0, b1);
        mma_16816(accu[t], au, b0, b1);
      }
    }
  }
  reduce_tile(accg, red, ntile, M, [&](int row, int tok, float s) { gsum[row * SHARED_MAXM + tok] = s; });
  __syncthreads();
  reduce_tile(accu, red, ntile, M, [&](int row, int tok, float u) {
    act[(int64_t)tok * Is + 16 * b + row] = __float2bfloat16_rn(silu(gsum[row * SHARED_MAXM + tok]) * u);
  });
  if (b == 0) {  // the shared expert's gate: one warp per token, lanes over h, a fixed shuffle order
    for (int t = warp; t < M; t += NW) {
      float s = 0.f;
      for (int h = lane; h < H; h += 32)
        s += __bfloat162float(x[(int64_t)t * H + h]) * __bfloat162float(wsg[h]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) sg[t] = 1.0f / (1.0f + expf(-s));
    }
  }
}

// rows[t][16 b + j] = sg[t] * sum_i act[t][i] * Wd[16 b + j][i]
__global__ void __launch_bounds__(THREADS) shared_down_kernel(const __nv_bfloat16* act, int M, int H, int Is,
                                                              const uint8_t* wd, const uint8_t* sd, const float* sg,
                                                              float* rows) {
  __shared__ float red[NW * 16 * SHARED_MAXM];
  pdl_wait();  // act and sg of the gate_up kernel
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int b = blockIdx.x, ntile = (M + 7) >> 3, ks = Is / NW, nsc = Is / 32;
  float acc[MAXT][4];
#pragma unroll
  for (int t = 0; t < MAXT; t++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[t][i] = 0.f;
  const int r = 16 * b + g;
  for (int k = warp * ks; k < (warp + 1) * ks; k += 16) {
    const int kk = k + 2 * c, sb = k >> 5;
    uint32_t a[4];
    a_frag_mx(wd + (int64_t)r * Is, wd + (int64_t)(r + 8) * Is, kk, e8m0_factor2(sd[(int64_t)r * nsc + sb]),
              e8m0_factor2(sd[(int64_t)(r + 8) * nsc + sb]), a);
#pragma unroll
    for (int t = 0; t < MAXT; t++) {
      if (t < ntile) {
        uint32_t b0, b1;
        b_frag(act, M, Is, 8 * t + g, kk, b0, b1);
        mma_16816(acc[t], a, b0, b1);
      }
    }
  }
  reduce_tile(acc, red, ntile, M, [&](int row, int tok, float s) {
    rows[(int64_t)tok * H + 16 * b + row] = __fmul_rn(sg[tok], s);
  });
}

}  // namespace sh

cudaError_t launch_router_gate(const __nv_bfloat16* x, int M, int H, const __nv_bfloat16* wg, int E, float* logits,
                               cudaStream_t st) {
  return launch_pdl(sh::router_gate_kernel, dim3(E / 16), dim3(sh::THREADS), 0, st, x, M, H, wg, E, logits);
}

cudaError_t launch_shared_expert(const __nv_bfloat16* x, int M, int H, int Is, const uint8_t* wgu, const uint8_t* sgu,
                                 const uint8_t* wd, const uint8_t* sd, const __nv_bfloat16* wsg, __nv_bfloat16* act,
                                 float* sg, float* rows, cudaStream_t st) {
  cudaError_t e = launch_pdl(sh::shared_gate_up_kernel, dim3(Is / 16), dim3(sh::THREADS), 0, st, x, M, H, Is, wgu, sgu,
                             wsg, act, sg);
  if (e != cudaSuccess) return e;
  return launch_pdl(sh::shared_down_kernel, dim3(H / 16), dim3(sh::THREADS), 0, st, static_cast<const __nv_bfloat16*>(act),
                    M, H, Is, wd, sd, static_cast<const float*>(sg), rows);
}

}  // namespace moek
