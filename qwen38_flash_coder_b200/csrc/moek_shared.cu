// The decode-regime neighbours of the routed experts in the same MoE block, sm_100a: the router gate GEMM and the
// MXFP8 shared expert (vllm/model_executor/models/qwen3_next.py:125-204, the block the kit's model subclasses at
// files/v54/model.py:193-210; the shared expert is vllm/model_executor/models/qwen2_moe.py:114-122's MLP with its
// sigmoid expert gate, MXFP8 in the kit's checkpoint, README.md:38).
//
// Both are weight-streaming GEMMs at decode sizes (M <= 64 tokens): the gate reads E x H bf16 (2 MB at E = 512,
// H = 2048), the shared expert 3 x Is x H e4m3 bytes plus one E8M0 scale per 32 (3.1 MB at Is = 512). Each CTA owns
// 16 weight rows (the 16-row A operand of mma.sync m16n8k16, tokens as the 8-column B operand): one thread brings the
// rows (and their scale rows) into shared memory with bulk copies on one mbarrier (bounded wait), rows padded by 16
// bytes so that the fragment reads are free of bank conflicts; its eight warps split K, and their fp32 partials are
// added in warp order, so every call gives the same bits.
//
// MXFP8 dequantisation is exact: the e4m3 byte's exponent and mantissa bits placed at bf16 bits 4-10 (sign at 15)
// are the bf16 value e4m3 x 2^-120 (normal and subnormal e4m3 alike), and one bf16 multiply by 2^(s - 7) (the E8M0
// scale s, bf16 exponent field s + 120) gives e4m3 x 2^(s - 127) with no rounding for scales 10 <= s <= 134 (every
// product a normal bf16).
//
// Kernels (one launch each, chained with programmatic dependent launch):
//   router_gate_kernel      logits fp32 [M, E] = x @ W_gate^T, 16 experts per CTA
//   shared_gate_up_kernel   act bf16 [M, Is] = bf16(silu(x @ Wg^T) * (x @ Wu^T)) for 8 act columns per CTA (its 16
//                           rows: 8 gate rows then their 8 up rows), and (CTA 0) the expert gate sg fp32 [M] =
//                           sigmoid(x @ w_sg)
//   shared_down_kernel      rows fp32 [M, H] = sg * (act @ Wd^T) for 16 output columns per CTA
// The routed layer adds the rows to each token's fp32 sum before its one bf16 rounding (moek_layer.cu).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "moek_common.cuh"
#include "moek_kernels.cuh"
#include "moek_route.cuh"

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

// Bring 16 weight rows of `bytes` bytes (row r from src + row_of[r] * bytes) into shared memory, dst_pitch apart, and,
// when sdst, their scale rows of `sbytes` bytes as two runs of 8 consecutive rows (from ssrc + row_of[0] * sbytes and
// ssrc + row_of[8] * sbytes; rows 0-7 and 8-15 are consecutive in the source) to sdst, sbytes apart; then wait
// (bounded) until everything landed. Sizes and addresses are multiples of 16 bytes (the callers' H, Is % 128 == 0).
__device__ __forceinline__ bool load_rows(uint8_t* dst, int dst_pitch, const uint8_t* src, int bytes, const int* row_of,
                                          uint8_t* sdst, const uint8_t* ssrc, int sbytes, uint64_t* bar,
                                          uint64_t timeout_ns, int* err) {
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_expect_tx(bar, 16 * bytes + (sdst ? 16 * sbytes : 0));
    for (int r = 0; r < 16; r++) bulk_g2s(dst + r * dst_pitch, src + (int64_t)row_of[r] * bytes, bytes, bar);
    if (sdst) {
      bulk_g2s(sdst, ssrc + (int64_t)row_of[0] * sbytes, 8 * sbytes, bar);
      bulk_g2s(sdst + 8 * sbytes, ssrc + (int64_t)row_of[8] * sbytes, 8 * sbytes, bar);
    }
  }
  return mbar_wait(bar, 0, globaltimer() + timeout_ns, err);
}

// shared memory of the kernels below besides the dynamic weight rows
struct Smem {
  float red[NW * 16 * SHARED_MAXM];
  uint64_t bar;
  int row_of[16];
};

// logits[t][e] = sum_h x[t][h] * Wg[e][h]: CTA cta = 16 experts, warp w = K slice [w H / 8, (w + 1) H / 8).
__device__ __forceinline__ void router_gate_cta(uint8_t* smem, Smem& S, int cta, const __nv_bfloat16* x, int M, int H,
                                                const __nv_bfloat16* wg, int E, float* logits, uint64_t timeout_ns,
                                                int* err) {
  float* red = S.red;
  uint64_t& bar = S.bar;
  int* row_of = S.row_of;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int e0 = cta * 16, ntile = (M + 7) >> 3, ks = H / NW, pitch = H * 2 + 16;
  if (threadIdx.x < 16) row_of[threadIdx.x] = e0 + threadIdx.x;
  // the weights do not depend on the kernel before: they stream in while it finishes; x may come from it
  const bool ok = load_rows(smem, pitch, reinterpret_cast<const uint8_t*>(wg), H * 2, row_of, nullptr, nullptr, 0,
                            &bar, timeout_ns, err);
  pdl_wait();
  pdl_launch_dependents();
  float acc[MAXT][4];
#pragma unroll
  for (int t = 0; t < MAXT; t++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[t][i] = 0.f;
  if (ok) {
    const uint8_t* r0 = smem + g * pitch;
    const uint8_t* r1 = r0 + 8 * pitch;
#pragma unroll 2
    for (int k = warp * ks; k < (warp + 1) * ks; k += 16) {
      const int kb = 2 * (k + 2 * c);
      const uint32_t a[4] = {*reinterpret_cast<const uint32_t*>(r0 + kb), *reinterpret_cast<const uint32_t*>(r1 + kb),
                             *reinterpret_cast<const uint32_t*>(r0 + kb + 16),
                             *reinterpret_cast<const uint32_t*>(r1 + kb + 16)};
#pragma unroll
      for (int t = 0; t < MAXT; t++) {
        if (t < ntile) {
          uint32_t b0, b1;
          b_frag(x, M, H, 8 * t + g, k + 2 * c, b0, b1);
          mma_16816(acc[t], a, b0, b1);
        }
      }
    }
  }
  reduce_tile(acc, red, ntile, M, [&](int row, int tok, float s) { logits[(int64_t)tok * E + e0 + row] = s; });
}

// A fragment of 16 MXFP8 rows in shared memory (r0 = row g, r1 = row g + 8) at byte kk, scaled: the bf16 weights.
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

// The shared expert's 16-row MXFP8 GEMM of one CTA: acc[t] += W[rows] . B[tokens], W rows and scale rows in shared
// memory (pitch bytes apart; scale rows K / 32 bytes apart), B = bf16 [M, K] in global memory, warp = K slice.
__device__ __forceinline__ void mx_gemm(const uint8_t* w, int pitch, const uint8_t* sc, const __nv_bfloat16* B, int M,
                                        int K, int ntile, float (*acc)[4]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3, ks = K / NW, nsc = K / 32;
  const uint8_t* r0 = w + g * pitch;
  const uint8_t* r1 = r0 + 8 * pitch;
#pragma unroll 2
  for (int k = warp * ks; k < (warp + 1) * ks; k += 16) {
    const int kk = k + 2 * c;
    uint32_t a[4];
    a_frag_mx(r0, r1, kk, e8m0_factor2(sc[g * nsc + (k >> 5)]), e8m0_factor2(sc[(g + 8) * nsc + (k >> 5)]), a);
#pragma unroll
    for (int t = 0; t < MAXT; t++) {
      if (t < ntile) {
        uint32_t b0, b1;
        b_frag(B, M, K, 8 * t + g, kk, b0, b1);
        mma_16816(acc[t], a, b0, b1);
      }
    }
  }
}

// act[t][8 b + j] = bf16(silu(gate row 8 b + j) * (up row Is + 8 b + j)); CTA b = 0 also sg[t].
__device__ __forceinline__ void shared_gate_up_cta(uint8_t* smem, Smem& S, int b, const __nv_bfloat16* x, int M, int H,
                                                   int Is, const uint8_t* wgu, const uint8_t* sgu,
                                                   const __nv_bfloat16* wsg, __nv_bfloat16* act, float* sg,
                                                   uint64_t timeout_ns, int* err) {
  float* red = S.red;
  uint64_t& bar = S.bar;
  int* row_of = S.row_of;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ntile = (M + 7) >> 3, pitch = H + 16;
  if (threadIdx.x < 16) row_of[threadIdx.x] = threadIdx.x < 8 ? 8 * b + threadIdx.x : Is + 8 * b + threadIdx.x - 8;
  uint8_t* sc = smem + 16 * pitch;
  const bool ok = load_rows(smem, pitch, wgu, H, row_of, sc, sgu, H / 32, &bar, timeout_ns, err);
  pdl_wait();  // x may come from the kernel before
  pdl_launch_dependents();
  float acc[MAXT][4];
#pragma unroll
  for (int t = 0; t < MAXT; t++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[t][i] = 0.f;
  if (ok) mx_gemm(smem, pitch, sc, x, M, H, ntile, acc);
  // tile rows 0-7 are the gate rows of act columns 8b..8b+7, rows 8-15 their up rows
  float* gsum = reinterpret_cast<float*>(smem);  // the weights are read: reuse their space for the gate sums
  __syncthreads();
  reduce_tile(acc, red, ntile, M, [&](int row, int tok, float s) { gsum[row * SHARED_MAXM + tok] = s; });
  for (int idx = threadIdx.x; idx < 8 * M; idx += THREADS) {
    const int j = idx / M, tok = idx - j * M;
    const float gt = gsum[j * SHARED_MAXM + tok], up = gsum[(j + 8) * SHARED_MAXM + tok];
    act[(int64_t)tok * Is + 8 * b + j] = __float2bfloat16_rn(silu(gt) * up);
  }
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
__device__ __forceinline__ void shared_down_cta(uint8_t* smem, Smem& S, int b, const __nv_bfloat16* act, int M, int H,
                                                int Is, const uint8_t* wd, const uint8_t* sd, const float* sg,
                                                float* rows, uint64_t timeout_ns, int* err) {
  float* red = S.red;
  uint64_t& bar = S.bar;
  int* row_of = S.row_of;
  const int ntile = (M + 7) >> 3, pitch = Is + 16;
  if (threadIdx.x < 16) row_of[threadIdx.x] = 16 * b + threadIdx.x;
  uint8_t* sc = smem + 16 * pitch;
  // the weights do not depend on the kernel before: they are in flight while it finishes
  const bool ok = load_rows(smem, pitch, wd, Is, row_of, sc, sd, Is / 32, &bar, timeout_ns, err);
  pdl_wait();  // act and sg of the gate_up kernel
  pdl_launch_dependents();
  float acc[MAXT][4];
#pragma unroll
  for (int t = 0; t < MAXT; t++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[t][i] = 0.f;
  if (ok) mx_gemm(smem, pitch, sc, act, M, Is, ntile, acc);
  reduce_tile(acc, red, ntile, M, [&](int row, int tok, float s) {
    rows[(int64_t)tok * H + 16 * b + row] = __fmul_rn(sg[tok], s);
  });
}

__global__ void __launch_bounds__(THREADS) router_gate_kernel(const __nv_bfloat16* x, int M, int H,
                                                              const __nv_bfloat16* wg, int E, float* logits,
                                                              uint64_t timeout_ns, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ Smem S;
  router_gate_cta(smem, S, blockIdx.x, x, M, H, wg, E, logits, timeout_ns, err);
}
__global__ void __launch_bounds__(THREADS) shared_gate_up_kernel(const __nv_bfloat16* x, int M, int H, int Is,
                                                                 const uint8_t* wgu, const uint8_t* sgu,
                                                                 const __nv_bfloat16* wsg, __nv_bfloat16* act,
                                                                 float* sg, uint64_t timeout_ns, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ Smem S;
  shared_gate_up_cta(smem, S, blockIdx.x, x, M, H, Is, wgu, sgu, wsg, act, sg, timeout_ns, err);
}
__global__ void __launch_bounds__(THREADS) shared_down_kernel(const __nv_bfloat16* act, int M, int H, int Is,
                                                              const uint8_t* wd, const uint8_t* sd, const float* sg,
                                                              float* rows, uint64_t timeout_ns, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ Smem S;
  shared_down_cta(smem, S, blockIdx.x, act, M, H, Is, wd, sd, sg, rows, timeout_ns, err);
}

// The MoE block's two kernels before the whole-layer kernel (moek_moe_block): the router gate and the shared
// expert's gate_up share one grid (CTAs [0, E / 16) the gate, the rest the gate_up); then the shared expert's down and
// the routing of the logits (softmax, top-k, renormalised: the router kernel's per-token code, one warp per token, in
// the grid's last CTA), so that the layer kernel reads ids and weights.
__global__ void __launch_bounds__(THREADS) block_pre_kernel(const __nv_bfloat16* x, int M, int H, int E, int Is,
                                                            const __nv_bfloat16* wg, float* logits, const uint8_t* wgu,
                                                            const uint8_t* sgu, const __nv_bfloat16* wsg,
                                                            __nv_bfloat16* act, float* sg, uint64_t timeout_ns,
                                                            int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ Smem S;
  const int ng = E / 16;
  if ((int)blockIdx.x < ng)
    router_gate_cta(smem, S, blockIdx.x, x, M, H, wg, E, logits, timeout_ns, err);
  else
    shared_gate_up_cta(smem, S, blockIdx.x - ng, x, M, H, Is, wgu, sgu, wsg, act, sg, timeout_ns, err);
}
__global__ void __launch_bounds__(THREADS) block_post_kernel(const __nv_bfloat16* act, int M, int H, int E, int Is,
                                                             const uint8_t* wd, const uint8_t* sd, const float* sg,
                                                             float* rows, const float* logits, int k, int renorm,
                                                             int32_t* ids, float* w, uint64_t timeout_ns, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ Smem S;
  const int nd = Is > 0 ? H / 16 : 0;
  if ((int)blockIdx.x < nd) {
    shared_down_cta(smem, S, blockIdx.x, act, M, H, Is, wd, sd, sg, rows, timeout_ns, err);
  } else {
    pdl_wait();  // the logits of the kernel before
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    for (int t = threadIdx.x >> 5; t < M; t += NW) {
      int es;
      float ws;
      route_token<16>(logits + (int64_t)t * E, E, k, renorm, es, ws);
      if (lane < k) {
        ids[t * k + lane] = es;
        w[t * k + lane] = ws;
      }
    }
  }
}

}  // namespace sh

cudaError_t launch_router_gate(const __nv_bfloat16* x, int M, int H, const __nv_bfloat16* wg, int E, float* logits,
                               uint64_t timeout_ns, int* err, cudaStream_t st) {
  const int smem = 16 * (H * 2 + 16);
  cudaError_t e = cudaFuncSetAttribute(sh::router_gate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(sh::router_gate_kernel, dim3(E / 16), dim3(sh::THREADS), smem, st, x, M, H, wg, E, logits,
                    timeout_ns, err);
}

cudaError_t launch_block_pre_post(const __nv_bfloat16* x, int M, int H, int E, int Is, const __nv_bfloat16* wg,
                                  float* logits, const uint8_t* wgu, const uint8_t* sgu, const uint8_t* wd,
                                  const uint8_t* sd, const __nv_bfloat16* wsg, __nv_bfloat16* act, float* sg,
                                  float* rows, int k, int renorm, int32_t* ids, float* w, uint64_t timeout_ns, int* err,
                                  cudaStream_t st) {
  const int smem1 = std::max(16 * (H * 2 + 16), Is > 0 ? 16 * (H + 16) + 16 * (H / 32) : 0);
  const int smem2 = Is > 0 ? 16 * (Is + 16) + 16 * (Is / 32) : 0;
  cudaError_t e = cudaFuncSetAttribute(sh::block_pre_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(sh::block_post_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2);
  if (e != cudaSuccess) return e;
  e = launch_pdl(sh::block_pre_kernel, dim3(E / 16 + (Is > 0 ? Is / 8 : 0)), dim3(sh::THREADS), smem1, st, x, M, H,
                 E, Is, wg, logits, wgu, sgu, wsg, act, sg, timeout_ns, err);
  if (e != cudaSuccess) return e;
  return launch_pdl(sh::block_post_kernel, dim3((Is > 0 ? H / 16 : 0) + 1), dim3(sh::THREADS), smem2, st,
                    static_cast<const __nv_bfloat16*>(act), M, H, E, Is, wd, sd, static_cast<const float*>(sg), rows,
                    static_cast<const float*>(logits), k, renorm, ids, w, timeout_ns, err);
}

cudaError_t launch_shared_expert(const __nv_bfloat16* x, int M, int H, int Is, const uint8_t* wgu, const uint8_t* sgu,
                                 const uint8_t* wd, const uint8_t* sd, const __nv_bfloat16* wsg, __nv_bfloat16* act,
                                 float* sg, float* rows, uint64_t timeout_ns, int* err, cudaStream_t st) {
  const int smem1 = 16 * (H + 16) + 16 * (H / 32), smem2 = 16 * (Is + 16) + 16 * (Is / 32);
  cudaError_t e = cudaFuncSetAttribute(sh::shared_gate_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(sh::shared_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2);
  if (e != cudaSuccess) return e;
  e = launch_pdl(sh::shared_gate_up_kernel, dim3(Is / 8), dim3(sh::THREADS), smem1, st, x, M, H, Is, wgu, sgu, wsg, act,
                 sg, timeout_ns, err);
  if (e != cudaSuccess) return e;
  return launch_pdl(sh::shared_down_kernel, dim3(H / 16), dim3(sh::THREADS), smem2, st,
                    static_cast<const __nv_bfloat16*>(act), M, H, Is, wd, sd, static_cast<const float*>(sg), rows,
                    timeout_ns, err);
}

}  // namespace moek
