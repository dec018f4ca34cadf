// Load-time conversion of checkpoint NVFP4 experts into the kernels' formats, on the GPU (sm_100a): the work that
// the kit does with vLLM's Marlin repack and scale helpers plus its own Python codec (files/mbx_moek.py:61-172,
// vllm/.../marlin_utils_fp4.py:30-146,355-386), in five kernels per matrix:
//   scale_max_kernel     largest E4M3 block scale of the matrix (the shared power-of-two factor is chosen on the
//                        host from it, as vLLM's _nvfp4_compute_scale_factor does)
//   weights_kernel       codes uint8 [E, N, K/2] -> this build's tiled words int32 [E, K/16, 2N] (one thread per word:
//                        8 codes, each code's 4 bits moved to their CODE_BITS positions, halves swapped on rows with
//                        bit 2 set)
//   scales_kernel        one warp per block of 8 positions x 8 k-groups: the 64 Marlin S0E5M3 bytes (scale_perm,
//                        [0, 2, 1, 3] swap, x scale factor x 2^7 in fp16), the base (the value whose window
//                        [v, v + 15] holds the most values, the smallest such v), the nibbles into the item-tiled packed
//                        runs, the block's exception count
//   exc_scan_kernels     per (expert, item, run) list: the blocks' counts scanned into list offsets (exc_off)
//   exc_write_kernel     the exception entries (position | k-group << 16 | byte << 24) in list order
// The bytes are the torch restatement's in qwen38_flash_coder_b200/prep.py, which is bit-exact against the
// reference's own codec output; the test compares the two on the GPU.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "moek_kernels.cuh"

namespace moek {
namespace prep {

constexpr int KGR = 8;          // k-groups per packed run
constexpr int RUNB = 16 + KGR * 64;  // 528 packed bytes per (run of 8 k-groups, 128 positions)

// bit positions (m, e0, e1, sign) of code i of a tiled word (prep.py CODE_BITS)
__constant__ uint8_t c_code_bits[8][4] = {{6, 7, 8, 15},   {22, 23, 24, 31}, {10, 11, 12, 19}, {26, 27, 28, 3},
                                          {16, 17, 18, 25}, {0, 1, 2, 9},    {20, 13, 14, 21}, {4, 29, 30, 5}};

__global__ void scale_max_kernel(const uint8_t* s, int64_t n, unsigned int* out) {
  unsigned int m = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const unsigned int b = s[i];
    if (b < 0x7F) m = max(m, b);  // positive E4M3 patterns order as their values; negatives and NaN are no scale
  }
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m) atomicMax(out, m);
}

// Logical column of item slot r of item t (prep.item_columns)
__device__ __forceinline__ int item_column(int t, int r, int N, bool gate_up) {
  return gate_up ? (r < 128 ? 128 * t + r : N / 2 + 128 * t + r - 128) : 256 * t + r;
}

// out[e][(t * nst + s) * 2048 + r * 8 + slot]: word w = slot ^ (4 if bit 2 of r) of row r, k 64s + 8w .. + 7
__global__ void weights_kernel(const uint8_t* codes, int E, int N, int K, int gate_up, uint32_t* out) {
  const int64_t total = (int64_t)E * N * K / 8;
  const int nst = K / 64, nt = N / 256;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int slot = (int)(idx & 7), r = (int)((idx >> 3) & 255);
    const int64_t blk = idx >> 11;  // (e, t, s)
    const int s = (int)(blk % nst), t = (int)((blk / nst) % nt), e = (int)(blk / ((int64_t)nst * nt));
    const int w = slot ^ (((r >> 2) & 1) << 2);
    const int col = item_column(t, r, N, gate_up != 0);
    const uint32_t q = *reinterpret_cast<const uint32_t*>(codes + ((int64_t)e * N + col) * (K / 2) + 32 * s + 4 * w);
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint32_t code = (q >> (4 * i)) & 0xF;  // element 2j in the low nibble of byte j
#pragma unroll
      for (int b = 0; b < 4; b++) word |= ((code >> b) & 1u) << c_code_bits[i][b];
    }
    out[idx] = word;
  }
}

// The Marlin S0E5M3 byte of processed position p (within N), k-group kg, from E4M3 scales [E, N, K/16]: position
// q = p mod 64 holds column 8 j + i of its 64 where 8 i + j = 4 (q / 4) + [0, 2, 1, 3][q mod 4]; the value times the
// scale factor times 2^7 in fp16 (exact), zero below 2, then bits 7..14 of the fp16 pattern.
__device__ __forceinline__ uint32_t marlin_byte(const uint8_t* scales, int e, int N, int KG16, int p, int kg, float sf) {
  const int q = p & 63, perm = (q & 3) == 1 ? 2 : (q & 3) == 2 ? 1 : (q & 3), qq = (q & ~3) | perm;
  const int col = (p & ~63) + 8 * (qq & 7) + (qq >> 3);
  const uint32_t b = scales[((int64_t)e * N + col) * KG16 + kg];
  if (b & 0x80) return 0u;  // a negative scale is below 2: zero, as in the fp16 conversion
  const uint32_t ex = (b >> 3) & 15, m = b & 7;
  const float v = ex ? ldexpf(1.0f + m * 0.125f, (int)ex - 7) : ldexpf((float)m, -9);  // E4M3 (non-negative scales)
  const float h = v * sf * 128.0f;
  if (!(h >= 2.0f)) return 0u;
  return ((uint32_t)__half_as_ushort(__float2half_rn(h)) >> 7) & 0xFF;
}

// The list of block (e, b, ic): key = (e * nt + item) * nb + b, and the block's place j among the list's 32 chunks
__device__ __forceinline__ void block_key(int e, int b, int ic, int N, int nb, bool gate_up, int& key, int& j) {
  const int nt = N / 256, run = ic >> 4;
  int item;
  if (gate_up) {
    item = run % nt;
    j = (run < nt ? 0 : 16) + (ic & 15);
  } else {
    item = run >> 1;
    j = ((run & 1) << 4) + (ic & 15);
  }
  key = (e * nt + item) * nb + b;
}

// One warp per block (e, b, ic) of 8 positions x 8 k-groups: lane l holds value l (k-group l / 8, position l % 8)
// and value l + 32. Returns the two bytes and the block's base.
__device__ __forceinline__ void block_values(const uint8_t* scales, int e, int b, int ic, int N, int K, float sf,
                                             uint32_t& v0, uint32_t& v1, uint32_t& base) {
  const int lane = threadIdx.x & 31, KG16 = K / 16;
  v0 = marlin_byte(scales, e, N, KG16, ic * 8 + (lane & 7), b * KGR + (lane >> 3), sf);
  v1 = marlin_byte(scales, e, N, KG16, ic * 8 + (lane & 7), b * KGR + 4 + (lane >> 3), sf);
  // score of candidate v: (values in [v, v + 15]) * 256 + 255 - v; the base is the best candidate's value
  uint32_t c0 = 0, c1 = 0;
  for (int i = 0; i < 32; i++) {
    const uint32_t a = __shfl_sync(0xffffffffu, v0, i), a2 = __shfl_sync(0xffffffffu, v1, i);
    c0 += (a >= v0 && a <= v0 + 15) + (a2 >= v0 && a2 <= v0 + 15);
    c1 += (a >= v1 && a <= v1 + 15) + (a2 >= v1 && a2 <= v1 + 15);
  }
  uint32_t best = max(c0 * 256 + 255 - v0, c1 * 256 + 255 - v1);
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  base = 255 - (best & 255);
}

// Packed run bytes (into the item-tiled layout sp [E, N/256, nb, 1056]) and the exception count of every block.
__global__ void scales_kernel(const uint8_t* scales, int E, int N, int K, int gate_up, float sf, uint8_t* sp,
                              int* cnt) {
  const int nb = K / 128, nic = N / 8, nt = N / 256;
  const int64_t nblk = (int64_t)E * nb * nic;
  const int lane = threadIdx.x & 31;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < nblk;
       w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int ic = (int)(w % nic), b = (int)((w / nic) % nb), e = (int)(w / ((int64_t)nic * nb));
    uint32_t v0, v1, base;
    block_values(scales, e, b, ic, N, K, sf, v0, v1, base);
    const int o0 = (int)v0 - (int)base, o1 = (int)v1 - (int)base;
    const bool x0 = o0 < 0 || o0 > 15, x1 = o1 < 0 || o1 > 15;
    const uint32_t n0 = x0 ? 0u : (uint32_t)o0, n1 = x1 ? 0u : (uint32_t)o1;
    // the run's place in the tiled scales: item t, half h
    const int run = ic >> 4, t = gate_up ? (run < nt ? run : run - nt) : run >> 1;
    const int h = gate_up ? (run < nt ? 0 : 1) : (run & 1);
    uint8_t* dst = sp + (((int64_t)e * nt + t) * nb + b) * (2 * RUNB) + h * RUNB;
    // byte 16 + kg * 64 + chunk * 4 + j = nibble of position j | nibble of position j + 4 << 4: lane l (kg l / 8,
    // position l % 8) pairs with lane l + 4 (positions 0-3 take the low nibble)
    const uint32_t hi0 = __shfl_down_sync(0xffffffffu, n0, 4), hi1 = __shfl_down_sync(0xffffffffu, n1, 4);
    if ((lane & 7) < 4) {
      const int kg = lane >> 3, c16 = ic & 15, j = lane & 3;
      dst[16 + kg * 64 + c16 * 4 + j] = (uint8_t)(n0 | (hi0 << 4));
      dst[16 + (kg + 4) * 64 + c16 * 4 + j] = (uint8_t)(n1 | (hi1 << 4));
    }
    if (lane == 0) dst[ic & 15] = (uint8_t)base;
    const int nx = __popc(__ballot_sync(0xffffffffu, x0)) + __popc(__ballot_sync(0xffffffffu, x1));
    if (lane == 0) {
      int key, j;
      block_key(e, b, ic, N, nb, gate_up != 0, key, j);
      cnt[(int64_t)key * 32 + j] = nx;
    }
  }
}

// Per list (warp per key): the 32 blocks' counts -> their exclusive prefix (in place) and the list's total.
__global__ void exc_list_kernel(int* cnt, int nkeys, int* total) {
  const int lane = threadIdx.x & 31;
  for (int64_t k = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; k < nkeys;
       k += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int c = cnt[k * 32 + lane];
    int inc = c;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    cnt[k * 32 + lane] = inc - c;
    if (lane == 31) total[k] = inc;
  }
}

// exc_off[0] = 0, exc_off[k + 1] = sum of the totals of lists 0..k (one CTA of 1024 threads: per-thread runs, then a
// scan of the thread sums in shared memory).
__global__ void __launch_bounds__(1024) exc_offsets_kernel(const int* total, int nkeys, int* exc_off) {
  __shared__ int part[1024];
  const int per = (nkeys + 1023) / 1024, t = threadIdx.x, k0 = t * per;
  int s = 0;
  for (int k = k0; k < min(k0 + per, nkeys); k++) s += total[k];
  part[t] = s;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const int v = t >= o ? part[t - o] : 0;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  int run = part[t] - s;  // exclusive prefix of this thread's run
  if (t == 0) exc_off[0] = 0;
  for (int k = k0; k < min(k0 + per, nkeys); k++) {
    run += total[k];
    exc_off[k + 1] = run;
  }
}

// The entries: block (e, b, ic)'s exceptions at exc_off[key] + its prefix, in (k-group, position) order.
__global__ void exc_write_kernel(const uint8_t* scales, int E, int N, int K, int gate_up, float sf,
                                 const int* cnt_prefix, const int* exc_off, int* ent) {
  const int nb = K / 128, nic = N / 8;
  const int64_t nblk = (int64_t)E * nb * nic;
  const int lane = threadIdx.x & 31;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < nblk;
       w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int ic = (int)(w % nic), b = (int)((w / nic) % nb), e = (int)(w / ((int64_t)nic * nb));
    int key, j;
    block_key(e, b, ic, N, nb, gate_up != 0, key, j);
    if (exc_off[key + 1] == exc_off[key]) continue;  // an empty list (the common case): nothing to write
    uint32_t v0, v1, base;
    block_values(scales, e, b, ic, N, K, sf, v0, v1, base);
    const bool x0 = (int)v0 - (int)base < 0 || (int)v0 - (int)base > 15;
    const bool x1 = (int)v1 - (int)base < 0 || (int)v1 - (int)base > 15;
    const uint32_t m0 = __ballot_sync(0xffffffffu, x0), m1 = __ballot_sync(0xffffffffu, x1);
    const int at = exc_off[key] + cnt_prefix[(int64_t)key * 32 + j];
    const uint32_t below = (1u << lane) - 1u;
    const int pos = ic * 8 + (lane & 7);
    if (x0) ent[at + __popc(m0 & below)] = (int)((uint32_t)pos | ((uint32_t)(lane >> 3) << 16) | (v0 << 24));
    if (x1) ent[at + __popc(m0) + __popc(m1 & below)] =
        (int)((uint32_t)pos | ((uint32_t)((lane >> 3) + 4) << 16) | (v1 << 24));
  }
}

__global__ void global_scale_kernel(const float* gs, int E, float sf, float* g) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e < E) g[e] = (gs[e] * 0x1p119f) / sf;
}

}  // namespace prep

static int grid_for(int64_t work, int per_cta) {
  return (int)std::min<int64_t>((work + per_cta - 1) / per_cta, 148 * 16);
}

cudaError_t launch_prep_scale_max(const uint8_t* scales, int64_t n, unsigned int* out, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return e;
  prep::scale_max_kernel<<<grid_for(n, 256 * 16), 256, 0, st>>>(scales, n, out);
  return cudaGetLastError();
}

cudaError_t launch_prep_weights(const uint8_t* codes, int E, int N, int K, int gate_up, uint32_t* out,
                                cudaStream_t st) {
  const int64_t total = (int64_t)E * N * K / 8;
  prep::weights_kernel<<<grid_for(total, 256), 256, 0, st>>>(codes, E, N, K, gate_up, out);
  return cudaGetLastError();
}

cudaError_t launch_prep_scales(const uint8_t* scales, const float* gs, int E, int N, int K, int gate_up, float sf,
                               uint8_t* sp, float* g, int* cnt, int* total, int* exc_off, cudaStream_t st) {
  const int64_t nblk = (int64_t)E * (K / 128) * (N / 8);
  const int nkeys = E * (N / 256) * (K / 128);
  prep::scales_kernel<<<grid_for(nblk * 32, 256), 256, 0, st>>>(scales, E, N, K, gate_up, sf, sp, cnt);
  prep::exc_list_kernel<<<grid_for((int64_t)nkeys * 32, 256), 256, 0, st>>>(cnt, nkeys, total);
  prep::exc_offsets_kernel<<<1, 1024, 0, st>>>(total, nkeys, exc_off);
  prep::global_scale_kernel<<<(E + 255) / 256, 256, 0, st>>>(gs, E, sf, g);
  return cudaGetLastError();
}

cudaError_t launch_prep_exceptions(const uint8_t* scales, int E, int N, int K, int gate_up, float sf,
                                   const int* cnt_prefix, const int* exc_off, int* ent, cudaStream_t st) {
  const int64_t nblk = (int64_t)E * (K / 128) * (N / 8);
  prep::exc_write_kernel<<<grid_for(nblk * 32, 256), 256, 0, st>>>(scales, E, N, K, gate_up, sf, cnt_prefix,
                                                                   exc_off, ent);
  return cudaGetLastError();
}

}  // namespace moek
