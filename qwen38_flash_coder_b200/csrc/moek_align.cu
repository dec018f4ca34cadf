// moe_align on sm_100a: group the flat (token, slot) indices by expert, ascending inside an expert, each expert padded
// to a multiple of block_size with the sentinel numel (the contract of vLLM's moe_align_block_size,
// vllm/model_executor/layers/fused_moe/moe_align_block_size.py:11-103, as the kit calls it at files/mbx_moek.py:266
// with ignore_invalid_experts=True: ids outside [0, E) are skipped).
//
// Tiles of 1024 indices. Inside a tile the stable rank of index i among equal experts comes from warp match masks
// (rank inside the warp) plus a [32 warps x E] table of per-warp counts scanned down each expert's column (rank of
// the warp). One tile (numel <= 1024, every decode batch) is handled start to finish by one CTA; more tiles take
// three launches: per-tile counts and ranks, one CTA for the expert and tile offsets, then the scatter.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "moek_common.cuh"
#include "moek_kernels.cuh"

namespace moek {

constexpr int AT = 1024;  // indices per tile = threads per CTA

// Stable in-tile ranks. tab: [32][E] shared ints (zeroed here). Returns this thread's expert (or -1) and rank;
// afterwards tab[w][e] holds the number of expert-e indices in warps before w, and tot[e] the tile's count.
__device__ __forceinline__ void tile_ranks(const int32_t* ids, int64_t numel, int64_t i0, int E, int* tab, int* tot,
                                           int& e_out, int& r_out) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  for (int j = t; j < 32 * E; j += AT) tab[j] = 0;
  __syncthreads();
  const int64_t i = i0 + t;
  int e = i < numel ? ids[i] : -1;
  if (e >= E) e = -1;
  const unsigned same = __match_any_sync(0xffffffffu, e);
  const int rw = __popc(same & ((1u << lane) - 1));
  if (e >= 0 && rw == 0) tab[w * E + e] = __popc(same);  // the group's first lane publishes its size
  __syncthreads();
  for (int x = t; x < E; x += AT) {  // exclusive scan down each expert's column
    int s = 0;
    for (int ww = 0; ww < 32; ww++) {
      const int c = tab[ww * E + x];
      tab[ww * E + x] = s;
      s += c;
    }
    tot[x] = s;
  }
  __syncthreads();
  e_out = e;
  r_out = e >= 0 ? tab[w * E + e] + rw : 0;
}

// Block-wide exclusive scan of one int per thread (any multiple of 32 threads up to 1024); returns the exclusive
// prefix, *total the block's sum.
__device__ __forceinline__ int block_scan(int v, int* wsum, int* total) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  if (w == 0) {
    int s = lane < nw ? wsum[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, d);
      if (lane >= d) s += y;
    }
    if (lane < nw) wsum[lane] = s;  // inclusive over warps
  }
  __syncthreads();
  const int before = (w ? wsum[w - 1] : 0) + x - v;
  *total = wsum[nw - 1];
  __syncthreads();  // wsum may be reused by the caller's next scan
  return before;
}

// One CTA of n2 threads (n2 = numel rounded up to a power of two, at least 64, at most AT): keys
// (expert << 11 | index) sorted in shared memory (bitonic), so equal experts come out in ascending index order; then
// group starts, padded offsets by a block scan, and the scatter.
__global__ void __launch_bounds__(AT) align_one_kernel(const int32_t* __restrict__ ids, int numel, int E, int bs,
                                                        int32_t* __restrict__ sorted_ids, int sorted_len,
                                                        int32_t* __restrict__ expert_ids, int expert_len,
                                                        int32_t* __restrict__ npad) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ uint32_t key[AT];
  __shared__ int gstart[AT + 1], goff[AT + 1], wsum[32];
  const int t = threadIdx.x;
  const int n2 = blockDim.x;
  if (t < n2) {
    const int e = t < numel ? ids[t] : -1;
    key[t] = (e >= 0 && e < E) ? ((uint32_t)e << 11) | (uint32_t)t : 0xFFFFFFFFu;
  }
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (t < n2) {
        const int q = t ^ j;
        if (q > t) {
          const uint32_t a = key[t], b = key[q];
          const bool up = (t & k) == 0;
          if ((a > b) == up) {
            key[t] = b;
            key[q] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // valid keys form a prefix; a group starts where the expert changes
  const uint32_t kt = t < n2 ? key[t] : 0xFFFFFFFFu;
  const bool valid = kt != 0xFFFFFFFFu;
  const bool head = valid && (t == 0 || (key[t - 1] >> 11) != (kt >> 11));
  int ngroups;
  const int gidx = block_scan(head ? 1 : 0, wsum, &ngroups);
  if (head) gstart[gidx] = t;
  int nvalid;
  block_scan(valid ? 1 : 0, wsum, &nvalid);
  if (t == 0) gstart[ngroups] = nvalid;
  __syncthreads();
  int padded = 0;
  if (t < ngroups) padded = (gstart[t + 1] - gstart[t] + bs - 1) / bs * bs;
  int total;
  const int off = block_scan(padded, wsum, &total);
  if (t < ngroups) goff[t] = off;
  if (t == 0) npad[0] = total;
  for (int j = t; j < sorted_len; j += blockDim.x) sorted_ids[j] = numel;
  for (int b = t; b < expert_len; b += blockDim.x) expert_ids[b] = -1;
  __syncthreads();
  if (t < ngroups) {
    const int e = (int)(key[gstart[t]] >> 11);
    for (int b = goff[t] / bs; b < (goff[t] + padded) / bs; b++) expert_ids[b] = e;
  }
  if (valid) {
    // the group of sorted position t: the last group start <= t
    int lo = 0, hi = ngroups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (gstart[mid] <= t) lo = mid; else hi = mid - 1;
    }
    sorted_ids[goff[lo] + t - gstart[lo]] = (int32_t)(kt & 2047u);
  }
}

// Multi-tile pass 1: per-tile expert counts [ntiles][E] and every index's in-tile rank.
__global__ void __launch_bounds__(AT) align_count_kernel(const int32_t* __restrict__ ids, int64_t numel, int E,
                                                          int32_t* __restrict__ counts, int32_t* __restrict__ ranks) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm[];
  int* tab = sm;
  int* tot = tab + 32 * E;
  int e, r;
  const int64_t i0 = (int64_t)blockIdx.x * AT;
  tile_ranks(ids, numel, i0, E, tab, tot, e, r);
  for (int x = threadIdx.x; x < E; x += AT) counts[(int64_t)blockIdx.x * E + x] = tot[x];
  if (i0 + threadIdx.x < numel) ranks[i0 + threadIdx.x] = r;
}

// Multi-tile pass 2 (one CTA): counts -> per-(tile, expert) start positions, npad, expert_ids, sentinel fill.
__global__ void __launch_bounds__(AT) align_offsets_kernel(int32_t* __restrict__ counts, int ntiles, int E, int bs,
                                                            int numel, int32_t* __restrict__ sorted_ids,
                                                            int64_t sorted_len, int32_t* __restrict__ expert_ids,
                                                            int expert_len, int32_t* __restrict__ npad) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm[];
  int* off = sm;  // [E + 1]
  const int t = threadIdx.x;
  // per expert: the total over tiles (loads issued 16 tiles at a time, not one dependent round trip per tile)
  for (int x = t; x < E; x += AT) {
    int s = 0;
    for (int tl0 = 0; tl0 < ntiles; tl0 += 16) {
      int c[16];
#pragma unroll
      for (int i = 0; i < 16; i++) c[i] = tl0 + i < ntiles ? counts[(int64_t)(tl0 + i) * E + x] : 0;
#pragma unroll
      for (int i = 0; i < 16; i++) s += c[i];
    }
    off[x] = s;
  }
  __syncthreads();
  {  // padded expert offsets: block scans over chunks of AT experts
    __shared__ int wsum[32];
    int carry = 0;
    for (int x0 = 0; x0 < E; x0 += AT) {
      const int x = x0 + t;
      const int c = x < E ? off[x] : 0;
      int tot;
      const int before = block_scan((c + bs - 1) / bs * bs, wsum, &tot);
      if (x < E) off[x] = carry + before;
      carry += tot;
    }
    if (t == 0) {
      off[E] = carry;
      npad[0] = carry;
    }
  }
  __syncthreads();
  // each (tile, expert) count becomes the expert's padded offset plus the counts of the tiles before it
  for (int x = t; x < E; x += AT) {
    int s = off[x];
    for (int tl0 = 0; tl0 < ntiles; tl0 += 16) {
      int c[16];
#pragma unroll
      for (int i = 0; i < 16; i++) c[i] = tl0 + i < ntiles ? counts[(int64_t)(tl0 + i) * E + x] : 0;
#pragma unroll
      for (int i = 0; i < 16; i++) {
        if (tl0 + i < ntiles) counts[(int64_t)(tl0 + i) * E + x] = s;
        s += c[i];
      }
    }
  }
  const int total = off[E];
  for (int64_t j = t; j < sorted_len; j += AT) sorted_ids[j] = numel;
  for (int b = t; b < expert_len; b += AT) {
    int x = -1;
    if ((int64_t)b * bs < total) {
      int lo = 0, hi = E - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= b * bs) lo = mid; else hi = mid - 1;
      }
      x = lo;
    }
    expert_ids[b] = x;
  }
}

// Multi-tile pass 3: scatter.
__global__ void __launch_bounds__(AT) align_scatter_kernel(const int32_t* __restrict__ ids, int64_t numel, int E,
                                                            const int32_t* __restrict__ starts,
                                                            const int32_t* __restrict__ ranks,
                                                            int32_t* __restrict__ sorted_ids) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * AT + threadIdx.x;
  if (i >= numel) return;
  const int e = ids[i];
  if (e < 0 || e >= E) return;
  sorted_ids[starts[(int64_t)blockIdx.x * E + e] + ranks[i]] = (int32_t)i;
}

size_t align_smem_one(int E) { return sizeof(int) * (33 * (size_t)E + 1); }  // largest dynamic smem (count pass)
size_t align_workspace_bytes(int64_t numel, int E) {
  const int64_t ntiles = (numel + AT - 1) / AT;
  return ntiles <= 1 ? 0 : sizeof(int32_t) * (size_t)(ntiles * E + numel);
}

cudaError_t launch_align(const int32_t* ids, int64_t numel, int E, int bs, int32_t* sorted_ids, int64_t sorted_len,
                         int32_t* expert_ids, int64_t expert_len, int32_t* npad, void* ws, cudaStream_t st) {
  const int64_t ntiles = (numel + AT - 1) / AT;
  if (ntiles <= 1) {
    int n2 = 64;
    while (n2 < numel) n2 <<= 1;
    cudaError_t e = launch_pdl(align_one_kernel, dim3(1), dim3(n2), 0, st, ids, (int)numel, E, bs, sorted_ids,
                               (int)sorted_len, expert_ids, (int)expert_len, npad);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  int32_t* counts = static_cast<int32_t*>(ws);
  int32_t* ranks = counts + ntiles * E;
  const size_t smem1 = sizeof(int) * 33 * (size_t)E;
  cudaFuncSetAttribute(align_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
  align_count_kernel<<<(unsigned)ntiles, AT, smem1, st>>>(ids, numel, E, counts, ranks);
  const size_t smem2 = sizeof(int) * ((size_t)E + 1);
  align_offsets_kernel<<<1, AT, smem2, st>>>(counts, (int)ntiles, E, bs, (int)numel, sorted_ids, sorted_len,
                                             expert_ids, (int)expert_len, npad);
  align_scatter_kernel<<<(unsigned)ntiles, AT, 0, st>>>(ids, numel, E, counts, ranks, sorted_ids);
  return cudaGetLastError();
}

}  // namespace moek

// ------------------------------------------------------------------------------------------ allocation-free variant
// moek_align_noalloc: the same sort-and-pad as moek_align, for callers that cannot hand the library any scratch
// buffer because they may not allocate device memory on the path that calls it (a host runtime that owns a fixed
// memory plan, or a binding that only passes the tensors it already holds). The multi-tile path's scratch (per-tile
// expert counts and per-index ranks) lives instead in the fixed array below, which every GPU that loads this library
// keeps until the process exits.
namespace moek {
constexpr int64_t NOALLOC_MAX_NUMEL = 65536;  // flattened (token, slot) indices per call
constexpr int NOALLOC_MAX_EXPERTS = 1024;
constexpr int64_t NOALLOC_MAX_TILES = NOALLOC_MAX_NUMEL / AT;
constexpr int64_t NOALLOC_INTS = NOALLOC_MAX_TILES * NOALLOC_MAX_EXPERTS + NOALLOC_MAX_NUMEL;  // 512 KiB
static __device__ __align__(256) int32_t g_align_scratch[NOALLOC_INTS];

// Device address of g_align_scratch on the current device. In host code the symbol's name is only a host-side
// stand-in, so the address is looked up once per device (with that device current) and cached.
static cudaError_t noalloc_scratch(int32_t** out) {
  static std::mutex mu;
  static int32_t* ptr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_align_scratch);
    if (e != cudaSuccess) return e;
    ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = ptr[dev];
  return cudaSuccess;
}
}  // namespace moek

extern "C" __attribute__((visibility("default"))) int moek_align_noalloc(
    const int32_t* topk_ids, int64_t numel, int32_t num_experts, int32_t block_size, int32_t* sorted_ids,
    int64_t sorted_len, int32_t* expert_ids, int64_t expert_len, int32_t* num_post_pad, void* stream) {
  using namespace moek;
  if (numel < 0 || numel > NOALLOC_MAX_NUMEL || num_experts <= 0 || num_experts > NOALLOC_MAX_EXPERTS ||
      block_size <= 0)
    return set_error(1, "moek_b200: moe_align_noalloc takes 0..%lld indices, 1..%d experts and block_size > 0 "
                        "(got %lld, %d, %d); use moek_align with a workspace for larger calls",
                     (long long)NOALLOC_MAX_NUMEL, NOALLOC_MAX_EXPERTS, (long long)numel, num_experts, block_size);
  int64_t need = numel + (int64_t)num_experts * (block_size - 1);
  if (numel < num_experts) need = std::min<int64_t>(need, numel * block_size);
  if (sorted_len < need || expert_len < (need + block_size - 1) / block_size)
    return set_error(1, "moek_b200: moe_align_noalloc outputs too small (sorted %lld < %lld or expert_ids %lld)",
                     (long long)sorted_len, (long long)need, (long long)expert_len);
  if ((sorted_len && !sorted_ids) || (expert_len && !expert_ids) || !num_post_pad || (numel && !topk_ids))
    return set_error(1, "moek_b200: moe_align_noalloc null pointer");
  int32_t* scratch = nullptr;  // a single-tile call (numel <= AT) needs no scratch and looks nothing up
  cudaError_t e = numel > AT ? noalloc_scratch(&scratch) : cudaSuccess;
  if (e != cudaSuccess)
    return set_error(2, "moek_b200: moe_align_noalloc scratch lookup: %s", cudaGetErrorString(e));
  e = launch_align(topk_ids, numel, num_experts, block_size, sorted_ids, sorted_len, expert_ids, expert_len,
                   num_post_pad, scratch, (cudaStream_t)stream);
  if (e != cudaSuccess) return set_error(2, "moek_b200: moe_align_noalloc launch: %s", cudaGetErrorString(e));
  return 0;
}
