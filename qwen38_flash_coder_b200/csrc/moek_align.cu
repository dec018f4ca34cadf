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

// One CTA: numel <= AT.
__global__ void __launch_bounds__(AT) align_one_kernel(const int32_t* __restrict__ ids, int numel, int E, int bs,
                                                        int32_t* __restrict__ sorted_ids, int sorted_len,
                                                        int32_t* __restrict__ expert_ids, int expert_len,
                                                        int32_t* __restrict__ npad) {
  extern __shared__ int sm[];
  int* tab = sm;            // [32][E]
  int* tot = tab + 32 * E;  // [E]
  int* off = tot + E;       // [E + 1] padded offsets
  int e, r;
  tile_ranks(ids, numel, 0, E, tab, tot, e, r);
  const int t = threadIdx.x;
  if (t == 0) {  // serial scan over experts: E is small (<= a few thousand)
    int s = 0;
    for (int x = 0; x < E; x++) {
      off[x] = s;
      s += (tot[x] + bs - 1) / bs * bs;
    }
    off[E] = s;
    npad[0] = s;
  }
  __syncthreads();
  const int total = off[E];
  for (int j = t; j < sorted_len; j += AT) sorted_ids[j] = numel;
  for (int b = t; b < expert_len; b += AT) {
    int x = -1;
    if (b * bs < total) {  // the expert whose padded range holds block b
      int lo = 0, hi = E - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= b * bs) lo = mid; else hi = mid - 1;
      }
      x = lo;
    }
    expert_ids[b] = x;
  }
  __syncthreads();
  if (e >= 0) sorted_ids[off[e] + r] = t;
}

// Multi-tile pass 1: per-tile expert counts [ntiles][E] and every index's in-tile rank.
__global__ void __launch_bounds__(AT) align_count_kernel(const int32_t* __restrict__ ids, int64_t numel, int E,
                                                          int32_t* __restrict__ counts, int32_t* __restrict__ ranks) {
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
  extern __shared__ int sm[];
  int* off = sm;  // [E + 1]
  const int t = threadIdx.x;
  for (int x = t; x < E; x += AT) {  // per expert: exclusive scan over tiles (in place), total kept in off
    int s = 0;
    for (int tl = 0; tl < ntiles; tl++) {
      const int c = counts[(int64_t)tl * E + x];
      counts[(int64_t)tl * E + x] = s;
      s += c;
    }
    off[x] = s;
  }
  __syncthreads();
  if (t == 0) {
    int s = 0;
    for (int x = 0; x < E; x++) {
      const int c = off[x];
      off[x] = s;
      s += (c + bs - 1) / bs * bs;
    }
    off[E] = s;
    npad[0] = s;
  }
  __syncthreads();
  for (int x = t; x < E; x += AT)
    for (int tl = 0; tl < ntiles; tl++) counts[(int64_t)tl * E + x] += off[x];
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
  const int64_t i = (int64_t)blockIdx.x * AT + threadIdx.x;
  if (i >= numel) return;
  const int e = ids[i];
  if (e < 0 || e >= E) return;
  sorted_ids[starts[(int64_t)blockIdx.x * E + e] + ranks[i]] = (int32_t)i;
}

size_t align_smem_one(int E) { return sizeof(int) * (33 * (size_t)E + E + 1); }
size_t align_workspace_bytes(int64_t numel, int E) {
  const int64_t ntiles = (numel + AT - 1) / AT;
  return ntiles <= 1 ? 0 : sizeof(int32_t) * (size_t)(ntiles * E + numel);
}

cudaError_t launch_align(const int32_t* ids, int64_t numel, int E, int bs, int32_t* sorted_ids, int64_t sorted_len,
                         int32_t* expert_ids, int64_t expert_len, int32_t* npad, void* ws, cudaStream_t st) {
  const int64_t ntiles = (numel + AT - 1) / AT;
  if (ntiles <= 1) {
    const size_t smem = align_smem_one(E);
    cudaFuncSetAttribute(align_one_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    align_one_kernel<<<1, AT, smem, st>>>(ids, (int)numel, E, bs, sorted_ids, (int)sorted_len, expert_ids,
                                          (int)expert_len, npad);
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
  int32_t* scratch = nullptr;
  cudaError_t e = noalloc_scratch(&scratch);
  if (e != cudaSuccess)
    return set_error(2, "moek_b200: moe_align_noalloc scratch lookup: %s", cudaGetErrorString(e));
  e = launch_align(topk_ids, numel, num_experts, block_size, sorted_ids, sorted_len, expert_ids, expert_len,
                   num_post_pad, scratch, (cudaStream_t)stream);
  if (e != cudaSuccess) return set_error(2, "moek_b200: moe_align_noalloc launch: %s", cudaGetErrorString(e));
  return 0;
}
