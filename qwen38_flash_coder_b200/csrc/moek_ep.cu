// Expert-parallel (EP) dispatch and combine around the routed-expert GEMMs, sm_100a.
//
// The 512 experts are split contiguously over `world` ranks (rank d owns experts [d * E/world, (d + 1) * E/world));
// every rank owns its own tokens. A token is sent once to every rank that owns at least one of its top-k experts,
// with the k slots' local expert ids (-1 for slots owned elsewhere) and router weights; the receiving rank runs the
// same gate_up / SwiGLU / down kernels on the rows it received, sums each row's local slots in fp32 and sends the
// partial row back; the source rank adds the returned partials in rank order and rounds once to bf16. The byte
// movement between ranks is NCCL's (all-to-allv through torch.distributed on the caller's stream); these kernels do
// the index work and the row copies on each rank's own memory:
//
//   ep_plan     one CTA: for every destination rank, the position of each token in that rank's send segment
//               (ascending token order, -1 when nothing goes there), the per-rank row counts and their offsets.
//   ep_pack     one CTA per token: the token's bf16 row into each destination segment (16-byte vector copies) and
//               the slot metadata (k local ids, then k router weights as fp32 bits), at caller-given row strides so
//               that rows and metadata can share one buffer (one all-to-all); with `fill`, one more CTA per
//               destination marks the segment's unused rows (fixed-capacity exchange) as having no valid slot.
//   ep_partial  out[r][n] = sum over the row's local slots j (slot order) of rows[r * k + j][n], fp32.
//   ep_unpack   out[t][n] = bf16(sum over ranks d in order of back[offset[d] + pos[t][d]][n]).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "moek_common.cuh"
#include "moek_kernels.cuh"

namespace moek {

constexpr int EP_PLAN_THREADS = 1024;

__global__ void __launch_bounds__(EP_PLAN_THREADS) ep_plan_kernel(const int32_t* __restrict__ ids, int M, int k,
                                                                  int E, int world, int32_t* __restrict__ pos,
                                                                  int32_t* __restrict__ counts,
                                                                  int32_t* __restrict__ offsets) {
  __shared__ int wcnt[32][EP_MAX_WORLD];  // per-warp counts of the chunk, then their exclusive prefix
  __shared__ int base[EP_MAX_WORLD];      // rows already placed per destination
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const int per = E / world;
  if (tid < world) base[tid] = 0;
  __syncthreads();
  for (int t0 = 0; t0 < M; t0 += blockDim.x) {
    const int t = t0 + tid;
    uint32_t mask = 0;
    if (t < M)
      for (int j = 0; j < k; j++) {
        const int e = ids[(int64_t)t * k + j];
        if (e >= 0 && e < E) mask |= 1u << (e / per);
      }
    for (int d = 0; d < world; d++) {
      const uint32_t b = __ballot_sync(0xffffffffu, (mask >> d) & 1u);
      if (lane == 0) wcnt[warp][d] = __popc(b);
    }
    __syncthreads();
    if (tid < world) {  // exclusive prefix over the warps, per destination
      int run = base[tid];
      for (int w = 0; w < nw; w++) {
        const int c = wcnt[w][tid];
        wcnt[w][tid] = run;
        run += c;
      }
      base[tid] = run;
    }
    __syncthreads();
    for (int d = 0; d < world; d++) {
      const uint32_t b = __ballot_sync(0xffffffffu, (mask >> d) & 1u);  // the same ballot as above
      if (t < M)
        pos[(int64_t)t * world + d] = (mask >> d) & 1u ? wcnt[warp][d] + __popc(b & ((1u << lane) - 1u)) : -1;
    }
    __syncthreads();  // wcnt is rewritten by the next chunk
  }
  if (tid == 0) {
    int off = 0;
    for (int d = 0; d < world; d++) {
      counts[d] = base[d];
      offsets[d] = off;
      off += base[d];
    }
    offsets[world] = off;
  }
}

__global__ void ep_pack_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ ids,
                               const float* __restrict__ topk_w, const int32_t* __restrict__ pos,
                               const int32_t* __restrict__ offsets, const int32_t* __restrict__ counts, int M,
                               int H16, int k, int E, int world, uint4* __restrict__ send_x, int64_t xs16,
                               int32_t* __restrict__ send_meta, int64_t ms) {
  const int per = E / world;
  if (blockIdx.x >= M) {  // fill: the rows of destination d's segment that no token uses get invalid slots
    const int d = blockIdx.x - M;
    for (int64_t row = (int64_t)offsets[d] + counts[d] + threadIdx.x; row < offsets[d + 1]; row += blockDim.x)
      for (int j = 0; j < k; j++) {
        send_meta[row * ms + j] = -1;
        send_meta[row * ms + k + j] = 0;
      }
    return;
  }
  const int t = blockIdx.x;
  for (int d = 0; d < world; d++) {
    const int p = pos[(int64_t)t * world + d];
    if (p < 0) continue;
    const int64_t row = (int64_t)offsets[d] + p;
    for (int c = threadIdx.x; c < H16; c += blockDim.x) send_x[row * xs16 + c] = x[(int64_t)t * H16 + c];
    if (threadIdx.x < k) {
      const int j = threadIdx.x;
      const int e = ids[(int64_t)t * k + j];
      const bool mine = e >= 0 && e < E && e / per == d;
      send_meta[row * ms + j] = mine ? e - d * per : -1;
      send_meta[row * ms + k + j] = __float_as_int(mine ? topk_w[(int64_t)t * k + j] : 0.f);
    }
  }
}

__global__ void ep_partial_kernel(const float* __restrict__ rows, const int32_t* __restrict__ meta, int64_t ms,
                                  int E_local, int R, int N, int k, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)R * N) return;
  const int64_t r = i / N;
  const int n = (int)(i - r * N);
  float o = 0.f;
  for (int j = 0; j < k; j++) {
    const int e = meta[r * ms + j];
    if (e >= 0 && e < E_local) o += rows[(r * k + j) * N + n];
  }
  out[i] = o;
}

__global__ void ep_unpack_kernel(const float* __restrict__ back, const int32_t* __restrict__ pos,
                                 const int32_t* __restrict__ offsets, int M, int H, int world,
                                 __nv_bfloat16* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * H) return;
  const int64_t t = i / H;
  const int n = (int)(i - t * H);
  float o = 0.f;
  for (int d = 0; d < world; d++) {
    const int p = pos[t * world + d];
    if (p >= 0) o += back[((int64_t)offsets[d] + p) * H + n];
  }
  out[i] = __float2bfloat16_rn(o);
}

cudaError_t launch_ep_plan(const int32_t* ids, int M, int k, int E, int world, int32_t* pos, int32_t* counts,
                           int32_t* offsets, cudaStream_t st) {
  ep_plan_kernel<<<1, EP_PLAN_THREADS, 0, st>>>(ids, M, k, E, world, pos, counts, offsets);
  return cudaGetLastError();
}

cudaError_t launch_ep_pack(const __nv_bfloat16* x, const int32_t* ids, const float* topk_w, const int32_t* pos,
                           const int32_t* offsets, const int32_t* counts, int fill, int M, int H, int k, int E,
                           int world, __nv_bfloat16* send_x, int64_t x_stride, int32_t* send_meta,
                           int64_t meta_stride, cudaStream_t st) {
  const int grid = M + (fill ? world : 0);
  if (grid == 0) return cudaSuccess;
  ep_pack_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const uint4*>(x), ids, topk_w, pos, offsets, counts, M, H / 8,
                                       k, E, world, reinterpret_cast<uint4*>(send_x), x_stride / 8, send_meta,
                                       meta_stride);
  return cudaGetLastError();
}

cudaError_t launch_ep_partial(const float* rows, const int32_t* meta, int64_t meta_stride, int E_local, int R, int N,
                              int k, float* out, cudaStream_t st) {
  const int64_t n = (int64_t)R * N;
  if (n == 0) return cudaSuccess;
  ep_partial_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, meta, meta_stride, E_local, R, N, k, out);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack(const float* back, const int32_t* pos, const int32_t* offsets, int M, int H, int world,
                             __nv_bfloat16* out, cudaStream_t st) {
  const int64_t n = (int64_t)M * H;
  if (n == 0) return cudaSuccess;
  ep_unpack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(back, pos, offsets, M, H, world, out);
  return cudaGetLastError();
}

}  // namespace moek
