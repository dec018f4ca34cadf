// Expert-parallel (EP) dispatch and combine around the routed-expert GEMMs, sm_100a.
//
// The 512 experts are split contiguously over `world` ranks (rank d owns experts [d * E/world, (d + 1) * E/world));
// every rank owns its own tokens. A token is sent once to every rank that owns at least one of its top-k experts,
// with the k slots' local expert ids (-1 for slots owned elsewhere) and router weights; the receiving rank runs the
// same gate_up / SwiGLU / down kernels on the rows it received, sums each row's local slots in fp32 and sends the
// partial row back; the source rank adds the returned partials in rank order and rounds once to bf16. The byte
// movement between ranks is NCCL's (all-to-allv through torch.distributed on the caller's stream); these kernels do
// the index work and the row copies on each rank's own memory (the fixed-capacity exchange can instead run over peer
// memory with this file's own kernels: the section "peer-memory exchange" below):
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

#include <algorithm>

#include "moek_common.cuh"
#include "moek_ep.cuh"
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

// ------------------------------------------------------------------------- peer-memory exchange (fixed capacity)
// Every rank holds one exchange block (P2PLayout), shared by CUDA IPC; the kernels below write straight into the
// peers' blocks over NVLink (plain stores, no multicast) and hand segments over with system-scope flags that carry
// the call number c (every rank counts its completed calls in its own block; the current call is that count + 1), so
// no flag is ever reset and no kernel waits before writing:
//   dispatch  CTAs (d, g), G per destination d: place my tokens in d's segment for me (ascending token order, as
//             moek_ep_plan), copy rows g, g + G, ... with their slot ids (local id, or -1 for slots owned elsewhere)
//             and router weights, mark the unused rows as having no valid slot; the last CTA of d fences and sets
//             d's receive flag for me to c. No wait is needed before writing: d had finished reading my previous
//             rows before it returned my partials of call c - 1, and my own unpack of call c - 1 (earlier on my
//             stream) waited for those.
//   wait      my receive flags all c (bounded); the whole-layer kernel does this wait itself.
//   combine   CTAs (s, g): for the rows of receive segment s, the fp32 sum (slot order) of the row's local slots into
//             segment s of my own back buffer; the last CTA of s sets s's back flag for me to c (a release store: my
//             writes are local, so no system-wide fence is needed first). No wait is needed before writing: s sent
//             call c's rows after its unpack of call c - 1 had read that segment.
//   unpack    wait until my back flags are all c, out[t] = bf16(sum over ranks d in order of my segment of d's back
//             buffer, read over NVLink); the last CTA to finish advances my completed-call count to c.
// Every wait is bounded by the caller's deadline; on expiry the kernel records MOEK_DEV_TIMEOUT and stops waiting (the
// counts of the ranks may then disagree: build the exchange again).
constexpr int P2P_THREADS = 256;

__global__ void __launch_bounds__(P2P_THREADS) ep_dispatch_p2p_kernel(P2PArgs q, const uint4* __restrict__ x,
                                                                      const int32_t* __restrict__ ids,
                                                                      const float* __restrict__ topk_w, int M, int E,
                                                                      int G, int32_t* __restrict__ pos) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) MOEK_TR(0);
  __shared__ int spos[EP_P2P_MAXM];
  __shared__ int wcnt[P2P_THREADS / 32];
  const int d = blockIdx.x / G, g = blockIdx.x - d * G;
  ep_dispatch_cta<P2P_THREADS, 8, 2>(q, x, ids, topk_w, M, E, d, g, G, current_call(q), pos, spos, wcnt);
}

__global__ void ep_wait_kernel(const int* __restrict__ flags, const int* __restrict__ calls, int world, int* err,
                               uint64_t timeout_ns) {
  pdl_wait();
  pdl_launch_dependents();
  const uint64_t deadline = globaltimer() + timeout_ns;
  const int call = *reinterpret_cast<const volatile int*>(calls) + 1;
  for (int s = threadIdx.x; s < world; s += blockDim.x) wait_flag(flags + s, call, deadline, err);
}

__global__ void __launch_bounds__(P2P_THREADS) ep_combine_p2p_kernel(P2PArgs q, const float* __restrict__ rows,
                                                                     int E_local, int G) {
  pdl_wait();
  pdl_launch_dependents();
  const int s = blockIdx.x / G, g = blockIdx.x - s * G, k = q.k;
  const int call = current_call(q);
  uint8_t* mine = reinterpret_cast<uint8_t*>(q.peer[q.rank]);
  const int32_t* rid = reinterpret_cast<const int32_t*>(mine + q.lay.ids);
  float* back = reinterpret_cast<float*>(mine + q.lay.back) +
                (int64_t)s * q.mcap * q.H;  // s's segment of my back buffer (s reads it over NVLink)
  const int H4 = q.H / 4;
  for (int p = g; p < q.mcap; p += G) {
    const int64_t r = (int64_t)s * q.mcap + p;  // the row's index in my receive buffers (and in rows)
    bool any = false;
    for (int j = 0; j < k; j++) any |= rid[r * k + j] >= 0 && rid[r * k + j] < E_local;
    if (!any) continue;  // an unused row
    for (int c = threadIdx.x; c < H4; c += P2P_THREADS) {
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < k; j++) {
        const int e = rid[r * k + j];
        if (e < 0 || e >= E_local) continue;
        const float4 v = reinterpret_cast<const float4*>(rows + (r * k + j) * q.H)[c];
        o.x += v.x;
        o.y += v.y;
        o.z += v.z;
        o.w += v.w;
      }
      reinterpret_cast<float4*>(back + (int64_t)p * q.H)[c] = o;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    int* ctr = reinterpret_cast<int*>(mine + q.lay.ctr) + q.world + s;
    if (last_arrival(ctr, G)) st_sys(p2p_flags(q, s) + q.world + q.rank, call);
  }
}

__global__ void __launch_bounds__(P2P_THREADS) ep_unpack_p2p_kernel(P2PArgs q, const int32_t* __restrict__ pos, int M,
                                                                    __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) MOEK_TR(8);
  __shared__ int ok;
  uint8_t* mine = reinterpret_cast<uint8_t*>(q.peer[q.rank]);
  int* my_flags = reinterpret_cast<int*>(mine + q.lay.flags);
  const int call = current_call(q);
  if (threadIdx.x < 32) {
    bool good = true;
    const uint64_t deadline = globaltimer() + q.timeout_ns;
    for (int s = threadIdx.x; s < q.world; s += 32) good &= wait_flag(my_flags + q.world + s, call, deadline, q.err);
    good = __all_sync(0xffffffffu, good);
    if (threadIdx.x == 0) ok = good;
    if (threadIdx.x == 0) MOEK_TR(9);
  }
  __syncthreads();
  if (!ok) return;
  ep_unpack_slice<P2P_THREADS>(q, pos, M, out, blockIdx.x, gridDim.x);
  __syncthreads();
  if (threadIdx.x == 0) {  // every CTA has read `call`: the last one to finish completes the call
    MOEK_TR(10);
    if (last_arrival(p2p_call(q) + 1, gridDim.x)) {
      __threadfence();
      *p2p_call(q) = call;
    }
  }
}

MOEK_TRACE_COPY_FN(trace_copy_ep)

static int p2p_split(int rows) { return rows <= 8 ? 1 : rows <= 64 ? (rows + 7) / 8 : 8; }  // CTAs per peer

cudaError_t launch_ep_dispatch_p2p(const P2PArgs& a, const __nv_bfloat16* x, const int32_t* ids, const float* topk_w,
                                   int M, int E, int32_t* pos, cudaStream_t st) {
  const int G = p2p_split(M);
  cudaError_t e = launch_pdl(ep_dispatch_p2p_kernel, dim3(a.world * G), dim3(P2P_THREADS), 0, st, a,
                             reinterpret_cast<const uint4*>(x), ids, topk_w, M, E, G, pos);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_ep_wait(const int* flags, int world, int* err, uint64_t timeout_ns, cudaStream_t st) {
  // the completed-call count sits after the flags and the 2 world arrival counters (p2p_layout)
  const int* calls = flags + up256(2 * world * 4) / 4 + 2 * world;
  cudaError_t e = launch_pdl(ep_wait_kernel, dim3(1), dim3(32), 0, st, flags, calls, world, err, timeout_ns);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_ep_combine_p2p(const P2PArgs& a, const float* rows, int E_local, cudaStream_t st) {
  const int G = p2p_split(a.mcap);
  cudaError_t e = launch_pdl(ep_combine_p2p_kernel, dim3(a.world * G), dim3(P2P_THREADS), 0, st, a, rows, E_local, G);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack_p2p(const P2PArgs& a, const int32_t* pos, int M, __nv_bfloat16* out, cudaStream_t st) {
  const int64_t n4 = (int64_t)M * a.H / 4;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n4 + P2P_THREADS - 1) / P2P_THREADS, 1184));
  cudaError_t e = launch_pdl(ep_unpack_p2p_kernel, dim3(grid), dim3(P2P_THREADS), 0, st, a, pos, M, out);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace moek
