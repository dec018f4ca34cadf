// Launch interfaces shared by the kernel files and the C ABI (moek_abi.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace moek {

// Launch with programmatic stream serialisation: the kernel may start while the previous kernel in the stream is
// finishing; it orders itself behind that kernel's results with pdl_wait() (moek_common.cuh).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Launch as a cooperative grid (every CTA resident at once, or the launch fails instead of running), with
// programmatic stream serialisation as well when the runtime accepts both attributes together (pdl = 1). Kernels
// whose CTAs wait on one another use this: the co-residency their waits rely on is then guaranteed, also when other
// kernels hold part of the GPU.
template <typename... KArgs, typename... Args>
cudaError_t launch_coop(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int pdl,
                        Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

struct GemmParams {
  const __nv_bfloat16* A;  // gate_up: hidden [M, K]; down: act [num_ids, K]
  const uint8_t* W;        // tiled codes [E, N/256, K/64, 8 KB]
  const float* G;          // processed global scales [E]
  const int32_t* sorted_ids;
  const int32_t* expert_ids;
  const int32_t* num_post_pad;
  const uint8_t* SP;        // tiled packed scales [E, N/256, K/128, 1056]
  const int32_t* exc_off;   // [E * N/256 * K/128 + 1]
  const uint32_t* exc_ent;  // exception entries
  float* part;              // mode 2 / split: [nsplit, num_ids, N] fp32 partials; down, nsplit 1: fp32 rows
  int* err;                 // device error word (cnt[0])
  int* counters;            // split-k arrival counters (cnt[1..]), zero between launches
  const int32_t* topk_ids;  // mode 3 down combine: [num_ids] (slots whose expert is invalid are left out)
  const float* topk_w;      // [num_ids] router weights (down)
  void* out;                // mode 3: gate_up -> act bf16 [num_ids, N/2]; down (split) -> bf16 [M, N] top-k sums
  uint64_t timeout_ns;
  int num_ids, N, K, E, a_div, block_m, nsplit, max_blocks;
  int a_rows;  // tcgen05 path: rows of A (x: num_ids / a_div; sorted-order down: the sorted act rows)
  int gate_up, mode, combine_k;
  int sorted_act;  // tcgen05 path: act rows at their position in moe_align's sorted order (moek_gemm mode 5)
  int down_bf16;   // tcgen05 path, down: bf16 rows topk_w * sum into out (modes 0/1) instead of fp32 rows into part
};

// moek_ep.cu / moek_ep.cuh: the fixed-capacity expert-parallel exchange over peer memory
constexpr int EP_MAX_WORLD = 32;
constexpr int EP_P2P_MAXM = 1024;  // tokens per rank and call of the peer-memory exchange
constexpr int EP_P2P_MAXH = 4096;  // hidden size of the peer-memory exchange
// The exchange block of the fixed-capacity peer-memory EP path, the same layout on every rank (R = world x mcap rows;
// segment s = rows [s mcap, (s + 1) mcap), the rows rank s sent): byte offsets of the received bf16 rows [R, H], their
// local expert ids int32 [R, k] (-1: slot owned elsewhere or unused row) and router weights fp32 [R, k], this rank's
// fp32 partial rows of the received rows [R, H] (segment s = the partials for rank s's rows, which rank s reads over
// NVLink), the flags int32 [2 world] ([s]: the call number whose rows rank s wrote into receive segment s; [world + d]:
// the call number whose partials for this rank rank d has written into its own back buffer) and counters int32
// [2 world + 2] (arrival counters; [2 world] = the number of
// calls this rank has completed, advanced by its unpack; [2 world + 1] = the unpack's arrival counter).
struct P2PLayout {
  int64_t x, ids, w, back, flags, ctr, total;
};
__host__ __device__ inline int64_t up256(int64_t b) { return (b + 255) / 256 * 256; }
__host__ __device__ inline P2PLayout p2p_layout(int world, int mcap, int H, int k) {
  const int64_t R = (int64_t)world * mcap;
  P2PLayout l;
  l.x = 0;
  l.ids = l.x + up256(R * H * 2);
  l.w = l.ids + up256(R * k * 4);
  l.back = l.w + up256(R * k * 4);
  l.flags = l.back + up256(R * H * 4);
  l.ctr = l.flags + up256(2 * world * 4);
  l.total = l.ctr + up256((2 * world + 2) * 4);
  return l;
}
struct P2PArgs {  // peer-memory exchange of the fixed-capacity EP path (moek_ep.cu)
  const uint64_t* peer;  // [world] device table: base of each rank's exchange block (CUDA IPC mappings)
  P2PLayout lay;
  int world, rank, mcap, H, k;
  int* err;
  uint64_t timeout_ns;
};
// moek_layer.cu: the whole decode-regime layer in one persistent kernel
constexpr int LAYER_MAXIDS = 512;      // routed slots (tokens x top_k) per call
constexpr int LAYER_XFLAG_CTAS = 1024; // CTAs of the grid at most
// gate_up partial records of one call: one per (CTA, pair) whose ranges meet; record index = CTA + pair, so at most
// grid + pairs, pairs = blocks x (2I / 256) <= LAYER_MAXIDS x (2I / 256)
inline int64_t layer_max_records(int64_t grid, int64_t num_ids, int I) {
  return grid + num_ids * (2 * (int64_t)I / 256);
}
constexpr int LAYER_NCW = 8;           // consumer warps per CTA
struct LayerMat {                  // one weight matrix in this build's layout (gate_up: N = 2I, K = H; down: N = H, K = I)
  const uint8_t* W;
  const uint8_t* SP;
  const float* G;
  const int32_t* exc_off;
  const uint32_t* exc_ent;
  int N, K, nt, nstage;  // nt = N / 256 items, nstage = K / 128
};
struct LayerParams {
  LayerMat m[2];  // 0 = gate_up, 1 = down
  const __nv_bfloat16* x;  // [M, H]
  const int32_t* ids;      // [M * top_k] expert per slot (outside [0, E): not routed)
  const float* tw;         // [M * top_k] router weights
  float* xpart;            // workspace [records, XR, 256]: fp32 gate_up partials, record = CTA + pair
  float* part2;            // workspace [I / 128, num_ids, H]: down partials per k-slice
  float* out_rows;         // caller's fp32 rows [num_ids, H] instead of the top-k sum (or null)
  __nv_bfloat16* out;      // caller's bf16 [M, H] top-k sums (or null)
  const float* shared;     // fp32 [M, H] rows added to each token's sum before its rounding (the shared expert), or
                           // null
  int* ctr;                // persistent int32 state: epoch, barrier and arrival counters, exchange flags (zeroed once)
  int* err;                // device error word
  uint64_t timeout_ns;
  int M, top_k, num_ids, E, H, I;
  int off_epoch, off_done, off_ep, off_xflag;  // int offsets into ctr (xflag: [records][consumer warp])
  int max_records;                             // records the workspace and the flags hold
  // Expert-parallel receive side (ep_peer non-null, out and out_rows null): x / ids / tw are this rank's receive
  // buffers of the peer-memory exchange (row s * ep_mcap + p came from rank s), the kernel waits for the receive
  // flags before routing, and each row's fp32 sum of its local slots goes to the same row of this rank's own back
  // buffer (rank s reads segment s over NVLink); once every row is written, rank s's back flag for this rank is
  // raised.
  const uint64_t* ep_peer;   // [ep_world] device table: base of each rank's exchange block
  const int* ep_recv_flags;  // this rank's flags [0, ep_world)
  const int* ep_call;        // this rank's completed-call counter (the current call is *ep_call + 1)
  int64_t ep_back_off, ep_flags_off;  // byte offsets of the back buffer and the flags in an exchange block
  int ep_world, ep_rank, ep_mcap;
  // Fused exchange (ep_x non-null, with ep_peer): the kernel also runs this rank's side of the exchange, so that the
  // layer is one launch: CTAs [0, world x G) dispatch this rank's ep_M tokens (rows ep_x, global expert ids ep_ids,
  // router weights ep_w) into the owners' receive segments and write ep_pos [ep_M, world] before the receive wait, and
  // once the owners' back flags read this call, CTAs unpack ep_out bf16 [ep_M, H] = the owners' partials summed in
  // rank order; the last CTA to finish completes the call.
  P2PArgs ep_q;
  const uint4* ep_x;
  const int32_t* ep_ids;
  const float* ep_w;
  int32_t* ep_pos;
  __nv_bfloat16* ep_out;
  int ep_M, ep_E;
  // Fused router (logits non-null): every CTA routes the M tokens itself from the router logits [M, E] (fp32, or bf16
  // when logits_bf16): softmax, top_k, renormalised when renorm; ids and tw are not read, and CTA 0 writes the
  // routing to ids_out / w_out (when non-null) for the caller.
  const void* logits;
  int logits_bf16, renorm;
  int32_t* ids_out;
  float* w_out;
};
// rows per block: 8/16/32; coop: cooperative launch (every CTA resident together, the default)
cudaError_t launch_layer(const LayerParams& p, int block_rows, int sms, int coop, cudaStream_t st);

// moek_prep.cu: load-time conversion of checkpoint NVFP4 matrices (E4M3 scales [E, N, K/16], codes [E, N, K/2])
cudaError_t launch_prep_scale_max(const uint8_t* scales, int64_t n, unsigned int* out, cudaStream_t st);
cudaError_t launch_prep_weights(const uint8_t* codes, int E, int N, int K, int gate_up, uint32_t* out,
                                cudaStream_t st);
// sp [E, N/256, K/128, 1056], g [E], cnt [nkeys, 32] (the blocks' exclusive prefixes within their list on return),
// total [nkeys], exc_off [nkeys + 1]; nkeys = E * N/256 * K/128
cudaError_t launch_prep_scales(const uint8_t* scales, const float* gs, int E, int N, int K, int gate_up, float sf,
                               uint8_t* sp, float* g, int* cnt, int* total, int* exc_off, cudaStream_t st);
cudaError_t launch_prep_exceptions(const uint8_t* scales, int E, int N, int K, int gate_up, float sf,
                                   const int* cnt_prefix, const int* exc_off, int* ent, cudaStream_t st);

// moek_shared.cu: the router gate GEMM and the MXFP8 shared expert at decode sizes (M <= SHARED_MAXM tokens)
constexpr int SHARED_MAXM = 64;
cudaError_t launch_router_gate(const __nv_bfloat16* x, int M, int H, const __nv_bfloat16* wg, int E, float* logits,
                               uint64_t timeout_ns, int* err, cudaStream_t st);
// The MoE block's two kernels before the whole-layer kernel: [router gate | shared gate_up], then [shared down | the
// routing of the logits into ids / w (softmax, top k, renormalised when renorm)]; Is = 0: no shared expert
cudaError_t launch_block_pre_post(const __nv_bfloat16* x, int M, int H, int E, int Is, const __nv_bfloat16* wg,
                                  float* logits, const uint8_t* wgu, const uint8_t* sgu, const uint8_t* wd,
                                  const uint8_t* sd, const __nv_bfloat16* wsg, __nv_bfloat16* act, float* sg,
                                  float* rows, int k, int renorm, int32_t* ids, float* w, uint64_t timeout_ns, int* err,
                                  cudaStream_t st);
// act bf16 [M, Is] and sg fp32 [M] are scratch; rows fp32 [M, H] the output
cudaError_t launch_shared_expert(const __nv_bfloat16* x, int M, int H, int Is, const uint8_t* wgu, const uint8_t* sgu,
                                 const uint8_t* wd, const uint8_t* sd, const __nv_bfloat16* wsg, __nv_bfloat16* act,
                                 float* sg, float* rows, uint64_t timeout_ns, int* err, cudaStream_t st);

// moek_router.cu: softmax -> top-k -> optional renormalisation (dtype 0 = fp32 logits, 1 = bf16)
cudaError_t launch_router_topk(const void* logits, int dtype, int M, int E, int k, int renorm, int32_t* ids,
                               float* weights, int32_t* tok_idx, cudaStream_t st);

// Timeline stamps of MOEK_TRACE builds (moek_common.cuh): copy up to `bytes` of a translation unit's stamp array
// [CTA][slot] to host memory (dst may be null) and optionally zero it; cudaErrorNotSupported without MOEK_TRACE.
cudaError_t trace_copy_layer(void* dst, size_t bytes, int clear);
cudaError_t trace_copy_prefill(void* dst, size_t bytes, int clear);
cudaError_t trace_copy_ep(void* dst, size_t bytes, int clear);

// moek_abi.cu: record the calling thread's error message (read back by moek_last_error) and return code
int set_error(int code, const char* fmt, ...);

// moek_align.cu
cudaError_t launch_align(const int32_t* ids, int64_t numel, int E, int bs, int32_t* sorted_ids, int64_t sorted_len,
                         int32_t* expert_ids, int64_t expert_len, int32_t* npad, void* ws, cudaStream_t st);
size_t align_workspace_bytes(int64_t numel, int E);
size_t align_smem_one(int E);

// moek_prefill.cu: tcgen05 grouped GEMM for large batches (blocks of <= prefill_block_m() rows)
int prefill_block_m();
cudaError_t launch_prefill(const GemmParams& p, int sms, cudaStream_t st);

// moek_decode.cu
cudaError_t launch_decode(const GemmParams& p, int max_rows, int sms, cudaStream_t st);
cudaError_t launch_gate_epilogue(const float* part, int nsplit, int num_ids, int N, __nv_bfloat16* act,
                                 cudaStream_t st);
cudaError_t launch_down_combine(const float* part, int nsplit, int num_ids, int N, int top_k, const float* topk_w,
                                __nv_bfloat16* out, cudaStream_t st);
cudaError_t launch_down_rows(const float* part, int nsplit, int num_ids, int N, const float* topk_w, float* dout,
                             cudaStream_t st);
cudaError_t launch_combine_f32(const float* rows, int m, int N, int top_k, __nv_bfloat16* out, cudaStream_t st);
// the top-k sum over the slots whose id lies in [0, E) (unrouted slots left out; none routed: a zero row)
cudaError_t launch_combine_routed(const float* rows, const int32_t* ids, int E, int m, int N, int top_k,
                                  __nv_bfloat16* out, cudaStream_t st);
cudaError_t launch_combine_bf16(const __nv_bfloat16* rows, int m, int N, int top_k, __nv_bfloat16* out,
                                cudaStream_t st);

// moek_ep.cu: expert-parallel dispatch plan, row packing, partial combine and ordered unpack (the exchange
// structures are declared before the whole-layer kernel, which can run the peer exchange itself)
cudaError_t launch_ep_dispatch_p2p(const P2PArgs& a, const __nv_bfloat16* x, const int32_t* ids, const float* topk_w,
                                   int M, int E, int32_t* pos, cudaStream_t st);
cudaError_t launch_ep_wait(const int* flags, int world, int* err, uint64_t timeout_ns, cudaStream_t st);
cudaError_t launch_ep_combine_p2p(const P2PArgs& a, const float* rows, int E_local, cudaStream_t st);
cudaError_t launch_ep_unpack_p2p(const P2PArgs& a, const int32_t* pos, int M, __nv_bfloat16* out, cudaStream_t st);
cudaError_t launch_ep_plan(const int32_t* ids, int M, int k, int E, int world, int32_t* pos, int32_t* counts,
                           int32_t* offsets, cudaStream_t st);
cudaError_t launch_ep_pack(const __nv_bfloat16* x, const int32_t* ids, const float* topk_w, const int32_t* pos,
                           const int32_t* offsets, const int32_t* counts, int fill, int M, int H, int k, int E,
                           int world, __nv_bfloat16* send_x, int64_t x_stride, int32_t* send_meta,
                           int64_t meta_stride, cudaStream_t st);
cudaError_t launch_ep_partial(const float* rows, const int32_t* meta, int64_t meta_stride, int E_local, int R, int N,
                              int k, float* out, cudaStream_t st);
cudaError_t launch_ep_unpack(const float* back, const int32_t* pos, const int32_t* offsets, int M, int H, int world,
                             __nv_bfloat16* out, cudaStream_t st);

}  // namespace moek
