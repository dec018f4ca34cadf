// C ABI of the routed-expert MoE kernels: plain pointers, sizes and a cudaStream_t, an int status (0 = ok) and a
// thread-local message behind moek_last_error(). Declared in include/moek_b200.h (each entry point's comment names
// the reference interface it replaces).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstring>

#include "moek_common.cuh"
#include "moek_kernels.cuh"

#define MOEK_API extern "C" __attribute__((visibility("default")))

enum { MOEK_OK = 0, MOEK_ERR_ARG = 1, MOEK_ERR_CUDA = 2, MOEK_ERR_UNSUPPORTED = 3 };

static thread_local char g_msg[512];

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}
namespace moek {
int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace moek

static int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MOEK_OK;
  return fail(MOEK_ERR_CUDA, "moek_b200: %s: %s", what, cudaGetErrorString(e));
}

static int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (!v) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

static uint64_t g_timeout_ns = 2000000000ull;  // 2 s bound on every device-side wait

MOEK_API const char* moek_last_error(void) { return g_msg; }

MOEK_API int moek_version(void) { return 1; }

MOEK_API int moek_build_flags(void) {
  int f = 0;
#ifdef MOEK_TRACE
  f |= 1;
#endif
#ifdef MOEK_DEBUG_CHECKS
  f |= 2;
#endif
  return f;
}

// Timeline stamps (MOEK_TRACE builds): kind 0 = the whole-layer kernel, 1 = the tcgen05 GEMM, 2 = the EP peer
// exchange kernels; dst is host memory of `bytes` (at most 1024 CTAs x 128 slots x 8 bytes are copied).
MOEK_API int moek_trace_read(int32_t kind, void* dst, size_t bytes) {
  if (!dst || kind < 0 || kind > 2) return fail(MOEK_ERR_ARG, "moek_b200: trace_read needs kind 0-2 and a buffer");
  cudaError_t e = kind == 0 ? moek::trace_copy_layer(dst, bytes, 0)
                : kind == 1 ? moek::trace_copy_prefill(dst, bytes, 0)
                            : moek::trace_copy_ep(dst, bytes, 0);
  if (e == cudaErrorNotSupported)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: this library was built without MOEK_TRACE (use the trace variant)");
  return cuda_status(e, "trace_read");
}
MOEK_API int moek_trace_clear(void) {
  cudaError_t e = moek::trace_copy_layer(nullptr, 0, 1);
  if (e == cudaErrorNotSupported)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: this library was built without MOEK_TRACE (use the trace variant)");
  if (e == cudaSuccess) e = moek::trace_copy_prefill(nullptr, 0, 1);
  if (e == cudaSuccess) e = moek::trace_copy_ep(nullptr, 0, 1);
  return cuda_status(e, "trace_clear");
}

MOEK_API int moek_set_wait_timeout_ns(uint64_t ns) {
  if (ns == 0) return fail(MOEK_ERR_ARG, "moek_b200: the wait timeout must be positive");
  g_timeout_ns = ns;
  return MOEK_OK;
}

MOEK_API int moek_align_workspace_bytes(int64_t numel, int32_t num_experts, size_t* bytes) {
  if (!bytes || numel < 0 || num_experts <= 0) return fail(MOEK_ERR_ARG, "moek_b200: bad align workspace query");
  *bytes = moek::align_workspace_bytes(numel, num_experts);
  return MOEK_OK;
}

MOEK_API int moek_align(const int32_t* topk_ids, int64_t numel, int32_t num_experts, int32_t block_size,
                        int32_t* sorted_ids, int64_t sorted_len, int32_t* expert_ids, int64_t expert_len,
                        int32_t* num_post_pad, void* workspace, size_t workspace_bytes, void* stream) {
  if (numel < 0 || num_experts <= 0 || block_size <= 0)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_align needs numel >= 0, num_experts > 0, block_size > 0");
  if (moek::align_smem_one(num_experts) > 220 * 1024)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: moe_align supports up to 1600 experts (got %d)", num_experts);
  int64_t need = numel + (int64_t)num_experts * (block_size - 1);
  if (numel < num_experts) need = std::min<int64_t>(need, numel * block_size);
  if (sorted_len < need || expert_len < (need + block_size - 1) / block_size)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_align outputs too small (sorted %lld < %lld or expert_ids %lld)",
                (long long)sorted_len, (long long)need, (long long)expert_len);
  if (numel > INT32_MAX / 2) return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: moe_align numel too large");
  if ((sorted_len && !sorted_ids) || (expert_len && !expert_ids) || !num_post_pad || (numel && !topk_ids))
    return fail(MOEK_ERR_ARG, "moek_b200: moe_align null pointer");
  const size_t ws = moek::align_workspace_bytes(numel, num_experts);
  if (ws > workspace_bytes || (ws && !workspace))
    return fail(MOEK_ERR_ARG, "moek_b200: moe_align needs %zu workspace bytes for %lld indices", ws, (long long)numel);
  return cuda_status(moek::launch_align(topk_ids, numel, num_experts, block_size, sorted_ids, sorted_len, expert_ids,
                                        expert_len, num_post_pad, workspace, (cudaStream_t)stream),
                     "moe_align launch");
}

MOEK_API int moek_gemm(const void* A, const void* W, const void* S, const float* G, const int32_t* sorted_ids,
                       int64_t sorted_len, const int32_t* expert_ids, const int32_t* num_post_pad,
                       const float* topk_w, void* out, int32_t num_ids, int32_t N, int32_t K, int32_t E,
                       int32_t top_k, int32_t gate_up, const uint8_t* SP, const int32_t* exc_off,
                       const int32_t* exc_ent, int32_t* cnt, int64_t cnt_len, int32_t mode, int32_t nsplit,
                       float* part, int64_t part_len, int32_t tiled, int32_t block_m, int32_t max_rows,
                       const int32_t* topk_ids, int32_t combine_k, void* stream) {
  if (num_ids == 0) return MOEK_OK;  // empty batch
  if (num_ids < 0 || N <= 0 || K <= 0 || E <= 0 || block_m <= 0)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_gemm bad sizes (num_ids %d, N %d, K %d, E %d, block %d)", num_ids, N,
                K, E, block_m);
  if (K % 128 || N % 256 || (gate_up && (N / 2) % 128))
    return fail(MOEK_ERR_ARG, "moek_b200: moe_gemm needs K %% 128 == 0 and N %% 256 == 0 (got N %d, K %d)", N, K);
  if (S) return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: plain (unpacked) scales are not supported; pass packed SP");
  if (!tiled) return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: weights must be in moek_b200's tiled layout");
  if (!A || !W || !G || !sorted_ids || !expert_ids || !num_post_pad || !SP || !exc_off || !exc_ent)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_gemm null pointer");
  if (!gate_up && top_k != 1) return fail(MOEK_ERR_ARG, "moek_b200: down reads one activation row per id (top_k 1)");
  if (top_k <= 0) return fail(MOEK_ERR_ARG, "moek_b200: top_k must be positive");
  if (mode < 0 || mode > 5)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: moe_gemm mode %d is not available in this build (0-5)", mode);
  // tcgen05 path, whole K per unit, direct epilogue. 0/1: the reference's output contract (gate_up: act to out; down:
  // bf16 rows bf16(topk_w * sum) to out); 4: down writes fp32 rows to part; 5: as 4 with act in sorted order.
  const bool tc = mode == 0 || mode == 1 || mode == 4 || mode == 5;
  if (tc) {
    const bool kit = mode <= 1;
    if (K / 128 > 32) return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: mode %d supports K <= 4096 (got %d)", mode, K);
    if (nsplit != 1) return fail(MOEK_ERR_ARG, "moek_b200: mode %d takes whole K per unit (nsplit 1, got %d)", mode,
                                 nsplit);
    if (block_m > moek::prefill_block_m())
      return fail(MOEK_ERR_ARG, "moek_b200: mode %d takes moe_align blocks of <= %d rows (got %d)", mode,
                  moek::prefill_block_m(), block_m);
    if (gate_up && !out) return fail(MOEK_ERR_ARG, "moek_b200: mode %d gate_up writes act to out", mode);
    if (!gate_up && kit && (!topk_w || !out))
      return fail(MOEK_ERR_ARG, "moek_b200: mode %d down writes bf16(topk_w * sum) rows to out and needs topk_w",
                  mode);
    if (!gate_up && !kit && (!topk_w || !part || part_len < (int64_t)num_ids * N))
      return fail(MOEK_ERR_ARG, "moek_b200: mode %d down writes fp32 rows to part (num_ids * N floats) and needs "
                                "topk_w", mode);
    if (!cnt || cnt_len < 1) return fail(MOEK_ERR_ARG, "moek_b200: cnt[0] is the device error word");
    moek::GemmParams p{};
    p.A = static_cast<const __nv_bfloat16*>(A);
    p.W = static_cast<const uint8_t*>(W);
    p.G = G;
    p.sorted_ids = sorted_ids;
    p.expert_ids = expert_ids;
    p.num_post_pad = num_post_pad;
    p.SP = SP;
    p.exc_off = exc_off;
    p.exc_ent = reinterpret_cast<const uint32_t*>(exc_ent);
    p.part = part;
    p.err = cnt;
    p.topk_w = topk_w;
    p.out = out;
    p.timeout_ns = g_timeout_ns;
    p.num_ids = num_ids;
    p.N = N;
    p.K = K;
    p.E = E;
    p.a_div = top_k;
    p.block_m = block_m;
    p.nsplit = 1;
    p.max_blocks = (int)std::min<int64_t>(sorted_len / block_m,
                                          (num_ids + block_m - 1) / block_m + std::min<int64_t>(E, num_ids));
    p.gate_up = gate_up ? 1 : 0;
    p.mode = mode;
    p.sorted_act = mode == 5 ? 1 : 0;
    p.down_bf16 = kit && !gate_up ? 1 : 0;
    // sorted-order down reads A (act) by sorted position: sorted_len rows; otherwise A rows are tokens
    p.a_rows = (p.sorted_act && !gate_up) ? (int)sorted_len : std::max(1, num_ids / top_k);
    return cuda_status(moek::launch_prefill(p, sm_count(), (cudaStream_t)stream), "moe_gemm (tcgen05) launch");
  }
  const int nstage = K / moek::BK;
  if (nsplit < 1 || nstage % nsplit || (nstage / nsplit) % moek::STAGES_PER_RUN)
    return fail(MOEK_ERR_ARG, "moek_b200: nsplit %d must cut K/128 = %d into whole runs", nsplit, K / 128);
  if (K / 128 / nsplit > 32)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: at most 32 packed-scale runs (4096 k) per split (K %d, nsplit %d)",
                K, nsplit);
  const bool fused = mode == 3, direct = fused && nsplit == 1;
  const int64_t part_need = direct ? (gate_up ? 0 : (int64_t)num_ids * N)
                                   : (int64_t)(nsplit + (fused && !gate_up ? 1 : 0)) * num_ids * N;
  if (part_need && (!part || part_len < part_need))
    return fail(MOEK_ERR_ARG, "moek_b200: part needs %lld floats", (long long)part_need);
  if (max_rows <= 0 || max_rows > 96)
    return fail(MOEK_ERR_ARG, "moek_b200: max_rows %d must be in [1, 96]", max_rows);
  const int64_t maxb = std::min<int64_t>(sorted_len / block_m, (num_ids + block_m - 1) / block_m +
                                                                   std::min<int64_t>(E, num_ids));
  const int64_t mtok = combine_k > 0 ? num_ids / combine_k : 0;
  const int64_t cnt_need = fused && !direct ? 1 + maxb * (N / 256) + (gate_up ? 0 : mtok * (N / 256)) : 1;
  if (!cnt || cnt_len < std::max<int64_t>(4, cnt_need))
    return fail(MOEK_ERR_ARG, "moek_b200: cnt needs %lld int32 (error word + split counters, zero-filled)",
                (long long)std::max<int64_t>(4, cnt_need));
  if (fused && gate_up && !out) return fail(MOEK_ERR_ARG, "moek_b200: mode 3 gate_up writes act to out");
  if (fused && !gate_up && (!topk_w || (!direct && (!out || !topk_ids || combine_k <= 0 || num_ids % combine_k))))
    return fail(MOEK_ERR_ARG, "moek_b200: mode 3 down needs topk_w (and out, topk_ids, combine_k when split)");
  moek::GemmParams p{};
  p.A = static_cast<const __nv_bfloat16*>(A);
  p.W = static_cast<const uint8_t*>(W);
  p.G = G;
  p.sorted_ids = sorted_ids;
  p.expert_ids = expert_ids;
  p.num_post_pad = num_post_pad;
  p.SP = SP;
  p.exc_off = exc_off;
  p.exc_ent = reinterpret_cast<const uint32_t*>(exc_ent);
  p.part = part;
  p.err = cnt;
  p.counters = cnt + 1;
  p.topk_ids = topk_ids;
  p.topk_w = topk_w;
  p.out = out;
  p.mode = mode;
  p.combine_k = combine_k;
  p.timeout_ns = g_timeout_ns;
  p.num_ids = num_ids;
  p.N = N;
  p.K = K;
  p.E = E;
  p.a_div = top_k;
  p.block_m = block_m;
  p.nsplit = nsplit;
  p.max_blocks = (int)maxb;
  p.gate_up = gate_up ? 1 : 0;
  return cuda_status(moek::launch_decode(p, max_rows, sm_count(), (cudaStream_t)stream), "moe_gemm launch");
}

// --------------------------------------------------------------------------------------------------- router
MOEK_API int moek_router_topk(const void* logits, int32_t logits_bf16, int32_t M, int32_t E, int32_t top_k,
                              int32_t renormalize, int32_t* topk_ids, float* topk_weights,
                              int32_t* token_expert_indices, void* stream) {
  if (M < 0 || E <= 0 || E > 1024 || top_k <= 0 || top_k > 32 || top_k > E)
    return fail(MOEK_ERR_ARG, "moek_b200: router needs 0 < top_k <= min(32, E) and E <= 1024 (M %d, E %d, top_k %d)",
                M, E, top_k);
  if (M && (!logits || !topk_ids || !topk_weights)) return fail(MOEK_ERR_ARG, "moek_b200: router null pointer");
  return cuda_status(moek::launch_router_topk(logits, logits_bf16 ? 1 : 0, M, E, top_k, renormalize ? 1 : 0,
                                              topk_ids, topk_weights, token_expert_indices, (cudaStream_t)stream),
                     "router launch");
}

// ------------------------------------------------------------------------------------- whole decode layer
// Persistent int32 state of moek_moe_layer: [epoch, barrier counter, EP arrival counter], then the gate_up record
// flags [record][consumer warp] (stamped with the launch epoch), for the most records a call of this expert
// intermediate size can have (layer_max_records at the largest grid and LAYER_MAXIDS slots). One zeroed state buffer
// serves every call of the layer.
struct LayerLayout {
  int64_t xflag, total;
};
static LayerLayout layer_layout(int32_t, int32_t, int32_t I) {
  LayerLayout l;
  l.xflag = 3;
  l.total = l.xflag + moek::layer_max_records(moek::LAYER_XFLAG_CTAS, moek::LAYER_MAXIDS, I) * moek::LAYER_NCW;
  return l;
}

// Rows per block of the whole-layer kernel (8, 16 or 32): 8 unless set. An expert with more routed slots is cut into
// several blocks, its weights streamed once per block; the 16- and 32-row variants hold their tiles' accumulators and
// activation fragments in more registers and run each 16 KB stage slower (on B200, M = 32 with Zipf routing: 62 us
// per layer with 8-row blocks, 82 us with 16-row blocks).
static int g_layer_rows = 0;
static int layer_block_rows(int) { return g_layer_rows ? g_layer_rows : 8; }
static int64_t layer_grid_bound() { return std::min<int64_t>(2 * (int64_t)sm_count(), moek::LAYER_XFLAG_CTAS); }
// Workspace: the gate_up partial records [records][block rows][256] fp32 (record = CTA + pair, sized for the most
// pairs num_ids slots can form), then the down partials per k-slice [I / 128, num_ids, H] fp32.
static int64_t layer_rec_bytes(int64_t num_ids, int32_t I, int M) {
  return moek::layer_max_records(layer_grid_bound(), num_ids, I) * layer_block_rows(M) * moek::ITEM_COLS * 4;
}
static int64_t layer_ws_bytes(int64_t num_ids, int32_t H, int32_t I, int M) {
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  return up(layer_rec_bytes(num_ids, I, M)) + up((int64_t)(I / 128) * num_ids * H * 4);
}

MOEK_API int moek_layer_state_ints(int32_t num_experts, int32_t H, int32_t I, int64_t* n) {
  if (!n || num_experts <= 0 || H <= 0 || I <= 0) return fail(MOEK_ERR_ARG, "moek_b200: bad layer state query");
  *n = layer_layout(num_experts, H, I).total;
  return MOEK_OK;
}

MOEK_API int moek_layer_workspace_bytes(int32_t M, int32_t top_k, int32_t H, int32_t I, int32_t nsplit_gate,
                                        int32_t nsplit_down, int32_t rows_out, size_t* bytes) {
  if (!bytes || M < 0 || top_k <= 0 || H <= 0 || I <= 0 || nsplit_gate < 1 || nsplit_down < 1)
    return fail(MOEK_ERR_ARG, "moek_b200: bad layer workspace query");
  *bytes = (size_t)layer_ws_bytes((int64_t)M * top_k, H, I, M);
  return MOEK_OK;
}

MOEK_API int moek_set_layer_block_rows(int32_t rows) {
  if (rows != 0 && rows != 8 && rows != 16 && rows != 32)
    return fail(MOEK_ERR_ARG, "moek_b200: layer block rows must be 8, 16, 32 or 0 (automatic), got %d", rows);
  g_layer_rows = rows;
  return MOEK_OK;
}
// Kept for callers of the earlier unit plan: the stream-K plan cuts every CTA's ranges at stage granularity, so
// there is no tail to split.
MOEK_API int moek_set_layer_tail_split(int32_t) { return MOEK_OK; }
// Whether the whole-layer kernel is launched as a cooperative grid (default on): down units wait for the gate_up
// records of other CTAs and the grid barrier waits for every CTA, so every CTA must be resident at once; a
// cooperative launch makes the runtime guarantee it.
static int g_layer_coop = 1;
MOEK_API int moek_set_layer_cooperative(int32_t on) {
  g_layer_coop = on ? 1 : 0;
  return MOEK_OK;
}
// Checks and parameters shared by moek_moe_layer and moek_moe_layer_p2p (rows_ws: the fp32 slot rows live in the
// workspace, i.e. the caller does not take them).
static int layer_params(moek::LayerParams& p, const void* x, int32_t M, int32_t H, int32_t I, int32_t E,
                        const int32_t* topk_ids, const float* topk_w, int32_t top_k, const void* w13,
                        const uint8_t* sp13, const float* g13, const int32_t* exc_off13, const int32_t* exc_ent13,
                        const void* w2, const uint8_t* sp2, const float* g2, const int32_t* exc_off2,
                        const int32_t* exc_ent2, int32_t nsplit_gate, int32_t nsplit_down, void* workspace,
                        size_t workspace_bytes, int32_t* state, int64_t state_ints, int32_t* err, bool rows_ws,
                        bool from_logits = false) {
  if (M < 0 || top_k <= 0 || top_k > 32 || E <= 0 || H <= 0 || I <= 0)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer bad sizes (M %d, top_k %d, E %d, H %d, I %d)", M, top_k, E, H, I);
  const int64_t num_ids = (int64_t)M * top_k;
  if (num_ids > moek::LAYER_MAXIDS)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: moe_layer serves decode batches of <= %d routed slots (got M %d, "
                                      "top_k %d)", moek::LAYER_MAXIDS, M, top_k);
  if (H % 256 || I % 128 || H / 128 > 32 || I / 128 > 32)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer needs H %% 256 == 0, I %% 128 == 0, H and I <= 4096 (H %d, I %d)",
                H, I);
  const int nst1 = H / 128, nst2 = I / 128;  // the kernel's stages: one 128-k packed-scale run pair each
  if (nsplit_gate < 1 || nst1 % nsplit_gate || nsplit_down < 1 || nst2 % nsplit_down)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer k-splits (%d, %d) must cut H/128 = %d and I/128 = %d into whole "
                              "runs", nsplit_gate, nsplit_down, H / 128, I / 128);
  if (!x || (!from_logits && (!topk_ids || !topk_w)) || !w13 || !sp13 || !g13 || !exc_off13 || !exc_ent13 || !w2 ||
      !sp2 || !g2 ||
      !exc_off2 || !exc_ent2 || !state || !err)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer null pointer");
  const LayerLayout lay = layer_layout(E, H, I);
  if (state_ints < lay.total)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer state needs %lld int32 (zeroed once)", (long long)lay.total);
  const int64_t ws = layer_ws_bytes(num_ids, H, I, M);
  if ((int64_t)workspace_bytes < ws || !workspace)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer needs %lld workspace bytes", (long long)ws);
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  uint8_t* wp = static_cast<uint8_t*>(workspace);
  p = moek::LayerParams{};
  p.xpart = reinterpret_cast<float*>(wp);
  wp += up(layer_rec_bytes(num_ids, I, M));
  p.max_records = (int)moek::layer_max_records(layer_grid_bound(), num_ids, I);
  p.part2 = reinterpret_cast<float*>(wp);
  const moek::LayerMat m1{static_cast<const uint8_t*>(w13), sp13, g13, exc_off13,
                          reinterpret_cast<const uint32_t*>(exc_ent13), 2 * I, H, 2 * I / 256, nst1};
  const moek::LayerMat m2{static_cast<const uint8_t*>(w2), sp2, g2, exc_off2,
                          reinterpret_cast<const uint32_t*>(exc_ent2), H, I, H / 256, nst2};
  p.m[0] = m1;
  p.m[1] = m2;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ids = topk_ids;
  p.tw = topk_w;
  p.ctr = state;
  p.err = err;
  p.timeout_ns = g_timeout_ns;
  p.M = M;
  p.top_k = top_k;
  p.num_ids = (int)num_ids;
  p.E = E;
  p.H = H;
  p.I = I;
  p.off_epoch = 0;
  p.off_done = 1;
  p.off_ep = 2;
  p.off_xflag = (int)lay.xflag;
  return MOEK_OK;
}

MOEK_API int moek_moe_layer(const void* x, int32_t M, int32_t H, int32_t I, int32_t E, const int32_t* topk_ids,
                            const float* topk_w, int32_t top_k, const void* w13, const uint8_t* sp13,
                            const float* g13, const int32_t* exc_off13, const int32_t* exc_ent13, const void* w2,
                            const uint8_t* sp2, const float* g2, const int32_t* exc_off2, const int32_t* exc_ent2,
                            int32_t nsplit_gate, int32_t nsplit_down, void* workspace, size_t workspace_bytes,
                            int32_t* state, int64_t state_ints, int32_t* err, void* out, float* out_rows,
                            void* stream) {
  if (M == 0) return MOEK_OK;
  moek::LayerParams p;
  if (int rc = layer_params(p, x, M, H, I, E, topk_ids, topk_w, top_k, w13, sp13, g13, exc_off13, exc_ent13, w2, sp2,
                            g2, exc_off2, exc_ent2, nsplit_gate, nsplit_down, workspace, workspace_bytes, state,
                            state_ints, err, out != nullptr))
    return rc;
  if (!out && !out_rows) return fail(MOEK_ERR_ARG, "moek_b200: moe_layer null pointer");
  if (out && out_rows) return fail(MOEK_ERR_ARG, "moek_b200: moe_layer writes either out (bf16 sums) or out_rows");
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_rows = out_rows;
  return cuda_status(moek::launch_layer(p, layer_block_rows(M), sm_count(), g_layer_coop, (cudaStream_t)stream),
                     "moe_layer launch");
}

MOEK_API int moek_moe_layer_logits(const void* x, int32_t M, int32_t H, int32_t I, int32_t E, const void* logits,
                                   int32_t logits_bf16, int32_t top_k, int32_t renormalize, int32_t* topk_ids_out,
                                   float* topk_w_out, const void* w13, const uint8_t* sp13, const float* g13,
                                   const int32_t* exc_off13, const int32_t* exc_ent13, const void* w2,
                                   const uint8_t* sp2, const float* g2, const int32_t* exc_off2,
                                   const int32_t* exc_ent2, int32_t nsplit_gate, int32_t nsplit_down, void* workspace,
                                   size_t workspace_bytes, int32_t* state, int64_t state_ints, int32_t* err, void* out,
                                   void* stream) {
  if (M == 0) return MOEK_OK;
  if (E > 512 || top_k > E)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: the layer's fused router takes E <= 512 and top_k <= E (E %d, top_k "
                                      "%d); route with moek_router_topk and call moek_moe_layer", E, top_k);
  if (!logits || !out) return fail(MOEK_ERR_ARG, "moek_b200: moe_layer_logits null pointer");
  moek::LayerParams p;
  if (int rc = layer_params(p, x, M, H, I, E, nullptr, nullptr, top_k, w13, sp13, g13, exc_off13, exc_ent13, w2, sp2,
                            g2, exc_off2, exc_ent2, nsplit_gate, nsplit_down, workspace, workspace_bytes, state,
                            state_ints, err, true, true))
    return rc;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.logits = logits;
  p.logits_bf16 = logits_bf16 ? 1 : 0;
  p.renorm = renormalize ? 1 : 0;
  p.ids_out = topk_ids_out;
  p.w_out = topk_w_out;
  return cuda_status(moek::launch_layer(p, layer_block_rows(M), sm_count(), g_layer_coop, (cudaStream_t)stream),
                     "moe_layer_logits launch");
}

// ----------------------------------------------------------------------------- load-time weight preparation
static int prep_shape(int32_t E, int32_t N, int32_t K, int32_t gate_up) {
  if (E <= 0 || N <= 0 || K <= 0 || K % 128 || N % 256 || (gate_up && (N / 2) % 128))
    return fail(MOEK_ERR_ARG, "moek_b200: prep needs K %% 128 == 0, N %% 256 == 0 (and N/2 %% 128 == 0 for gate_up) "
                              "(E %d, N %d, K %d)", E, N, K);
  return MOEK_OK;
}
static int64_t prep_keys(int32_t E, int32_t N, int32_t K) { return (int64_t)E * (N / 256) * (K / 128); }
static int64_t prep_ws_bytes(int32_t E, int32_t N, int32_t K) {
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  return up(prep_keys(E, N, K) * 32 * 4) + up(prep_keys(E, N, K) * 4) + 256;
}

MOEK_API int moek_prep_workspace_bytes(int32_t E, int32_t N, int32_t K, size_t* bytes) {
  if (!bytes) return fail(MOEK_ERR_ARG, "moek_b200: prep workspace query needs an output");
  if (int rc = prep_shape(E, N, K, 0)) return rc;
  *bytes = (size_t)prep_ws_bytes(E, N, K);
  return MOEK_OK;
}

MOEK_API int moek_prep_weights(const uint8_t* codes, int32_t E, int32_t N, int32_t K, int32_t gate_up, int32_t* w_out,
                               void* stream) {
  if (int rc = prep_shape(E, N, K, gate_up)) return rc;
  if (!codes || !w_out || (reinterpret_cast<uintptr_t>(codes) & 3))
    return fail(MOEK_ERR_ARG, "moek_b200: prep_weights null or unaligned pointer");
  return cuda_status(moek::launch_prep_weights(codes, E, N, K, gate_up ? 1 : 0, reinterpret_cast<uint32_t*>(w_out),
                                               (cudaStream_t)stream),
                     "prep_weights launch");
}

MOEK_API int moek_prep_scales(const uint8_t* scales, const float* gs, int32_t E, int32_t N, int32_t K, int32_t gate_up,
                              void* workspace, size_t workspace_bytes, uint8_t* sp_out, float* g_out,
                              int32_t* exc_off_out, float* sf_out, int64_t* n_exc_out, void* stream) {
  if (int rc = prep_shape(E, N, K, gate_up)) return rc;
  if (!scales || !gs || !workspace || !sp_out || !g_out || !exc_off_out || !sf_out || !n_exc_out)
    return fail(MOEK_ERR_ARG, "moek_b200: prep_scales null pointer");
  if ((int64_t)workspace_bytes < prep_ws_bytes(E, N, K))
    return fail(MOEK_ERR_ARG, "moek_b200: prep_scales needs %lld workspace bytes", (long long)prep_ws_bytes(E, N, K));
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  const int64_t nkeys = prep_keys(E, N, K);
  uint8_t* wp = static_cast<uint8_t*>(workspace);
  int* cnt = reinterpret_cast<int*>(wp);
  int* total = reinterpret_cast<int*>(wp + up(nkeys * 32 * 4));
  unsigned int* mx = reinterpret_cast<unsigned int*>(wp + up(nkeys * 32 * 4) + up(nkeys * 4));
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = moek::launch_prep_scale_max(scales, (int64_t)E * N * (K / 16), mx, st);
  unsigned int m = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&m, mx, sizeof(m), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e, "prep_scales scale max");
  // the shared factor: the largest power of two sf with max * 2^7 * sf <= 448 * 2^7 (vllm/.../marlin_utils_fp4.py:
  // 30-60, _nvfp4_compute_scale_factor); 1 when no scale is positive
  float sf = 1.0f;
  if (m) {
    const float v = (m >> 3) ? ldexpf(1.0f + (m & 7) * 0.125f, (int)(m >> 3) - 7) : ldexpf((float)(m & 7), -9);
    const float mxv = v * 128.0f, lim = 448.0f * 128.0f;
    while (mxv < lim && mxv * sf * 2.0f <= lim) sf *= 2.0f;
  }
  e = moek::launch_prep_scales(scales, gs, E, N, K, gate_up ? 1 : 0, sf, sp_out, g_out, cnt, total, exc_off_out, st);
  int n = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&n, exc_off_out + nkeys, sizeof(n), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e, "prep_scales");
  *sf_out = sf;
  *n_exc_out = n;
  return MOEK_OK;
}

MOEK_API int moek_prep_exceptions(const uint8_t* scales, int32_t E, int32_t N, int32_t K, int32_t gate_up, float sf,
                                  const void* workspace, const int32_t* exc_off, int32_t* exc_ent, void* stream) {
  if (int rc = prep_shape(E, N, K, gate_up)) return rc;
  if (!scales || !workspace || !exc_off || !exc_ent)
    return fail(MOEK_ERR_ARG, "moek_b200: prep_exceptions null pointer");
  return cuda_status(moek::launch_prep_exceptions(scales, E, N, K, gate_up ? 1 : 0, sf,
                                                  static_cast<const int*>(workspace), exc_off, exc_ent,
                                                  (cudaStream_t)stream),
                     "prep_exceptions launch");
}

// ------------------------------------------------------------------ the rest of the MoE block (decode sizes)
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

MOEK_API int moek_router_gate(const void* x, int32_t M, int32_t H, const void* w_gate, int32_t E, float* logits,
                              int32_t* err, void* stream) {
  if (M < 0 || M > moek::SHARED_MAXM || H <= 0 || H % 128 || E <= 0 || E % 16)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: router_gate takes decode batches of <= %d tokens, H %% 128 == 0 and "
                                      "E %% 16 == 0 (M %d, H %d, E %d); larger batches are a plain bf16 GEMM",
                moek::SHARED_MAXM, M, H, E);
  if (M == 0) return MOEK_OK;
  if (!x || !w_gate || !logits || !aligned16(x) || !aligned16(w_gate))
    return fail(MOEK_ERR_ARG, "moek_b200: router_gate null or unaligned pointer");
  return cuda_status(moek::launch_router_gate(static_cast<const __nv_bfloat16*>(x), M, H,
                                              static_cast<const __nv_bfloat16*>(w_gate), E, logits, g_timeout_ns,
                                              err, (cudaStream_t)stream),
                     "router_gate launch");
}

static int64_t shared_ws_bytes(int64_t M, int64_t Is) {
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  return up(M * Is * 2) + up(M * 4);
}
MOEK_API int moek_shared_workspace_bytes(int32_t M, int32_t Is, size_t* bytes) {
  if (!bytes || M < 0 || Is < 0) return fail(MOEK_ERR_ARG, "moek_b200: bad shared-expert workspace query");
  *bytes = (size_t)shared_ws_bytes(M, Is);
  return MOEK_OK;
}

MOEK_API int moek_shared_expert(const void* x, int32_t M, int32_t H, int32_t Is, const uint8_t* w_gu,
                                const uint8_t* s_gu, const uint8_t* w_d, const uint8_t* s_d, const void* w_sg,
                                void* workspace, size_t workspace_bytes, float* rows, int32_t* err, void* stream) {
  if (M < 0 || M > moek::SHARED_MAXM || H <= 0 || H % 128 || Is <= 0 || Is % 128)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: shared_expert takes decode batches of <= %d tokens, H %% 128 == 0 "
                                      "and Is %% 128 == 0 (M %d, H %d, Is %d)", moek::SHARED_MAXM, M, H, Is);
  if (M == 0) return MOEK_OK;
  if (!x || !w_gu || !s_gu || !w_d || !s_d || !w_sg || !rows || !workspace || !aligned16(x) || !aligned16(w_gu) ||
      !aligned16(s_gu) || !aligned16(w_d) || !aligned16(s_d))
    return fail(MOEK_ERR_ARG, "moek_b200: shared_expert null or unaligned pointer");
  if ((int64_t)workspace_bytes < shared_ws_bytes(M, Is))
    return fail(MOEK_ERR_ARG, "moek_b200: shared_expert needs %lld workspace bytes", (long long)shared_ws_bytes(M, Is));
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  uint8_t* wp = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* act = reinterpret_cast<__nv_bfloat16*>(wp);
  float* sg = reinterpret_cast<float*>(wp + up((int64_t)M * Is * 2));
  return cuda_status(moek::launch_shared_expert(static_cast<const __nv_bfloat16*>(x), M, H, Is, w_gu, s_gu, w_d, s_d,
                                                static_cast<const __nv_bfloat16*>(w_sg), act, sg, rows, g_timeout_ns,
                                                err, (cudaStream_t)stream),
                     "shared_expert launch");
}

static int64_t block_ws_bytes(int64_t M, int32_t top_k, int32_t H, int32_t I, int32_t E, int32_t Is) {
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  return up(M * E * 4) + up(M * H * 4) + shared_ws_bytes(M, Is) + 2 * up(M * top_k * 4) +
         layer_ws_bytes(M * top_k, H, I, (int)M);
}
MOEK_API int moek_block_workspace_bytes(int32_t M, int32_t top_k, int32_t H, int32_t I, int32_t E, int32_t Is,
                                        size_t* bytes) {
  if (!bytes || M < 0 || top_k <= 0 || H <= 0 || I <= 0 || E <= 0 || Is < 0)
    return fail(MOEK_ERR_ARG, "moek_b200: bad MoE block workspace query");
  *bytes = (size_t)block_ws_bytes(M, top_k, H, I, E, Is);
  return MOEK_OK;
}

MOEK_API int moek_moe_block(const void* x, int32_t M, int32_t H, int32_t I, int32_t E, const void* w_gate,
                            int32_t top_k, int32_t renormalize, int32_t* topk_ids_out, float* topk_w_out,
                            const void* w13, const uint8_t* sp13, const float* g13, const int32_t* exc_off13,
                            const int32_t* exc_ent13, const void* w2, const uint8_t* sp2, const float* g2,
                            const int32_t* exc_off2, const int32_t* exc_ent2, int32_t nsplit_gate,
                            int32_t nsplit_down, int32_t Is, const uint8_t* w_gu, const uint8_t* s_gu,
                            const uint8_t* w_d, const uint8_t* s_d, const void* w_sg, void* workspace,
                            size_t workspace_bytes, int32_t* state, int64_t state_ints, int32_t* err, void* out,
                            void* stream) {
  if (M == 0) return MOEK_OK;
  if (M < 0 || M > moek::SHARED_MAXM || E > 512 || E % 16 || top_k <= 0 || top_k > 32 || top_k > E || Is < 0 ||
      Is % 128 || H % 128)
    return fail(MOEK_ERR_UNSUPPORTED, "moek_b200: moe_block takes decode batches of <= %d tokens, E <= 512 with "
                                      "E %% 16 == 0, 0 < top_k <= min(E, 32), H %% 128 == 0 and Is %% 128 == 0 (M %d, "
                                      "E %d, top_k %d, H %d, Is %d)", moek::SHARED_MAXM, M, E, top_k, H, Is);
  if (!out || !workspace || !x || !w_gate || !aligned16(x) || !aligned16(w_gate) ||
      (Is > 0 && (!w_gu || !s_gu || !w_d || !s_d || !w_sg || !aligned16(w_gu) || !aligned16(s_gu) ||
                  !aligned16(w_d) || !aligned16(s_d))))
    return fail(MOEK_ERR_ARG, "moek_b200: moe_block null or unaligned pointer");
  const int64_t need = block_ws_bytes(M, top_k, H, I, E, Is);
  if ((int64_t)workspace_bytes < need)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_block needs %lld workspace bytes", (long long)need);
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  uint8_t* wp = static_cast<uint8_t*>(workspace);
  float* logits = reinterpret_cast<float*>(wp);
  wp += up((int64_t)M * E * 4);
  float* rows = reinterpret_cast<float*>(wp);
  wp += up((int64_t)M * H * 4);
  __nv_bfloat16* act = reinterpret_cast<__nv_bfloat16*>(wp);
  float* sg = reinterpret_cast<float*>(wp + up((int64_t)M * Is * 2));
  wp += shared_ws_bytes(M, Is);
  int32_t* ids = topk_ids_out ? topk_ids_out : reinterpret_cast<int32_t*>(wp);
  wp += up((int64_t)M * top_k * 4);
  float* tw = topk_w_out ? topk_w_out : reinterpret_cast<float*>(wp);
  wp += up((int64_t)M * top_k * 4);
  moek::LayerParams p;
  if (int rc = layer_params(p, x, M, H, I, E, ids, tw, top_k, w13, sp13, g13, exc_off13, exc_ent13, w2, sp2, g2,
                            exc_off2, exc_ent2, nsplit_gate, nsplit_down, wp,
                            workspace_bytes - (size_t)(wp - static_cast<uint8_t*>(workspace)), state, state_ints, err,
                            true))
    return rc;
  cudaError_t e = moek::launch_block_pre_post(static_cast<const __nv_bfloat16*>(x), M, H, E, Is,
                                              static_cast<const __nv_bfloat16*>(w_gate), logits, w_gu, s_gu, w_d, s_d,
                                              static_cast<const __nv_bfloat16*>(w_sg), act, sg, rows, top_k,
                                              renormalize ? 1 : 0, ids, tw, g_timeout_ns, err, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_status(e, "moe_block gate and shared expert launch");
  if (Is > 0) p.shared = rows;
  p.out = static_cast<__nv_bfloat16*>(out);
  return cuda_status(moek::launch_layer(p, layer_block_rows(M), sm_count(), g_layer_coop, (cudaStream_t)stream),
                     "moe_block launch");
}

// ------------------------------------------------------------------------- EP peer-memory exchange (fixed capacity)
MOEK_API int moek_ipc_malloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(MOEK_ERR_ARG, "moek_b200: ipc_malloc needs a size and an output pointer");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  return cuda_status(e, "ipc_malloc");
}
MOEK_API int moek_ipc_free(void* ptr) { return cuda_status(cudaFree(ptr), "ipc_free"); }
MOEK_API int moek_ipc_handle(void* ptr, void* handle64) {
  if (!ptr || !handle64) return fail(MOEK_ERR_ARG, "moek_b200: ipc_handle null pointer");
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e == cudaSuccess) memcpy(handle64, &h, sizeof(h));
  return cuda_status(e, "ipc_handle");
}
MOEK_API int moek_ipc_open(const void* handle64, void** ptr) {
  if (!ptr || !handle64) return fail(MOEK_ERR_ARG, "moek_b200: ipc_open null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc_open");
}
MOEK_API int moek_ipc_close(void* ptr) { return cuda_status(cudaIpcCloseMemHandle(ptr), "ipc_close"); }

static int p2p_args(moek::P2PArgs& a, const uint64_t* peer, int32_t world, int32_t rank, int32_t mcap, int32_t H,
                    int32_t k, int32_t* err) {
  if (!peer || !err || world < 1 || world > moek::EP_MAX_WORLD || rank < 0 || rank >= world || mcap < 0 ||
      mcap > moek::EP_P2P_MAXM || H <= 0 || H % 8 || H > moek::EP_P2P_MAXH || k <= 0 || k > 32)
    return fail(MOEK_ERR_ARG, "moek_b200: EP peer exchange bad arguments (world %d, rank %d, mcap %d, H %d, k %d)",
                world, rank, mcap, H, k);
  a = moek::P2PArgs{peer, moek::p2p_layout(world, mcap, H, k), world, rank, mcap, H, k, err, g_timeout_ns};
  return MOEK_OK;
}

MOEK_API int moek_ep_p2p_layout(int32_t world, int32_t mcap, int32_t H, int32_t top_k, int64_t* offsets7) {
  if (!offsets7 || world < 1 || world > moek::EP_MAX_WORLD || mcap < 0 || mcap > moek::EP_P2P_MAXM || H <= 0 ||
      H % 8 || H > moek::EP_P2P_MAXH || top_k <= 0 || top_k > 32)
    return fail(MOEK_ERR_ARG, "moek_b200: EP peer exchange layout bad arguments (world %d, mcap %d, H %d, k %d)",
                world, mcap, H, top_k);
  const moek::P2PLayout l = moek::p2p_layout(world, mcap, H, top_k);
  const int64_t v[7] = {l.x, l.ids, l.w, l.back, l.flags, l.ctr, l.total};
  memcpy(offsets7, v, sizeof(v));
  return MOEK_OK;
}

MOEK_API int moek_ep_dispatch_p2p(const uint64_t* peer, int32_t world, int32_t rank, int32_t mcap, int32_t H,
                                  int32_t top_k, const void* x, const int32_t* topk_ids, const float* topk_w, int32_t M,
                                  int32_t num_experts, int32_t* pos, int32_t* err, void* stream) {
  moek::P2PArgs a;
  if (int rc = p2p_args(a, peer, world, rank, mcap, H, top_k, err)) return rc;
  if (M < 0 || M > mcap || num_experts <= 0 || num_experts % world || (M && (!x || !topk_ids || !topk_w || !pos)))
    return fail(MOEK_ERR_ARG, "moek_b200: EP dispatch needs 0 <= M <= mcap and experts split evenly (M %d, E %d)", M,
                num_experts);
  return cuda_status(moek::launch_ep_dispatch_p2p(a, static_cast<const __nv_bfloat16*>(x), topk_ids, topk_w, M,
                                                  num_experts, pos, (cudaStream_t)stream),
                     "ep dispatch launch");
}

MOEK_API int moek_ep_wait(const int32_t* flags, int32_t world, int32_t* err, void* stream) {
  if (!flags || !err || world < 1 || world > moek::EP_MAX_WORLD)
    return fail(MOEK_ERR_ARG, "moek_b200: EP wait bad arguments");
  return cuda_status(moek::launch_ep_wait(flags, world, err, g_timeout_ns, (cudaStream_t)stream), "ep wait launch");
}

MOEK_API int moek_ep_combine_p2p(const uint64_t* peer, int32_t world, int32_t rank, int32_t mcap, int32_t H,
                                 int32_t top_k, const float* rows, int32_t local_experts, int32_t* err, void* stream) {
  moek::P2PArgs a;
  if (int rc = p2p_args(a, peer, world, rank, mcap, H, top_k, err)) return rc;
  if ((mcap && !rows) || local_experts <= 0) return fail(MOEK_ERR_ARG, "moek_b200: EP combine bad arguments");
  return cuda_status(moek::launch_ep_combine_p2p(a, rows, local_experts, (cudaStream_t)stream), "ep combine launch");
}

MOEK_API int moek_ep_unpack_p2p(const uint64_t* peer, int32_t world, int32_t rank, int32_t mcap, int32_t H,
                                int32_t top_k, const int32_t* pos, int32_t M, void* out, int32_t* err, void* stream) {
  moek::P2PArgs a;
  if (int rc = p2p_args(a, peer, world, rank, mcap, H, top_k, err)) return rc;
  if (M < 0 || M > mcap || (M && (!pos || !out))) return fail(MOEK_ERR_ARG, "moek_b200: EP unpack bad arguments");
  return cuda_status(moek::launch_ep_unpack_p2p(a, pos, M, static_cast<__nv_bfloat16*>(out), (cudaStream_t)stream),
                     "ep unpack launch");
}

// The receive side of the peer exchange in the whole-layer kernel's parameters (moek_moe_layer_p2p, moek_moe_layer_ep).
static int layer_p2p_params(moek::LayerParams& p, moek::P2PArgs& a, const uint64_t* peer, const void* own,
                            int32_t world, int32_t rank, int32_t mcap, int32_t H, int32_t I, int32_t local_experts,
                            int32_t top_k, const void* w13, const uint8_t* sp13, const float* g13,
                            const int32_t* exc_off13, const int32_t* exc_ent13, const void* w2, const uint8_t* sp2,
                            const float* g2, const int32_t* exc_off2, const int32_t* exc_ent2, int32_t nsplit_gate,
                            int32_t nsplit_down, void* workspace, size_t workspace_bytes, int32_t* state,
                            int64_t state_ints, int32_t* err) {
  if (int rc = p2p_args(a, peer, world, rank, mcap, H, top_k, err)) return rc;
  if (!own) return fail(MOEK_ERR_ARG, "moek_b200: moe_layer_p2p needs this rank's exchange block");
  const int32_t R = world * mcap;
  if (R == 0) return fail(MOEK_ERR_ARG, "moek_b200: moe_layer_p2p needs mcap > 0");
  const uint8_t* blk = static_cast<const uint8_t*>(own);
  if (int rc = layer_params(p, blk + a.lay.x, R, H, I, local_experts, reinterpret_cast<const int32_t*>(blk + a.lay.ids),
                            reinterpret_cast<const float*>(blk + a.lay.w), top_k, w13, sp13, g13, exc_off13, exc_ent13,
                            w2, sp2, g2, exc_off2, exc_ent2, nsplit_gate, nsplit_down, workspace, workspace_bytes,
                            state, state_ints, err, true))
    return rc;
  p.ep_peer = peer;
  p.ep_recv_flags = reinterpret_cast<const int*>(blk + a.lay.flags);
  p.ep_call = reinterpret_cast<const int*>(blk + a.lay.ctr) + 2 * world;
  p.ep_back_off = a.lay.back;
  p.ep_flags_off = a.lay.flags;
  p.ep_world = world;
  p.ep_rank = rank;
  p.ep_mcap = mcap;
  return MOEK_OK;
}

MOEK_API int moek_moe_layer_p2p(const uint64_t* peer, const void* own, int32_t world, int32_t rank, int32_t mcap,
                                int32_t H, int32_t I, int32_t local_experts, int32_t top_k, const void* w13,
                                const uint8_t* sp13, const float* g13, const int32_t* exc_off13,
                                const int32_t* exc_ent13, const void* w2, const uint8_t* sp2, const float* g2,
                                const int32_t* exc_off2, const int32_t* exc_ent2, int32_t nsplit_gate,
                                int32_t nsplit_down, void* workspace, size_t workspace_bytes, int32_t* state,
                                int64_t state_ints, int32_t* err, void* stream) {
  moek::P2PArgs a;
  moek::LayerParams p;
  if (int rc = layer_p2p_params(p, a, peer, own, world, rank, mcap, H, I, local_experts, top_k, w13, sp13, g13,
                                exc_off13, exc_ent13, w2, sp2, g2, exc_off2, exc_ent2, nsplit_gate, nsplit_down,
                                workspace, workspace_bytes, state, state_ints, err))
    return rc;
  return cuda_status(moek::launch_layer(p, layer_block_rows(world * mcap), sm_count(), g_layer_coop,
                                        (cudaStream_t)stream),
                     "moe_layer_p2p launch");
}

MOEK_API int moek_moe_layer_ep(const uint64_t* peer, const void* own, int32_t world, int32_t rank, int32_t mcap,
                               int32_t H, int32_t I, int32_t num_experts, int32_t top_k, const void* x,
                               const int32_t* topk_ids, const float* topk_w, int32_t M, int32_t* pos, void* out,
                               const void* w13, const uint8_t* sp13, const float* g13, const int32_t* exc_off13,
                               const int32_t* exc_ent13, const void* w2, const uint8_t* sp2, const float* g2,
                               const int32_t* exc_off2, const int32_t* exc_ent2, int32_t nsplit_gate,
                               int32_t nsplit_down, void* workspace, size_t workspace_bytes, int32_t* state,
                               int64_t state_ints, int32_t* err, void* stream) {
  if (world < 1 || num_experts <= 0 || num_experts % world)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer_ep needs the experts split evenly (E %d, world %d)", num_experts,
                world);
  if (M < 0 || M > mcap || (M && (!x || !topk_ids || !topk_w || !pos || !out)))
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer_ep needs 0 <= M <= mcap (M %d, mcap %d) and its buffers", M, mcap);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(MOEK_ERR_ARG, "moek_b200: moe_layer_ep needs 16-byte aligned x and out");
  moek::P2PArgs a;
  moek::LayerParams p;
  if (int rc = layer_p2p_params(p, a, peer, own, world, rank, mcap, H, I, num_experts / world, top_k, w13, sp13, g13,
                                exc_off13, exc_ent13, w2, sp2, g2, exc_off2, exc_ent2, nsplit_gate, nsplit_down,
                                workspace, workspace_bytes, state, state_ints, err))
    return rc;
  p.ep_q = a;
  p.ep_x = static_cast<const uint4*>(x);
  p.ep_ids = topk_ids;
  p.ep_w = topk_w;
  p.ep_pos = pos;
  p.ep_out = static_cast<__nv_bfloat16*>(out);
  p.ep_M = M;
  p.ep_E = num_experts;
  return cuda_status(moek::launch_layer(p, layer_block_rows(world * mcap), sm_count(), g_layer_coop,
                                        (cudaStream_t)stream),
                     "moe_layer_ep launch");
}

MOEK_API int moek_split_epilogue(const float* part, int32_t nsplit, int32_t num_ids, int32_t N, int32_t gate_up,
                                 const float* topk_w, int32_t top_k, void* out, int32_t out_kind, void* stream) {
  if (num_ids == 0) return MOEK_OK;
  if (!part || !out || nsplit < 1 || num_ids < 0 || N <= 0 || (N & 1))
    return fail(MOEK_ERR_ARG, "moek_b200: split epilogue bad arguments");
  cudaStream_t st = (cudaStream_t)stream;
  if (gate_up) {
    return cuda_status(moek::launch_gate_epilogue(part, nsplit, num_ids, N, static_cast<__nv_bfloat16*>(out), st),
                       "gate epilogue");
  }
  if (!topk_w) return fail(MOEK_ERR_ARG, "moek_b200: down epilogue needs the router weights");
  switch (out_kind) {
    case 1:
      return cuda_status(moek::launch_down_rows(part, nsplit, num_ids, N, topk_w, static_cast<float*>(out), st),
                         "down rows epilogue");
    case 2:
      if (top_k <= 0 || num_ids % top_k) return fail(MOEK_ERR_ARG, "moek_b200: num_ids must be a multiple of top_k");
      return cuda_status(moek::launch_down_combine(part, nsplit, num_ids, N, top_k, topk_w,
                                                   static_cast<__nv_bfloat16*>(out), st),
                         "down combine epilogue");
    default:
      return fail(MOEK_ERR_ARG, "moek_b200: down out_kind %d (1 = fp32 rows, 2 = combined)", out_kind);
  }
}

MOEK_API int moek_combine(const void* rows, int32_t rows_fp32, void* out, int32_t m, int32_t N, int32_t top_k,
                          void* stream) {
  if (m == 0) return MOEK_OK;
  if (!rows || !out || m < 0 || N <= 0 || top_k <= 0) return fail(MOEK_ERR_ARG, "moek_b200: combine bad arguments");
  cudaStream_t st = (cudaStream_t)stream;
  if (rows_fp32)
    return cuda_status(moek::launch_combine_f32(static_cast<const float*>(rows), m, N, top_k,
                                                static_cast<__nv_bfloat16*>(out), st),
                       "combine");
  return cuda_status(moek::launch_combine_bf16(static_cast<const __nv_bfloat16*>(rows), m, N, top_k,
                                               static_cast<__nv_bfloat16*>(out), st),
                     "combine");
}

MOEK_API int moek_combine_routed(const float* rows, const int32_t* topk_ids, int32_t E, void* out, int32_t m,
                                 int32_t N, int32_t top_k, void* stream) {
  if (m == 0) return MOEK_OK;
  if (!rows || !topk_ids || !out || m < 0 || N <= 0 || top_k <= 0 || E <= 0)
    return fail(MOEK_ERR_ARG, "moek_b200: routed combine bad arguments");
  return cuda_status(moek::launch_combine_routed(rows, topk_ids, E, m, N, top_k, static_cast<__nv_bfloat16*>(out),
                                                 (cudaStream_t)stream),
                     "routed combine");
}

// ------------------------------------------------------------------------------------------- expert parallel
static int ep_world_ok(int32_t E, int32_t world) {
  if (world < 1 || world > moek::EP_MAX_WORLD)
    return fail(MOEK_ERR_ARG, "moek_b200: EP world size %d outside [1, %d]", world, moek::EP_MAX_WORLD);
  if (E <= 0 || E % world)
    return fail(MOEK_ERR_ARG, "moek_b200: %d experts do not split evenly over %d ranks", E, world);
  return MOEK_OK;
}

MOEK_API int moek_ep_plan(const int32_t* topk_ids, int32_t M, int32_t top_k, int32_t num_experts, int32_t world,
                          int32_t* pos, int32_t* counts, int32_t* offsets, void* stream) {
  if (int rc = ep_world_ok(num_experts, world)) return rc;
  if (M < 0 || top_k <= 0 || !counts || !offsets || (M > 0 && (!topk_ids || !pos)))
    return fail(MOEK_ERR_ARG, "moek_b200: ep_plan bad arguments");
  return cuda_status(moek::launch_ep_plan(topk_ids, M, top_k, num_experts, world, pos, counts, offsets,
                                          (cudaStream_t)stream),
                     "ep_plan");
}

MOEK_API int moek_ep_pack(const void* x, const int32_t* topk_ids, const float* topk_w, const int32_t* pos,
                          const int32_t* offsets, const int32_t* counts, int32_t fill, int32_t M, int32_t H,
                          int32_t top_k, int32_t num_experts, int32_t world, void* send_x, int64_t x_stride,
                          int32_t* send_meta, int64_t meta_stride, void* stream) {
  if (int rc = ep_world_ok(num_experts, world)) return rc;
  if (M == 0 && !fill) return MOEK_OK;
  if (M < 0 || H <= 0 || H % 8 || top_k <= 0 || top_k > 256 || !pos || !offsets || !send_x || !send_meta ||
      x_stride < H || x_stride % 8 || meta_stride < 2 * top_k || (M > 0 && (!x || !topk_ids || !topk_w)) ||
      (fill && !counts))
    return fail(MOEK_ERR_ARG, "moek_b200: ep_pack bad arguments (H and the row stride must be multiples of 8)");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(send_x) % 16 ||
      reinterpret_cast<uintptr_t>(send_meta) % 4)
    return fail(MOEK_ERR_ARG, "moek_b200: ep_pack rows must be 16-byte aligned");
  return cuda_status(moek::launch_ep_pack(static_cast<const __nv_bfloat16*>(x), topk_ids, topk_w, pos, offsets, counts,
                                          fill ? 1 : 0, M, H, top_k, num_experts, world,
                                          static_cast<__nv_bfloat16*>(send_x), x_stride, send_meta, meta_stride,
                                          (cudaStream_t)stream),
                     "ep_pack");
}

MOEK_API int moek_ep_partial(const float* rows, const int32_t* meta, int64_t meta_stride, int32_t local_experts,
                             int32_t R, int32_t N, int32_t top_k, float* out, void* stream) {
  if (R == 0) return MOEK_OK;
  if (R < 0 || N <= 0 || top_k <= 0 || local_experts <= 0 || !rows || !meta || !out || meta_stride < top_k)
    return fail(MOEK_ERR_ARG, "moek_b200: ep_partial bad arguments");
  return cuda_status(moek::launch_ep_partial(rows, meta, meta_stride, local_experts, R, N, top_k, out,
                                             (cudaStream_t)stream),
                     "ep_partial");
}

MOEK_API int moek_ep_unpack(const float* back, const int32_t* pos, const int32_t* offsets, int32_t M, int32_t H,
                            int32_t world, void* out, void* stream) {
  if (M == 0) return MOEK_OK;
  if (M < 0 || H <= 0 || world < 1 || world > moek::EP_MAX_WORLD || !pos || !offsets || !out)
    return fail(MOEK_ERR_ARG, "moek_b200: ep_unpack bad arguments");
  return cuda_status(moek::launch_ep_unpack(back, pos, offsets, M, H, world, static_cast<__nv_bfloat16*>(out),
                                            (cudaStream_t)stream),
                     "ep_unpack");
}
