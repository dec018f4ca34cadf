/* moek_b200: routed-expert NVFP4-weight / bf16-activation (W4A16) MoE kernels for NVIDIA B200 (sm_100a).
 *
 * C ABI of libmoek_b200.so. Every function takes plain device pointers, element counts and a cudaStream_t (as
 * void*), launches asynchronously on that stream and returns MOEK_OK or an error code; moek_last_error() returns the
 * calling thread's last message. The caller allocates every buffer (the library allocates nothing except through
 * moek_ipc_malloc, the expert-parallel exchange block that must be a whole allocation to be shared). Reference paths
 * are relative to the Alssndr0/qwen38-flash-coder project; "vllm/..." paths point into vLLM's Python sources.
 *
 * Tensor formats (produced at load time by qwen38_flash_coder_b200.prep):
 *   W    int32 [E, K/16, 2N], this build's tiled layout: per (expert, 256-column item, 64-k stage) 8 KB of E2M1
 *        codes (same bytes as the checkpoint's [E, N, K/2], reordered).
 *   SP   uint8 [E, N/256, K/128, 1056]: the kit's packed E4M3 block scales, tiled per item (files/mbx_moek.py:61-172).
 *   exc_off int32 [E * N/256 * K/128 + 1], exc_ent int32 [>= 1]: the packed format's exception lists.
 *   G    fp32 [E]: weight_scale_2 * 2^119 / scale_factor (vllm/.../marlin_utils_fp4.py:134-146,385-386).
 */
#ifndef MOEK_B200_H
#define MOEK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MOEK_OK = 0,
  MOEK_ERR_ARG = 1,         /* bad argument (shape, size, null pointer): nothing was launched */
  MOEK_ERR_CUDA = 2,        /* a CUDA call failed; the message names it */
  MOEK_ERR_UNSUPPORTED = 3  /* a valid request this build does not implement */
};

/* Device-side error codes written to the error word (cnt[0] of moek_gemm); 0 means none. */
enum { MOEK_DEV_TIMEOUT = 1, MOEK_DEV_BAD_EXPERT = 2, MOEK_DEV_TOO_MANY_ROWS = 3, MOEK_DEV_BAD_INPUT = 4 };

/* Last error message of the calling thread (empty if none). No reference counterpart (the reference raised
 * c10::Error from TORCH_CHECK, files/mbx_moek.cu:727-755). */
const char* moek_last_error(void);

/* ABI version of this header (1). */
int moek_version(void);

/* Build flags of the loaded library: bit 0 = MOEK_TRACE (timeline stamps), bit 1 = MOEK_DEBUG_CHECKS (every index
 * taken from an input is range-checked before use; a bad one records MOEK_DEV_BAD_INPUT and the access is skipped).
 * No reference counterpart (the reference's trace flag is a compile-time switch of its kernel, files/mbx_moek.cu:
 * 152-160). */
int moek_build_flags(void);
/* MOEK_TRACE builds: copy the %globaltimer stamps [1024 CTAs][128 slots] (uint64, nanoseconds; 0 = not reached) of the
 * last launches of one kernel family to host memory dst (bytes <= 1 MiB are copied). kind 0: the whole-layer kernel (0
 * start, 1 after the dependent-launch wait, 2 expert-parallel flags seen, 3 routing done, 4 first weight copy issued, 5
 * consumers done, 6 end, 7 unit count, 47 every role done, 51 grid barrier passed, 52 top-k sums written; per unit u <
 * 8 of the CTA: 8 + 3u first stage ready, 9 + 3u last stage done, 10 + 3u finished (gate_up: record published), 32 + u
 * the unit (phase << 28 | block << 16 | item << 8 | first k-stage); the first unit's stages s < 8 in SM clock cycles
 * (clock64): 64 + s consumer warp 0 before its wait, 80 + s data and scales ready, 88 + s done, 96 + s the scale warp
 * sees the weights, 104 + s it publishes the scales, 112 + s the producer issues the copy, 120 + s the act warp issues
 * its copies; the start-up in SM clock cycles: 39 start, 40 keys built, 41 counted, 42 ranked, 43 blocks cut, 44 plan
 * made, 45 published, 53 units counted, 54 the producer's units decoded, 55 their rows published); kind 1: the tcgen05
 * GEMM (0 start, 1 after the wait, 6 end; per unit: 8 + 3u first MMA, 9 + 3u last MMA issued, 10 + 3u accumulator
 * drained); kind 2: the peer-exchange kernels (dispatch: 0 start, 1 destination free, 2 rows written, 3 flag raised;
 * unpack: 8 start, 9 partials ready, 10 done). Other builds return MOEK_ERR_UNSUPPORTED. moek_trace_clear zeroes
 * them. */
int moek_trace_read(int32_t kind, void* dst, size_t bytes);
int moek_trace_clear(void);

/* Bound on every device-side wait (default 2 s). After it a kernel records MOEK_DEV_TIMEOUT and returns instead of
 * hanging. No reference counterpart (its waits are unbounded, files/mbx_moek.cu:87-93). */
int moek_set_wait_timeout_ns(uint64_t ns);

/* Workspace moek_align needs for numel indices (0 when numel <= 1024). */
int moek_align_workspace_bytes(int64_t numel, int32_t num_experts, size_t* bytes);

/* moe_align: replaces vLLM's torch.ops._moe_C.moe_align_block_size as the kit calls it
 * (vllm/model_executor/layers/fused_moe/moe_align_block_size.py:11-103 via vllm/_custom_ops.py:2247-2265; called at
 * files/mbx_moek.py:266 with ignore_invalid_experts=True, expert_map=None).
 * topk_ids int32 [numel] (flattened [M, top_k]) -> sorted_ids int32 [sorted_len >= numel + E*(bs-1), or
 * min(numel*bs, that) when numel < E], expert_ids int32 [expert_len >= ceil(sorted_len/bs)], num_post_pad int32 [1].
 * Indices grouped by expert in ascending expert order, ascending inside an expert, each expert padded to a multiple
 * of block_size with the sentinel numel (also in every entry past num_post_pad); expert_ids is -1 past the last
 * block; ids outside [0, E) are skipped. workspace: moek_align_workspace_bytes() bytes (may be NULL when 0). */
int moek_align(const int32_t* topk_ids, int64_t numel, int32_t num_experts, int32_t block_size, int32_t* sorted_ids,
               int64_t sorted_len, int32_t* expert_ids, int64_t expert_len, int32_t* num_post_pad, void* workspace,
               size_t workspace_bytes, void* stream);

/* moe_align without a workspace argument, for callers that cannot allocate device memory on the path that calls
 * it (a host runtime with a fixed memory plan, or a foreign-language binding that only passes the tensors it already
 * owns). No counterpart in the reference. Same outputs as moek_align. Limits: numel <= 65536, num_experts <= 1024;
 * larger calls are rejected with MOEK_ERR_ARG (use moek_align with a workspace). The scratch it needs for more than
 * 1024 indices is a fixed 512 KiB array inside the library, held on every GPU that loads the library until the
 * process exits, and shared by all calls on that GPU: calls that overlap on the GPU (two streams at once) race on
 * it, so serialise them. It keeps the last call's contents, and nothing in it needs to start at zero (every call
 * writes what it reads). The first call on a device with more than 1024 indices looks up the array's device address
 * (cudaGetSymbolAddress) and caches it; make that first call before any stream capture on that device (calls of up to
 * 1024 indices use no scratch and look nothing up). The cached address belongs to the device's primary context: after
 * cudaDeviceReset on that device, do not call this entry point again in the same process. */
int moek_align_noalloc(const int32_t* topk_ids, int64_t numel, int32_t num_experts, int32_t block_size,
                       int32_t* sorted_ids, int64_t sorted_len, int32_t* expert_ids, int64_t expert_len,
                       int32_t* num_post_pad, void* stream);

/* Grouped GEMM of one routed-expert matrix: replaces the kit's moe_gemm (pybind, files/mbx_moek.cu:714-795) with the
 * same fields: A, W, S, G, sorted_ids, expert_ids, num_post_pad, topk_w, out, top_k, gate_up, SP, exc_off, exc_ent,
 * cnt, mode, nsplit, part, tiled (the reference's stream-k ws and schedule order have no use here).
 *   A       bf16: gate_up: hidden states [M, K] (row id / top_k); down: act [num_ids, K] (row id, top_k = 1).
 *   S       must be NULL (plain Marlin scales go with Marlin's untiled weight layout, which this build does not use);
 *           tiled must be 1.
 *   mode    0, 1: the reference's output contract (files/mbx_moek.cu:620-647; the kit's prefill call,
 *           files/mbx_moek.py:276-283), on this build's tcgen05 path (block_m <= 128, K <= 4096, nsplit 1; the
 *           reference's item-counter and stream-k schedules are one schedule here): gate_up writes act bf16
 *           [num_ids, N/2] = bf16(silu(g) * u) to out; down writes dout bf16 [num_ids, N] = bf16(topk_w[id] * sum)
 *           to out. part is unused.
 *           2: split-k; the kernel writes fp32 partial sums part[nsplit][num_ids][N] (gate_up: gate at column c, up
 *           at N/2 + c) and moek_split_epilogue finishes (the reference's mode 2).
 *           3: the epilogue is fused. nsplit 1: gate_up writes act bf16 [num_ids, N/2] = bf16(silu(g) * u) to out;
 *           down writes fp32 rows topk_w[id] * sum to part [num_ids, N] (finish with moek_combine, or with
 *           moek_combine_routed when some slots are unrouted: their rows are not written). nsplit > 1: the warp
 *           whose arrival completes a (block, item) (counters in cnt[1..]) adds the partials in split
 *           order; gate_up writes act to out; down writes fp32 rows topk_w * sum to part after the partials
 *           (part holds (nsplit + 1) * num_ids * N floats) and the arrival that completes a token's valid slots
 *           writes out bf16 [num_ids/combine_k, N] = their sum in slot order (slots whose topk_ids entry is outside
 *           [0, E) are left out).
 *           4: the tcgen05 path with fp32 rows: gate_up as mode 0; down writes the fp32 rows topk_w[id] * sum to
 *           part [num_ids, N] (finish with moek_combine_routed, which leaves out the unrouted slots' unwritten
 *           rows), out unused.
 *           5: as 4, but act is kept in moe_align's sorted order: gate_up writes act row sorted position (out holds
 *           sorted_len rows) and down reads A by sorted position, one 128-row tile per stage instead of a gather.
 *           Modes 3-5 are this build's own; other values are rejected with MOEK_ERR_UNSUPPORTED.
 *   nsplit  K/64/nsplit must be even (whole packed-scale runs), K/128/nsplit <= 32.
 *   cnt     int32, zero-filled before the first call; cnt[0] is the device error word (MOEK_DEV_*), cnt[1..] the
 *           split counters (mode 3, nsplit > 1: 1 + max_blocks * N/256 entries, down + (num_ids/combine_k) * N/256,
 *           max_blocks = min(sorted_len / block_m, ceil(num_ids / block_m) + min(E, num_ids))), which every
 *           completed launch leaves at zero.
 *   block_m the block size moek_align used; max_rows >= the most valid rows of any block (min(M, block_m) for top-k
 *           routing with distinct experts per token), <= 96.
 * The weights are dequantised exactly as the fp32 oracle does (bench/moek/problem.py:31-38: bf16(e2m1 * s * gs)),
 * products summed in fp32. topk_w, out, topk_ids and combine_k are unused in mode 2. */
int moek_gemm(const void* A, const void* W, const void* S, const float* G, const int32_t* sorted_ids,
              int64_t sorted_len, const int32_t* expert_ids, const int32_t* num_post_pad, const float* topk_w,
              void* out, int32_t num_ids, int32_t N, int32_t K, int32_t E, int32_t top_k, int32_t gate_up,
              const uint8_t* SP, const int32_t* exc_off, const int32_t* exc_ent, int32_t* cnt, int64_t cnt_len,
              int32_t mode, int32_t nsplit, float* part, int64_t part_len, int32_t tiled, int32_t block_m,
              int32_t max_rows, const int32_t* topk_ids, int32_t combine_k, void* stream);

/* Split-k epilogue: replaces the kit's moe_split_epilogue (files/mbx_moek.cu:797-851). Adds the nsplit partials in
 * split order (deterministic), then
 *   gate_up: out = act bf16 [num_ids, N/2] = bf16(silu(g) * u) with g, u the fp32 sums (the oracle's rounding point,
 *            bench/moek/problem.py:63-65);
 *   down, out_kind 1: out = fp32 rows [num_ids, N] = topk_w[id] * sum;
 *   down, out_kind 2: out = bf16 [num_ids/top_k, N] = bf16(sum_j topk_w * sum) over the top_k slots of each token in
 *            slot order: the down epilogue fused with the top-k combine (files/mbx_moek.py:284-289). */
int moek_split_epilogue(const float* part, int32_t nsplit, int32_t num_ids, int32_t N, int32_t gate_up,
                        const float* topk_w, int32_t top_k, void* out, int32_t out_kind, void* stream);

/* Top-k combine: replaces torch.sum(dout.view(-1, top_k, N), 1, out=output) / vLLM's moe_sum (files/mbx_moek.py:
 * 284-289): out bf16 [m, N] = bf16(sum_j rows[t*top_k + j]) in fp32, slot order. rows: fp32 if rows_fp32 else bf16. */
int moek_combine(const void* rows, int32_t rows_fp32, void* out, int32_t m, int32_t N, int32_t top_k, void* stream);

/* Top-k combine over the routed slots: the same sum for routings that leave slots unrouted (an expert map marks the
 * experts it does not hold with -1, vllm/.../fused_moe/moe_align_block_size.py:11-103, and moe_align skips them; the
 * oracle leaves such slots out, bench/moek/problem.py:51-67). out bf16 [m, N] = bf16(sum_j rows[t*top_k + j]) over
 * the slots j whose topk_ids[t*top_k + j] lies in [0, E), in slot order, in fp32; a token with no such slot gets a
 * zero row. The rows of unrouted slots may hold any value (the down GEMM never writes them); with every slot routed
 * the result equals moek_combine's bit for bit. rows fp32 [m * top_k, N]. */
int moek_combine_routed(const float* rows, const int32_t* topk_ids, int32_t E, void* out, int32_t m, int32_t N,
                        int32_t top_k, void* stream);

/* ---- Router. Replaces vLLM's fused_topk with scoring "softmax" (vllm/.../router/fused_topk_router.py:69-108, the
 * topk_softmax op), the gating step in front of the layer (vllm/.../models/qwen3_next.py:158-165): per token t,
 * p = softmax(logits[t]) in fp32, the top_k largest p (the lowest expert index among equal p, largest first) into
 * topk_ids[t, :] and their p into topk_weights[t, :], divided by their sum when renormalize != 0; when
 * token_expert_indices is not NULL it receives j * M + t for slot j. logits: fp32, or bf16 when logits_bf16 != 0,
 * [M, E] row-major; E <= 1024, top_k <= 32. */
int moek_router_topk(const void* logits, int32_t logits_bf16, int32_t M, int32_t E, int32_t top_k,
                     int32_t renormalize, int32_t* topk_ids, float* topk_weights, int32_t* token_expert_indices,
                     void* stream);

/* ---- Whole decode layer in one launch. Replaces, for decode batches, the sequence the kit's forward wrap runs
 * (files/mbx_moek.py:236-289: moe_align, gate_up moe_gemm, split epilogue, down moe_gemm, split epilogue + top-k sum)
 * with one persistent kernel: routing in shared memory; the gate_up stages of every (block, gate_up item) pair cut
 * into equal contiguous ranges, one per CTA, each CTA publishing fp32 partial records; then the down items cut the
 * same way, each CTA forming a pair's act (SwiGLU) from the pair's records before its down items; after a grid
 * barrier, the router-weighted top-k sums. */

/* int32 count of the persistent state: launch epoch, barrier and arrival counters, the gate_up record flags (their
 * number depends on I only; num_experts and H are accepted for the geometry). Zero it once before the first
 * call; every completed call leaves it valid for the next one (after a device error, zero it again). Calls that share
 * a state buffer must be ordered (one stream). */
int moek_layer_state_ints(int32_t num_experts, int32_t H, int32_t I, int64_t* n);

/* Scratch bytes of one call: the fp32 gate_up partial records ((the grid bound 2 x SMs + M * top_k * 2I / 256)
 * records of block-rows x 256 values, block rows as moek_set_layer_block_rows sets them for this M at the time of the
 * query and of the call) and the fp32 down partials per 128-k slice [I / 128, M * top_k, H]. rows_out is accepted for
 * the earlier layout and changes nothing. Contents need not be preserved between calls. */
int moek_layer_workspace_bytes(int32_t M, int32_t top_k, int32_t H, int32_t I, int32_t nsplit_gate,
                               int32_t nsplit_down, int32_t rows_out, size_t* bytes);

/* out bf16 [M, H] = bf16(sum over valid slots j in order of topk_w[t, j] * down_e(bf16(silu(g) * u))) with
 * (g, u) = gate_up_e(x[t]) in fp32, e = topk_ids[t, j] in [0, E) (other ids are not routed; a token with none gets
 * zeros), the weights dequantised as the oracle does (bf16(e2m1 * s * gs)). With out = NULL and out_rows set, the
 * fp32 rows [M * top_k, H] = topk_w * down_e(...) are written instead (rows of unrouted slots are left as they were).
 *   x       bf16 [M, H]; M * top_k <= 512 (decode batches; larger ones take the moek_gemm path).
 *   w13/sp13/g13/exc_off13/exc_ent13  gate_up in the tiled formats above (N = 2I, K = H); w2.. likewise (N = H,
 *           K = I). H % 256 == 0, I % 128 == 0, both <= 4096.
 *   nsplit_gate, nsplit_down  checked as before (whole 128-k runs) and otherwise unused: the kernel cuts the
 *           gate_up stages over the CTAs itself (from the number of blocks and the grid), which changes only the
 *           order of fp32 partial sums; the same routing always gives the same plan and the same bits.
 *   err     int32 device error word (MOEK_DEV_*), zero before the call. */
/* ---- Load-time preparation on the GPU: checkpoint NVFP4 matrices (codes uint8 [E, N, K/2], element 2i in the low
 * nibble; E4M3 block scales [E, N, K/16]; global scales fp32 [E]) into the kernels' formats. Replaces, at model load,
 * vLLM's prepare_nvfp4_moe_layer_for_marlin (vllm/.../marlin_utils_fp4.py:288-386: the Marlin repack and scale
 * processing) plus the kit's codec and tiling (files/mbx_moek.py:61-172), with the same scale bytes. K % 128 == 0,
 * N % 256 == 0 (gate_up: N/2 % 128 == 0). Order: moek_prep_scales (its workspace from moek_prep_workspace_bytes; it
 * synchronises the stream twice to read the matrix's largest scale and the exception count back), then
 * moek_prep_exceptions with the same workspace and an exc_ent of max(1, *n_exc_out) int32; moek_prep_weights any
 * time. */
int moek_prep_workspace_bytes(int32_t E, int32_t N, int32_t K, size_t* bytes);
/* w_out int32 [E, K/16, 2N]: the tiled code words (per (expert, 256-row item, 64-k stage) an 8 KB block). */
int moek_prep_weights(const uint8_t* codes, int32_t E, int32_t N, int32_t K, int32_t gate_up, int32_t* w_out,
                      void* stream);
/* sp_out uint8 [E, N/256, K/128, 1056] (the kit's packed scales, an item's two runs side by side), g_out fp32 [E]
 * (gs * 2^119 / sf), exc_off_out int32 [E * N/256 * K/128 + 1]; *sf_out the shared power-of-two scale factor,
 * *n_exc_out the number of exception entries. */
int moek_prep_scales(const uint8_t* scales, const float* gs, int32_t E, int32_t N, int32_t K, int32_t gate_up,
                     void* workspace, size_t workspace_bytes, uint8_t* sp_out, float* g_out, int32_t* exc_off_out,
                     float* sf_out, int64_t* n_exc_out, void* stream);
/* exc_ent int32 [n_exc]: position | k-group << 16 | scale byte << 24, per (expert, item, run) list in order. */
int moek_prep_exceptions(const uint8_t* scales, int32_t E, int32_t N, int32_t K, int32_t gate_up, float sf,
                         const void* workspace, const int32_t* exc_off, int32_t* exc_ent, void* stream);

/* ---- The rest of the MoE block at decode sizes: the router gate GEMM and the MXFP8 shared expert, whose fp32 rows
 * the whole-layer kernel adds to each token's sum before its one bf16 rounding. They replace, for decode batches, the
 * block's other steps around the routed experts (files/v54/model.py:193-210 subclasses vLLM's
 * Qwen3NextSparseMoeBlock: vllm/model_executor/models/qwen3_next.py:125-131,193 the gate, qwen2_moe.py:114-122 the
 * shared expert with its sigmoid gate; the shared expert is MXFP8 in the kit's checkpoint, README.md:38). */

/* logits fp32 [M, E] = x bf16 [M, H] @ w_gate bf16 [E, H]^T (fp32 sums: eight K slices added in order, the same
 * bits on every call). M <= 64, H % 128 == 0, E % 16 == 0 (else MOEK_ERR_UNSUPPORTED: larger batches are a plain
 * library GEMM). x and w_gate 16-byte aligned. err: the int32 device error word (MOEK_DEV_TIMEOUT if a weight copy's
 * bounded wait ran out; may be NULL). */
int moek_router_gate(const void* x, int32_t M, int32_t H, const void* w_gate, int32_t E, float* logits, int32_t* err,
                     void* stream);

/* Scratch bytes of moek_shared_expert: act bf16 [M, Is] and the expert gate fp32 [M], each rounded up to 256. */
int moek_shared_workspace_bytes(int32_t M, int32_t Is, size_t* bytes);

/* rows fp32 [M, H] = sigmoid(x @ w_sg) * (bf16(silu(g) * u) @ W_d^T), [g | u] = x @ W_gu^T in fp32, with MXFP8
 * weights in the checkpoint layout: w_gu uint8 [2 Is, H] (float8_e4m3fn bytes; gate rows 0..Is-1, then the up rows),
 * s_gu uint8 [2 Is, H / 32] (E8M0 exponents, one per 32 inputs), w_d uint8 [H, Is], s_d uint8 [H, Is / 32]; w_sg
 * bf16 [H] (shared_expert_gate). Dequantisation is exact for scale bytes in [10, 134], the supported range (the
 * Python wrapper rejects others). M <= 64, H % 128 == 0, Is % 128 == 0; x and the weight and scale pointers
 * 16-byte aligned. err as moek_router_gate. */
int moek_shared_expert(const void* x, int32_t M, int32_t H, int32_t Is, const uint8_t* w_gu, const uint8_t* s_gu,
                       const uint8_t* w_d, const uint8_t* s_d, const void* w_sg, void* workspace,
                       size_t workspace_bytes, float* rows, int32_t* err, void* stream);

/* Scratch bytes of moek_moe_block: logits fp32 [M, E], the shared rows fp32 [M, H], the shared expert's scratch,
 * the routing (ids int32 and weights fp32 [M, top_k]) and the whole-layer kernel's workspace. */
int moek_block_workspace_bytes(int32_t M, int32_t top_k, int32_t H, int32_t I, int32_t E, int32_t Is, size_t* bytes);

/* The whole MoE block for a decode batch (M <= 64 tokens, E <= 512, E % 16 == 0, top_k <= 32), three launches chained
 * with programmatic dependent launch: the router gate GEMM beside the shared expert's gate_up (one grid), the shared
 * expert's down beside the routing of the logits (softmax, top_k, renormalised when renormalize != 0; the router
 * kernel's per-token code), then the whole-layer kernel from those ids and weights with the shared rows added:
 * out bf16 [M, H] = bf16(sum over valid slots j in order of topk_w * down_e(...) + shared row). The routed weights and
 * the state as moek_moe_layer; the shared expert's tensors as moek_shared_expert (ignored when Is = 0);
 * topk_ids_out / topk_w_out (may be NULL) receive the routing. No reference counterpart as one call: the reference
 * runs these steps as separate vLLM layers. */
int moek_moe_block(const void* x, int32_t M, int32_t H, int32_t I, int32_t E, const void* w_gate, int32_t top_k,
                   int32_t renormalize, int32_t* topk_ids_out, float* topk_w_out, const void* w13, const uint8_t* sp13,
                   const float* g13, const int32_t* exc_off13, const int32_t* exc_ent13, const void* w2,
                   const uint8_t* sp2, const float* g2, const int32_t* exc_off2, const int32_t* exc_ent2,
                   int32_t nsplit_gate, int32_t nsplit_down, int32_t Is, const uint8_t* w_gu, const uint8_t* s_gu,
                   const uint8_t* w_d, const uint8_t* s_d, const void* w_sg, void* workspace, size_t workspace_bytes,
                   int32_t* state, int64_t state_ints, int32_t* err, void* out, void* stream);

/* Rows per block of the whole-layer kernel: 8, 16 or 32, or 0 (automatic: 8).
 * An expert with more routed slots than that is cut into several blocks, its weights streamed once per block.
 * Process-wide; a tuning knob with no effect on the results. */
int moek_set_layer_block_rows(int32_t rows);
/* Accepted for callers of the earlier unit plan; no effect (the stream-K plan has no tail to split). */
int moek_set_layer_tail_split(int32_t on);
/* Whether the whole-layer kernel is launched as a cooperative grid (on != 0, the default). A CTA's down items wait
 * (bounded) on the gate_up records of other CTAs and every CTA waits at a grid barrier before the top-k sums,
 * so all of its CTAs must be resident at once; a cooperative launch makes the runtime start the grid only when they
 * all are, also while kernels of other streams hold part of the GPU (with on = 0 such a stream could hold CTAs back
 * past the wait bound and the layer would end in MOEK_DEV_TIMEOUT).
 * Process-wide. No reference counterpart (the reference's kernels do not wait across CTAs). */
int moek_set_layer_cooperative(int32_t on);

int moek_moe_layer(const void* x, int32_t M, int32_t H, int32_t I, int32_t E, const int32_t* topk_ids,
                   const float* topk_w, int32_t top_k, const void* w13, const uint8_t* sp13, const float* g13,
                   const int32_t* exc_off13, const int32_t* exc_ent13, const void* w2, const uint8_t* sp2,
                   const float* g2, const int32_t* exc_off2, const int32_t* exc_ent2, int32_t nsplit_gate,
                   int32_t nsplit_down, void* workspace, size_t workspace_bytes, int32_t* state, int64_t state_ints,
                   int32_t* err, void* out, float* out_rows, void* stream);

/* The same layer with the router fused into the kernel: replaces, for decode batches, vLLM's fused_topk (scoring
 * "softmax", vllm/.../router/fused_topk_router.py:69-108) followed by the layer (moek_router_topk then moek_moe_layer:
 * one launch instead of two). Every CTA routes the M tokens itself from logits [M, E] (fp32, or bf16 when
 * logits_bf16 != 0): the same softmax, top_k and renormalisation as moek_router_topk, bit for bit; the ids and
 * weights also go to topk_ids_out / topk_w_out [M, top_k] when those are not NULL. E <= 512; the other arguments as
 * moek_moe_layer (out is required; the workspace as moek_layer_workspace_bytes with rows_out = 0). */
int moek_moe_layer_logits(const void* x, int32_t M, int32_t H, int32_t I, int32_t E, const void* logits,
                          int32_t logits_bf16, int32_t top_k, int32_t renormalize, int32_t* topk_ids_out,
                          float* topk_w_out, const void* w13, const uint8_t* sp13, const float* g13,
                          const int32_t* exc_off13, const int32_t* exc_ent13, const void* w2, const uint8_t* sp2,
                          const float* g2, const int32_t* exc_off2, const int32_t* exc_ent2, int32_t nsplit_gate,
                          int32_t nsplit_down, void* workspace, size_t workspace_bytes, int32_t* state,
                          int64_t state_ints, int32_t* err, void* out, void* stream);

/* ---- Expert parallelism. The reference has none (its hook rejects expert_map, files/mbx_moek.py:248-255); these
 * are the dispatch / combine steps around the same GEMMs when the experts are split contiguously over `world` ranks
 * (rank d owns [d * E/world, (d + 1) * E/world)). The all-to-all transfers are the caller's (NCCL). */

/* Dispatch plan: for tokens t < M and ranks d < world, pos[t * world + d] = position of token t in rank d's send
 * segment (tokens with at least one of their top_k experts on d, ascending t), else -1; counts[d] = rows for d;
 * offsets[0..world] = exclusive prefix of counts. Ids outside [0, num_experts) go nowhere. */
int moek_ep_plan(const int32_t* topk_ids, int32_t M, int32_t top_k, int32_t num_experts, int32_t world,
                 int32_t* pos, int32_t* counts, int32_t* offsets, void* stream);

/* Packs the send buffer: rows bf16 at send_x + row * x_stride (x_stride >= H elements, a multiple of 8; row
 * offsets[d] + pos[t*world + d] = x[t]) and slot metadata int32 at send_meta + row * meta_stride (meta_stride >=
 * 2 * top_k: the slots' expert ids local to d, -1 for slots owned elsewhere, then the router weights as fp32 bits, 0
 * for slots owned elsewhere). Rows and metadata may share one buffer (meta inside each row's tail). With fill != 0
 * the rows offsets[d] + counts[d] .. offsets[d + 1] of each segment (a fixed-capacity layout) get ids -1. */
int moek_ep_pack(const void* x, const int32_t* topk_ids, const float* topk_w, const int32_t* pos,
                 const int32_t* offsets, const int32_t* counts, int32_t fill, int32_t M, int32_t H, int32_t top_k,
                 int32_t num_experts, int32_t world, void* send_x, int64_t x_stride, int32_t* send_meta,
                 int64_t meta_stride, void* stream);

/* Receiving side, after the down GEMM wrote fp32 rows (router weight applied) for the R received rows' slots:
 * out fp32 [R, N] = sum over slots j with 0 <= meta[r * meta_stride + j] < local_experts, slot order, of
 * rows[r * top_k + j]. */
int moek_ep_partial(const float* rows, const int32_t* meta, int64_t meta_stride, int32_t local_experts, int32_t R,
                    int32_t N, int32_t top_k, float* out, void* stream);

/* Source side, after the partial rows came back (back fp32 [offsets[world], H], same order as the send buffer):
 * out bf16 [M, H] = bf16(sum over d = 0..world-1 with pos >= 0 of back[offsets[d] + pos[t*world + d]]). */
int moek_ep_unpack(const float* back, const int32_t* pos, const int32_t* offsets, int32_t M, int32_t H,
                   int32_t world, void* out, void* stream);

/* ---- Expert parallelism over peer memory (the fixed-capacity decode exchange without a collective library; no
 * counterpart in the reference, like the rest of EP). Each rank allocates one exchange block of moek_ep_p2p_layout's
 * total bytes with moek_ipc_malloc (zeroed; a whole cudaMalloc allocation, so that CUDA IPC can share it), shares it
 * with moek_ipc_handle / moek_ipc_open, and passes `peer`, a device array of every rank's block base (its own
 * included). With R = world * mcap rows (segment s = rows [s mcap, (s + 1) mcap), the rows rank s sent),
 * moek_ep_p2p_layout gives the byte offsets of: received rows bf16 [R, H], their local expert ids int32 [R, top_k]
 * (-1: slot owned elsewhere, or unused row), router weights fp32 [R, top_k], this rank's fp32 partials of the
 * received rows [R, H] (segment s: those of rank s's rows, which rank s reads over NVLink), flags int32 [2 world],
 * counters int32 [2 world + 2], and the total. Per layer call, on one stream, every rank runs:
 *   moek_ep_dispatch_p2p (plans the token order itself, writes pos [M, world] for the unpack, and copies rows, ids
 *   and weights straight into the owners' receive segments), then either
 *     moek_moe_layer_p2p (R * top_k <= 512: the whole-layer kernel waits for the receive flags itself, writes each
 *     row's fp32 partial into its own back buffer and raises the senders' flags), or
 *     moek_ep_wait(own flags), the local layer on the receive rows (fp32 slot rows), moek_ep_combine_p2p,
 *   then moek_ep_unpack_p2p (waits for every rank's flag, reads the partials from the owners' back buffers, sums them
 *   in rank order, rounds once to bf16).
 * Or, when R * top_k <= 512, the one launch moek_moe_layer_ep, which runs all three steps in the whole-layer kernel.
 * The flags carry the call number, so they never need resetting and the sequence can be captured in a CUDA graph.
 * Waits are bounded (moek_set_wait_timeout_ns) and record MOEK_DEV_TIMEOUT in err; after one, build the exchange
 * again. mcap <= 1024 tokens per rank and call, H <= 4096. */
int moek_ipc_malloc(size_t bytes, void** ptr);
int moek_ipc_free(void* ptr);
int moek_ipc_handle(void* ptr, void* handle64);
int moek_ipc_open(const void* handle64, void** ptr);
int moek_ipc_close(void* ptr);
/* offsets7: x, ids, w, back, flags, counters, total (bytes). */
int moek_ep_p2p_layout(int32_t world, int32_t mcap, int32_t H, int32_t top_k, int64_t* offsets7);
int moek_ep_dispatch_p2p(const uint64_t* peer, int32_t world, int32_t rank, int32_t mcap, int32_t H, int32_t top_k,
                         const void* x, const int32_t* topk_ids, const float* topk_w, int32_t M, int32_t num_experts,
                         int32_t* pos, int32_t* err, void* stream);
int moek_ep_wait(const int32_t* flags, int32_t world, int32_t* err, void* stream);
int moek_ep_combine_p2p(const uint64_t* peer, int32_t world, int32_t rank, int32_t mcap, int32_t H, int32_t top_k,
                        const float* rows, int32_t local_experts, int32_t* err, void* stream);
int moek_ep_unpack_p2p(const uint64_t* peer, int32_t world, int32_t rank, int32_t mcap, int32_t H, int32_t top_k,
                       const int32_t* pos, int32_t M, void* out, int32_t* err, void* stream);
/* The whole-layer kernel on this rank's receive segments (own = this rank's block), the same arguments as
 * moek_moe_layer otherwise; its rows' fp32 partials go to this rank's back buffer, where the senders read them. */
int moek_moe_layer_p2p(const uint64_t* peer, const void* own, int32_t world, int32_t rank, int32_t mcap, int32_t H,
                       int32_t I, int32_t local_experts, int32_t top_k, const void* w13, const uint8_t* sp13,
                       const float* g13, const int32_t* exc_off13, const int32_t* exc_ent13, const void* w2,
                       const uint8_t* sp2, const float* g2, const int32_t* exc_off2, const int32_t* exc_ent2,
                       int32_t nsplit_gate, int32_t nsplit_down, void* workspace, size_t workspace_bytes,
                       int32_t* state, int64_t state_ints, int32_t* err, void* stream);
/* The whole expert-parallel decode layer in one launch (R * top_k <= 512): the whole-layer kernel dispatches this
 * rank's M <= mcap tokens (x bf16 [M, H], global expert ids topk_ids [M, top_k], router weights topk_w, experts split
 * evenly: rank d owns [d E / world, (d + 1) E / world)) as moek_ep_dispatch_p2p does (pos [M, world] is written), runs
 * the layer on the receive segments as moek_moe_layer_p2p does, and writes out bf16 [M, H] as moek_ep_unpack_p2p
 * does; the same bits as that three-launch sequence. x and out 16-byte aligned. */
int moek_moe_layer_ep(const uint64_t* peer, const void* own, int32_t world, int32_t rank, int32_t mcap, int32_t H,
                      int32_t I, int32_t num_experts, int32_t top_k, const void* x, const int32_t* topk_ids,
                      const float* topk_w, int32_t M, int32_t* pos, void* out, const void* w13, const uint8_t* sp13,
                      const float* g13, const int32_t* exc_off13, const int32_t* exc_ent13, const void* w2,
                      const uint8_t* sp2, const float* g2, const int32_t* exc_off2, const int32_t* exc_ent2,
                      int32_t nsplit_gate, int32_t nsplit_down, void* workspace, size_t workspace_bytes,
                      int32_t* state, int64_t state_ints, int32_t* err, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MOEK_B200_H */
