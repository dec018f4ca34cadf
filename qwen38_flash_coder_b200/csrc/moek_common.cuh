// Shared device helpers for the routed-expert NVFP4 (W4A16) MoE kernels (sm_100a).
//
// Weight decode. A tiled weight word holds 8 E2M1 codes (sign = bit 3) of 8 consecutive k of one output column,
// bit-scattered at load time (prep.CODE_BITS) so that the bf16 pairs come out with few integer ops: codes 0 and 1
// already have their signs at bits 15 / 31 and their three magnitude bits at 8..6 / 24..22, codes 2-3 and 4-5 hold
// that pattern rotated left by 4 and 10 bits (one funnel-shift rotate and one mask each), codes 6-7 hold their
// mantissa bits rotated by 14 and the other bits by 6 (two rotates, two masks). A code's sign at bit 15 and its
// three magnitude bits at 8..6 of a bf16 give exactly e2m1 * 2^-126 (exponent field = the code's exponent, top
// mantissa bit = its mantissa bit; code 1 becomes the subnormal 2^-127). That value D is exact, and the weight the
// reference's oracle uses, bf16(e2m1 * s * gs) with s the E4M3 block scale and gs the expert's fp32 global scale
// (bench/moek/problem.py:31-38), is then rebuilt per pair of codes with two bf16 FMAs:
//     Y  = fp32(s * gs) * 2^126            (once per 16 weights, from the packed scale byte and the global scale)
//     B  = bf16(Y), R = bf16(Y - B)         (B carries 8 bits of Y, R the next 8)
//     w  = bf16(D * B + bf16(D * R))        (D * B is exact inside the FMA; one rounding of the sum)
// which equals bf16(e2m1 * fp32(s * gs)) except when e2m1 * Y lies within 2^-18 (relative) of a bf16 rounding
// midpoint (about 1 weight in 2000 then differs by one bf16 ulp).
//
// Scale bytes. The kit's packed scales hold vLLM's Marlin "S0E5M3" bytes: the high byte of (fp16(s * sf * 2^7) << 1)
// (vllm/.../marlin_utils_fp4.py:53-114), 0 for values below 2. As fp32: bits = (b << 20) + (112 << 23) for b != 0.
// The global scale the kernels receive is G = gs * 2^119 / sf (marlin_utils_fp4.py:134-146,385-386), so
// fp32(S0E5M3(b) * G) = fp32(s * gs) * 2^126 exactly: Y needs one multiply.
//
// Waits. Every spin (mbarrier phase) is bounded by a %globaltimer deadline; on expiry the waiting thread records
// MOEK_DEV_TIMEOUT in the caller's error word and the kernel winds down instead of hanging the GPU.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace moek {

constexpr int BK = 64;                       // k per pipeline stage
constexpr int ITEM_COLS = 256;               // output columns (weight rows) per item
constexpr int STAGE_BYTES = BK * ITEM_COLS / 2;  // 8 KB of packed codes per (item, stage)
constexpr int KG = 8;                        // k-groups of 16 per packed-scale run
constexpr int RUN_BYTES = 16 + KG * 64;      // 528
constexpr int PAIR_BYTES = 2 * RUN_BYTES;    // an item's two runs
constexpr int STAGES_PER_RUN = KG * 16 / BK; // 2

// Device error codes (the caller's error word; 0 = fine)
constexpr int MOEK_DEV_TIMEOUT = 1;
constexpr int MOEK_DEV_BAD_EXPERT = 2;
constexpr int MOEK_DEV_TOO_MANY_ROWS = 3;
constexpr int MOEK_DEV_BAD_INPUT = 4;  // an input index out of range (checked in MOEK_DEBUG_CHECKS builds)

__device__ __forceinline__ uint64_t globaltimer();
__device__ __forceinline__ void report(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ----------------------------------------------------------------------------------------- timeline stamps
// Built with -DMOEK_TRACE, a kernel writes %globaltimer stamps of its phases: MOEK_TR(slot) stores the time in
// g_moek_trace[blockIdx.x][slot] (CTAs and slots beyond the array are not recorded), MOEK_TR_CLK the SM's cycle
// counter (clock64: fine-grained intervals inside a CTA; %globaltimer may advance in steps of a microsecond),
// MOEK_TR_VAL a value.
// Each translation unit has its own array (a static __device__ array defined here), read back by that unit's
// trace_copy_* function (moek_trace_read). Without the flag the macros are empty.
constexpr int MOEK_TRACE_CTAS = 1024, MOEK_TRACE_SLOTS = 128;
#ifdef MOEK_TRACE
static __device__ unsigned long long g_moek_trace[MOEK_TRACE_CTAS][MOEK_TRACE_SLOTS];
#define MOEK_TR_VAL(slot, v)                                                      \
  do {                                                                            \
    if (blockIdx.x < (unsigned)moek::MOEK_TRACE_CTAS && (slot) < moek::MOEK_TRACE_SLOTS) \
      moek::g_moek_trace[blockIdx.x][(slot)] = (unsigned long long)(v);          \
  } while (0)
#define MOEK_TR(slot) MOEK_TR_VAL(slot, moek::globaltimer())
#define MOEK_TR_CLK(slot) MOEK_TR_VAL(slot, clock64())
#define MOEK_TRACE_COPY_FN(name)                                                                      \
  cudaError_t name(void* dst, size_t bytes, int clear) {                                              \
    if (bytes > sizeof(g_moek_trace)) bytes = sizeof(g_moek_trace);                                   \
    cudaError_t e = dst ? cudaMemcpyFromSymbol(dst, g_moek_trace, bytes) : cudaSuccess;              \
    if (e == cudaSuccess && clear) {                                                                  \
      void* a = nullptr;                                                                              \
      e = cudaGetSymbolAddress(&a, g_moek_trace);                                                     \
      if (e == cudaSuccess) e = cudaMemset(a, 0, sizeof(g_moek_trace));                               \
    }                                                                                                 \
    return e;                                                                                         \
  }
#else
#define MOEK_TR_VAL(slot, v) \
  do {                       \
  } while (0)
#define MOEK_TR(slot) \
  do {                \
  } while (0)
#define MOEK_TR_CLK(slot) \
  do {                    \
  } while (0)
#define MOEK_TRACE_COPY_FN(name) \
  cudaError_t name(void*, size_t, int) { return cudaErrorNotSupported; }
#endif

// ------------------------------------------------------------------------------------------ input checks
// Built with -DMOEK_DEBUG_CHECKS, MOEK_CHECK(cond, err) is false (after recording MOEK_DEV_BAD_INPUT) when an index
// taken from an input is out of range, and the caller skips the access; otherwise it is always true.
#ifdef MOEK_DEBUG_CHECKS
#define MOEK_CHECK(cond, err) ((cond) ? true : (moek::report((err), moek::MOEK_DEV_BAD_INPUT), false))
#else
#define MOEK_CHECK(cond, err) true
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch: wait until the grid this one depends on has completed and its memory is visible
// (a no-op when the launch did not ask for programmatic serialisation), and let the next grid in the stream start
// launching (its CTAs stop at their own pdl_wait until this grid completes).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------- mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, int bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking test of the phase with the given parity (a completed phase reads true).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
#ifndef MOEK_WAIT_HINT_NS
#define MOEK_WAIT_HINT_NS 0
#endif
// try_wait with a suspend-time hint: the thread is suspended in hardware (issuing nothing) until the phase completes
// or about `ns` nanoseconds have passed.
__device__ __forceinline__ bool mbar_try_for(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity. Returns false (after reporting) once the deadline passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t deadline, int* err) {
  if (mbar_try(bar, parity)) return true;
  for (uint32_t i = 1;; i++) {
#if MOEK_WAIT_HINT_NS > 0
    if (mbar_try_for(bar, parity, MOEK_WAIT_HINT_NS)) return true;
    if (globaltimer() > deadline) {
#else
    if (mbar_try(bar, parity)) return true;
    if ((i & 255) == 0 && globaltimer() > deadline) {
#endif
      report(err, MOEK_DEV_TIMEOUT);
      return false;
    }
  }
}
// The same wait with a sleep between tests (growing to about 0.25 us), for warps whose wake-up latency is hidden
// (they run ahead of the warps they feed): waiting warps then leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint64_t deadline, int* err) {
  if (mbar_try(bar, parity)) return true;
#if MOEK_WAIT_HINT_NS > 0
  for (;;) {
    if (mbar_try_for(bar, parity, MOEK_WAIT_HINT_NS)) return true;
#else
  for (uint32_t ns = 32;; ns = ns < 256 ? 2 * ns : ns) {
    __nanosleep(ns);
    if (mbar_try(bar, parity)) return true;
#endif
    if (globaltimer() > deadline) {
      report(err, MOEK_DEV_TIMEOUT);
      return false;
    }
  }
}

// ------------------------------------------------------------------------------ flags shared with other GPUs
// int32 flags in peer-visible memory (CUDA IPC): system-scope acquire loads and release stores, bounded waits.
__device__ __forceinline__ int ld_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool wait_flag(const int* p, int want, uint64_t deadline, int* err) {
  for (uint32_t i = 0;; i++) {
    if (ld_sys(p) == want) return true;
    if ((i & 63) == 63 && globaltimer() > deadline) {
      report(err, MOEK_DEV_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
}

// ------------------------------------------------------------------------------------------------ bulk copies
// Non-tensor bulk copy global -> this CTA's shared memory, completion counted on an mbarrier (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// -------------------------------------------------------------------------------------------------- decoding
// The four pairs of a tiled word as bf16x2 of e2m1 * 2^-126: pair d = codes 2d, 2d + 1 (prep.CODE_BITS).
__device__ __forceinline__ void fp4_pairs(uint32_t q, uint32_t* d) {
  constexpr uint32_t P = 0x81C081C0u;  // sign and magnitude bits of a bf16 pair
  d[0] = q & P;
  d[1] = __funnelshift_r(q, q, 4) & P;
  d[2] = __funnelshift_r(q, q, 10) & P;
  d[3] = (__funnelshift_r(q, q, 14) & 0x00400040u) | (__funnelshift_r(q, q, 6) & 0x81808180u);
}
// S0E5M3 byte -> fp32 value (s * sf * 2^7)
__device__ __forceinline__ float s0e5m3_to_f32(uint32_t b) {
  return __uint_as_float(b ? (b << 20) + (112u << 23) : 0u);
}
// Per-scale constants: B and R of the module comment, each broadcast to both halves of a bf16x2.
struct ScaleBR {
  uint32_t b2, r2;
};
__device__ __forceinline__ ScaleBR scale_br(uint32_t byte, float g) {
  const float y = s0e5m3_to_f32(byte) * g;
  const __nv_bfloat16 b = __float2bfloat16_rn(y);
  const __nv_bfloat16 r = __float2bfloat16_rn(y - __bfloat162float(b));
  const uint32_t bu = __bfloat16_as_ushort(b), ru = __bfloat16_as_ushort(r);
  return {bu | (bu << 16), ru | (ru << 16)};
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Pair d (codes 2d, 2d + 1) of a tiled word as bf16x2 of e2m1 * 2^-126 (fp4_pairs, one pair).
template <int D>
__device__ __forceinline__ uint32_t fp4_pair(uint32_t q) {
  constexpr uint32_t P = 0x81C081C0u;
  if constexpr (D == 0) return q & P;
  if constexpr (D == 1) return __funnelshift_r(q, q, 4) & P;
  if constexpr (D == 2) return __funnelshift_r(q, q, 10) & P;
  return (__funnelshift_r(q, q, 14) & 0x00400040u) | (__funnelshift_r(q, q, 6) & 0x81808180u);
}
// The oracle's bf16 weights of pair D of a word (dequant_word, one pair).
template <int D>
__device__ __forceinline__ uint32_t dequant_pair(uint32_t q, const ScaleBR& s) {
  const uint32_t d = fp4_pair<D>(q);
  return bf2_fma(d, s.b2, bf2_mul(d, s.r2));
}
// The oracle's bf16 weights for the 8 codes of one word: out[d] = bf16x2 of codes 2d, 2d + 1.
__device__ __forceinline__ void dequant_word(uint32_t q, const ScaleBR& s, uint32_t* out) {
  uint32_t dv[4];
  fp4_pairs(q, dv);
#pragma unroll
  for (int d = 0; d < 4; d++) out[d] = bf2_fma(dv[d], s.b2, bf2_mul(dv[d], s.r2));
}

// Processed position (within its 128-position run) of item slot s: vLLM's scale_perm (new 8i + j <- old i + 8j)
// followed by the [0, 2, 1, 3] swap of every 4, inverted (vllm/.../marlin_utils.py:296-316,
// marlin_utils_fp4.py:91-93).
__device__ __forceinline__ int slot_position(int s) {
  const int c = s & 63;
  const int m = 8 * (c & 7) + (c >> 3);
  const int r = m & 3;
  return (s & 64) | (m & ~3) | (r == 1 ? 2 : r == 2 ? 1 : r);
}
// Logical slot offset (within its 64-column group) held at processed position p (the forward permutation).
__device__ __forceinline__ int position_slot(int p) {
  const int q = p & 63;
  const int r = q & 3;
  const int m = (q & ~3) | (r == 1 ? 2 : r == 2 ? 1 : r);
  return (p & 64) | ((m >> 3) + 8 * (m & 7));
}
// S0E5M3 byte of run position p, k-group kg (0..7) from a 528-byte packed run (exceptions not applied).
__device__ __forceinline__ uint32_t run_byte(const uint8_t* run, int p, int kg) {
  const uint32_t base = run[p >> 3];
  const uint32_t nb = run[16 + kg * 64 + (p >> 3) * 4 + (p & 3)];
  return base + ((p & 4) ? (nb >> 4) : (nb & 15));
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ uint32_t prmt_b(uint32_t a, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %1, %2;" : "=r"(r) : "r"(a), "r"(sel));
  return r;
}
// (bf16 B | bf16 R << 16) for a scale byte and the expert's global scale G (the B / R split described above)
__device__ __forceinline__ uint32_t scale_word(uint32_t byte, float g) {
  const float y = s0e5m3_to_f32(byte) * g;
  const __nv_bfloat16 b = __float2bfloat16_rn(y);
  const __nv_bfloat16 r = __float2bfloat16_rn(y - __bfloat162float(b));
  return (uint32_t)__bfloat16_as_ushort(b) | ((uint32_t)__bfloat16_as_ushort(r) << 16);
}

}  // namespace moek
