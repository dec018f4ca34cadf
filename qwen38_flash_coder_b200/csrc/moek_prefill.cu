// Prefill-regime W4A16 grouped GEMM on the 5th-generation tensor cores (tcgen05, TMEM operands), sm_100a.
//
// Same work as the decode kernel (moek_decode.cu) but for large batches, where every expert has tens to thousands of
// rows and the layer sits at the tensor-core ridge. The weights are the MMA's M side ("swap AB"): an item's 256
// weight rows are two M = 128 halves; the block's token rows are the N side (N = valid rows rounded up to 16,
// <= 128), so ragged experts cost no padded MMA rows beyond that rounding.
//
// The dequantised weights never touch shared memory: each dequant thread owns one weight row, turns its 64 codes of
// a stage into the oracle's bf16 weights in registers and writes them straight into tensor memory
// (tcgen05.st 32x32b), and the MMA reads A from TMEM (tcgen05.mma ... [d], [a], b_desc): shared memory only carries
// the packed codes, the packed scales and the activation tiles.
//
//   unit      = (moe_align block of <= 128 rows, 256-row item); units dealt round-robin to one persistent CTA per SM.
//   producer  = warp 0: per 64-k stage, bulk-copies (cp.async.bulk, no multicast) the 8 KB of packed codes (lane 0)
//               and the 1056-byte packed-scale run pair (lane 1, same instruction) into a ring slot (mbarrier
//               complete_tx).
//   MMA       = warps 1-4 (one lane each): per stage 2 halves x 4 k16 steps of tcgen05.mma.cta_group::1.kind::f16
//               (bf16 x bf16 -> fp32), A from a TMEM ring slot, B from a shared-memory K-major SWIZZLE_128B tile, D in
//               TMEM. Warp 1 + 2h + p issues the MMAs of accumulator (half h, k16 parity p) (with two accumulators,
//               warp 1 + 2h issues half h's): one thread's tcgen05.mma issue is latency-bound, so four issuing warps
//               keep four times as many in flight. Each warp's tcgen05.commit releases the A and B slots (four
//               arrivals) and, after a unit's last stage, hands D to the epilogue.
//               Warp 1 also allocates and frees the 512 TMEM columns: D = columns 0-319 (four accumulators of <= 80
//               columns for blocks of <= 80 padded rows, else two of <= 128), A ring = columns 320-511 (3 slots x two
//               halves x 32 columns of bf16 pairs). An MMA costs about the same for any N <= 256 and chained MMAs
//               into one accumulator wait on each other, so more independent accumulators means more MMAs in flight.
//   loaders   = warps 5-6: the block's activation rows gathered by TMA (cp.async.bulk.tensor tile::gather4, no
//               multicast: 4 rows of 64 k per instruction, one instruction per lane, the two warps taking alternate
//               gathers) into the 128-byte-swizzled B tile of the stage; rows past the block's valid ones read out of
//               bounds and arrive as zeros.
//   scales    = warp 7: per unit the (B | R) table of the expert's scale bytes (moek_common.cuh) and the unit's
//               exception lists (held in registers, loaded one unit ahead); per stage the scale byte of each of the
//               256 rows x 4 k-groups (base + 4-bit offset, then the exceptions), one 32-bit word per row.
//   dequant   = warps 8-23, two groups of eight taking alternate stages (a stage's dequant is a chain of shared-
//               memory loads, table lookups, bf16 FMAs and a tcgen05.st + wait, so two stages in flight hide half
//               of its latency): warp 8 + 8s + 4h + i owns rows 128h + 32q .. +31 of the item, q = warp % 4 (its TMEM
//               lane quarter); per stage a thread reads its row's 32 bytes of codes and its scale word, and stores
//               32 columns of bf16 pairs into the A slot.
//   epilogue  = warps 24-31 (lane quarter = warp % 4; two warps per quarter take alternate 8-column chunks, so the
//               accumulator is drained twice as fast and the next unit's MMAs wait less): tcgen05.ld 8 columns at a
//               time; gate_up writes act = bf16(silu(gate) * up) (gate row r and its up partner are lane r of halves
//               0 and 1), down writes the fp32 rows topk_w * acc that moek_combine sums over the top-k slots, or
//               (down_bf16: the kit's moe_gemm mode 0 contract) the bf16 rows bf16(topk_w * acc) into out.
//   sorted    = (sorted_act) gate_up writes act at the row's position in moe_align's sorted order instead of its
//               id, so that the down GEMM loads a block's rows as one 128-row TMA tile per stage instead of
//               gathering them.
//
// Every wait is bounded (%globaltimer); on expiry the CTA raises an abort flag, every role skips its remaining work
// in step, and TMEM is freed before the kernel returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "moek_common.cuh"
#include "moek_kernels.cuh"

namespace moek {
namespace pf {

constexpr int BMP = 128;  // rows per moe_align block (the MMA's N, at most)
constexpr int NW = 6;     // shared-memory ring of packed codes + packed scales + scale words
constexpr int NB = 6;     // shared-memory ring of activation tiles
constexpr int NA = 3;     // TMEM ring of dequantised weight tiles
constexpr int NDQ = 16;   // dequant warps: two groups of 8 taking alternate stages
constexpr int NEPI = 8;   // epilogue warps: two per TMEM lane quarter, taking alternate 8-column chunks
constexpr int NMMA = 4;   // MMA-issuing warps: one per accumulator (half h, k16-step parity p) = warp W_MMA + 2h + p
constexpr int NLOAD = 2;  // activation-gather warps (a TMA issue is latency-bound per thread: two warps, twice the rate)
constexpr int W_PROD = 0, W_MMA = 1, W_LOAD = W_MMA + NMMA, W_SCALE = W_LOAD + NLOAD, DQ0 = W_SCALE + 1,
              EPI0 = DQ0 + NDQ;
constexpr int THREADS = (EPI0 + NEPI) * 32;
// TMEM columns. D: a block of N <= QUAD_N padded rows keeps four accumulators (half h, k16-step parity p at column
// (2h + p) * QUAD_N), so four independent MMA chains are in flight; larger blocks keep two (half h at column 128h).
// The A ring follows.
constexpr int QUAD_N = 80, D_COLS = 4 * QUAD_N, A_COL0 = D_COLS, A_SLOT_COLS = 64;

constexpr int B_BYTES = BMP * 128;  // up to 128 token rows x 64 k bf16, 128-byte swizzled rows
constexpr int B_OFF = 0;
constexpr int TBL_BYTES = ITEM_COLS * 4;  // one scale word (4 k-groups) per row
constexpr int W_SLOT = STAGE_BYTES + PAIR_BYTES + TBL_BYTES;
constexpr int W_OFF = B_OFF + NB * B_BYTES;
constexpr int S_REL = STAGE_BYTES, TBL_REL = STAGE_BYTES + PAIR_BYTES;
constexpr int LUT_OFF = W_OFF + NW * W_SLOT;  // 2 x 256 {B B, R R} word pairs (units alternate; no per-use prmt)
constexpr int IDS_OFF = LUT_OFF + 2 * 256 * 8;                   // 128 activation rows per loader warp
constexpr int MISC_OFF = IDS_OFF + NLOAD * BMP * 4;              // tmem base, abort flag
constexpr int BAR_OFF = (MISC_OFF + 16 + 7) / 8 * 8;
constexpr int NBARS = 3 * NW + 2 * NB + 2 * NA + 2 + 2;
constexpr int SMEM_USED = BAR_OFF + NBARS * 8;
// + slack to align the base to 1024; at least 116 KB so that two CTAs never share an SM (each holds all 512 columns)
constexpr int SMEM = std::max(SMEM_USED + 1024, 116 * 1024);
static_assert(B_BYTES % 1024 == 0 && W_OFF % 1024 == 0, "swizzled tiles stay 1024-byte aligned");
static_assert(W_SLOT % 16 == 0 && S_REL % 16 == 0, "bulk copies need 16-byte alignment");
static_assert(A_COL0 >= 256 && A_COL0 + NA * A_SLOT_COLS <= 512, "D and the A ring share the 512 TMEM columns");

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMA gather of 4 rows of a 2-D tensor (box: 64 bf16 x 1 row, 128-byte swizzle) into 512 bytes of shared memory;
// completion counted on an mbarrier. No multicast.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int x, int4 rows, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(rows.x), "r"(rows.y), "r"(rows.z), "r"(rows.w),
      "r"(smem_u32(bar))
      : "memory");
}

// TMA load of a 2-D tile (box: 64 bf16 x 128 rows, 128-byte swizzle) into shared memory, completion on an mbarrier.
// No multicast.
__device__ __forceinline__ void tma_tile2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// K-major, 128-byte swizzle UMMA shared-memory descriptor of a tile whose 128-byte rows are contiguous and whose
// 8-row groups are 1024 bytes apart (SBO); LBO is unused for swizzled K-major layouts (1); version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;           // LBO
  d |= (uint64_t)(1024 >> 4) << 32; // SBO
  d |= (uint64_t)1 << 46;           // version
  d |= (uint64_t)2 << 61;           // SWIZZLE_128B
  return d;
}
// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
// D[tmem] (+)= A[tmem] x B[smem]: A is 128 lanes (rows) x 8 columns of bf16 pairs (k 2c, 2c + 1 in column c).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 8-column loads (32 lanes x 8 columns each) issued together, then one wait.
#define MOEK_LD8(T, X)                                                                                   \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"                  \
               : "=r"(X[0]), "=r"(X[1]), "=r"(X[2]), "=r"(X[3]), "=r"(X[4]), "=r"(X[5]), "=r"(X[6]), "=r"(X[7]) \
               : "r"(T))
__device__ __forceinline__ void tmem_ld8x2(uint32_t ta, uint32_t tb, float* va, float* vb) {
  uint32_t r[8], q[8];
  MOEK_LD8(ta, r);
  MOEK_LD8(tb, q);
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; i++) {
    va[i] = __uint_as_float(r[i]);
    vb[i] = __uint_as_float(q[i]);
  }
}
__device__ __forceinline__ void tmem_ld8x4(uint32_t ta, uint32_t tb, uint32_t tc, uint32_t td, float* va, float* vb,
                                           float* vc, float* vd) {
  uint32_t r[8], q[8], x[8], y[8];
  MOEK_LD8(ta, r);
  MOEK_LD8(tb, q);
  MOEK_LD8(tc, x);
  MOEK_LD8(td, y);
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; i++) {
    va[i] = __uint_as_float(r[i]);
    vb[i] = __uint_as_float(q[i]);
    vc[i] = __uint_as_float(x[i]);
    vd[i] = __uint_as_float(y[i]);
  }
}
#undef MOEK_LD8
// SiLU with the hardware exponent and the approximate divide (a few fp32 ulps; the product is rounded to bf16 next).
// x -> -inf gives x * 0 = -0, the limit.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

struct Bars {
  uint64_t *wfull, *wempty, *sfull, *bfull, *bempty, *afull, *aempty, *accfull, *accempty, *lutempty;
};

__device__ __forceinline__ bool wait_ab(uint64_t* bar, uint32_t par, uint64_t deadline, int* err, volatile int* ab) {
  if (*ab) return false;
  if (mbar_wait(bar, par, deadline, err)) return true;
  *ab = 1;
  return false;
}
// Warp-uniform bounded wait: every role is a whole warp and some of them go on to warp-wide instructions, so the
// lanes agree on the outcome (a lane that saw the deadline pass makes the whole warp give up).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t par, uint64_t deadline, int* err, volatile int* ab) {
  return __all_sync(0xffffffffu, wait_ab(bar, par, deadline, err, ab));
}

struct UnitInfo {
  int blk, item, e;
};
__device__ __forceinline__ UnitInfo unit_info(const GemmParams& p, int64_t u, int nt) {
  UnitInfo r;
  r.blk = (int)(u / nt);
  r.item = (int)(u - (int64_t)r.blk * nt);
  r.e = p.expert_ids[r.blk];
  return r;
}

__global__ void __launch_bounds__(THREADS, 1)
    moek_prefill_kernel(GemmParams p, const __grid_constant__ CUtensorMap tmap_a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  Bars B;
  B.wfull = bars;
  B.wempty = B.wfull + NW;
  B.sfull = B.wempty + NW;
  B.bfull = B.sfull + NW;
  B.bempty = B.bfull + NB;
  B.afull = B.bempty + NB;
  B.aempty = B.afull + NA;
  B.accfull = B.aempty + NA;
  B.accempty = B.accfull + 1;
  B.lutempty = B.accempty + 1;
  uint2* lut = reinterpret_cast<uint2*>(smem + LUT_OFF);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + MISC_OFF + 4);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nt = p.N / ITEM_COLS, nstage = p.K / BK, nb = p.K / 128;

  if (tid == 0) {
    *abort_flag = 0;
    for (int i = 0; i < NW; i++) {
      mbar_init(B.wfull + i, 1);
      mbar_init(B.wempty + i, NDQ / 2);
      mbar_init(B.sfull + i, 1);
    }
    for (int i = 0; i < NB; i++) {
      mbar_init(B.bfull + i, 1);
      mbar_init(B.bempty + i, NMMA);  // every MMA warp commits
    }
    for (int i = 0; i < NA; i++) {
      mbar_init(B.afull + i, NDQ / 2);
      mbar_init(B.aempty + i, NMMA);
    }
    mbar_init(B.accfull, NMMA);
    mbar_init(B.accempty, NEPI);
    mbar_init(B.lutempty, NDQ);
    mbar_init(B.lutempty + 1, NDQ);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == W_MMA) {  // TMEM: all 512 columns (D, then the A ring)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32((const void*)tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) MOEK_TR(0);
  pdl_wait();  // sorted ids, experts and activations come from the previous kernels
  pdl_launch_dependents();
  if (tid == 0) MOEK_TR(1);
  const uint64_t deadline = globaltimer() + p.timeout_ns;
  const int nblocks = min(p.num_post_pad[0] / p.block_m, p.max_blocks);
  const int64_t nunits = (int64_t)nblocks * nt;

  if (warp == W_PROD) {  // ---------------------------------------------------------------------- producer
    uint32_t g = 0;
    bool ok = true;
    UnitInfo nx = blockIdx.x < nunits ? unit_info(p, blockIdx.x, nt) : UnitInfo{0, 0, -1};  // one unit ahead
    for (int64_t u = blockIdx.x; u < nunits && ok && !*abort_flag; u += gridDim.x) {
      const UnitInfo ui = nx;
      if (u + gridDim.x < nunits) nx = unit_info(p, u + gridDim.x, nt);
      if (ui.e < 0 || ui.e >= p.E) continue;
      for (int st = 0; st < nstage; st++, g++) {
        const int s = g % NW;
        if (g >= NW && !wait_warp(B.wempty + s, ((g / NW) - 1) & 1, deadline, p.err, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* dst = smem + W_OFF + s * W_SLOT;
        if (lane == 0) mbar_expect_tx(B.wfull + s, STAGE_BYTES + PAIR_BYTES);
        __syncwarp();
        // the codes from lane 0 and the scale pair from lane 1, in one instruction
        if (lane == 0) {
          const int64_t wi = ((int64_t)ui.e * nt + ui.item) * nstage + st;
          bulk_g2s(dst, p.W + wi * STAGE_BYTES, STAGE_BYTES, B.wfull + s);
        } else if (lane == 1) {
          const int64_t si = ((int64_t)ui.e * nt + ui.item) * nb + (st >> 1);
          bulk_g2s(dst + S_REL, p.SP + si * PAIR_BYTES, PAIR_BYTES, B.wfull + s);
        }
        __syncwarp();
      }
    }
  } else if (warp >= W_MMA && warp < W_MMA + NMMA) {  // ------------------------------------------------ MMA
    const int mh = (warp - W_MMA) >> 1, mp = (warp - W_MMA) & 1;  // this warp's accumulator
    uint32_t g = 0, un = 0;
    for (int64_t u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
      const UnitInfo ui = unit_info(p, u, nt);
      if (ui.e < 0 || ui.e >= p.E) continue;
      int ids[BMP / 32], nv = 0;
#pragma unroll
      for (int j = 0; j < BMP / 32; j++) {  // all loads first, then the ballots
        const int r = lane + 32 * j;
        ids[j] = r < p.block_m ? p.sorted_ids[(int64_t)ui.blk * p.block_m + r] : p.num_ids;
        if (!MOEK_CHECK(ids[j] >= 0 && ids[j] <= p.num_ids, p.err)) ids[j] = p.num_ids;
      }
#pragma unroll
      for (int j = 0; j < BMP / 32; j++) nv += __popc(__ballot_sync(0xffffffffu, ids[j] < p.num_ids));
      const int nalloc = max(16, (nv + 15) & ~15);
      const uint32_t idesc = idesc_bf16(nalloc);
      const bool quad = nalloc <= QUAD_N;
      if (un >= 1 && !wait_warp(B.accempty, (un - 1) & 1, deadline, p.err, abort_flag)) break;
      tc_fence_after();
      bool ok = true;
      for (int st = 0; st < nstage; st++, g++) {
        const int a = g % NA, b = g % NB;
        if (!wait_warp(B.afull + a, (g / NA) & 1, deadline, p.err, abort_flag) ||
            !wait_warp(B.bfull + b, (g / NB) & 1, deadline, p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (warp == W_MMA && lane == 0 && st == 0 && un < 16) MOEK_TR(8 + 3 * un);
        if (lane == 0) {
          const uint32_t b0 = smem_u32(smem + B_OFF + b * B_BYTES);
          const uint32_t a0 = tmem + A_COL0 + a * A_SLOT_COLS;
#pragma unroll
          for (int ks = 0; ks < 4; ks++) {
            // four accumulators (half h, parity ks & 1): this warp's; two (half h): warp p = 0 of each half
            if (quad ? (ks & 1) != mp : mp != 0) continue;
            const uint64_t bd = umma_desc_k_sw128(b0 + 32 * ks);
            const uint32_t d = quad ? (2 * mh + mp) * QUAD_N : mh * 128;
            umma_ts(tmem + d, a0 + mh * 32 + ks * 8, bd, idesc, (st > 0 || ks >= (quad ? 2 : 1)) ? 1u : 0u);
          }
          umma_commit(B.aempty + a);  // the A and B slots may be refilled once these MMAs completed
          umma_commit(B.bempty + b);
          if (st == nstage - 1) umma_commit(B.accfull);
          if (warp == W_MMA && st == nstage - 1 && un < 16) MOEK_TR(9 + 3 * un);
        }
        __syncwarp();
      }
      if (!ok) break;
      un++;
    }
  } else if (warp >= W_LOAD && warp < W_LOAD + NLOAD) {  // --------------------------------------- activation loaders
    int* rowc = reinterpret_cast<int*>(smem + IDS_OFF) + (warp - W_LOAD) * BMP;  // each loader warp its own copy
    const int lw = warp - W_LOAD;                // gathers lw, lw + NLOAD, ... of a stage are this warp's
    const int rows_a = p.a_rows;  // rows of A; a coordinate of rows_a reads zeros
    const bool tile_rows = p.sorted_act && !p.gate_up;  // act in sorted order: the block's rows are contiguous
    uint32_t g = 0;
    for (int64_t u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
      const UnitInfo ui = unit_info(p, u, nt);
      if (ui.e < 0 || ui.e >= p.E) continue;
      const int64_t row0 = (int64_t)ui.blk * p.block_m;
      __syncwarp();  // the previous unit's gathers were issued from these rows
      int nv = 0;
#pragma unroll
      for (int j = 0; j < BMP / 32; j++) {
        const int r = lane + 32 * j;
        int id = r < p.block_m ? p.sorted_ids[row0 + r] : p.num_ids;
        if (!MOEK_CHECK(id >= 0 && id <= p.num_ids, p.err)) id = p.num_ids;
        rowc[r] = id < p.num_ids ? id / p.a_div : rows_a;
      }
#pragma unroll
      for (int j = 0; j < BMP / 32; j++) nv += __popc(__ballot_sync(0xffffffffu, rowc[lane + 32 * j] < rows_a));
      __syncwarp();
      const int ng = (nv + 3) >> 2;  // gathers of 4 rows; the block's valid rows come first
      bool ok = true;
      for (int st = 0; st < nstage; st++, g++) {
        const int b = g % NB;
        if (g >= NB && !wait_warp(B.bempty + b, ((g / NB) - 1) & 1, deadline, p.err, abort_flag)) {
          ok = false;
          break;
        }
        // the first loader's arrival carries the stage's byte count; the other's copies may complete before it
        // (the phase cannot end before that arrival)
        if (tile_rows) {  // one TMA for the block's 128 rows (rows past the block's valid ones are not read)
          if (lw == 0 && lane == 0) {
            mbar_expect_tx(B.bfull + b, BMP * 128);
            tma_tile2d(smem + B_OFF + b * B_BYTES, &tmap_a, st * BK, (int)row0, B.bfull + b);
          }
          __syncwarp();
          continue;
        }
        if (lw == 0 && lane == 0) mbar_expect_tx(B.bfull + b, ng * 4 * 128);
        __syncwarp();
        const int j = lane * NLOAD + lw;  // this lane's gather of the stage
        if (j < ng)
          tma_gather4(smem + B_OFF + b * B_BYTES + j * 512, &tmap_a, st * BK,
                      *reinterpret_cast<const int4*>(rowc + 4 * j), B.bfull + b);
      }
      if (!ok) break;
    }
  } else if (warp == W_SCALE) {  // ------------------------------------------------------------------ scale words
    // Per unit: the expert's global scale, the unit's run offsets (lane j: run j's first exception entry) and up to 64
    // exception entries, held in registers and loaded one unit ahead, so that no unit starts behind a chain of
    // dependent global loads. Per stage: the 4 k-group scale bytes of each row as one word, then the exceptions.
    const int run = lane >> 4, chk = lane & 15;  // this lane's 8 positions: run `run`, positions 8 chk .. 8 chk + 7
    int rows[8];
#pragma unroll
    for (int i = 0; i < 8; i++) rows[i] = run * 128 + position_slot(8 * chk + i);
    auto next_valid = [&](int64_t u2) -> int64_t {
      for (; u2 < nunits; u2 += gridDim.x) {
        const int e = unit_info(p, u2, nt).e;
        if (e >= 0 && e < p.E) break;
      }
      return u2;
    };
    int ro_n = 0, end_n = 0;
    float g_n = 0.f;
    auto fetch = [&](int64_t u2) {  // loads only: consumed when the unit starts
      const UnitInfo v = unit_info(p, u2, nt);
      const int64_t key0 = ((int64_t)v.e * nt + v.item) * nb;
      ro_n = lane < nb ? p.exc_off[key0 + lane] : 0;
      end_n = p.exc_off[key0 + nb];
      g_n = p.G[v.e];
    };
    uint32_t g = 0, un = 0;
    int64_t u = next_valid(blockIdx.x);
    if (u < nunits) fetch(u);
    while (u < nunits && !*abort_flag) {
      const UnitInfo ui = unit_info(p, u, nt);
      const int lb = un & 1;
      const int o0 = __shfl_sync(0xffffffffu, ro_n, 0);
      const int ro = ro_n - o0, cnt = end_n - o0;
      const float gsc = g_n;
      const uint32_t* eg = p.exc_ent + o0;
      const uint32_t ex0 = lane < cnt ? eg[lane] : 0u, ex1 = lane + 32 < cnt ? eg[lane + 32] : 0u;
      const int64_t u_next = next_valid(u + gridDim.x);
      if (u_next < nunits) fetch(u_next);
      const int r0g = p.gate_up ? ui.item : 2 * ui.item;
      const int r1g = p.gate_up ? nt + ui.item : r0g + 1;  // the pair's second run (gate_up: the up rows' run)
      // the (B | R) table of this expert, once the dequant warps finished the unit that used this buffer last
      if (un >= 2 && !wait_warp(B.lutempty + lb, ((un >> 1) - 1) & 1, deadline, p.err, abort_flag)) break;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const ScaleBR br = scale_br(lane + 32 * j, gsc);
        lut[lb * 256 + lane + 32 * j] = make_uint2(br.b2, br.r2);
      }
      __syncwarp();
      bool ok = true;
      for (int st = 0; st < nstage; st++, g++) {
        const int s = g % NW;
        if (!wait_warp(B.wfull + s, (g / NW) & 1, deadline, p.err, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* slot = smem + W_OFF + s * W_SLOT;
        uint32_t* tbl = reinterpret_cast<uint32_t*>(slot + TBL_REL);
        const uint8_t* runp = slot + S_REL + run * RUN_BYTES;
        const uint32_t b4 = runp[chk] * 0x01010101u;
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const int kg = (st & 1) * 4 + kk;
          const uint32_t q = *reinterpret_cast<const uint32_t*>(runp + 16 + kg * 64 + chk * 4);
          lo[kk] = (q & 0x0F0F0F0Fu) + b4;         // positions 8 chk + 0..3
          hi[kk] = ((q >> 4) & 0x0F0F0F0Fu) + b4;  // positions 8 chk + 4..7
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const uint32_t* src = i < 4 ? lo : hi;
          const uint32_t bi = i & 3, sel = bi | ((bi + 4) << 4);
          tbl[rows[i]] = prmt(prmt(src[0], src[1], sel), prmt(src[2], src[3], sel), 0x5410);
        }
        __syncwarp();
        // exceptions of this stage's run (rn) whose k-group falls in this stage's half overwrite their bytes
        const int rn = st >> 1;
        const int eo0 = __shfl_sync(0xffffffffu, ro, rn);
        const int eo1 = rn + 1 < nb ? __shfl_sync(0xffffffffu, ro, rn + 1) : cnt;
        auto patch = [&](uint32_t en) {
          const int ppos = en & 0xFFFF, kg = (en >> 16) & 0xFF;
          if (!MOEK_CHECK(kg < KG && ((ppos >> 7) == r0g || (ppos >> 7) == r1g), p.err)) return;
          if ((kg >> 2) != (st & 1)) return;
          const int row = ((ppos >> 7) == r0g ? 0 : 128) + position_slot(ppos & 127);
          reinterpret_cast<uint8_t*>(tbl)[row * 4 + (kg & 3)] = (uint8_t)(en >> 24);
        };
        if (lane >= eo0 && lane < eo1) patch(ex0);
        if (lane + 32 >= eo0 && lane + 32 < eo1) patch(ex1);
        for (int j = max(eo0, 64) + lane; j < eo1; j += 32) patch(eg[j]);  // long lists: the rest from memory
        __syncwarp();
        if (lane == 0) mbar_arrive(B.sfull + s);
      }
      if (!ok) break;
      un++;
      u = u_next;
    }
  } else if (warp < EPI0) {  // ------------------------------------------------------------------- dequant
    const int dw = warp - DQ0, h = (dw >> 2) & 1, grp = dw >> 3, q = warp & 3;
    const int row = 128 * h + 32 * q + lane;  // this thread's weight row within the item
    const int sw = ((row >> 2) & 1) << 4;     // byte offset of the row's first 16-byte half (swizzle)
    const uint32_t t_row = tmem + ((uint32_t)(32 * q) << 16) + A_COL0 + 32 * h;
    uint32_t g = 0, un = 0;
    // the next unit's expert is loaded one unit ahead (only its validity is needed here)
    int e_next = blockIdx.x < nunits ? unit_info(p, blockIdx.x, nt).e : -1;
    for (int64_t u = blockIdx.x; u < nunits; u += gridDim.x) {
      const int e = e_next;
      e_next = u + gridDim.x < nunits ? unit_info(p, u + gridDim.x, nt).e : -1;
      if (e < 0 || e >= p.E) {
        if (dw == 0 && lane == 0) report(p.err, MOEK_DEV_BAD_EXPERT);
        continue;
      }
      const uint2* lt = lut + (un & 1) * 256;
      for (int st = 0; st < nstage; st++, g++) {
        if ((int)(g & 1) != grp) continue;  // the other group's stage
        const int s = g % NW, a = g % NA;
        const bool have_w = wait_warp(B.wfull + s, (g / NW) & 1, deadline, p.err, abort_flag) &&
                            wait_warp(B.sfull + s, (g / NW) & 1, deadline, p.err, abort_flag);
        const bool free_a = g < NA || wait_warp(B.aempty + a, ((g / NA) - 1) & 1, deadline, p.err, abort_flag);
        // warp-uniform: tcgen05.st is a warp-wide instruction
        const bool live = __all_sync(0xffffffffu, have_w && free_a && !*abort_flag);
        if (live) {
          tc_fence_after();
          const uint8_t* slot = smem + W_OFF + s * W_SLOT;
          const uint4 c0 = *reinterpret_cast<const uint4*>(slot + row * 32 + sw);
          const uint4 c1 = *reinterpret_cast<const uint4*>(slot + row * 32 + (sw ^ 16));
          const uint32_t sc = reinterpret_cast<const uint32_t*>(slot + TBL_REL)[row];
          const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          uint32_t v[32];
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const uint2 lw = lt[(sc >> (8 * kk)) & 0xFF];
            const ScaleBR sbr{lw.x, lw.y};
            dequant_word(words[2 * kk], sbr, v + 8 * kk);
            dequant_word(words[2 * kk + 1], sbr, v + 8 * kk + 4);
          }
          tmem_st32(t_row + a * A_SLOT_COLS, v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (have_w) mbar_arrive(B.wempty + s);  // packed codes and scale words consumed
          mbar_arrive(B.afull + a);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(B.lutempty + (un & 1));
      un++;
    }
  } else {  // ------------------------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int part = (warp - EPI0) >> 2;  // this warp's chunks: c0 = 8 part (mod 8 NEPI / 4)
    const int I = p.N / 2;
    uint32_t un = 0;
    for (int64_t u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
      const UnitInfo ui = unit_info(p, u, nt);
      if (ui.e < 0 || ui.e >= p.E) continue;
      const int64_t row0 = (int64_t)ui.blk * p.block_m;
      int ids[4];
      float wts[4];
      int nv = 0;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int r = lane + 32 * j;
        ids[j] = r < p.block_m ? p.sorted_ids[row0 + r] : p.num_ids;
        if (!MOEK_CHECK(ids[j] >= 0 && ids[j] <= p.num_ids, p.err)) ids[j] = p.num_ids;
        nv += __popc(__ballot_sync(0xffffffffu, ids[j] < p.num_ids));
        wts[j] = (!p.gate_up && ids[j] < p.num_ids) ? p.topk_w[ids[j]] : 0.f;
      }
      if (!wait_warp(B.accfull, un & 1, deadline, p.err, abort_flag)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16);
      const int row = 32 * q + lane;  // weight row within the half
      const bool quad = max(16, (nv + 15) & ~15) <= QUAD_N;
      for (int c0 = 8 * part; c0 < nv; c0 += 8 * (NEPI / 4)) {
        float v0[8], v1[8];
        if (quad) {  // sum the two k-parity accumulators of each half
          float g1[8], u1[8];
          tmem_ld8x4(tbase + c0, tbase + QUAD_N + c0, tbase + 2 * QUAD_N + c0, tbase + 3 * QUAD_N + c0, v0, g1, v1, u1);
#pragma unroll
          for (int j = 0; j < 8; j++) {
            v0[j] += g1[j];
            v1[j] += u1[j];
          }
        } else {
          tmem_ld8x2(tbase + c0, tbase + 128 + c0, v0, v1);
        }
        const int jj = c0 >> 5, l0 = c0 & 24;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          if (c0 + j >= nv) break;
          const int id = __shfl_sync(0xffffffffu, ids[jj], l0 + j);
          if (p.gate_up) {  // sorted order: act row = the row's sorted position, else its id
            const int64_t arow = p.sorted_act ? row0 + c0 + j : (int64_t)id;
            static_cast<__nv_bfloat16*>(p.out)[arow * I + 128 * ui.item + row] =
                __float2bfloat16_rn(silu_fast(v0[j]) * v1[j]);
          } else {
            const float w = __shfl_sync(0xffffffffu, wts[jj], l0 + j);
            if (p.down_bf16) {  // the kit's dout row: bf16(topk_w * sum)
              __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + (int64_t)id * p.N + 256 * ui.item;
              orow[row] = __float2bfloat16_rn(w * v0[j]);
              orow[128 + row] = __float2bfloat16_rn(w * v1[j]);
            } else {
              float* orow = p.part + (int64_t)id * p.N + 256 * ui.item;
              orow[row] = w * v0[j];
              orow[128 + row] = w * v1[j];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(B.accempty);
      if (warp == EPI0 && lane == 0 && un < 16) MOEK_TR(10 + 3 * un);
      un++;
    }
  }
  // ------------------------------------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (tid == 0) MOEK_TR(6);
  if (warp == W_MMA) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace pf

MOEK_TRACE_COPY_FN(trace_copy_prefill)

int prefill_block_m() { return pf::BMP; }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against the driver library).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

cudaError_t launch_prefill(const GemmParams& p, int sms, cudaStream_t st) {
  const int nt = p.N / ITEM_COLS;
  const int64_t units = (int64_t)p.max_blocks * nt;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sms, units));
  // A as a 2-D bf16 tensor [rows, K] (K contiguous), read 64 k x 1 row per gathered row, 128-byte swizzle
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap tmap;
  const cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)std::max(1, p.a_rows)};
  const cuuint64_t strides[1] = {(cuuint64_t)p.K * 2};
  // gathered rows: a 1-row box (tile::gather4); sorted-order down: the block's 128 consecutive rows in one box
  const cuuint32_t box[2] = {BK, (p.sorted_act && !p.gate_up) ? (cuuint32_t)pf::BMP : 1u}, estr[2] = {1, 1};
  if (encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(p.A), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(pf::moek_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM);
  if (e != cudaSuccess) return e;
  e = launch_pdl(pf::moek_prefill_kernel, dim3(grid), dim3(pf::THREADS), pf::SMEM, st, p, tmap);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace moek
