// Prefill-regime W4A16 grouped GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulators), sm_100a.
//
// Same work as the decode kernel (moek_decode.cu) but for large batches, where every expert has tens to thousands of
// rows and the layer is at the tensor-core / HBM ridge. The weights are the MMA's M side ("swap AB"): an item's 256
// weight rows are two M=128 halves, the block's token rows are the N side (N = valid rows rounded up to 16, <= 128),
// so ragged experts cost no padded MMA rows beyond that rounding.
//
//   unit      = (moe_align block of <= 128 rows, 256-row item); units dealt round-robin to one persistent CTA per SM.
//   producer  = warp 0: per 64-k stage, bulk-copies (cp.async.bulk, no multicast) the 8 KB of packed codes and the
//               1056-byte packed-scale run pair into a ring slot (mbarrier complete_tx).
//   MMA       = warp 1 (one elected lane): per stage 2 halves x 4 k16 steps of tcgen05.mma.cta_group::1.kind::f16
//               (bf16 x bf16 -> fp32), A and B from shared memory through K-major SWIZZLE_128B descriptors, D in TMEM;
//               tcgen05.commit releases the stage and, after a unit's last stage, hands the accumulator to the
//               epilogue. Two accumulator buffers (2 x 2 halves x 128 columns = all 512 TMEM columns) let the next
//               unit's MMAs run while the epilogue drains the previous one. Warp 1 also allocates and frees TMEM.
//   dequant   = warps 2-9: per stage, the scale bytes of the 4 k-groups x 256 rows (base + 4-bit offset, then the
//               unit's exception entries), then the oracle's bf16 weights (moek_common.cuh: bf16(e2m1 * s * gs))
//               written as two 128 x 64 K-major tiles in the 128-byte swizzle (16-byte chunk c of row r at c ^ (r % 8)),
//               and the block's activation rows gathered with cp.async into the same swizzled layout;
//               fence.proxy.async then makes the generic-proxy writes visible to the tensor core.
//   epilogue  = warps 10-13 (TMEM lane quarter = warp % 4): tcgen05.ld 32 columns at a time; gate_up writes
//               act = bf16(silu(gate) * up) (gate row r and its up partner are lane r of halves 0 and 1), down writes
//               the fp32 rows topk_w * acc that moek_combine sums over the top-k slots.
//
// Every wait is bounded (%globaltimer); on expiry the CTA raises an abort flag, every role skips its remaining work
// in step, and TMEM is freed before the kernel returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "moek_common.cuh"
#include "moek_kernels.cuh"

namespace moek {
namespace pf {

constexpr int BMP = 128;           // rows per moe_align block (the MMA's N, at most)
constexpr int NST = 3;             // ring stages
constexpr int NDQ = 8;             // dequant warps
constexpr int NEPI = 4;            // epilogue warps
constexpr int THREADS = (2 + NDQ + NEPI) * 32;
constexpr int DQ0 = 2, EPI0 = 2 + NDQ;  // first dequant warp, first epilogue warp
constexpr int A_BYTES = 2 * 128 * 128;  // two 128-row x 64-k bf16 tiles
constexpr int B_BYTES = BMP * 128;      // up to 128 token rows x 64 k bf16
constexpr int SCB_STRIDE = 288;         // scale-byte row per k-group (256 + 32)
constexpr int A_OFF = 0, B_OFF = A_OFF + A_BYTES, W_OFF = B_OFF + B_BYTES, S_OFF = W_OFF + STAGE_BYTES,
              SCB_OFF = S_OFF + PAIR_BYTES, STAGE_END = SCB_OFF + 4 * SCB_STRIDE;
constexpr int STAGE_STRIDE = (STAGE_END + 1023) / 1024 * 1024;  // tiles stay 1024-byte aligned
constexpr int EXC_CAP = 2048;           // exception entries of one unit cached in shared memory
constexpr int RING_END = NST * STAGE_STRIDE;
constexpr int LUT_OFF = RING_END;                     // 2 x 256 (B | R) words (units alternate)
constexpr int EXC_OFF = LUT_OFF + 2 * 256 * 4;        // 2 x EXC_CAP entries
constexpr int RUNOFF_OFF = EXC_OFF + 2 * EXC_CAP * 4; // 2 x 33 run offsets
constexpr int MISC_OFF = RUNOFF_OFF + 2 * 33 * 4;     // tmem base, abort flag
constexpr int BAR_OFF = (MISC_OFF + 16 + 7) / 8 * 8;
constexpr int NBARS = 4 * NST + 4;
constexpr int SMEM = BAR_OFF + NBARS * 8 + 1024;      // + slack to align the base to 1024

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void dq_sync() { asm volatile("bar.sync 2, %0;" ::"n"(NDQ * 32) : "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

struct Bars {
  uint64_t *wfull, *wempty, *afull, *aempty, *accfull, *accempty;
};

__device__ __forceinline__ bool wait_ab(uint64_t* bar, uint32_t par, uint64_t deadline, int* err, volatile int* ab) {
  if (*ab) return false;
  if (mbar_wait(bar, par, deadline, err)) return true;
  *ab = 1;
  return false;
}

struct UnitInfo {
  int blk, item, e, nv;
};
__device__ __forceinline__ UnitInfo unit_info(const GemmParams& p, int64_t u, int nt) {
  UnitInfo r;
  r.blk = (int)(u / nt);
  r.item = (int)(u - (int64_t)r.blk * nt);
  r.e = p.expert_ids[r.blk];
  return r;
}

__global__ void __launch_bounds__(THREADS, 1) moek_prefill_kernel(GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  const Bars B{bars, bars + NST, bars + 2 * NST, bars + 3 * NST, bars + 4 * NST, bars + 4 * NST + 2};
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem + LUT_OFF);
  uint32_t* excs = reinterpret_cast<uint32_t*>(smem + EXC_OFF);
  int* runoffs = reinterpret_cast<int*>(smem + RUNOFF_OFF);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + MISC_OFF + 4);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nt = p.N / ITEM_COLS, nstage = p.K / BK, nb = p.K / 128, nruns = nb;

  if (tid == 0) {
    *abort_flag = 0;
    for (int i = 0; i < NST; i++) {
      mbar_init(B.wfull + i, 1);
      mbar_init(B.wempty + i, NDQ);
      mbar_init(B.afull + i, NDQ);
      mbar_init(B.aempty + i, 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(B.accfull + i, 1);
      mbar_init(B.accempty + i, NEPI);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // TMEM: all 512 columns (2 accumulator buffers x 2 halves x 128 columns)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32((const void*)tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // sorted ids, experts and activations come from the previous kernels
  pdl_launch_dependents();
  const uint64_t deadline = globaltimer() + p.timeout_ns;
  const int nblocks = min(p.num_post_pad[0] / p.block_m, p.max_blocks);
  const int64_t nunits = (int64_t)nblocks * nt;

  if (warp == 0) {  // --------------------------------------------------------------------------- producer
    uint32_t g = 0;
    for (int64_t u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
      const UnitInfo ui = unit_info(p, u, nt);
      if (ui.e < 0 || ui.e >= p.E) continue;
      for (int st = 0; st < nstage; st++, g++) {
        const int s = g % NST;
        if (g >= NST && !wait_ab(B.wempty + s, ((g / NST) - 1) & 1, deadline, p.err, abort_flag)) break;
        if (lane == 0) {
          uint8_t* dst = smem + s * STAGE_STRIDE;
          mbar_expect_tx(B.wfull + s, STAGE_BYTES + PAIR_BYTES);
          const int64_t wi = ((int64_t)ui.e * nt + ui.item) * nstage + st;
          bulk_g2s(dst + W_OFF, p.W + wi * STAGE_BYTES, STAGE_BYTES, B.wfull + s);
          const int64_t si = ((int64_t)ui.e * nt + ui.item) * nb + (st >> 1);
          bulk_g2s(dst + S_OFF, p.SP + si * PAIR_BYTES, PAIR_BYTES, B.wfull + s);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {  // ------------------------------------------------------------------------ MMA
    uint32_t g = 0, un = 0;
    for (int64_t u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
      const UnitInfo ui = unit_info(p, u, nt);
      if (ui.e < 0 || ui.e >= p.E) continue;
      int nv = 0;
      for (int r0 = 0; r0 < BMP; r0 += 32) {
        const int r = r0 + lane;
        nv += __popc(__ballot_sync(0xffffffffu, r < p.block_m &&
                                                    p.sorted_ids[(int64_t)ui.blk * p.block_m + r] < p.num_ids));
      }
      const int n = max(16, (nv + 15) & ~15);
      const uint32_t idesc = idesc_bf16(n);
      const int buf = un & 1;
      if (un >= 2 && !wait_ab(B.accempty + buf, ((un >> 1) - 1) & 1, deadline, p.err, abort_flag)) break;
      tc_fence_after();
      bool ok = true;
      for (int st = 0; st < nstage; st++, g++) {
        const int s = g % NST;
        if (!wait_ab(B.afull + s, (g / NST) & 1, deadline, p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a0 = smem_u32(smem + s * STAGE_STRIDE + A_OFF), b0 = smem_u32(smem + s * STAGE_STRIDE + B_OFF);
#pragma unroll
          for (int ks = 0; ks < 4; ks++) {
            const uint64_t bd = umma_desc_k_sw128(b0 + 32 * ks);
#pragma unroll
            for (int h = 0; h < 2; h++) {
              const uint64_t ad = umma_desc_k_sw128(a0 + h * (128 * 128) + 32 * ks);
              umma_bf16(tmem + buf * 256 + h * 128, ad, bd, idesc, (st > 0 || ks > 0) ? 1u : 0u);
            }
          }
          umma_commit(B.aempty + s);  // the stage's tiles may be overwritten once these MMAs completed
          if (st == nstage - 1) umma_commit(B.accfull + buf);
        }
        __syncwarp();
      }
      if (!ok) break;
      un++;
    }
  } else if (warp < EPI0) {  // ------------------------------------------------------------------- dequant
    const int dw = warp - DQ0, dt = tid - DQ0 * 32;  // dequant warp 0..7, thread 0..255
    const int gq = lane >> 2, c = lane & 3;
    // scale-byte decode: thread dt < 128 owns chunk (dt & 15) of run (dt >> 4) & 1 for k-group kk = dt >> 5
    const int s_kk = dt >> 5, s_run = (dt >> 4) & 1, s_ch = dt & 15;
    int s_dst[8];
#pragma unroll
    for (int i = 0; i < 8; i++) s_dst[i] = s_run * 128 + position_slot(8 * s_ch + i);
    uint32_t g = 0, un = 0;
    // no abort test in the loop header: the dequant warps share a named barrier, so they all run every unit and
    // stage; after an abort every wait fails at once and the work is skipped
    for (int64_t u = blockIdx.x; u < nunits; u += gridDim.x) {
      const UnitInfo ui = unit_info(p, u, nt);
      if (ui.e < 0 || ui.e >= p.E) {
        if (dt == 0) report(p.err, MOEK_DEV_BAD_EXPERT);
        continue;
      }
      const int lb = un & 1;
      uint32_t* lt = lut + lb * 256;
      uint32_t* ex = excs + lb * EXC_CAP;
      int* ro = runoffs + lb * 33;
      const int64_t row0 = (int64_t)ui.blk * p.block_m;
      // per unit: the (B | R) table for this expert, the exception lists of the item, the valid rows
      const float gsc = p.G[ui.e];
      lt[dt] = scale_word(dt, gsc);
      const int64_t key0 = ((int64_t)ui.e * nt + ui.item) * nb;
      const int o0 = p.exc_off[key0];
      if (dt <= nruns) ro[dt] = p.exc_off[key0 + dt] - o0;
      dq_sync();
      const int nexc = ro[nruns];
      const bool exc_smem = nexc <= EXC_CAP;
      if (exc_smem)
        for (int j = dt; j < nexc; j += NDQ * 32) ex[j] = p.exc_ent[o0 + j];
      const uint32_t* exl = exc_smem ? ex : p.exc_ent + o0;
      int my_id[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int r = (dt >> 3) + 32 * j;  // the rows this thread copies (8 16-byte chunks per row)
        my_id[j] = r < p.block_m ? p.sorted_ids[row0 + r] : p.num_ids;
      }
      dq_sync();
      const int r0g = p.gate_up ? ui.item : 2 * ui.item;
      for (int st = 0; st < nstage; st++, g++) {
        const int s = g % NST;
        uint8_t* sb = smem + s * STAGE_STRIDE;
        const bool have_w = wait_ab(B.wfull + s, (g / NST) & 1, deadline, p.err, abort_flag);
        const bool free_a = g < NST || wait_ab(B.aempty + s, ((g / NST) - 1) & 1, deadline, p.err, abort_flag);
        const bool live = have_w && free_a && !*abort_flag;
        // 1. activation rows of this stage into the swizzled B tile (cp.async, 16 bytes each)
        if (live) {
          const uint32_t bbase = smem_u32(sb + B_OFF);
          const int ch = dt & 7;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int r = (dt >> 3) + 32 * j;
            const int id = my_id[j];
            if (id < p.num_ids) {
              const __nv_bfloat16* src = p.A + (int64_t)(id / p.a_div) * p.K + st * BK + ch * 8;
              cp_async16(bbase + r * 128 + ((ch ^ (r & 7)) << 4), src);
            }
          }
        }
        // 2. scale bytes of the stage (4 k-groups x 256 rows), then the exceptions that fall in it
        uint8_t* scb = sb + SCB_OFF;
        if (live && dt < 128) {
          const uint8_t* runp = sb + S_OFF + s_run * RUN_BYTES;
          const uint32_t b4 = runp[s_ch] * 0x01010101u;
          const int kg = (st & 1) * 4 + s_kk;
          const uint32_t q = *reinterpret_cast<const uint32_t*>(runp + 16 + kg * 64 + s_ch * 4);
          const uint32_t lo = (q & 0x0F0F0F0Fu) + b4, hi = ((q >> 4) & 0x0F0F0F0Fu) + b4;
          uint8_t* row = scb + s_kk * SCB_STRIDE;
#pragma unroll
          for (int i = 0; i < 8; i++) row[s_dst[i]] = (uint8_t)(((i < 4 ? lo : hi) >> (8 * (i & 3))) & 0xFF);
        }
        dq_sync();
        if (live) {
          const int rr = st >> 1;
          for (int j = ro[rr] + dt; j < ro[rr + 1]; j += NDQ * 32) {
            const uint32_t en = exl[j];
            const int ppos = en & 0xFFFF, kg = (en >> 16) & 0xFF;
            if ((kg >> 2) != (st & 1)) continue;
            const int slot_e = ((ppos >> 7) == r0g ? 0 : 128) + position_slot(ppos & 127);
            scb[(kg & 3) * SCB_STRIDE + slot_e] = (uint8_t)(en >> 24);
          }
        }
        dq_sync();
        // 3. the oracle's bf16 weights of this warp's two 16-row groups (one per half) into the A tiles
        if (live) {
          const uint8_t* scr = scb + c * SCB_STRIDE;
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int G = h * 8 + dw;
            const uint4 q = *reinterpret_cast<const uint4*>(sb + W_OFF + (G * 32 + lane) * 16);
            const int rA = 16 * dw + gq, rB = rA + 8;  // rows within the half
            const uint32_t wa = lt[scr[h * 128 + rA]], wb = lt[scr[h * 128 + rB]];
            const ScaleBR sa{prmt_b(wa, 0x1010), prmt_b(wa, 0x3232)}, sbv{prmt_b(wb, 0x1010), prmt_b(wb, 0x3232)};
            uint8_t* at = sb + A_OFF + h * (128 * 128);
            const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const int r = (j & 1) ? rB : rA, chunk = 2 * c + (j >> 1);
              uint32_t o[4];
              dequant_word(words[j], (j & 1) ? sbv : sa, o);
              *reinterpret_cast<uint4*>(at + r * 128 + ((chunk ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0 && have_w) mbar_arrive(B.wempty + s);  // packed codes and scales consumed
        cp_async_wait_all();
        fence_async_smem();  // generic-proxy writes (st.shared, cp.async) -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(B.afull + s);
        dq_sync();  // the scale-byte table of this slot is rewritten next time round
      }
      un++;
    }
  } else {  // ------------------------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
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
        nv += __popc(__ballot_sync(0xffffffffu, ids[j] < p.num_ids));
        wts[j] = (!p.gate_up && ids[j] < p.num_ids) ? p.topk_w[ids[j]] : 0.f;
      }
      const int buf = un & 1;
      if (!wait_ab(B.accfull + buf, (un >> 1) & 1, deadline, p.err, abort_flag)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + buf * 256;
      const int row = 32 * q + lane;  // weight row within the half
      for (int c0 = 0; c0 < nv; c0 += 32) {
        float v0[32], v1[32];
        tmem_ld32(tbase + c0, v0);
        tmem_ld32(tbase + 128 + c0, v1);
        const int jj = c0 >> 5;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          if (c0 + j >= nv) break;
          const int id = __shfl_sync(0xffffffffu, ids[jj], j);
          if (p.gate_up) {
            static_cast<__nv_bfloat16*>(p.out)[(int64_t)id * I + 128 * ui.item + row] =
                __float2bfloat16_rn(silu(v0[j]) * v1[j]);
          } else {
            const float w = __shfl_sync(0xffffffffu, wts[jj], j);
            float* orow = p.part + (int64_t)id * p.N + 256 * ui.item;
            orow[row] = w * v0[j];
            orow[128 + row] = w * v1[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(B.accempty + buf);
      un++;
    }
  }
  // ------------------------------------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace pf

int prefill_block_m() { return pf::BMP; }

cudaError_t launch_prefill(const GemmParams& p, int sms, cudaStream_t st) {
  const int nt = p.N / ITEM_COLS;
  const int64_t units = (int64_t)p.max_blocks * nt;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sms, units));
  cudaError_t e = cudaFuncSetAttribute(pf::moek_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM);
  if (e != cudaSuccess) return e;
  e = launch_pdl(pf::moek_prefill_kernel, dim3(grid), dim3(pf::THREADS), pf::SMEM, st, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace moek
