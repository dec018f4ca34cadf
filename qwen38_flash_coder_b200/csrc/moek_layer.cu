// The whole decode-regime routed-expert layer in one persistent kernel, sm_100a: routing, gate_up GEMM + SwiGLU,
// down GEMM x router weight and the top-k sum, with no launch between the steps.
//
// The layer's data is small next to the latencies of a launch: a decode batch touches ~40 experts (about 60 MB of
// packed weights), which one B200 streams in ~10 us, while a launch boundary costs a few microseconds of pipeline
// drain and refill. So the steps that the reference runs as separate kernels (files/mbx_moek.py:252-289: moe_align,
// the gate_up GEMM, SwiGLU, the down GEMM, the top-k sum) run here inside one grid of persistent CTAs (two per SM).
//
// Work plan (stream-K, two phases). A block is a run of at most XR routed slots of one expert (moe_align's blocks);
// a pair is (block, gate_up item t): item t's 256 weight rows (128 gate rows and their up partners) give the block's
// act columns [128 t, 128 t + 128), which are exactly the k-slice t of the down GEMM.
//   gate_up   the sequence of every pair's 128-k stages (pair-major) is cut into C equal contiguous ranges, one per
//             CTA; a CTA's range meets a few pairs, and for each it writes its fp32 partial sums (a record: record
//             index = CTA + pair, unique because both grow along the sequence) and raises one flag per consumer warp
//             (stamped with the launch epoch). No CTA waits for another in this phase.
//   down      the sequence of every pair's down items (256 output rows over the pair's k-slice) is cut the same way;
//             before its first item of a pair a CTA waits for the pair's records (the CTAs whose gate_up ranges met
//             the pair: at most H / 128 of them), adds them in CTA order and forms the act (SwiGLU, rounded to bf16).
//             Each item's fp32 partial rows of k-slice t are written with plain stores. A CTA's down pairs are about
//             the pairs its own gate_up range covered, so the records it waits for are its own and its neighbours',
//             which finish at about the same time, and the weights of its down items stream in while it waits.
//   sums      after a grid barrier every CTA sums a slice of the outputs: per token, per valid slot in slot order,
//             w * (sum of the k-slices in order), then the slots in order, rounded once to bf16 (the fp32 oracle's
//             order, bench/moek/problem.py:51-67).
// Every CTA streams the same number of stages (+- 1 per phase), whatever the batch. The plan is a function of the
// number of blocks and the grid only, so every call with the same routing gives the same bits.
//
// Roles of a CTA (per 128-k stage = one 16 KB bulk copy of packed codes + a 1056-byte packed-scale run pair):
//   producer  warp 8: decodes the CTA's units (the unit list of the plan, two metadata rounds in flight) and issues
//             the stage copies (cp.async.bulk, no multicast) into a ring slot. It never waits on another CTA.
//   act warp  warp 9: gate_up stages: the block's hidden rows by bulk copy; down stages read the act buffer in shared
//             memory (formed by the consumers from the records) and need nothing.
//   scales    warp 10: per stage the scale byte of each k-group x run position (base + 4-bit offset, then the
//             exceptions); per table change the {B B, R R} table of the expert (moek_common.cuh).
//   consumers warps 0-7: swap-AB mma.sync m16n8k16 (weights = the 16-row A operand, up to 8 tokens = B), fp32
//             accumulators per unit.
//
// Every wait is bounded (%globaltimer); a CTA whose wait expires records MOEK_DEV_TIMEOUT and winds down; the state
// buffer must then be zeroed again. The exchange flags and the grid barrier carry a launch epoch, so the state is
// zeroed once at allocation and never between launches.
//
// Co-residency: down units and the grid barrier wait on other CTAs, so the launcher sizes the grid to the
// occupancy the kernel reaches (cudaOccupancyMaxActiveBlocksPerMultiprocessor x SMs) and launches it as a cooperative
// grid, so that the runtime starts it only with every CTA resident, also while kernels of other streams hold part of
// the GPU.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "moek_common.cuh"
#include "moek_ep.cuh"
#include "moek_kernels.cuh"
#include "moek_route.cuh"

namespace moek {
namespace dl {

constexpr int NCW = 8;  // consumer warps
constexpr int W_PROD = NCW, W_ACT = NCW + 1, W_SCALE = NCW + 2;
constexpr int THREADS = (NCW + 3) * 32;
constexpr int LBK = 2 * BK;                  // k per pipeline stage: one packed-scale run pair
constexpr int LSTAGE = 2 * STAGE_BYTES;      // 16 KB of packed codes per (item, stage): one bulk copy
constexpr int X_STRIDE = LBK * 2 + 16;       // bytes per activation row in a slot (+16: conflict-free reads)
constexpr int SC_BYTES = ITEM_COLS * KG;     // scale table of a stage: one byte per (weight row, k-group)
constexpr int NLUT = 4;  // {B B, R R} tables in flight (>= ring slots: a table is rewritten only once the consumers
                         // have released every stage of the NLUT tables before it; each table spans >= 1 stage)
constexpr int MAXU = 8;  // units per metadata round; two rounds in flight
constexpr int LUT_NEW = 1 << 30;  // UnitMeta::lut: the unit starts a new table

// A unit: ph 0 = a gate_up range of pair `pair`: item `item`'s 128-k stages [st0, st0 + nst), written to record
// `rec`; ph 1 = a down run of pair `pair`: items [item, item + nst) each over the 128-k stage st0 (the pair's k-slice),
// after the records of CTAs [c0, c1]. Stage j of a unit is (unit_item(j), unit_kstage(j)).
struct UnitMeta {
  int ph, blk, item, st0, nst;
  int e, nv, flags;  // expert, valid rows (<= XR), 2 = block has more rows than XR
  int lut;           // table index (| LUT_NEW when the scale warp writes it at this unit)
  int pair, rec, c0, c1;
  __device__ __forceinline__ int unit_item(int j) const { return ph ? item + j : item; }
  __device__ __forceinline__ int unit_kstage(int j) const { return ph ? st0 : st0 + j; }
};

// v / d for 0 <= v < 2^22 and 1 <= d <= 2^10, without the long dependent chain of an integer division: a quotient
// estimate from the approximate fp32 reciprocal (relative error about 2^-23, so the estimate is off by at most one)
// and one correction each way.
__device__ __forceinline__ int div_small(int v, int d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"((float)d));
  int q = __float2int_rz((float)v * r);
  const int rem = v - q * d;
  q += (rem >= d) - (rem < 0);
  return q;
}

// The stream-K plan: S1 = pairs x nst1 gate_up stages cut into C1 = min(C, S1) ranges (so that every range holds at
// least one stage and at most H / 128 CTAs meet a pair), CTA c < C1's = [floor(c S1 / C1), floor((c + 1) S1 / C1)),
// CTAs from C1 on have none; S2 = pairs x nt2 down items cut into C ranges the same way. The bounds are evaluated as
// c q + floor(c r / C) (S = q C + r, c r < 2^20) with the reciprocal-estimate division, so that no thread runs an
// integer division routine on the start-up path.
struct SKPlan {
  int npairs, nt1, nst1, nt2, C;
  int s1, c1n, q1, r1, q2, r2;
  __device__ __forceinline__ SKPlan(int nblk, int nt1_, int nst1_, int nt2_, int C_)
      : npairs(nblk * nt1_), nt1(nt1_), nst1(nst1_), nt2(nt2_), C(C_) {
    s1 = npairs * nst1;
    c1n = min(C, s1);
    q1 = c1n ? div_small(s1, c1n) : 0;
    r1 = s1 - q1 * c1n;
    const int s2 = npairs * nt2;
    q2 = div_small(s2, C);
    r2 = s2 - q2 * C;
  }
  __device__ __forceinline__ int lo1(int c) const {
    c = min(c, c1n);
    return c1n ? c * q1 + div_small(c * r1, c1n) : 0;
  }
  __device__ __forceinline__ int lo2(int c) const { return c * q2 + div_small(c * r2, C); }
  // the CTA whose gate_up range holds stage q (q < S1): the largest c with lo1(c) <= q (an fp32 estimate, off by at
  // most one, then corrected)
  __device__ __forceinline__ int owner1(int q) const {
    int c = min(max(__float2int_rz(__fdividef(((float)q + 1.f) * (float)c1n, (float)s1)), 0), c1n - 1);
    if (c + 1 < c1n && lo1(c + 1) <= q) c++;
    if (lo1(c) > q) c--;
    return c;
  }
  __device__ __forceinline__ int n_gate(int c) const {
    const int a = lo1(c), b = lo1(c + 1);
    return b > a ? div_small(b - 1, nst1) - div_small(a, nst1) + 1 : 0;
  }
  __device__ __forceinline__ int n_down(int c) const {
    const int a = lo2(c), b = lo2(c + 1);
    return b > a ? div_small(b - 1, nt2) - div_small(a, nt2) + 1 : 0;
  }
  __device__ __forceinline__ int units(int c) const { return n_gate(c) + n_down(c); }
  // unit j of CTA c: its gate_up units (pairs in order), then its down units
  __device__ __forceinline__ void unit(int c, int j, UnitMeta& u) const {
    const int ng = n_gate(c);
    if (j < ng) {
      const int a = lo1(c), b = lo1(c + 1);
      const int pr = div_small(a, nst1) + j, s0 = pr * nst1;
      u.ph = 0;
      u.pair = pr;
      u.st0 = max(a - s0, 0);
      u.nst = min(b - s0, nst1) - u.st0;
      u.rec = c + pr;
      u.c0 = u.c1 = c;
    } else {
      const int a = lo2(c), b = lo2(c + 1);
      const int pr = div_small(a, nt2) + (j - ng), i0 = pr * nt2;
      u.ph = 1;
      u.pair = pr;
      u.item = max(a - i0, 0);
      u.nst = min(b - i0, nt2) - u.item;
      u.rec = -1;
      u.c0 = owner1(pr * nst1);
      u.c1 = owner1(pr * nst1 + nst1 - 1);
    }
    u.blk = pr_blk(u.pair);
    const int t = u.pair - u.blk * nt1;
    if (u.ph == 0)
      u.item = t;
    else
      u.st0 = t;
  }
  __device__ __forceinline__ int pr_blk(int pr) const { return div_small(pr, nt1); }
};

template <int XR>
struct Cfg {
  static constexpr int X_OFF = LSTAGE + PAIR_BYTES;
  static constexpr int SC_OFF = X_OFF + XR * X_STRIDE;
  static constexpr int SLOT = SC_OFF + SC_BYTES;
  static constexpr int NS = XR <= 8 ? 4 : 3;  // ring slots: two CTAs per SM
  static constexpr int ACT_OFF = NS * SLOT;   // the pair's act rows [XR, 128] bf16, X_STRIDE apart (down's B operand)
  static constexpr int META_OFF = ACT_OFF + XR * X_STRIDE;
  static constexpr int IDS_OFF = META_OFF + 2 * MAXU * (int)sizeof(UnitMeta);
  static constexpr int LUT_OFF = IDS_OFF + 2 * MAXU * XR * 4;
  static constexpr int ROUTE_OFF = LUT_OFF + NLUT * 256 * 8;  // srow[MAXIDS], bexp[MAXIDS], bstart[MAXIDS + 1]
  static constexpr int TOK_OFF = ROUTE_OFF + (3 * LAYER_MAXIDS + 1) * 4;  // the batch's slots: sid[], stw[]
  static constexpr int MISC_OFF = TOK_OFF + 2 * LAYER_MAXIDS * 4;
  static constexpr int BAR_OFF = (MISC_OFF + 16 + 7) / 8 * 8;  // mbarriers: 8-byte aligned
  static constexpr int SMEM = BAR_OFF + (3 * NS + 4) * 8;
  static constexpr int T = XR / 8;
  static constexpr int MINB = 2;
  static_assert(XR <= 32, "at most 32 rows per block");
  static_assert(BAR_OFF % 8 == 0 && LUT_OFF % 8 == 0 && META_OFF % 4 == 0 && X_OFF % 16 == 0 && ACT_OFF % 16 == 0 &&
                    SLOT % 16 == 0 && X_STRIDE % 16 == 0,
                "shared-memory sections aligned for their widest access");
  static_assert(2 * LAYER_MAXIDS * 4 <= SLOT, "routing scratch fits in ring slot 0");
  static_assert(XR > 16 || 2 * SMEM + 2048 <= 228 * 1024, "two CTAs per SM (32-row blocks: one)");
};

__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, uint64_t deadline, int* err,
                                              volatile int* abort_flag) {
  if (mbar_try(bar, parity)) return true;  // the common case: the phase is complete, no shared-memory load first
  if (*abort_flag) return false;
  if (mbar_wait_sleep(bar, parity, deadline, err)) return true;
  *abort_flag = 1;
  return false;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory"); }
// The same barrier, returning whether v was set in any consumer thread (every consumer warp gets the same answer, so
// they all take the same path through the barriers that follow).
__device__ __forceinline__ bool consumer_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\n"
      "setp.ne.u32 p, %1, 0;\n"
      "bar.red.or.pred q, 1, %2, p;\n"
      "selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(NCW * 32)
      : "memory");
  return r != 0;
}

// Raise, on every rank s, s's back flag for this rank to this call's number (all of this rank's returned rows are
// written).
__device__ __forceinline__ void ep_signal(const LayerParams& p, int call) {
  for (int s = 0; s < p.ep_world; s++)
    st_sys(reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(p.ep_peer[s]) + p.ep_flags_off) + p.ep_world + p.ep_rank,
           call);
}

// CTAs per destination of the fused exchange's dispatch: up to one per token, at least one (the flag must be raised)
__device__ __forceinline__ int ep_dispatch_ctas(const LayerParams& p) {
  return max(1, min((int)gridDim.x / p.ep_world, p.ep_M));
}

template <int XR>
__global__ void __launch_bounds__(THREADS, Cfg<XR>::MINB) moek_layer_kernel(LayerParams p) {
  using C = Cfg<XR>;
  extern __shared__ __align__(128) uint8_t smem[];
  UnitMeta* meta = reinterpret_cast<UnitMeta*>(smem + C::META_OFF);  // [2][MAXU]
  int* mids = reinterpret_cast<int*>(smem + C::IDS_OFF);             // [2][MAXU][XR]
  uint2* lut = reinterpret_cast<uint2*>(smem + C::LUT_OFF);  // per table: scale byte -> {B B, R R} (moek_common.cuh)
  int* srow = reinterpret_cast<int*>(smem + C::ROUTE_OFF);
  int* bexp = srow + LAYER_MAXIDS;
  int* bstart = bexp + LAYER_MAXIDS;
  // [0] blocks, [1] valid slots, [2] abort, [3] the blocks the plan covers
  volatile int* misc = reinterpret_cast<volatile int*>(smem + C::MISC_OFF);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + C::NS;
  uint64_t* scaled = empty + C::NS;
  uint64_t* mfull = scaled + C::NS;  // [2]
  uint64_t* mempty = mfull + 2;      // [2]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  volatile int* abort_flag = misc + 2;

  if (tid == 0) {
    misc[1] = 0;
    misc[2] = 0;
    for (int i = 0; i < C::NS; i++) {
      mbar_init(full + i, 2);  // the producer's and the act warp's arrivals (each with its byte count)
      mbar_init(empty + i, NCW);
      mbar_init(scaled + i, 32);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(mfull + i, 32);
      mbar_init(mempty + i, NCW + 2);  // consumers, scale warp, act warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) MOEK_TR(0);
  pdl_wait();  // x, routing and weights of the previous kernels; the workspace of the previous launch
  pdl_launch_dependents();
  if (tid == 0) MOEK_TR(1);
  if (tid == 0) MOEK_TR_CLK(39);
  const uint64_t deadline = globaltimer() + p.timeout_ns;
  // expert-parallel: this exchange call's number (the flags carry it, so they never need resetting)
  const int ep_call = p.ep_peer ? *reinterpret_cast<volatile const int*>(p.ep_call) + 1 : 0;
  if (p.ep_x) {  // fused exchange: CTAs [0, world x G) first send this rank's tokens to their experts' owners
    const int G = ep_dispatch_ctas(p);
    if ((int)blockIdx.x < p.ep_world * G) {
      if (tid == 0) MOEK_TR(48);
      const int d = blockIdx.x / G;
      int* spos = reinterpret_cast<int*>(smem);  // scratch in ring slot 0, as the routing's below
      ep_dispatch_cta<THREADS, 4, 46>(p.ep_q, p.ep_x, p.ep_ids, p.ep_w, p.ep_M, p.ep_E, d, blockIdx.x - d * G, G,
                                      ep_call, p.ep_pos, spos, spos + LAYER_MAXIDS);
    }
  }
  const int n = p.num_ids, k = p.top_k;
  // the batch's routing in shared memory for the whole kernel (ids and router weights of every slot): loaded first
  // (each thread's at most two slots: n <= 512 < 2 x THREADS), or computed from the router logits by every CTA (one
  // warp per token); expert-parallel receive buffers are read only after their flags (below)
  int* sid = reinterpret_cast<int*>(smem + C::TOK_OFF);
  float* stw = reinterpret_cast<float*>(sid + LAYER_MAXIDS);
  int e_in[2] = {-1, -1};
  float w_in[2] = {0.f, 0.f};
  if (p.logits) {
    for (int t = warp; t < p.M; t += THREADS / 32) {
      int es;
      float ws;
      if (p.logits_bf16)
        route_token<16>(static_cast<const __nv_bfloat16*>(p.logits) + (int64_t)t * p.E, p.E, k, p.renorm, es, ws);
      else
        route_token<16>(static_cast<const float*>(p.logits) + (int64_t)t * p.E, p.E, k, p.renorm, es, ws);
      if (lane < k) {
        sid[t * k + lane] = es;
        stw[t * k + lane] = ws;
        if (blockIdx.x == 0 && p.ids_out) p.ids_out[t * k + lane] = es;
        if (blockIdx.x == 0 && p.w_out) p.w_out[t * k + lane] = ws;
      }
    }
    __syncthreads();
    if (tid < n) e_in[0] = sid[tid];
    if (tid + THREADS < n) e_in[1] = sid[tid + THREADS];
  } else if (!p.ep_peer) {
    if (tid < n) {
      e_in[0] = p.ids[tid];
      w_in[0] = p.tw[tid];
    }
    if (tid + THREADS < n) {
      e_in[1] = p.ids[tid + THREADS];
      w_in[1] = p.tw[tid + THREADS];
    }
  }
  const int epoch = *reinterpret_cast<volatile const int*>(p.ctr + p.off_epoch);
  if (p.ep_peer) {  // expert-parallel: wait until every sender's rows, ids and weights are in the receive buffers
    if (warp == 0) {
      bool good = true;
      for (int s = lane; s < p.ep_world; s += 32) good &= wait_flag(p.ep_recv_flags + s, ep_call, deadline, p.err);
      if (!__all_sync(0xffffffffu, good) && lane == 0) misc[2] = 1;
      if (lane == 0) MOEK_TR(2);
    }
    __syncthreads();
    asm volatile("fence.proxy.async.global;" ::: "memory");  // the bulk copies below read what the peers wrote
  }

  // ------------------------------------------------------------------------------------------------- routing
  {
    uint32_t* key = reinterpret_cast<uint32_t*>(smem);  // scratch in ring slot 0: nothing is copied there yet
    uint32_t* skey = key + LAYER_MAXIDS;
    const int n4 = (n + 3) & ~3;  // keys padded to whole uint4 with 0xFFFFFFFF (above every valid key)
    uint32_t kk[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int i = tid + h * THREADS;
      if (p.ep_peer && i < n) {
        e_in[h] = p.ids[i];
        w_in[h] = p.tw[i];
      }
      if (i < n && !p.logits) {
        sid[i] = e_in[h];
        stw[i] = w_in[h];
      }
      const bool v = i < n && e_in[h] >= 0 && e_in[h] < p.E;
      kk[h] = v ? ((uint32_t)e_in[h] << 9) | (uint32_t)i : 0xFFFFFFFFu;
      if (i < n4) key[i] = kk[h];
    }
    if (tid == 0) MOEK_TR_CLK(40);
    const int nvalid = __syncthreads_count(kk[0] != 0xFFFFFFFFu) + __syncthreads_count(kk[1] != 0xFFFFFFFFu);
    if (tid == 0) MOEK_TR_CLK(41);
#pragma unroll
    for (int h = 0; h < 2; h++) {  // rank of each valid key among all keys (they are distinct): 4 keys per load
      if (kk[h] == 0xFFFFFFFFu) continue;
      int r = 0;
      for (int j = 0; j < n4; j += 4) {
        const uint4 q = *reinterpret_cast<const uint4*>(key + j);
        r += (q.x < kk[h]) + (q.y < kk[h]) + (q.z < kk[h]) + (q.w < kk[h]);
      }
      skey[r] = kk[h];
    }
    if (tid == 0) MOEK_TR_CLK(42);
    __syncthreads();
    if (warp == 0) {  // blocks: one starts where the expert changes, and after every XR rows of the same expert
      int base = 0, run0 = 0;  // run0: where the expert run that reaches into this chunk started
      for (int p0 = 0; p0 < nvalid; p0 += 32) {
        const int pos = p0 + lane;
        uint32_t kv = 0;
        bool ehead = false;
        if (pos < nvalid) {
          kv = skey[pos];
          ehead = pos == 0 || (skey[pos - 1] >> 9) != (kv >> 9);
          srow[pos] = (int)(kv & 511u);
        }
        const uint32_t eh = __ballot_sync(0xffffffffu, ehead) & (0xffffffffu >> (31 - lane));  // at lanes <= mine
        const int rs = eh ? p0 + 31 - __clz(eh) : run0;  // start of my expert's run
        const bool head = pos < nvalid && (pos - rs) % XR == 0;
        const uint32_t hb = __ballot_sync(0xffffffffu, head);
        if (head) {
          const int bi = base + __popc(hb & ((1u << lane) - 1u));
          bstart[bi] = pos;
          bexp[bi] = (int)(kv >> 9);
        }
        base += __popc(hb);
        run0 = __shfl_sync(0xffffffffu, rs, 31);
      }
      if (lane == 0) {
        MOEK_TR_CLK(43);
        bstart[base] = nvalid;
        misc[0] = base;
        misc[3] = *abort_flag ? 0 : base;  // the blocks the plan covers
        MOEK_TR_CLK(44);
      }
    }
    __syncthreads();
  }
  if (tid == 0) MOEK_TR(3);
  if (tid == 0) MOEK_TR_CLK(45);

  const int nt1 = p.m[0].nt, nst1 = p.m[0].nstage, nt2 = p.m[1].nt, nst2 = p.m[1].nstage;
  const SKPlan plan(misc[3], nt1, nst1, nt2, (int)gridDim.x);
  const int n_mine = plan.units(blockIdx.x);
  const int rounds = (n_mine + MAXU - 1) / MAXU;
  if (tid == 0) MOEK_TR_VAL(7, n_mine);
  if (tid == 0) MOEK_TR_CLK(53);

  if (warp == W_PROD) {  // ------------------------------------------------------------------------- producer
    uint32_t g = 0;
    bool ok = true;
    int lut_cur = -1, prev_key = -1;  // the last table index and its (phase, expert)
    for (int r = 0; r < rounds && ok; r++) {
      const int b = r & 1, u0 = r * MAXU, nu = min(MAXU, n_mine - u0);
      UnitMeta* mb = meta + b * MAXU;
      int* ib = mids + b * MAXU * XR;
      if (r >= 2 && !wait_or_abort(mempty + b, ((r - 2) >> 1) & 1, deadline, p.err, abort_flag)) break;
      UnitMeta um;
      int key = -1, b0 = 0;
      if (lane < nu) {
        plan.unit(blockIdx.x, u0 + lane, um);
        um.e = bexp[um.blk];
        b0 = bstart[um.blk];
        const int cnt = bstart[um.blk + 1] - b0;
        um.nv = min(cnt, XR);
        um.flags = cnt > XR ? 2 : 0;
        key = (um.ph << 24) | um.e;
      }
      if (lane == 0 && r == 0) MOEK_TR_CLK(54);
      // table indices: a new {B B, R R} table wherever (phase, expert) changes from the unit before
      const int kprev = __shfl_up_sync(0xffffffffu, key, 1);
      const bool isnew = lane < nu && key != (lane == 0 ? prev_key : kprev);
      const uint32_t nbits = __ballot_sync(0xffffffffu, isnew);
      if (lane < nu) {
        um.lut = (lut_cur + __popc(nbits & ((2u << lane) - 1u))) | (isnew ? LUT_NEW : 0);
        mb[lane] = um;
        for (int rr = 0; rr < um.nv; rr++) ib[lane * XR + rr] = srow[b0 + rr];
      }
      lut_cur += __popc(nbits);
      prev_key = __shfl_sync(0xffffffffu, key, nu - 1);
      __syncwarp();
      if (lane == 0 && r == 0) MOEK_TR_CLK(55);
      mbar_arrive(mfull + b);  // units, experts and rows published
      for (int ci = 0; ci < nu && ok; ci++) {
        const UnitMeta& m = mb[ci];
        const LayerMat& mt = p.m[m.ph];
        const int e = m.e;
        for (int j = 0; j < m.nst; j++, g++) {
          const int slot = g % C::NS, st = m.unit_kstage(j), item = m.unit_item(j);
          if (g >= C::NS && !wait_or_abort(empty + slot, ((g / C::NS) - 1) & 1, deadline, p.err, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + slot * C::SLOT;
          if (lane == 0) mbar_expect_tx(full + slot, LSTAGE + PAIR_BYTES);
          __syncwarp();
          if (lane == 0) {  // the two consecutive 64-k blocks of the stage
            const int64_t wi = (((int64_t)e * mt.nt + item) * mt.nstage + st) * 2;
            bulk_g2s(dst, mt.W + wi * STAGE_BYTES, LSTAGE, full + slot);
            if (g == 0) MOEK_TR(4);
            if (r == 0 && ci == 0 && j < 8) MOEK_TR_CLK(112 + j);
          } else if (lane == 1) {
            const int64_t si = ((int64_t)e * mt.nt + item) * mt.nstage + st;
            bulk_g2s(dst + LSTAGE, mt.SP + si * PAIR_BYTES, PAIR_BYTES, full + slot);
          }
          __syncwarp();
        }
      }
    }
  } else if (warp == W_ACT) {  // ----------------------------------------------------------------------- act warp
    uint32_t g = 0;
    bool ok = true;
    for (int r = 0; r < rounds && ok; r++) {
      const int b = r & 1, nu = min(MAXU, n_mine - r * MAXU);
      const UnitMeta* mb = meta + b * MAXU;
      if (!wait_or_abort(mfull + b, (r >> 1) & 1, deadline, p.err, abort_flag)) break;
      for (int ci = 0; ci < nu && ok; ci++) {
        const UnitMeta& m = mb[ci];
        const int nv = m.nv;
        const int* ids = mids + (b * MAXU + ci) * XR;
        for (int j = 0; j < m.nst; j++, g++) {
          const int slot = g % C::NS, st = m.unit_kstage(j);
          if (g >= C::NS && !wait_or_abort(empty + slot, ((g / C::NS) - 1) & 1, deadline, p.err, abort_flag)) {
            ok = false;
            break;
          }
          if (m.ph == 0) {  // hidden rows of the block's tokens, 128 k each, by bulk copy
            uint8_t* xs = smem + slot * C::SLOT + C::X_OFF;
            if (lane == 0) mbar_expect_tx(full + slot, nv * LBK * 2);
            __syncwarp();
            for (int rr = lane; rr < nv; rr += 32)
              bulk_g2s(xs + rr * X_STRIDE, p.x + (int64_t)(ids[rr] / k) * p.H + st * LBK, LBK * 2, full + slot);
            if (lane == 0 && r == 0 && ci == 0 && j < 8) MOEK_TR_CLK(120 + j);
          } else if (lane == 0) {  // down: the act rows are in shared memory already
            mbar_arrive(full + slot);
          }
          __syncwarp();
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mempty + b);
    }
  } else if (warp == W_SCALE) {  // -------------------------------------------------------------------- scale warp
    // Per unit: the expert's global scale and each stage's exception run [a, b) of the kit's list (lane j: stage j's
    // run), loaded by all lanes at once and one unit ahead, then the unit's entries (up to 64 held in registers, two
    // per lane, numbered across the unit's runs in stage order), so that no stage waits on a chain of global loads.
    // Per stage: the slot's scale table in run-position order, one byte per (k-group, run, position) at
    // kg * 256 + run * 128 + position (the consumers map their rows to positions), then the run's exceptions. Lane L
    // decodes chunk L % 16 (8 positions) of run L / 16 of the pair: eight 8-byte stores, no byte shuffling, so that
    // the single scale warp keeps ahead of the consumers.
    uint32_t g = 0;
    const int run = lane >> 4, ch = lane & 15;
    bool ok = true;
    for (int r = 0; r < rounds && ok; r++) {
      const int b = r & 1, nu = min(MAXU, n_mine - r * MAXU);
      const UnitMeta* mb = meta + b * MAXU;
      if (!wait_or_abort(mfull + b, (r >> 1) & 1, deadline, p.err, abort_flag)) break;
      int ra_n = 0, rb_n = 0;
      float g_n = 0.f;
      auto fetch = [&](int ui) {  // loads only; consumed one unit later
        const UnitMeta& m = mb[ui];
        const LayerMat& mt = p.m[m.ph];
        if (lane < m.nst) {
          const int64_t key = ((int64_t)m.e * mt.nt + m.unit_item(lane)) * mt.nstage + m.unit_kstage(lane);
          ra_n = mt.exc_off[key];
          rb_n = mt.exc_off[key + 1];
        } else {
          ra_n = rb_n = 0;
        }
        g_n = mt.G[m.e];
      };
      if (nu > 0) fetch(0);
      for (int ui = 0; ui < nu && ok; ui++) {
        const UnitMeta& m = mb[ui];
        const LayerMat& mt = p.m[m.ph];
        const int ra = ra_n, len = rb_n - ra_n;
        int pre = len;  // exclusive prefix of the runs' lengths: stage j's entries are numbered [pre_j, pre_j + len_j)
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, pre, o);
          if (lane >= o) pre += v;
        }
        const int total = __shfl_sync(0xffffffffu, pre, 31);
        pre -= len;
        const float gsc = g_n;
        // entry number L of the unit: in the run of the last stage whose first number is <= L
        auto entry = [&](int L) -> uint32_t {
          int a = 0, p0 = 0;
          for (int jj = 0; jj < m.nst; jj++) {
            const int pj = __shfl_sync(0xffffffffu, pre, jj), aj = __shfl_sync(0xffffffffu, ra, jj);
            if (pj <= L) a = aj, p0 = pj;
          }
          return L < total ? mt.exc_ent[a + L - p0] : 0u;
        };
        const uint32_t ex0 = entry(lane), ex1 = entry(lane + 32);
        if (ui + 1 < nu) fetch(ui + 1);
        uint2* lt = lut + ((m.lut & 0xFFFF) % NLUT) * 256;
        for (int j = 0; j < m.nst; j++, g++) {
          const int slot = g % C::NS, item = m.unit_item(j);
          if (!wait_or_abort(full + slot, (g / C::NS) & 1, deadline, p.err, abort_flag)) {
            ok = false;
            break;
          }
          if (lane == 0 && r == 0 && ui == 0 && j < 8) MOEK_TR_CLK(96 + j);
          if (j == 0 && (m.lut & LUT_NEW)) {  // a new table: its slot's previous table is no longer read
#pragma unroll
            for (int jj = 0; jj < 8; jj++) {
              const ScaleBR br = scale_br(lane + 32 * jj, gsc);
              lt[lane + 32 * jj] = make_uint2(br.b2, br.r2);
            }
          }
          const uint8_t* runp = smem + slot * C::SLOT + LSTAGE + run * RUN_BYTES;
          uint8_t* tb = smem + slot * C::SLOT + C::SC_OFF;
          const uint32_t b4 = runp[ch] * 0x01010101u;
#pragma unroll
          for (int kk = 0; kk < KG; kk++) {  // k-group kk's bytes of positions 8 ch + 0..3 (low nibbles), + 4..7
            const uint32_t q = *reinterpret_cast<const uint32_t*>(runp + 16 + kk * 64 + ch * 4);
            *reinterpret_cast<uint2*>(tb + kk * 256 + run * 128 + 8 * ch) =
                make_uint2((q & 0x0F0F0F0Fu) + b4, ((q >> 4) & 0x0F0F0F0Fu) + b4);
          }
          __syncwarp();
          // this stage's run: entries [eo0, eo1) of the unit's numbering overwrite their bytes
          const int eo0 = __shfl_sync(0xffffffffu, pre, j);
          const int eo1 = eo0 + __shfl_sync(0xffffffffu, len, j), aj = __shfl_sync(0xffffffffu, ra, j);
          const int r0g = m.ph == 0 ? item : 2 * item;           // global run index of the pair's first run
          const int r1g = m.ph == 0 ? mt.nt + item : r0g + 1;    // and of its second (gate_up: the up rows' run)
          auto patch = [&](uint32_t en) {
            const int ppos = en & 0xFFFF, kg = (en >> 16) & 0xFF;
            if (!MOEK_CHECK(kg < KG && ((ppos >> 7) == r0g || (ppos >> 7) == r1g), p.err)) return;
            tb[kg * 256 + ((ppos >> 7) == r0g ? 0 : 128) + (ppos & 127)] = (uint8_t)(en >> 24);
          };
          if (lane >= eo0 && lane < eo1) patch(ex0);
          if (lane + 32 >= eo0 && lane + 32 < eo1) patch(ex1);
          for (int L = max(eo0, 64) + lane; L < eo1; L += 32) patch(mt.exc_ent[aj + L - eo0]);  // long runs
          __syncwarp();
          mbar_arrive(scaled + slot);
          if (lane == 0 && r == 0 && ui == 0 && j < 8) MOEK_TR_CLK(104 + j);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mempty + b);
    }
  } else {  // ------------------------------------------------------------------------------------------ consumers
    const int gq = lane >> 2, c = lane & 3;
    const int w_off = ((((c >> 1) ^ (gq >> 2)) & 1) << 4) | ((c & 1) << 3);  // k-group c's bytes in a 32-byte row
    const int H = p.H;
    __nv_bfloat16* act_s = reinterpret_cast<__nv_bfloat16*>(smem + C::ACT_OFF);
    uint32_t g = 0;
    for (int r = 0; r < rounds; r++) {
      const int b = r & 1, nu = min(MAXU, n_mine - r * MAXU);
      const UnitMeta* mb = meta + b * MAXU;
      wait_or_abort(mfull + b, (r >> 1) & 1, deadline, p.err, abort_flag);
      const bool have_meta = !consumer_sync_or(*abort_flag);
      bool pre_seen = false;  // this lane's record flag of the next (down) unit was seen set during this unit
      for (int ui = 0; ui < nu && have_meta; ui++) {
        const UnitMeta& m = mb[ui];
        const int ph = m.ph, nv = m.nv;
        const int* ids = mids + (b * MAXU + ui) * XR;
        if ((m.flags & 2) && tid == 0) report(p.err, MOEK_DEV_TOO_MANY_ROWS);
        // the warp's two 16-row groups of the item (gate_up: gate group w and its up partner w + 8)
        const int G0 = ph == 0 ? warp : 2 * warp, G1 = ph == 0 ? warp + 8 : 2 * warp + 1;
        const int slot00 = 16 * G0 + gq, slot10 = 16 * G1 + gq;
        // the scale-table offsets (run * 128 + position) of the lane's four rows
        auto tpos = [](int r) { return (r & 128) + slot_position(r & 127); };
        const int p00 = tpos(slot00), p01 = tpos(slot00 + 8), p10 = tpos(slot10), p11 = tpos(slot10 + 8);
        const uint2* lt = lut + ((m.lut & 0xFFFF) % NLUT) * 256;
        const int ntile = (nv + 7) >> 3;
        // one accumulator chain per (row group, tile) and gate_up share or down item
        float acc[2][C::T][4];
#pragma unroll
        for (int i = 0; i < 2; i++)
#pragma unroll
          for (int t = 0; t < C::T; t++)
#pragma unroll
            for (int v = 0; v < 4; v++) acc[i][t][v] = 0.f;
        bool ok = true;
        const int tu = r * MAXU + ui;  // the unit's index among this CTA's (timeline stamps)
        bool ready = false;  // the next stage's scales were seen published while this stage was computed
        // down: this CTA's fp32 partials of k-slice st0, one item per stage (summed after the grid barrier)
        float* dbase = p.part2 + ((int64_t)m.st0 * n) * H;
        if (ph == 1) {  // ------------------------------------------------------------- the pair's act from records
          // every warp is done with the previous unit's operands before the act buffer is rewritten
          consumer_sync();
          if (!*abort_flag) {
            // the records of CTAs [c0, c1] for this warp's act columns [16 w, 16 w + 16) (lane i polls CTA c0 + i;
            // at most H / 128 <= 32 CTAs meet a pair)
            const int nrec = m.c1 - m.c0 + 1;
            const int* flags = p.ctr + p.off_xflag;
            bool seen = lane >= nrec || pre_seen;
            pre_seen = false;
            for (uint32_t it = 0;; it++) {
              if (!seen) seen = ld_acquire(flags + (int64_t)(m.c0 + lane + m.pair) * NCW + warp) == epoch + 1;
              if (__all_sync(0xffffffffu, seen)) break;
              if ((it & 63) == 63 && globaltimer() > deadline) {
                if (lane == 0) {
                  report(p.err, MOEK_DEV_TIMEOUT);
                  *abort_flag = 1;
                }
                break;
              }
              __nanosleep(32);
            }
            __syncwarp();
            if (!*abort_flag) {
              // act = bf16(silu(gate) * up), gate and up the records' sums in CTA order. Lane 4 r + q takes columns
              // 16 w + 4 q .. + 3 of row r (8 rows per pass): two 16-byte loads per record, two records' loads in
              // flight before they are added, so a pair costs about one L2 round trip per two records.
              const float* rec0 = p.xpart + (int64_t)(m.c0 + m.pair) * XR * ITEM_COLS + 16 * warp + 4 * (lane & 3);
              for (int row = lane >> 2; row < nv; row += 8) {
                const float* b = rec0 + row * ITEM_COLS;
                float4 gs = make_float4(0.f, 0.f, 0.f, 0.f), us = gs;
                for (int s2 = 0; s2 < nrec; s2 += 2) {
                  float4 gv[2], uv[2];
#pragma unroll
                  for (int u = 0; u < 2; u++) {
                    if (s2 + u < nrec) {
                      gv[u] = __ldcg(reinterpret_cast<const float4*>(b + (s2 + u) * XR * ITEM_COLS));
                      uv[u] = __ldcg(reinterpret_cast<const float4*>(b + (s2 + u) * XR * ITEM_COLS + ITEM_COLS / 2));
                    }
                  }
#pragma unroll
                  for (int u = 0; u < 2; u++) {
                    if (s2 + u < nrec) {
                      gs.x += gv[u].x, gs.y += gv[u].y, gs.z += gv[u].z, gs.w += gv[u].w;
                      us.x += uv[u].x, us.y += uv[u].y, us.z += uv[u].z, us.w += uv[u].w;
                    }
                  }
                }
                const __nv_bfloat162 a01 = __floats2bfloat162_rn(silu(gs.x) * us.x, silu(gs.y) * us.y);
                const __nv_bfloat162 a23 = __floats2bfloat162_rn(silu(gs.z) * us.z, silu(gs.w) * us.w);
                uint2 pk;
                pk.x = *reinterpret_cast<const uint32_t*>(&a01);
                pk.y = *reinterpret_cast<const uint32_t*>(&a23);
                *reinterpret_cast<uint2*>(act_s + row * (X_STRIDE / 2) + 16 * warp + 4 * (lane & 3)) = pk;
              }
            }
          }
          consumer_sync();  // the act buffer holds the pair's act rows
        }
        for (int j = 0; j < m.nst; j++, g++) {
          const int slot = g % C::NS;
          const uint32_t par = (g / C::NS) & 1;
          const bool stamp = tid == 0 && tu == 0 && j < 8;
          if (stamp) MOEK_TR_CLK(64 + j);
          // one wait: the scale warp arrives on `scaled` only after its own wait on `full` (weights, scales and
          // activations of the slot landed), so the consumers' acquire of `scaled` orders their reads after those
          // writes as well. Usually the test made during the previous stage already saw the phase complete, and the
          // stage starts without a wait on its critical path.
          if (!ready && !wait_or_abort(scaled + slot, par, deadline, p.err, abort_flag)) {
            ok = false;
            continue;  // stay in step with the other roles' counters
          }
          ready = false;
          if (stamp) MOEK_TR_CLK(80 + j);
          if (tid == 0 && j == 0 && tu < 8) {
            MOEK_TR(8 + 3 * tu);
            MOEK_TR_VAL(32 + tu, (ph << 28) | (m.blk << 16) | (m.item << 8) | m.st0);
          }
          // B operand rows: gate_up the slot's hidden rows, down the pair's act rows
          const uint8_t* xrows = ph == 0 ? smem + slot * C::SLOT + C::X_OFF : smem + C::ACT_OFF;
#pragma unroll
          for (int hf = 0; hf < 2; hf++) {  // the stage's two 64-k halves: an 8 KB block of codes and 4 k-groups each
          if (hf == 1 && j + 1 < m.nst)  // test the next stage's scales (its latency hides behind this half's math)
            ready = mbar_test(scaled + (g + 1) % C::NS, ((g + 1) / C::NS) & 1);
          if (hf == 1 && j + 1 == m.nst && ui + 1 < nu && mb[ui + 1].ph == 1) {
            // the next unit is a down unit: test its records' flags now, so that the load's latency hides behind
            // this half's math and the unit's prologue usually needs no poll
            const UnitMeta& mn = mb[ui + 1];
            pre_seen = lane < mn.c1 - mn.c0 + 1 &&
                       ld_acquire(p.ctr + p.off_xflag + (int64_t)(mn.c0 + lane + mn.pair) * NCW + warp) == epoch + 1;
          }
          const uint8_t* sw = smem + slot * C::SLOT + hf * STAGE_BYTES;
          const uint8_t* sx = xrows + hf * BK * 2;
          const uint8_t* sc = smem + slot * C::SLOT + C::SC_OFF + (4 * hf + c) * 256;  // k-group 4 hf + c
          const uint2 s0a = lt[sc[p00]], s0b = lt[sc[p01]], s1a = lt[sc[p10]], s1b = lt[sc[p11]];
          // the tiles' activation fragments of this half, shared by both row groups (loaded once here for one-tile
          // blocks; larger blocks load them next to their MMAs, to keep registers free)
          uint4 xf[C::T][2];
          if constexpr (C::T == 1) {
            const uint8_t* xr = sx + gq * X_STRIDE + c * 32;
            xf[0][0] = *reinterpret_cast<const uint4*>(xr);
            xf[0][1] = *reinterpret_cast<const uint4*>(xr + 16);
          }
#pragma unroll
          for (int i = 0; i < 2; i++) {
            const uint2 wa = i ? s1a : s0a, wb = i ? s1b : s0b;
            const ScaleBR sa{wa.x, wa.y}, sbv{wb.x, wb.y};
            const uint8_t* wr = sw + (16 * (i ? G1 : G0) + gq) * 32 + w_off;
            const uint2 qa = *reinterpret_cast<const uint2*>(wr), qb = *reinterpret_cast<const uint2*>(wr + 8 * 32);
            if constexpr (C::T > 1) {
#pragma unroll
              for (int t = 0; t < C::T; t++) {
                if (t < ntile) {
                  const uint8_t* xr = sx + (t * 8 + gq) * X_STRIDE + c * 32;
                  xf[t][0] = *reinterpret_cast<const uint4*>(xr);
                  xf[t][1] = *reinterpret_cast<const uint4*>(xr + 16);
                }
              }
            }
            // four MMAs: MMA j takes pairs 2(j & 1) and 2(j & 1) + 1 of rows g and g + 8 from the first (j < 2) or
            // second word of the k-group; each A fragment is dequantised straight into its operand registers
            auto mma_j = [&](auto jc, uint32_t wa, uint32_t wb) {
              constexpr int J = decltype(jc)::value, P0 = 2 * (J & 1), P1 = P0 + 1;
              const uint32_t A[4] = {dequant_pair<P0>(wa, sa), dequant_pair<P0>(wb, sbv), dequant_pair<P1>(wa, sa),
                                     dequant_pair<P1>(wb, sbv)};
#pragma unroll
              for (int t = 0; t < C::T; t++) {
                if (C::T == 1 || t < ntile) {  // a unit has at least one row: one-tile blocks need no test
                  const uint4& xv = xf[t][J >> 1];
                  mma_16816(acc[i][t], A, (J & 1) ? xv.z : xv.x, (J & 1) ? xv.w : xv.y);
                }
              }
            };
            mma_j(std::integral_constant<int, 0>{}, qa.x, qb.x);
            mma_j(std::integral_constant<int, 1>{}, qa.x, qb.x);
            mma_j(std::integral_constant<int, 2>{}, qa.y, qb.y);
            mma_j(std::integral_constant<int, 3>{}, qa.y, qb.y);
          }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(empty + slot);
          if (stamp) MOEK_TR_CLK(88 + j);
          if (ph == 1) {  // this stage's item done: its partial rows, then a fresh accumulator for the next item
            // acc[i][t][2h + v] = weight row (16 G_i + g + 8h) x block row 8t + 2c + v
            float* base = dbase + 256 * m.unit_item(j);
#pragma unroll
            for (int t = 0; t < C::T; t++) {
              if (t >= ntile) break;
#pragma unroll
              for (int v = 0; v < 2; v++) {
                const int row = t * 8 + 2 * c + v;
                if (row >= nv) continue;
                float* prow = base + (int64_t)ids[row] * H;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                  prow[slot00 + 8 * h] = acc[0][t][2 * h + v];
                  prow[slot10 + 8 * h] = acc[1][t][2 * h + v];
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
              for (int t = 0; t < C::T; t++)
#pragma unroll
                for (int v = 0; v < 4; v++) acc[i][t][v] = 0.f;
          }
        }
        const bool good = __all_sync(0xffffffffu, ok) && !*abort_flag;
        if (tid == 0 && tu < 8) MOEK_TR(9 + 3 * tu);
        if (ph == 1) {
          if (tid == 0 && tu < 8) MOEK_TR(10 + 3 * tu);
          continue;
        }

        // ------------------------------------------------------------------ gate_up finishing: this CTA's record
        // acc[i][t][2h + v] = weight row (16 G_i + g + 8h) x block row 8t + 2c + v; the warp's rows are its act
        // columns' gate and up rows, so each warp publishes its own columns with its own flag
        if (good) {
          float* mine = p.xpart + (int64_t)m.rec * XR * ITEM_COLS;
#pragma unroll
          for (int t = 0; t < C::T; t++) {
            if (t >= ntile) break;
#pragma unroll
            for (int v = 0; v < 2; v++) {
              const int row = t * 8 + 2 * c + v;
              if (row >= nv) continue;
#pragma unroll
              for (int h = 0; h < 2; h++) {
                __stcg(mine + row * ITEM_COLS + slot00 + 8 * h, acc[0][t][2 * h + v]);
                __stcg(mine + row * ITEM_COLS + slot10 + 8 * h, acc[1][t][2 * h + v]);
              }
            }
          }
          __syncwarp();
          // the warp's partials (ordered before lane 0's release by the warp barrier) before its flag
          if (lane == 0) st_release(p.ctr + p.off_xflag + (int64_t)m.rec * NCW + warp, epoch + 1);
        }
        if (tid == 0 && tu < 8) MOEK_TR(10 + 3 * tu);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mempty + b);
    }
    if (tid == 0) MOEK_TR(5);
  }

  // ------------------------------------------------------------------------------------------- grid barrier
  // every CTA's down partials are written: the last CTA to arrive advances the launch epoch, every CTA waits for it
  __syncthreads();
  if (tid == 0) {
    MOEK_TR(47);
    __threadfence();
    if (atomicAdd(p.ctr + p.off_done, 1) == (int)gridDim.x - 1) {
      // the last arrival: release the epoch first (the waiting CTAs pass on it), then reset the counter for the next
      // launch (no CTA of this launch reads it again; stream order makes the reset visible to the next launch)
      st_release(p.ctr + p.off_epoch, epoch + 1);
      p.ctr[p.off_done] = 0;
    }
    for (uint32_t it = 0;; it++) {
      if (ld_acquire(p.ctr + p.off_epoch) != epoch) break;
      if ((it & 63) == 63 && globaltimer() > deadline) {
        report(p.err, MOEK_DEV_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      __nanosleep(64);
    }
    MOEK_TR(51);
    // fused exchange: every CTA has read this call's number, so the call can be recorded as this rank's current one
    if (p.ep_x && blockIdx.x == 0) *p2p_call(p.ep_q) = ep_call;
  }
  __syncthreads();

  // ------------------------------------------------------------------------------------ the top-k sums, a slice each
  // out[t] = bf16(sum over valid slots j in order of w_j * (sum over k-slices in order of the down partials)); with
  // out_rows the weighted slot rows instead; expert-parallel: the fp32 sum into this rank's back buffer. One output
  // element per thread, the loads of up to 8 slots x 4 k-slices issued together.
  {
    float* back = p.ep_peer ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(p.ep_peer[p.ep_rank]) +
                                                      p.ep_back_off)
                            : nullptr;
    // 32-bit indices: M * H <= 512 x 4096 and (I / 128) x num_ids x H <= 32 x 512 x 4096 < 2^31
    const int H = p.H, nout = p.M * H, sst = n * H;
    // chunks of 32 consecutive outputs (one coalesced warp access each) dealt over the warps CTA by CTA, so that
    // every SM takes part, not only the first nout / THREADS CTAs
    for (int ch = warp * (int)gridDim.x + (int)blockIdx.x; ch * 32 < nout; ch += (int)gridDim.x * (THREADS / 32)) {
      const int i = ch * 32 + lane;
      if (i >= nout) continue;
      const int tk = i / H, col = i - tk * H;
      float o = 0.f;
      for (int j0 = 0; j0 < k; j0 += 8) {
        bool val[8];
        float sj[8];
        const float* rp[8];  // the slot's row of k-slice 0 (unused slots read slot 0's row, in bounds, then dropped)
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          const bool in = j0 + jj < k;
          const int sl = tk * k + (in ? j0 + jj : 0);
          const int e = in ? sid[sl] : -1;
          val[jj] = e >= 0 && e < p.E;
          sj[jj] = 0.f;
          rp[jj] = p.part2 + sl * H + col;
        }
        for (int t0 = 0; t0 < nst2; t0 += 4) {  // 32 loads in flight (I = 512: every load of a token at once)
          float v[8][4];
#pragma unroll
          for (int jj = 0; jj < 8; jj++)
#pragma unroll
            for (int u = 0; u < 4; u++) v[jj][u] = __ldcg(rp[jj] + min(t0 + u, nst2 - 1) * sst);
#pragma unroll
          for (int jj = 0; jj < 8; jj++)
#pragma unroll
            for (int u = 0; u < 4; u++)
              if (val[jj] && t0 + u < nst2) sj[jj] += v[jj][u];
        }
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          if (!val[jj]) continue;
          const int sl = tk * k + j0 + jj;
          const float y = __fmul_rn(stw[sl], sj[jj]);  // rounded like a stored slot row (no contraction)
          if (p.out_rows) p.out_rows[(int64_t)sl * H + col] = y;
          o += y;
        }
      }
      if (p.shared) o += p.shared[i];  // the shared expert's row (the block output = routed + shared)
      if (p.out) p.out[i] = __float2bfloat16_rn(o);
      if (back) back[i] = o;
    }
  }
  if (tid == 0) MOEK_TR(52);

  if (p.ep_peer) {  // every returned row is written: the last CTA raises the senders' back flags
    __syncthreads();
    if (tid == 0) {
      // the partials are in this GPU's memory: a device-scope release orders them before the arrival, and the last
      // arrival's system-scope release stores of the flags carry them to the senders
      __threadfence();
      if (atomicAdd(p.ctr + p.off_ep, 1) == (int)gridDim.x - 1) {
        p.ctr[p.off_ep] = 0;
        __threadfence();
        ep_signal(p, ep_call);
      }
    }
  }

  // fused exchange: once every owner's partials of this rank's tokens are written, the last CTAs sum them into the
  // output, a slice each
  if (p.ep_x) {
    const int total = p.ep_M * (p.H / 4), ncta = min((int)gridDim.x, (total + THREADS - 1) / THREADS);
    const int cta = (int)gridDim.x - 1 - (int)blockIdx.x;
    __syncthreads();
    if (cta < ncta) {
      bool good = true;
      if (warp == 0) {
        const uint64_t until = globaltimer() + p.timeout_ns;
        for (int s = lane; s < p.ep_world; s += 32)
          good &= wait_flag(p.ep_recv_flags + p.ep_world + s, ep_call, until, p.err);
        good = __all_sync(0xffffffffu, good);
        if (lane == 0) MOEK_TR(49);
      }
      if (__syncthreads_and(good)) ep_unpack_slice<THREADS>(p.ep_q, p.ep_pos, p.ep_M, p.ep_out, cta, ncta);
      if (tid == 0) MOEK_TR(50);
    }
  }
  if (tid == 0) MOEK_TR(6);
}

template <int XR>
static cudaError_t launch_xr(const LayerParams& p, int sms, int coop, cudaStream_t st) {
  using C = Cfg<XR>;
  cudaError_t e = cudaFuncSetAttribute(moek_layer_kernel<XR>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, moek_layer_kernel<XR>, THREADS, C::SMEM);
  if (e != cudaSuccess) return e;
  if (occ < 1) return cudaErrorLaunchOutOfResources;
  // every CTA resident at once (shares of a pair and the grid barrier wait on other CTAs)
  const int grid = std::min(std::min(occ, C::MINB) * sms, LAYER_XFLAG_CTAS);
  if (!coop) {
    e = launch_pdl(moek_layer_kernel<XR>, dim3(grid), dim3(THREADS), C::SMEM, st, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  // cooperative: the runtime guarantees that all CTAs are resident together, whatever else runs on the GPU. With
  // programmatic serialisation too where the runtime takes both; if it refuses the pair (a launch-configuration
  // error, reported before anything runs), cooperative alone.
  static std::atomic<int> coop_pdl{1};
  if (coop_pdl.load(std::memory_order_relaxed)) {
    e = launch_coop(moek_layer_kernel<XR>, dim3(grid), dim3(THREADS), C::SMEM, st, 1, p);
    if (e == cudaSuccess) return cudaGetLastError();
    if (e != cudaErrorInvalidValue && e != cudaErrorNotSupported) return e;
    cudaGetLastError();
    coop_pdl.store(0, std::memory_order_relaxed);
  }
  e = launch_coop(moek_layer_kernel<XR>, dim3(grid), dim3(THREADS), C::SMEM, st, 0, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace dl

MOEK_TRACE_COPY_FN(trace_copy_layer)

cudaError_t launch_layer(const LayerParams& p, int block_rows, int sms, int coop, cudaStream_t st) {
  if (block_rows <= 8) return dl::launch_xr<8>(p, sms, coop, st);
  if (block_rows <= 16) return dl::launch_xr<16>(p, sms, coop, st);
  return dl::launch_xr<32>(p, sms, coop, st);
}

}  // namespace moek
