// The whole decode-regime routed-expert layer in one persistent kernel, sm_100a: routing, gate_up GEMM + SwiGLU,
// down GEMM x router weight and the top-k sum, with no launch between the steps.
//
// The layer's data is small next to the latencies of a launch: a decode batch touches ~40 experts (about 60 MB of
// packed weights), which one B200 streams in ~10 us, while a launch boundary costs a few microseconds of pipeline
// drain and refill. So the steps that the reference runs as separate kernels (files/mbx_moek.py:252-289: moe_align,
// the gate_up GEMM, SwiGLU, the down GEMM, the top-k sum) run here inside one grid of persistent CTAs (two per SM)
// that stream the two weight matrices back to back:
//
//   routing   every CTA sorts the batch's (expert, slot) keys in shared memory at start-up: blocks = the distinct
//             valid experts in ascending order, each with its slots in ascending order (moe_align's order,
//             files/mbx_moek.cu:32-140), an expert with more than XR slots cut into blocks of XR (its weights are
//             then streamed once per block: XR <= 32 keeps two CTAs on every SM for any batch); no global
//             workspace and no separate launch.
//   units     gate_up units (block, 256-row item, k-split) and then down units (block, item, k-split), dealt
//             round-robin over the CTAs in that order: a CTA runs its gate_up units first, and the CTAs that got
//             fewer of those start streaming down weights early. Items beyond the last whole wave of units get a
//             finer k-split (PhasePlan), so that a phase does not end with a few CTAs running one more long unit.
//   producer  warp 8: per 64-k stage, the 8 KB of packed codes (lane 0) and the 1056-byte packed-scale run pair
//             (lane 1) by bulk copy (cp.async.bulk, no multicast) into a ring slot. It never waits on another CTA:
//             the weights of every unit are known once the routing is.
//   act warp  warp 9: the stage's activation rows. gate_up: the tokens' hidden rows by bulk copy; down: the act rows
//             of the block, once the gate_up item that produced those act columns is complete in every CTA (one
//             ready stamp per (block, item, consumer warp), acquire-loaded by eight lanes at once with a bounded
//             wait), by plain loads into the slot.
//   scales    warp 10: per stage the scale byte of each k-group x run position (base + 4-bit offset, then the
//             exceptions), in the packed run's own position order; per unit the {B B, R R} table of the expert
//             (moek_common.cuh).
//   consumers warps 0-7: the swap-AB mma.sync m16n8k16 of moek_decode.cu (weights = the 16-row A operand, up to 8
//             tokens = B), fp32 accumulators per unit; they wait on the scale warp's barrier only (it has waited for
//             the slot's copies itself).
//   finishing gate_up: with one k-split the lane holds gate and up of the same column and writes
//             act = bf16(silu(gate) * up); with more, fp32 partials go to the workspace and the warp whose arrival
//             completes (block, item, warp) adds them in split order, then releases that warp's ready stamp.
//             down: partials likewise, then the router weight: fp32 row w * sum; the
//             arrival that completes a token's valid slots for (item, warp) adds the token's rows in slot order and
//             rounds once to bf16 (the fp32 oracle's order, bench/moek/problem.py:51-67).
//
// Counters reset themselves (the completing arrival zeroes its counter); ready stamps carry a launch epoch, so the
// workspace is zeroed once at allocation and never between launches. Every wait is bounded (%globaltimer); a CTA
// whose wait expires records MOEK_DEV_TIMEOUT and winds down; the workspace must then be zeroed again.
//
// Co-residency: a down unit may wait on a gate_up unit of any CTA, and every CTA runs all of its gate_up units
// before any down unit, so the grid makes progress whenever all its CTAs are resident at once: the launcher sizes
// the grid to the occupancy the kernel reaches (cudaOccupancyMaxActiveBlocksPerMultiprocessor x SMs) and launches it
// as a cooperative grid, so that the runtime starts it only with every CTA resident, also while kernels of other
// streams hold part of the GPU.
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
constexpr int NLUT = 4;  // per-unit {B B, R R} tables in flight: a unit's table is written once its first stage has
                         // landed, when the consumers have released every stage of the unit NLUT units before
constexpr int MAXU = 8;         // units per metadata round (a CTA has about U / grid units; more take more rounds)

struct UnitMeta {
  int ph, blk, item, ks, e, nv, flags;  // ph: 0 = gate_up, 1 = down; flags: 2 = block has more rows than XR
  int st0, st1, ns;                     // the unit's stages [st0, st1) of its item, the item's k-split count
};

// Units of one phase: items (block, 256-row item) in order, each cut into k-splits. The first ni_main items use the
// caller's split; when those units would spill a few items past a whole number of waves of the grid, the remaining
// items use the finest whole-stage split that still fits them in one more wave, so the phase ends about one short
// unit after the last full wave instead of one full unit (the idea of stream-K, with no fix-up beyond the split-k
// arrivals the kernel has anyway).
// v / d for 0 <= v < 2^22 and 1 <= d < 2^10, without the long dependent chain of an integer division: a quotient
// estimate from the approximate fp32 reciprocal (relative error about 2^-23, so the estimate is off by at most one)
// and one correction each way. The unit plan and the unit decode divide by runtime values on the start-up path.
__device__ __forceinline__ int div_small(int v, int d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"((float)d));
  int q = __float2int_rz((float)v * r);
  const int rem = v - q * d;
  q += (rem >= d) - (rem < 0);
  return q;
}

struct PhasePlan {
  int ni_main, s_main, s_tail, u_main, u_total;  // at most 512 blocks x 16 items x 32 splits: 32-bit
};
__device__ __forceinline__ PhasePlan plan_phase(const LayerMat& m, int nblk, int grid, bool tail) {
  PhasePlan q;
  const int ni = nblk * m.nt;
  q.s_main = q.s_tail = m.nsplit;
  q.ni_main = ni;
  const int main_units = ni * m.nsplit;
  if (tail && main_units > grid) {
    const int nim = div_small(div_small(main_units, grid) * grid, m.nsplit);
    const int rem = ni - nim;
    int st = m.nsplit;  // the finest whole-stage split (a divisor of nstage, precomputed) that fits the grid
    for (uint64_t dm = m.divmask >> (m.nsplit + 1) << (m.nsplit + 1); dm; dm &= dm - 1) {
      const int s = __ffsll((long long)dm) - 1;
      if (rem * s <= grid) st = s;
    }
    if (rem > 0 && st > m.nsplit) {
      q.ni_main = nim;
      q.s_tail = st;
    }
  }
  q.u_main = q.ni_main * q.s_main;
  q.u_total = q.u_main + (ni - q.ni_main) * q.s_tail;
  return q;
}

template <int XR>
struct Cfg {
  static constexpr int X_OFF = LSTAGE + PAIR_BYTES;
  static constexpr int SC_OFF = X_OFF + XR * X_STRIDE;
  static constexpr int SLOT = SC_OFF + SC_BYTES;
  static constexpr int NS = XR <= 16 ? 4 : 3;  // ring slots: two CTAs per SM (XR <= 32)
  static constexpr int META_OFF = NS * SLOT;
  static constexpr int IDS_OFF = META_OFF + MAXU * (int)sizeof(UnitMeta);
  static constexpr int LUT_OFF = IDS_OFF + MAXU * XR * 4;
  static constexpr int ROUTE_OFF = LUT_OFF + NLUT * 256 * 8;  // srow[MAXIDS], bexp[MAXIDS], bstart[MAXIDS + 1]
  static constexpr int TOK_OFF = ROUTE_OFF + (3 * LAYER_MAXIDS + 1) * 4;  // the batch's slots: sid[], stw[]
  static constexpr int MISC_OFF = TOK_OFF + 2 * LAYER_MAXIDS * 4;
  static constexpr int PLAN_OFF = MISC_OFF + 16;  // the two phase plans
  static constexpr int BAR_OFF = (PLAN_OFF + 2 * (int)sizeof(PhasePlan) + 7) / 8 * 8;
  static constexpr int SMEM = BAR_OFF + (3 * NS + 2) * 8;
  static constexpr int T = XR / 8;
  static constexpr int MINB = 2;
  static_assert(XR <= 32, "two CTAs per SM");
  static_assert(2 * LAYER_MAXIDS * 4 <= SLOT, "routing scratch fits in ring slot 0");
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

// Bounded wait of a whole warp until the NCW ready stamps of a (block, item) all read `want`: lane L polls stamp
// L % NCW (acquire loads, all eight in parallel), then a warp barrier orders every lane's later loads after all the
// acquires (the consumer warps released their stamps after writing their act columns). Between polls the warp sleeps
// briefly, leaving the issue slots to the consumers.
__device__ __forceinline__ bool wait_stamps(const int* stamps, int want, uint64_t deadline, int* err,
                                            volatile int* abort_flag) {
  const int* st = stamps + (threadIdx.x & 31) % NCW;
  bool seen = false;
  for (uint32_t i = 0;; i++) {
    if (*abort_flag) return false;
    if (!seen) seen = ld_acquire(st) == want;
    if (__all_sync(0xffffffffu, seen)) {
      __syncwarp();
      return true;
    }
    if ((i & 63) == 63 && globaltimer() > deadline) {
      report(err, MOEK_DEV_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
    __nanosleep(32);
  }
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

__device__ __forceinline__ void decode_unit(const LayerParams& p, const PhasePlan& q0, const PhasePlan& q1, int u,
                                            UnitMeta& um) {
  um.ph = u >= q0.u_total ? 1 : 0;
  const LayerMat& m = p.m[um.ph];
  const PhasePlan& q = um.ph ? q1 : q0;
  const int v = um.ph ? u - q0.u_total : u;
  int ii;
  if (v < q.u_main) {
    ii = div_small(v, q.s_main);
    um.ks = v - ii * q.s_main;
    um.ns = q.s_main;
  } else {
    const int w = v - q.u_main;
    const int t = div_small(w, q.s_tail);
    ii = q.ni_main + t;
    um.ks = w - t * q.s_tail;
    um.ns = q.s_tail;
  }
  um.blk = div_small(ii, m.nt);
  um.item = ii - um.blk * m.nt;
  const int su = div_small(m.nstage, um.ns);
  um.st0 = um.ks * su;
  um.st1 = um.st0 + su;
}

template <int XR>
__global__ void __launch_bounds__(THREADS, Cfg<XR>::MINB) moek_layer_kernel(LayerParams p) {
  using C = Cfg<XR>;
  extern __shared__ __align__(128) uint8_t smem[];
  UnitMeta* meta = reinterpret_cast<UnitMeta*>(smem + C::META_OFF);
  int* mids = reinterpret_cast<int*>(smem + C::IDS_OFF);
  uint2* lut = reinterpret_cast<uint2*>(smem + C::LUT_OFF);  // per unit: scale byte -> {B B, R R} (moek_common.cuh)
  int* srow = reinterpret_cast<int*>(smem + C::ROUTE_OFF);
  int* bexp = srow + LAYER_MAXIDS;
  int* bstart = bexp + LAYER_MAXIDS;
  volatile int* misc = reinterpret_cast<volatile int*>(smem + C::MISC_OFF);  // [0] blocks, [1] valid slots, [2] abort,
                                                                              // [3] rows returned (expert-parallel)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + C::NS;
  uint64_t* scaled = empty + C::NS;
  uint64_t* mfull = scaled + C::NS;
  uint64_t* mempty = mfull + 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  volatile int* abort_flag = misc + 2;

  if (tid == 0) {
    misc[1] = 0;
    misc[2] = 0;
    misc[3] = 0;
    for (int i = 0; i < C::NS; i++) {
      mbar_init(full + i, 2);  // the producer's and the act warp's arrivals (each with its byte count)
      mbar_init(empty + i, NCW);
      mbar_init(scaled + i, 32);
    }
    mbar_init(mfull, 32);
    mbar_init(mempty, NCW + 2);  // consumers, scale warp, act warp
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
    if (p.ep_peer) {  // rows with at least one valid slot: the rows this rank returns (p.M * k <= 512)
      int rows = 0;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int t = tid + h * THREADS;
        bool any = false;
        if (t < p.M)
          for (int j = 0; j < k; j++) any |= key[t * k + j] != 0xFFFFFFFFu;
        rows += __syncthreads_count(any);
      }
      if (tid == 0) misc[3] = rows;
    }
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
      }
      if (lane < 2) {  // the two phases' plans, once per CTA, one lane each (every thread reads them after the barrier)
        const int nb = *abort_flag ? 0 : base;
        reinterpret_cast<PhasePlan*>(smem + C::PLAN_OFF)[lane] = plan_phase(p.m[lane], nb, gridDim.x, p.tail);
        if (lane == 0) MOEK_TR_CLK(44);
      }
    }
    __syncthreads();
  }
  const int nblk = *abort_flag ? 0 : misc[0];
  const int ep_rows = misc[3];
  if (tid == 0) MOEK_TR(3);
  if (tid == 0) MOEK_TR_CLK(45);
  if (p.ep_peer && ep_rows == 0 && !*abort_flag && blockIdx.x == 0 && tid == 0)
    ep_signal(p, ep_call);  // nothing to return: release the senders' waits at once


  const PhasePlan plan0 = reinterpret_cast<const PhasePlan*>(smem + C::PLAN_OFF)[0],
                  plan1 = reinterpret_cast<const PhasePlan*>(smem + C::PLAN_OFF)[1];
  const int U = plan0.u_total + plan1.u_total;
  const int n_mine = U > (int)blockIdx.x ? (U - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int rounds = (n_mine + MAXU - 1) / MAXU;
  if (tid == 0) MOEK_TR_VAL(7, n_mine);

  if (warp == W_PROD) {  // ------------------------------------------------------------------------- producer
    uint32_t g = 0;
    bool ok = true;
    for (int r = 0; r < rounds && ok; r++) {
      const int u0 = r * MAXU, nu = min(MAXU, n_mine - u0);
      if (r > 0 && !wait_or_abort(mempty, (r - 1) & 1, deadline, p.err, abort_flag)) break;
      for (int i = lane; i < nu; i += 32) {
        UnitMeta& m = meta[i];
        decode_unit(p, plan0, plan1, (int)blockIdx.x + (u0 + i) * (int)gridDim.x, m);
        m.e = bexp[m.blk];
        const int b0 = bstart[m.blk], cnt = bstart[m.blk + 1] - b0;
        m.nv = min(cnt, XR);
        m.flags = cnt > XR ? 2 : 0;
        for (int rr = 0; rr < m.nv; rr++) mids[i * XR + rr] = srow[b0 + rr];
      }
      __syncwarp();
      mbar_arrive(mfull);  // units, experts and rows published
      for (int ci = 0; ci < nu && ok; ci++) {
        const LayerMat& mt = p.m[meta[ci].ph];
        const int e = meta[ci].e, item = meta[ci].item;
        for (int st = meta[ci].st0; st < meta[ci].st1; st++, g++) {
          const int slot = g % C::NS;
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
            if (r == 0 && ci == 0 && st - meta[0].st0 < 8) MOEK_TR_CLK(112 + st - meta[0].st0);
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
    int n_wait = 0;  // act waits so far (the first four are stamped in MOEK_TRACE builds)
    for (int r = 0; r < rounds && ok; r++) {
      const int nu = min(MAXU, n_mine - r * MAXU);
      if (!wait_or_abort(mfull, r & 1, deadline, p.err, abort_flag)) break;
      for (int ci = 0; ci < nu && ok; ci++) {
        const UnitMeta& m = meta[ci];
        const int nv = m.nv;
        const int* ids = mids + ci * XR;
        int ready_item = -1;
        for (int st = m.st0; st < m.st1; st++, g++) {
          const int slot = g % C::NS;
          if (g >= C::NS && !wait_or_abort(empty + slot, ((g / C::NS) - 1) & 1, deadline, p.err, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* xs = smem + slot * C::SLOT + C::X_OFF;
          if (m.ph == 0) {  // hidden rows of the block's tokens, 64 k each, by bulk copy
            if (lane == 0) mbar_expect_tx(full + slot, nv * LBK * 2);
            __syncwarp();
            for (int rr = lane; rr < nv; rr += 32)
              bulk_g2s(xs + rr * X_STRIDE, p.x + (int64_t)(ids[rr] / k) * p.H + st * LBK, LBK * 2, full + slot);
            if (lane == 0 && r == 0 && ci == 0 && st - m.st0 < 8) MOEK_TR_CLK(120 + st - m.st0);
          } else {  // act rows: columns [128 st, 128 st + 128) are gate_up item st's (ITEM_COLS / 2 act columns)
            const int need = st;
            if (need != ready_item) {
              if (lane == 0 && n_wait < 4) MOEK_TR(56 + 2 * n_wait);
              if (!wait_stamps(p.ctr + p.off_ready + (m.blk * p.m[0].nt + need) * NCW, epoch + 1, deadline, p.err,
                               abort_flag)) {
                ok = false;
              }
              if (lane == 0 && n_wait < 4) MOEK_TR(57 + 2 * n_wait);
              n_wait++;
              ok = __all_sync(0xffffffffu, ok);
              if (!ok) break;
              ready_item = need;
            }
            for (int idx = lane; idx < nv * 16; idx += 32) {
              const int rr = idx >> 4, c = idx & 15;
              const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p.act + (int64_t)ids[rr] * p.I + st * LBK) + c);
              *reinterpret_cast<uint4*>(xs + rr * X_STRIDE + c * 16) = v;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(full + slot);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mempty);
    }
  } else if (warp == W_SCALE) {  // -------------------------------------------------------------------- scale warp
    // Per unit: the expert's global scale and the unit's exception offsets (lane j: run j's first entry) and entries
    // (up to 64 held in registers, two per lane), loaded by all lanes at once and one unit ahead, so that no stage
    // waits on a chain of global loads. Per stage: the slot's scale table in run-position order, one byte per
    // (k-group, run, position) at kg * 256 + run * 128 + position (the consumers map their rows to positions), then
    // the run's exceptions. Lane L decodes chunk L % 16 (8 positions) of run L / 16 of the pair: eight 8-byte stores,
    // no byte shuffling, so that the single scale warp keeps ahead of the consumers.
    uint32_t g = 0, kq = 0;
    const int run = lane >> 4, ch = lane & 15;
    bool ok = true;
    for (int r = 0; r < rounds && ok; r++) {
      const int nu = min(MAXU, n_mine - r * MAXU);
      if (!wait_or_abort(mfull, r & 1, deadline, p.err, abort_flag)) break;
      int ro_n = 0, end_n = 0;
      float g_n = 0.f;
      auto fetch = [&](int ui) {  // loads only; consumed one unit later
        const UnitMeta& m = meta[ui];
        const LayerMat& mt = p.m[m.ph];
        const int nruns = m.st1 - m.st0;
        const int64_t key0 = ((int64_t)m.e * mt.nt + m.item) * mt.nstage + m.st0;
        ro_n = lane < nruns ? mt.exc_off[key0 + lane] : 0;
        end_n = mt.exc_off[key0 + nruns];
        g_n = mt.G[m.e];
      };
      if (nu > 0) fetch(0);
      for (int ui = 0; ui < nu && ok; ui++) {
        const UnitMeta& m = meta[ui];
        const LayerMat& mt = p.m[m.ph];
        const int su = m.st1 - m.st0;
        const int o0 = __shfl_sync(0xffffffffu, ro_n, 0);
        const int ro = ro_n - o0, cnt = end_n - o0;
        const float gsc = g_n;
        const uint32_t* eg = mt.exc_ent + o0;
        const uint32_t ex0 = lane < cnt ? eg[lane] : 0u, ex1 = lane + 32 < cnt ? eg[lane + 32] : 0u;
        if (ui + 1 < nu) fetch(ui + 1);
        uint2* lt = lut + (kq % NLUT) * 256;
        kq++;
        const int r0g = m.ph == 0 ? m.item : 2 * m.item;  // global run index of the pair's first run
        const int r1g = m.ph == 0 ? mt.nt + m.item : r0g + 1;  // and of its second (gate_up: the up rows' run)
        for (int st = m.st0; st < m.st1; st++, g++) {
          const int slot = g % C::NS;
          if (!wait_or_abort(full + slot, (g / C::NS) & 1, deadline, p.err, abort_flag)) {
            ok = false;
            break;
          }
          if (lane == 0 && r == 0 && ui == 0 && st - m.st0 < 8) MOEK_TR_CLK(96 + st - m.st0);
          if (st == m.st0) {  // the unit's table: its slot's previous unit is done (the first stage has landed)
#pragma unroll
            for (int j = 0; j < 8; j++) {
              const ScaleBR br = scale_br(lane + 32 * j, gsc);
              lt[lane + 32 * j] = make_uint2(br.b2, br.r2);
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
          // this stage's run: entries [eo0, eo1) of the unit's list overwrite their bytes
          const int rr = st - m.st0;
          const int eo0 = __shfl_sync(0xffffffffu, ro, rr);
          const int eo1 = rr + 1 < su ? __shfl_sync(0xffffffffu, ro, rr + 1) : cnt;
          auto patch = [&](uint32_t en) {
            const int ppos = en & 0xFFFF, kg = (en >> 16) & 0xFF;
            if (!MOEK_CHECK(kg < KG && ((ppos >> 7) == r0g || (ppos >> 7) == r1g), p.err)) return;
            tb[kg * 256 + ((ppos >> 7) == r0g ? 0 : 128) + (ppos & 127)] = (uint8_t)(en >> 24);
          };
          if (lane >= eo0 && lane < eo1) patch(ex0);
          if (lane + 32 >= eo0 && lane + 32 < eo1) patch(ex1);
          for (int j = max(eo0, 64) + lane; j < eo1; j += 32) patch(eg[j]);  // long lists: the rest from memory
          __syncwarp();
          mbar_arrive(scaled + slot);
          if (lane == 0 && r == 0 && ui == 0 && st - m.st0 < 8) MOEK_TR_CLK(104 + st - m.st0);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mempty);
    }
  } else {  // ------------------------------------------------------------------------------------------ consumers
    const int gq = lane >> 2, c = lane & 3;
    const int w_off = ((((c >> 1) ^ (gq >> 2)) & 1) << 4) | ((c & 1) << 3);  // k-group c's bytes in a 32-byte row
    const int I = p.I, H = p.H;
    uint32_t g = 0, kq = 0;
    for (int r = 0; r < rounds; r++) {
      const int nu = min(MAXU, n_mine - r * MAXU);
      wait_or_abort(mfull, r & 1, deadline, p.err, abort_flag);
      consumer_sync();
      const bool have_meta = !*abort_flag;
      for (int ui = 0; ui < nu && have_meta; ui++) {
        const UnitMeta& m = meta[ui];
        const LayerMat& mt = p.m[m.ph];
        const int ph = m.ph, item = m.item, ks = m.ks, nv = m.nv, blk = m.blk, ns = m.ns;
        const int* ids = mids + ui * XR;
        if ((m.flags & 2) && tid == 0) report(p.err, MOEK_DEV_TOO_MANY_ROWS);
        // the warp's two 16-row groups of the item (gate_up: gate group w and its up partner w + 8)
        const int G0 = ph == 0 ? warp : 2 * warp, G1 = ph == 0 ? warp + 8 : 2 * warp + 1;
        const int slot00 = 16 * G0 + gq, slot10 = 16 * G1 + gq;
        // the scale-table offsets (run * 128 + position) of the lane's four rows
        auto tpos = [](int r) { return (r & 128) + slot_position(r & 127); };
        const int p00 = tpos(slot00), p01 = tpos(slot00 + 8), p10 = tpos(slot10), p11 = tpos(slot10 + 8);
        const uint2* lt = lut + (kq % NLUT) * 256;
        kq++;
        const int ntile = (nv + 7) >> 3;
        // one accumulator chain per (row group, tile): every block size adds the same terms in the same order, so
        // the rows per block never change the results (more chains per tile measured no faster: the consumers are
        // bound by issue slots, not by the MMA chain)
        constexpr int NH = 1;
        float acc[NH][2][C::T][4];
#pragma unroll
        for (int h = 0; h < NH; h++)
#pragma unroll
          for (int i = 0; i < 2; i++)
#pragma unroll
            for (int t = 0; t < C::T; t++)
#pragma unroll
              for (int v = 0; v < 4; v++) acc[h][i][t][v] = 0.f;
        bool ok = true;
        const int tu = r * MAXU + ui;  // the unit's index among this CTA's (timeline stamps)
        bool ready = false;  // the next stage's scales were seen published while this stage was computed
        for (int st = m.st0; st < m.st1; st++, g++) {
          const int slot = g % C::NS;
          const uint32_t par = (g / C::NS) & 1;
          const bool stamp = tid == 0 && tu == 0 && st - m.st0 < 8;
          if (stamp) MOEK_TR_CLK(64 + st - m.st0);
          // one wait: the scale warp arrives on `scaled` only after its own wait on `full` (weights, scales and
          // activations of the slot landed), so the consumers' acquire of `scaled` orders their reads after those
          // writes as well. Usually the test made during the previous stage already saw the phase complete, and the
          // stage starts without a wait on its critical path.
          if (!ready && !wait_or_abort(scaled + slot, par, deadline, p.err, abort_flag)) {
            ok = false;
            continue;  // stay in step with the other roles' counters
          }
          ready = false;
          if (stamp) MOEK_TR_CLK(80 + st - m.st0);
          if (tid == 0 && st == m.st0 && tu < 8) {
            MOEK_TR(8 + 3 * tu);
            MOEK_TR_VAL(32 + tu, (ph << 28) | (blk << 16) | (item << 8) | ks);
          }
#pragma unroll
          for (int hf = 0; hf < 2; hf++) {  // the stage's two 64-k halves: an 8 KB block of codes and 4 k-groups each
          if (hf == 1 && st + 1 < m.st1)  // test the next stage's scales (its latency hides behind this half's math)
            ready = mbar_test(scaled + (g + 1) % C::NS, ((g + 1) / C::NS) & 1);
          const uint8_t* sw = smem + slot * C::SLOT + hf * STAGE_BYTES;
          const uint8_t* sx = smem + slot * C::SLOT + C::X_OFF + hf * BK * 2;
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
                  mma_16816(acc[hf % NH][i][t], A, (J & 1) ? xv.z : xv.x, (J & 1) ? xv.w : xv.y);
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
          if (stamp) MOEK_TR_CLK(88 + st - m.st0);
        }
        ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
        if (!ok) continue;
        if (tid == 0 && tu < 8) MOEK_TR(9 + 3 * tu);
        if constexpr (NH == 2) {
#pragma unroll
          for (int i = 0; i < 2; i++)
#pragma unroll
            for (int t = 0; t < C::T; t++)
#pragma unroll
              for (int v = 0; v < 4; v++) acc[0][i][t][v] += acc[NH - 1][i][t][v];
        }

        // ------------------------------------------------------------------------------------------ finishing
        // acc[0][i][t][2h + v] = weight row (16 G_i + g + 8h) x block row 8t + 2c + v
        const int N = mt.N;
        if (ph == 0) {
          const int nt1 = mt.nt;
          bool complete = ns == 1;
          if (complete) {  // gate row and up row + 128 share the column: act straight from the accumulators
#pragma unroll
            for (int t = 0; t < C::T; t++) {
              if (t >= ntile) break;
#pragma unroll
              for (int v = 0; v < 2; v++) {
                const int row = t * 8 + 2 * c + v;
                if (row >= nv) continue;
#pragma unroll
                for (int h = 0; h < 2; h++)
                  p.act[(int64_t)ids[row] * I + 128 * item + slot00 + 8 * h] =
                      __float2bfloat16_rn(silu(acc[0][0][t][2 * h + v]) * acc[0][1][t][2 * h + v]);
              }
            }
          } else {
            float* base = p.part1 + (int64_t)ks * n * N;
#pragma unroll
            for (int t = 0; t < C::T; t++) {
              if (t >= ntile) break;
#pragma unroll
              for (int v = 0; v < 2; v++) {
                const int row = t * 8 + 2 * c + v;
                if (row >= nv) continue;
                float* prow = base + (int64_t)ids[row] * N;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                  prow[128 * item + slot00 + 8 * h] = acc[0][0][t][2 * h + v];
                  prow[I + 128 * item + slot00 + 8 * h] = acc[0][1][t][2 * h + v];
                }
              }
            }
            __threadfence();
            __syncwarp();
            int old = 0;
            int* cn = p.ctr + p.off_cnt1 + ((int64_t)blk * nt1 + item) * NCW + warp;
            if (lane == 0) old = atomicAdd(cn, 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            complete = old == ns - 1;
            if (complete) {  // every split of (block, item, warp) is in: add them in split order
              if (lane == 0) *cn = 0;
              __threadfence();
              for (int idx = lane; idx < nv * 16; idx += 32) {
                const int row = idx >> 4, col = 128 * item + 16 * warp + (idx & 15);
                const float* pr = p.part1 + (int64_t)ids[row] * N;
                float gs = 0.f, us = 0.f;
                for (int s2 = 0; s2 < ns; s2++) {
                  gs += __ldcg(pr + (int64_t)s2 * n * N + col);
                  us += __ldcg(pr + (int64_t)s2 * n * N + I + col);
                }
                p.act[(int64_t)ids[row] * I + col] = __float2bfloat16_rn(silu(gs) * us);
              }
            }
          }
          if (complete) {  // this warp's act columns of (block, item) are written: its ready stamp
            __threadfence();
            __syncwarp();
            if (lane == 0) st_release(p.ctr + p.off_ready + ((int64_t)blk * nt1 + item) * NCW + warp, epoch + 1);
          }
          if (tid == 0 && tu < 8) MOEK_TR(10 + 3 * tu);
          continue;
        }
        // down: weighted fp32 rows of (block, item), then the token sums
        const int nt2 = mt.nt;
        float* rows = p.out_rows ? p.out_rows : p.rows;
        bool complete = ns == 1;
        if (complete) {
#pragma unroll
          for (int t = 0; t < C::T; t++) {
            if (t >= ntile) break;
#pragma unroll
            for (int v = 0; v < 2; v++) {
              const int row = t * 8 + 2 * c + v;
              if (row >= nv) continue;
              const int id = ids[row];
              const float w = stw[id];
#pragma unroll
              for (int h = 0; h < 2; h++) {
                rows[(int64_t)id * H + 256 * item + slot00 + 8 * h] = w * acc[0][0][t][2 * h + v];
                rows[(int64_t)id * H + 256 * item + slot10 + 8 * h] = w * acc[0][1][t][2 * h + v];
              }
            }
          }
        } else {
          float* base = p.part2 + (int64_t)ks * n * N;
#pragma unroll
          for (int t = 0; t < C::T; t++) {
            if (t >= ntile) break;
#pragma unroll
            for (int v = 0; v < 2; v++) {
              const int row = t * 8 + 2 * c + v;
              if (row >= nv) continue;
              float* prow = base + (int64_t)ids[row] * N + 256 * item;
#pragma unroll
              for (int h = 0; h < 2; h++) {
                prow[slot00 + 8 * h] = acc[0][0][t][2 * h + v];
                prow[slot10 + 8 * h] = acc[0][1][t][2 * h + v];
              }
            }
          }
          __threadfence();
          __syncwarp();
          int old = 0;
          int* cn = p.ctr + p.off_cnt2 + ((int64_t)blk * nt2 + item) * NCW + warp;
          if (lane == 0) old = atomicAdd(cn, 1);
          old = __shfl_sync(0xffffffffu, old, 0);
          complete = old == ns - 1;
          if (complete) {
            if (lane == 0) *cn = 0;
            __threadfence();
            const int col = 256 * item + 32 * warp + lane;  // the warp's 32 output columns: one per lane
            for (int row = 0; row < nv; row++) {
              const int id = ids[row];
              const float* pr = p.part2 + (int64_t)id * N + col;
              float s = 0.f;
              for (int s2 = 0; s2 < ns; s2++) s += __ldcg(pr + (int64_t)s2 * n * N);
              rows[(int64_t)id * H + col] = stw[id] * s;
            }
          }
        }
        if (tid == 0 && tu < 8) MOEK_TR(10 + 3 * tu);
        if (!complete || p.out_rows) continue;
        __threadfence();
        __syncwarp();
        // each row's token: the arrival that completes the token's valid slots for (item, warp) adds them in order
        const int col = 256 * item + 32 * warp + lane;
        int pieces = 0;  // expert-parallel: (token, item, warp) sums written to the senders' back buffers
        for (int row = 0; row < nv; row++) {
          const int tk = ids[row] / k;
          const int ej = lane < k ? sid[tk * k + lane] : -1;
          const int nslots = __popc(__ballot_sync(0xffffffffu, ej >= 0 && ej < p.E));
          int o2 = 0;
          int* tc = p.ctr + p.off_tok + ((int64_t)tk * nt2 + item) * NCW + warp;
          if (lane == 0) o2 = atomicAdd(tc, 1);
          o2 = __shfl_sync(0xffffffffu, o2, 0);
          if (o2 != nslots - 1) continue;
          if (lane == 0) *tc = 0;
          __threadfence();
          float o = 0.f;
          for (int sl = 0; sl < k; sl++) {
            const int ejs = sid[tk * k + sl];
            if (ejs < 0 || ejs >= p.E) continue;
            o += __ldcg(rows + (int64_t)(tk * k + sl) * H + col);
          }
          if (p.ep_peer) {  // fp32 partial of the row into its sender's back buffer, over NVLink
            // the row's partial into its sender's segment of this rank's own back buffer (the sender reads it)
            float* back = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(p.ep_peer[p.ep_rank]) + p.ep_back_off);
            back[(int64_t)tk * H + col] = o;
            pieces++;
          } else {
            p.out[(int64_t)tk * H + col] = __float2bfloat16_rn(o);
          }
        }
        if (pieces) {  // the arrival that completes every returned row raises the senders' back flags
          __syncwarp();
          if (lane == 0) {
            // the partials are in this GPU's memory: a device-scope release orders them before the arrival, and the
            // last arrival's system-scope release stores of the flags carry them to the senders
            __threadfence();
            const int want = ep_rows * p.m[1].nt * NCW;
            if (atomicAdd(p.ctr + p.off_ep, pieces) + pieces == want) {
              p.ctr[p.off_ep] = 0;
              __threadfence();
              ep_signal(p, ep_call);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mempty);
    }
    if (tid == 0) MOEK_TR(5);
  }

  // tokens with no valid slot get a zero output row (nothing else writes them): the last CTA, which has the fewest
  // units, once its own work is done, so that no CTA starts streaming late
  if (blockIdx.x == gridDim.x - 1 && p.out && warp < NCW) {
    for (int t = warp; t < p.M; t += NCW) {
      const int e = lane < k ? sid[t * k + lane] : -1;
      if (__any_sync(0xffffffffu, e >= 0 && e < p.E)) continue;
      for (int c = lane; c < p.H; c += 32) p.out[(int64_t)t * p.H + c] = __float2bfloat16_rn(0.f);
    }
  }

  // fused exchange: once every owner's partials of this rank's tokens are written, the last CTAs (the ones with the
  // fewest units) sum them into the output, a slice each
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

  // ------------------------------------------------------------------------------------------------ teardown
  __syncthreads();
  if (tid == 0) MOEK_TR(6);
  if (tid == 0) {  // the last CTA to finish advances the launch epoch of the ready stamps
    __threadfence();
    if (atomicAdd(p.ctr + p.off_done, 1) == (int)gridDim.x - 1) {
      p.ctr[p.off_done] = 0;
      __threadfence();
      atomicAdd(p.ctr + p.off_epoch, 1);
      // fused exchange: every CTA has read this call's number and unpacked its slice, so the call is complete
      if (p.ep_x) *p2p_call(p.ep_q) = ep_call;
    }
  }
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
  const int grid = std::min(occ, C::MINB) * sms;  // every CTA resident at once (down units wait on gate_up units)
  if (!coop) {
    e = launch_pdl(moek_layer_kernel<XR>, dim3(grid), dim3(THREADS), C::SMEM, st, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  // cooperative: the runtime guarantees that all CTAs are resident together (down units wait on gate_up units of
  // other CTAs), whatever else runs on the GPU. With programmatic serialisation too where the runtime takes both;
  // if it refuses the pair (a launch-configuration error, reported before anything runs), cooperative alone.
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
