// Decode-regime W4A16 grouped GEMM (gate_up and down of the routed experts) for sm_100a, plus its split-k
// epilogues and the top-k combine.
//
// The reference's kernel (files/mbx_moek.cu:665-712, mode 2 for batches of <= 16 tokens) does the same job; this one
// is written for B200 from the weight stream outwards:
//
//   unit      = (moe_align block, 256-column item, k-split). Units are dealt round-robin to the CTAs in
//               (block, item, split) order, so neighbouring CTAs stream the splits of one expert's item at once and
//               every SM keeps a stream going however few experts the batch touches.
//   producer  = warp 8. Per 64-k stage it bulk-copies (cp.async.bulk, no multicast) the stage's 8 KB of packed codes,
//               the item's 1056-byte packed-scale run pair and the block's activation rows (one 128-byte copy per
//               valid row, gathered through sorted_ids) into a ring slot, all counted on the slot's mbarrier.
//   consumers = warps 0-7. Warp w owns 32 of the item's 256 weight rows (gate_up: 16 gate rows and the matching 16 up
//               rows, so SwiGLU pairs stay in one thread). Per stage a lane (4g + c) decodes 4 x 8 bytes of codes
//               (k-group c of rows g and g + 8 of its two 16-row groups) plus the scales its k-group needs into the
//               oracle's bf16 weights (moek_common.cuh) and runs
//               mma.sync m16n8k16 with the WEIGHTS as the 16-row A operand and up to 8 activation rows as B
//               ("swap AB": a decode block has 1-8 valid rows, so no MMA row is padding). The k order inside an
//               MMA is the lane's own 16 consecutive k; activations are read in the same order.
//   output    = fp32 partial sums part[split][id][column] (gate at column c, up at I + c); the epilogue kernels add
//               the splits in split order (deterministic) and apply SwiGLU or router weight + top-k sum.
//
// Exception scales (the packed format's out-of-window values) are patched per stage: the run's list is read by the
// warp, an entry whose k-group and column belong to the warp is broadcast with a shuffle to the lane that owns it.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "moek_common.cuh"
#include "moek_kernels.cuh"

namespace moek {



constexpr int DC_WARPS = 8;                      // consumer warps
constexpr int DC_THREADS = DC_WARPS * 32 + 64;    // + the bulk-copy producer warp + the scale warp
constexpr int X_STRIDE = 144;   // bytes per activation row in a slot (128 + 16: conflict-free 16-byte reads)
constexpr int SC_STRIDE = 288;  // bytes per k-group row of a slot's scale-byte table (256 + 32: conflict-free reads)
constexpr int SC_BYTES = 4 * SC_STRIDE;
constexpr int NLUT = 4;         // per-unit (B | R) tables in flight (the scale warp runs at most 3 units ahead)
constexpr int MAXU = 64;        // units per metadata round
constexpr int MAXRUN = 32;      // packed-scale runs per unit (K / 128 / nsplit)
constexpr int EXC_POOL = 1024;  // exception entries cached in shared memory per round

// Per-unit metadata, gathered once per round (MAXU units) so that no thread waits on a global load inside the stage
// loop. The producer fills the first group (units, experts, rows) and publishes it with mfull; the scale warp, the
// only reader of the second group (global scale, exception lists), fills it itself afterwards, so that those
// dependent loads overlap the producer's streaming instead of delaying it.
struct UnitMeta {
  int blk, item, ks, e, nv, flags;  // flags: 2 = block has more rows than XR
  float g;                           // the expert's global scale
  int from_global;                   // 1 = the exception list is read from global memory (did not fit the pool)
  int exc_g0;                        // global index of the unit's first exception entry
  int exc_s0;                        // shared-pool index of the unit's first entry (from_global == 0)
  int run_off[MAXRUN + 1];           // entry offsets, relative to the first, at each run boundary
};

// Ring slot: [8 KB codes][1056 B packed-scale run pair][XR activation rows][scale bytes: 4 k-groups x 256 rows,
// exceptions applied, written by the scale warp]. Per unit the scale warp also fills one of NLUT tables mapping every
// byte value to (bf16 B | bf16 R << 16) for the unit's expert.
template <int XR>
struct DecodeCfg {
  static constexpr int X_OFF = STAGE_BYTES + PAIR_BYTES;
  static constexpr int SC_OFF = X_OFF + XR * X_STRIDE;
  static constexpr int SLOT = SC_OFF + SC_BYTES;
  static constexpr int NS = XR <= 8 ? 7 : XR <= 32 ? (XR <= 16 ? 6 : 5) : 4;
  static constexpr int META_OFF = NS * SLOT;
  static constexpr int IDS_OFF = META_OFF + MAXU * (int)sizeof(UnitMeta);
  static constexpr int POOL_OFF = IDS_OFF + MAXU * XR * 4;
  static constexpr int LUT_OFF = POOL_OFF + EXC_POOL * 4;
  static constexpr int RED_OFF = LUT_OFF + NLUT * 256 * 4;
  static constexpr int BAR_OFF = RED_OFF + 16;
  static constexpr int SMEM = BAR_OFF + (3 * NS + 2) * 8;
  static constexpr int T = XR / 8;  // token tiles of 8 rows
  static constexpr int MINB = XR <= 32 ? 2 : 1;
};

__device__ __forceinline__ void mma_bf16_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Bounded wait honouring the CTA-wide abort flag: once any thread of the CTA gave up, every later wait fails at once,
// so all warps keep their control flow (and the named barriers) in step and the kernel ends.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, uint64_t deadline, int* err,
                                              volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity, deadline, err)) return true;
  *abort_flag = 1;
  return false;
}
__device__ __forceinline__ int atom_add_acq_rel(int* addr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(DC_WARPS * 32) : "memory"); }

// Item slot -> output column of the N-wide weight matrix
__device__ __forceinline__ int slot_column(const GemmParams& p, int item, int slot) {
  if (p.gate_up) return slot < 128 ? 128 * item + slot : p.N / 2 + 128 * item + slot - 128;
  return 256 * item + slot;
}

template <int XR>
__global__ void __launch_bounds__(DC_THREADS, DecodeCfg<XR>::MINB) moek_decode_kernel(GemmParams p) {
  using C = DecodeCfg<XR>;
  extern __shared__ __align__(128) uint8_t smem[];
  UnitMeta* meta = reinterpret_cast<UnitMeta*>(smem + C::META_OFF);
  int* mids = reinterpret_cast<int*>(smem + C::IDS_OFF);
  uint32_t* pool = reinterpret_cast<uint32_t*>(smem + C::POOL_OFF);
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem + C::LUT_OFF);
  volatile int* red = reinterpret_cast<volatile int*>(smem + C::RED_OFF);  // [0] last-arriver flag, [1] abort
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + C::NS;
  uint64_t* scaled = empty + C::NS;   // the scale warp filled the slot's scale table (32 arrivals)
  uint64_t* mfull = scaled + C::NS;   // a round's metadata is published (32 producer lanes arrive)
  uint64_t* mempty = mfull + 1;       // a round's units are all consumed (consumer warps + the scale warp)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nt = p.N / ITEM_COLS, nstage = p.K / BK, nb = p.K / 128;
  const int su = nstage / p.nsplit, nruns = su / 2;
  if (tid == 0) {
    red[1] = 0;
    for (int i = 0; i < C::NS; i++) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, DC_WARPS);
      mbar_init(scaled + i, 32);
    }
    mbar_init(mfull, 32);
    mbar_init(mempty, DC_WARPS + 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();  // sorted_ids / expert_ids / activations come from the previous kernel
  pdl_launch_dependents();
  const uint64_t deadline = globaltimer() + p.timeout_ns;
  const int nblocks = min(p.num_post_pad[0] / p.block_m, p.max_blocks);
  const int64_t nunits = (int64_t)nblocks * nt * p.nsplit;
  const int n_mine = nunits > blockIdx.x ? (int)((nunits - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  const int rounds = (n_mine + MAXU - 1) / MAXU;
  volatile int* abort_flag = red + 1;

  if (warp == DC_WARPS) {  // ------------------------------------------------------------------ producer
    uint32_t g = 0;
    for (int r = 0; r < rounds; r++) {
      const int u0 = r * MAXU, nu = min(MAXU, n_mine - u0);
      if (r > 0 && !wait_or_abort(mempty, (r - 1) & 1, deadline, p.err, abort_flag)) return;
      // units, experts, row ids (valid rows are a prefix of a block)
      for (int i = lane; i < nu; i += 32) {
        const int64_t u = blockIdx.x + (int64_t)(u0 + i) * gridDim.x;
        const int per = nt * p.nsplit;
        UnitMeta& m = meta[i];
        m.blk = (int)(u / per);
        const int rem = (int)(u - (int64_t)m.blk * per);
        m.item = rem / p.nsplit;
        m.ks = rem - m.item * p.nsplit;
        m.e = p.expert_ids[m.blk];
        const int lim = min(XR, p.block_m);
        const int64_t row0 = (int64_t)m.blk * p.block_m;
        int nv = 0;
        for (int rr = 0; rr < lim; rr++) {
          const int id = p.sorted_ids[row0 + rr];
          mids[i * XR + rr] = id;
          nv += id < p.num_ids;
        }
        m.nv = nv;
        m.flags = (lim < p.block_m && p.sorted_ids[row0 + lim] < p.num_ids) ? 2 : 0;
      }
      __syncwarp();
      // stream: the copies need only the expert and the rows
      int ci = 0, cst = -1;  // cursor: unit index and stage of the next copy
      auto issue = [&](int limit) -> bool {
        int issued = 0;
        for (; ci < nu; ci++) {
          const int e = meta[ci].e, item = meta[ci].item, ks = meta[ci].ks, nv = meta[ci].nv;
          if (e < 0 || e >= p.E) continue;
          if (cst < 0) cst = ks * su;
          for (; cst < (ks + 1) * su; cst++, g++) {
            if (issued == limit) return true;
            const int slot = g % C::NS;
            if (g >= C::NS && !wait_or_abort(empty + slot, ((g / C::NS) - 1) & 1, deadline, p.err, abort_flag))
              return false;
            uint8_t* dst = smem + slot * C::SLOT;
            if (lane == 0) mbar_expect_tx(full + slot, STAGE_BYTES + PAIR_BYTES + nv * BK * 2);
            __syncwarp();
            // every copy of the stage from its own lane in one instruction (a bulk copy's issue latency is paid once
            // per instruction, not once per copy): lane 0 the codes, lane 1 the scale pair, lanes 2.. the rows
            for (int c = lane; c < 2 + nv; c += 32) {
              if (c == 0) {
                const int64_t wi = ((int64_t)e * nt + item) * nstage + cst;
                bulk_g2s(dst, p.W + wi * STAGE_BYTES, STAGE_BYTES, full + slot);
              } else if (c == 1) {
                const int64_t si = ((int64_t)e * nt + item) * nb + (cst >> 1);
                bulk_g2s(dst + STAGE_BYTES, p.SP + si * PAIR_BYTES, PAIR_BYTES, full + slot);
              } else {
                const int rr = c - 2;
                const int id = mids[ci * XR + rr];
                const __nv_bfloat16* src = p.A + (int64_t)(id / p.a_div) * p.K + cst * BK;
                bulk_g2s(dst + C::X_OFF + rr * X_STRIDE, src, BK * 2, full + slot);
              }
            }
            issued++;
          }
          cst = -1;
        }
        return true;
      };
      mbar_arrive(mfull);  // ids, rows and experts published: consumers and the scale warp may start
      if (!issue(1 << 30)) return;
    }
    return;
  }

  if (warp == DC_WARPS + 1) {  // ------------------------------------------------------------- scale warp
    // Per stage: the 4 k-groups x 256 rows of scale bytes (base + 4-bit offset, then the unit's exception entries)
    // into the slot's byte table; per unit: the (B | R) table of all 256 byte values for the unit's expert. Lane L
    // decodes chunk L % 16 (8 positions) of run L / 16 of the item's run pair.
    uint32_t g = 0, k = 0;
    const int run = lane >> 4, ch = lane & 15;
    int dst[8];  // the rows (item slots) of the lane's 8 positions
#pragma unroll
    for (int i = 0; i < 8; i++) dst[i] = run * 128 + position_slot(8 * ch + i);
    for (int r = 0; r < rounds; r++) {
      const int nu = min(MAXU, n_mine - r * MAXU);
      if (!wait_or_abort(mfull, r & 1, deadline, p.err, abort_flag)) return;
      // the round's global scales and exception-list bounds (one unit per lane), then the lists into the pool
      for (int i = lane; i < nu; i += 32) {
        UnitMeta& m = meta[i];
        const bool valid = m.e >= 0 && m.e < p.E;
        m.g = valid ? p.G[m.e] : 0.f;
        const int64_t key0 = ((int64_t)(valid ? m.e : 0) * nt + m.item) * nb + (int64_t)m.ks * nruns;
        const int o0 = valid ? p.exc_off[key0] : 0;
        m.exc_g0 = o0;
        for (int j = 0; j <= nruns; j++) m.run_off[j] = valid ? p.exc_off[key0 + j] - o0 : 0;
      }
      __syncwarp();
      if (lane == 0) {  // pool places; a unit whose list does not fit reads it from global memory
        int used = 0;
        for (int i = 0; i < nu; i++) {
          const int n = meta[i].run_off[nruns];
          meta[i].from_global = used + n > EXC_POOL;
          if (!meta[i].from_global) {
            meta[i].exc_s0 = used;
            used += n;
          }
        }
      }
      __syncwarp();
      for (int i = lane; i < nu; i += 32) {  // each lane copies its own units' lists: loads in parallel
        if (meta[i].from_global) continue;
        const int n = meta[i].run_off[nruns], s0 = meta[i].exc_s0, g0 = meta[i].exc_g0;
        for (int j = 0; j < n; j++) pool[s0 + j] = p.exc_ent[g0 + j];
      }
      __syncwarp();
      for (int ui = 0; ui < nu; ui++) {
        const UnitMeta& m = meta[ui];
        const int e = m.e, item = m.item, ks = m.ks;
        if (e < 0 || e >= p.E) continue;
        const float gsc = m.g;
        uint32_t* lt = lut + (k % NLUT) * 256;
#pragma unroll
        for (int j = 0; j < 8; j++) lt[lane + 32 * j] = scale_word(lane + 32 * j, gsc);
        k++;
        const uint32_t* exc = m.from_global ? p.exc_ent + m.exc_g0 : pool + m.exc_s0;
        const int r0g = p.gate_up ? item : 2 * item;  // global run index of the pair's first run
        for (int st = ks * su; st < (ks + 1) * su; st++, g++) {
          const int slot = g % C::NS;
          if (!wait_or_abort(full + slot, (g / C::NS) & 1, deadline, p.err, abort_flag)) return;
          const uint8_t* runp = smem + slot * C::SLOT + STAGE_BYTES + run * RUN_BYTES;
          uint8_t* sc = smem + slot * C::SLOT + C::SC_OFF;
          const uint32_t b4 = runp[ch] * 0x01010101u;  // the chunk's base, in every byte
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const int kg = (st & 1) * 4 + kk;
            const uint32_t q = *reinterpret_cast<const uint32_t*>(runp + 16 + kg * 64 + ch * 4);
            const uint32_t lo = (q & 0x0F0F0F0Fu) + b4;         // positions 8ch + 0..3
            const uint32_t hi = ((q >> 4) & 0x0F0F0F0Fu) + b4;  // positions 8ch + 4..7
            uint8_t* row = sc + kk * SC_STRIDE;
#pragma unroll
            for (int i = 0; i < 8; i++) row[dst[i]] = (uint8_t)(((i < 4 ? lo : hi) >> (8 * (i & 3))) & 0xFF);
          }
          __syncwarp();
          // exception entries of this run that fall in this stage: overwrite their bytes
          const int rr = (st - ks * su) >> 1;
          const int eo0 = m.run_off[rr], eo1 = m.run_off[rr + 1];
          for (int j = eo0 + lane; j < eo1; j += 32) {
            const uint32_t en = exc[j];
            const int ppos = en & 0xFFFF, kg = (en >> 16) & 0xFF;
            if ((kg >> 2) != (st & 1)) continue;
            const int slot_e = ((ppos >> 7) == r0g ? 0 : 128) + position_slot(ppos & 127);
            sc[(kg & 3) * SC_STRIDE + slot_e] = (uint8_t)(en >> 24);
          }
          __syncwarp();
          mbar_arrive(scaled + slot);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mempty);
    }
    return;
  }

  // -------------------------------------------------------------------------------------------- consumers
  const int gq = lane >> 2, c = lane & 3;
  // the warp's two 16-row groups of the item (gate_up: gate group w and its up partner w + 8)
  const int G0 = p.gate_up ? warp : 2 * warp, G1 = p.gate_up ? warp + 8 : 2 * warp + 1;
  const int slot00 = 16 * G0 + gq, slot10 = 16 * G1 + gq;  // rows (g) of the two groups; g + 8 follows
  const int w_off = ((((c >> 1) ^ (gq >> 2)) & 1) << 4) | ((c & 1) << 3);  // byte of k-group c in a 32-byte row
  const int I = p.N / 2;
  uint32_t g = 0, k = 0;
  for (int r = 0; r < rounds; r++) {
    const int nu = min(MAXU, n_mine - r * MAXU);
    wait_or_abort(mfull, r & 1, deadline, p.err, abort_flag);
    consumer_sync();  // one decision for all consumer warps
    const bool have_meta = !*abort_flag;
    for (int ui = 0; ui < nu; ui++) {
      if (!have_meta) break;  // aborted: nothing was published (uniform across the consumer warps)
      const UnitMeta& m = meta[ui];
      const int e = m.e, item = m.item, ks = m.ks, nv = m.nv, blk = m.blk, flags = m.flags;
      const int* ids = mids + ui * XR;
      if (e < 0 || e >= p.E) {
        if (tid == 0) report(p.err, MOEK_DEV_BAD_EXPERT);
        continue;
      }
      if ((flags & 2) && tid == 0) report(p.err, MOEK_DEV_TOO_MANY_ROWS);
      const uint32_t* lt = lut + (k % NLUT) * 256;  // filled by the scale warp before the unit's first stage
      k++;
      const int ntile = (nv + 7) >> 3;
      float acc[2][C::T][4];
#pragma unroll
      for (int i = 0; i < 2; i++)
#pragma unroll
        for (int t = 0; t < C::T; t++)
#pragma unroll
          for (int v = 0; v < 4; v++) acc[i][t][v] = 0.f;

      for (int st = ks * su; st < (ks + 1) * su; st++, g++) {
        const int slot = g % C::NS;
        const uint32_t par = (g / C::NS) & 1;
        if (!wait_or_abort(full + slot, par, deadline, p.err, abort_flag) ||
            !wait_or_abort(scaled + slot, par, deadline, p.err, abort_flag))
          continue;  // aborted: skip, stay in step
        const uint8_t* sw = smem + slot * C::SLOT;
        const uint8_t* sx = sw + C::X_OFF;
        const uint8_t* sc = sw + C::SC_OFF + c * SC_STRIDE;
        const uint32_t s0a = lt[sc[slot00]], s0b = lt[sc[slot00 + 8]], s1a = lt[sc[slot10]], s1b = lt[sc[slot10 + 8]];
#pragma unroll
        for (int i = 0; i < 2; i++) {
          const uint32_t wa = i ? s1a : s0a, wb = i ? s1b : s0b;
          const ScaleBR sa{prmt_b(wa, 0x1010), prmt_b(wa, 0x3232)}, sbv{prmt_b(wb, 0x1010), prmt_b(wb, 0x3232)};
          // k-group c of rows g and g + 8 of the group: 8 bytes of each 32-byte row (halves swizzled by row bit 2)
          const uint8_t* wr = sw + (16 * (i ? G1 : G0) + gq) * 32 + w_off;
          const uint2 qa = *reinterpret_cast<const uint2*>(wr), qb = *reinterpret_cast<const uint2*>(wr + 8 * 32);
          uint32_t wa0[4], wb0[4], wa1[4], wb1[4];
          dequant_word(qa.x, sa, wa0);
          dequant_word(qb.x, sbv, wb0);
          dequant_word(qa.y, sa, wa1);
          dequant_word(qb.y, sbv, wb1);
          const uint32_t A0[4] = {wa0[0], wb0[0], wa0[1], wb0[1]};
          const uint32_t A1[4] = {wa0[2], wb0[2], wa0[3], wb0[3]};
          const uint32_t A2[4] = {wa1[0], wb1[0], wa1[1], wb1[1]};
          const uint32_t A3[4] = {wa1[2], wb1[2], wa1[3], wb1[3]};
#pragma unroll
          for (int t = 0; t < C::T; t++) {
            if (t < ntile) {
              const uint8_t* xr = sx + (t * 8 + gq) * X_STRIDE + c * 32;
              const uint4 x0 = *reinterpret_cast<const uint4*>(xr);
              const uint4 x1 = *reinterpret_cast<const uint4*>(xr + 16);
              mma_bf16_16816(acc[i][t], A0, x0.x, x0.y);
              mma_bf16_16816(acc[i][t], A1, x0.z, x0.w);
              mma_bf16_16816(acc[i][t], A2, x1.x, x1.y);
              mma_bf16_16816(acc[i][t], A3, x1.z, x1.w);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
      }

      // ---------------------------------------------------------------------------------------- epilogue
      // acc[i][t][2h + v] = weight row (16 G_i + g + 8h) x block row 8t + 2c + v
      if (p.mode == 3 && p.nsplit == 1) {
#pragma unroll
        for (int t = 0; t < C::T; t++) {
          if (t >= ntile) break;
#pragma unroll
          for (int v = 0; v < 2; v++) {
            const int row = t * 8 + 2 * c + v;
            if (row >= nv) continue;
            const int id = ids[row];
#pragma unroll
            for (int h = 0; h < 2; h++) {
              if (p.gate_up) {  // gate row and up row + 128 share the column
                const int col = 128 * item + slot00 + 8 * h;
                static_cast<__nv_bfloat16*>(p.out)[(int64_t)id * I + col] =
                    __float2bfloat16_rn(silu(acc[0][t][2 * h + v]) * acc[1][t][2 * h + v]);
              } else {
                const float w = p.topk_w[id];
                p.part[(int64_t)id * p.N + slot_column(p, item, slot00 + 8 * h)] = w * acc[0][t][2 * h + v];
                p.part[(int64_t)id * p.N + slot_column(p, item, slot10 + 8 * h)] = w * acc[1][t][2 * h + v];
              }
            }
          }
        }
        continue;
      }
      float* base = p.part + (int64_t)ks * p.num_ids * p.N;
#pragma unroll
      for (int t = 0; t < C::T; t++) {
        if (t >= ntile) break;
#pragma unroll
        for (int v = 0; v < 2; v++) {
          const int row = t * 8 + 2 * c + v;
          if (row >= nv) continue;
          float* prow = base + (int64_t)ids[row] * p.N;
#pragma unroll
          for (int h = 0; h < 2; h++) {
            prow[slot_column(p, item, slot00 + 8 * h)] = acc[0][t][2 * h + v];
            prow[slot_column(p, item, slot10 + 8 * h)] = acc[1][t][2 * h + v];
          }
        }
      }
      if (p.mode != 3) continue;
      // split-k completion, per warp (no CTA barrier): the warp whose arrival completes the (block, item) adds the
      // partials of every split in split order (deterministic) and finishes the item's rows.
      __threadfence();
      __syncwarp();
      int old = 0;
      if (lane == 0) old = atom_add_acq_rel(p.counters + (int64_t)blk * nt + item, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old != DC_WARPS * p.nsplit - 1) continue;
      if (lane == 0) p.counters[(int64_t)blk * nt + item] = 0;  // every arrival is in: ready for the next launch
      __threadfence();
      const int64_t stride = (int64_t)p.num_ids * p.N;
      if (p.gate_up) {
        for (int row = 0; row < nv; row++) {
          const int id = ids[row];
          const float* pr = p.part + (int64_t)id * p.N;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int col = 128 * item + lane + 32 * j;
            float gs = 0.f, us = 0.f;
            for (int s2 = 0; s2 < p.nsplit; s2++) {
              gs += __ldcg(pr + s2 * stride + col);
              us += __ldcg(pr + s2 * stride + I + col);
            }
            static_cast<__nv_bfloat16*>(p.out)[(int64_t)id * I + col] = __float2bfloat16_rn(silu(gs) * us);
          }
        }
        continue;
      }
      // down: weighted fp32 rows of this (block, item) into the row buffer after the partials
      float* rows_f32 = p.part + (int64_t)p.nsplit * stride;
      for (int row = 0; row < nv; row++) {
        const int id = ids[row];
        const float w = p.topk_w[id];
        const float* pr = p.part + (int64_t)id * p.N;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int col = 256 * item + lane + 32 * j;
          float sum = 0.f;
          for (int s2 = 0; s2 < p.nsplit; s2++) sum += __ldcg(pr + s2 * stride + col);
          rows_f32[(int64_t)id * p.N + col] = w * sum;
        }
      }
      __threadfence();
      __syncwarp();
      // each row's token: the arrival that completes the token's valid slots for this item adds them (slot order)
      int* tok_ctr = p.counters + (int64_t)p.max_blocks * nt;
      for (int row = 0; row < nv; row++) {
        const int tk = ids[row] / p.combine_k;
        int nslots = 0;
        if (lane < p.combine_k) {
          const int ej = p.topk_ids[tk * p.combine_k + lane];
          nslots = ej >= 0 && ej < p.E;
        }
        nslots = __popc(__ballot_sync(0xffffffffu, nslots != 0));
        int o2 = 0;
        if (lane == 0) o2 = atom_add_acq_rel(tok_ctr + (int64_t)tk * nt + item, 1);
        o2 = __shfl_sync(0xffffffffu, o2, 0);
        if (o2 != nslots - 1) continue;
        if (lane == 0) tok_ctr[(int64_t)tk * nt + item] = 0;
        __threadfence();
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int col = 256 * item + lane + 32 * j;
          float o = 0.f;
          for (int sl = 0; sl < p.combine_k; sl++) {
            const int id = tk * p.combine_k + sl;
            const int ej = p.topk_ids[id];
            if (ej < 0 || ej >= p.E) continue;
            o += __ldcg(rows_f32 + (int64_t)id * p.N + col);
          }
          static_cast<__nv_bfloat16*>(p.out)[(int64_t)tk * p.N + col] = __float2bfloat16_rn(o);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(mempty);
  }
}

// Sum of the nsplit partials at p[0], p[stride], ... in split order, with all loads issued before the adds (the
// partials are independent loads; the order of the fp32 additions is fixed, so the result is deterministic).
__device__ __forceinline__ float split_sum(const float* __restrict__ p, int64_t stride, int nsplit) {
  float acc = 0.f;
  for (int s0 = 0; s0 < nsplit; s0 += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = s0 + j < nsplit ? __ldcg(p + (s0 + j) * stride) : 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (s0 + j < nsplit) acc += v[j];
  }
  return acc;
}

// gate_up epilogue: act[id][c] = bf16(silu(sum_s g) * sum_s u), sums over the splits in split order.
__global__ void moek_gate_epilogue_kernel(const float* __restrict__ part, int nsplit, int num_ids, int N,
                                          __nv_bfloat16* __restrict__ act) {
  pdl_wait();
  pdl_launch_dependents();
  const int I = N / 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)num_ids * I) return;
  const int64_t id = i / I;
  const int col = (int)(i - id * I);
  const int64_t stride = (int64_t)num_ids * N;
  const float* r = part + id * N;
  const float gsum = split_sum(r + col, stride, nsplit);
  const float usum = split_sum(r + I + col, stride, nsplit);
  act[i] = __float2bfloat16_rn(silu(gsum) * usum);
}

// down epilogue fused with the top-k sum: out[t][n] = bf16(sum_j w[t,j] * sum_s part[s][t*k+j][n]) in fp32, slots in
// order j = 0..k-1 (one rounding, as the fp32 oracle).
__global__ void moek_down_combine_kernel(const float* __restrict__ part, int nsplit, int num_ids, int N, int top_k,
                                         const float* __restrict__ topk_w, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int m = num_ids / top_k;
  if (i >= (int64_t)m * N) return;
  const int64_t t = i / N;
  const int n = (int)(i - t * N);
  const int64_t stride = (int64_t)num_ids * N;
  float o = 0.f;
  for (int j0 = 0; j0 < top_k; j0 += 8) {
    float sums[8];
#pragma unroll
    for (int j = 0; j < 8; j++)
      sums[j] = j0 + j < top_k ? split_sum(part + (t * top_k + j0 + j) * N + n, stride, nsplit) : 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (j0 + j < top_k) o += topk_w[t * top_k + j0 + j] * sums[j];
  }
  out[i] = __float2bfloat16_rn(o);
}

// down epilogue without the sum: dout[id][n] = fp32 w[id] * sum_s part (kept in fp32 for the combine)
__global__ void moek_down_rows_kernel(const float* __restrict__ part, int nsplit, int num_ids, int N,
                                      const float* __restrict__ topk_w, float* __restrict__ dout) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)num_ids * N) return;
  const int64_t id = i / N;
  const int64_t stride = (int64_t)num_ids * N;
  float s = 0.f;
  for (int sp = 0; sp < nsplit; sp++) s += part[sp * stride + i];
  dout[i] = topk_w[id] * s;
}

// top-k combine of fp32 rows: out[t][n] = bf16(sum_j rows[t*k + j][n]) (slot order)
__global__ void moek_combine_f32_kernel(const float* __restrict__ rows, int m, int N, int top_k,
                                        __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)m * N) return;
  const int64_t t = i / N;
  const int n = (int)(i - t * N);
  float o = 0.f;
  for (int j = 0; j < top_k; j++) o += rows[(t * top_k + j) * N + n];
  out[i] = __float2bfloat16_rn(o);
}

// The same for N % 4 == 0, four columns per thread: the k slots' 16-byte loads issued together, one 8-byte store; an
// HBM stream of k fp32 rows in and one bf16 row out per token.
__global__ void __launch_bounds__(256) moek_combine_f32x4_kernel(const float4* __restrict__ rows, int m, int N4,
                                                                 int top_k, uint2* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t n = (int64_t)m * N4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / N4;
    const int64_t c = i - t * N4;
    const float4* r = rows + t * top_k * N4 + c;
    float4 v[8];
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = 0; j0 < top_k; j0 += 8) {
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j0 + j < top_k) v[j] = __ldcs(r + (int64_t)(j0 + j) * N4);  // read once: do not keep in L2
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j0 + j < top_k) o.x += v[j].x, o.y += v[j].y, o.z += v[j].z, o.w += v[j].w;
    }
    const __nv_bfloat162 a = __floats2bfloat162_rn(o.x, o.y), b = __floats2bfloat162_rn(o.z, o.w);
    out[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  }
}

// The top-k sum over the routed slots only: a slot whose expert id lies outside [0, E) was not computed (its row
// holds whatever the buffer held) and is left out, so a token with no routed slot gets a zero row. Every slot's row is
// loaded (all rows lie inside the buffer) and the ids only choose which ones are added, so the row loads do not wait
// for the id loads; with every slot routed the additions are the plain combine's, bit for bit.
__global__ void __launch_bounds__(256) moek_combine_routed_f32x4_kernel(const float4* __restrict__ rows,
                                                                        const int32_t* __restrict__ ids, int E, int m,
                                                                        int N4, int top_k, uint2* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t n = (int64_t)m * N4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / N4;
    const int64_t c = i - t * N4;
    const float4* r = rows + t * top_k * N4 + c;
    const int32_t* tid = ids + t * top_k;
    float4 v[8];
    int e[8];
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = 0; j0 < top_k; j0 += 8) {
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j0 + j < top_k) {
          e[j] = __ldg(tid + j0 + j);
          v[j] = __ldcs(r + (int64_t)(j0 + j) * N4);  // read once: do not keep in L2
        }
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j0 + j < top_k && e[j] >= 0 && e[j] < E) o.x += v[j].x, o.y += v[j].y, o.z += v[j].z, o.w += v[j].w;
    }
    const __nv_bfloat162 a = __floats2bfloat162_rn(o.x, o.y), b = __floats2bfloat162_rn(o.z, o.w);
    out[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  }
}

// The same, one column per thread (any N or alignment).
__global__ void moek_combine_routed_f32_kernel(const float* __restrict__ rows, const int32_t* __restrict__ ids, int E,
                                               int m, int N, int top_k, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)m * N) return;
  const int64_t t = i / N;
  const int n = (int)(i - t * N);
  float o = 0.f;
  for (int j = 0; j < top_k; j++) {
    const int e = ids[t * top_k + j];
    const float v = rows[(t * top_k + j) * N + n];
    if (e >= 0 && e < E) o += v;
  }
  out[i] = __float2bfloat16_rn(o);
}

// top-k combine of bf16 rows (the reference's torch.sum over dim 1: fp32 accumulation, one rounding)
__global__ void moek_combine_bf16_kernel(const __nv_bfloat16* __restrict__ rows, int m, int N, int top_k,
                                         __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)m * N) return;
  const int64_t t = i / N;
  const int n = (int)(i - t * N);
  float o = 0.f;
  for (int j = 0; j < top_k; j++) o += __bfloat162float(rows[(t * top_k + j) * N + n]);
  out[i] = __float2bfloat16_rn(o);
}

// ------------------------------------------------------------------------------------------------- launchers
template <int XR>
static cudaError_t launch_decode_xr(const GemmParams& p, int grid, cudaStream_t st) {
  using C = DecodeCfg<XR>;
  cudaError_t e = cudaFuncSetAttribute(moek_decode_kernel<XR>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  e = launch_pdl(moek_decode_kernel<XR>, dim3(grid), dim3(DC_THREADS), C::SMEM, st, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_decode(const GemmParams& p, int max_rows, int sms, cudaStream_t st) {
  const int nt = p.N / ITEM_COLS;
  const int64_t units = (int64_t)p.max_blocks * nt * p.nsplit;
  const int per_sm = max_rows <= 32 ? 2 : 1;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)per_sm * sms, units));
  if (max_rows <= 8) return launch_decode_xr<8>(p, grid, st);
  if (max_rows <= 16) return launch_decode_xr<16>(p, grid, st);
  if (max_rows <= 32) return launch_decode_xr<32>(p, grid, st);
  return launch_decode_xr<96>(p, grid, st);
}

cudaError_t launch_gate_epilogue(const float* part, int nsplit, int num_ids, int N, __nv_bfloat16* act,
                                 cudaStream_t st) {
  const int64_t n = (int64_t)num_ids * (N / 2);
  if (n == 0) return cudaSuccess;
  cudaError_t e = launch_pdl(moek_gate_epilogue_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, part,
                             nsplit, num_ids, N, act);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_down_combine(const float* part, int nsplit, int num_ids, int N, int top_k, const float* topk_w,
                                __nv_bfloat16* out, cudaStream_t st) {
  const int64_t n = (int64_t)(num_ids / top_k) * N;
  if (n == 0) return cudaSuccess;
  cudaError_t e = launch_pdl(moek_down_combine_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, part,
                             nsplit, num_ids, N, top_k, topk_w, out);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_down_rows(const float* part, int nsplit, int num_ids, int N, const float* topk_w, float* dout,
                             cudaStream_t st) {
  const int64_t n = (int64_t)num_ids * N;
  if (n == 0) return cudaSuccess;
  moek_down_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, nsplit, num_ids, N, topk_w, dout);
  return cudaGetLastError();
}

cudaError_t launch_combine_f32(const float* rows, int m, int N, int top_k, __nv_bfloat16* out, cudaStream_t st) {
  const int64_t n = (int64_t)m * N;
  if (n == 0) return cudaSuccess;
  if (N % 4 == 0 && ((reinterpret_cast<uintptr_t>(rows) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
    const int64_t n4 = n / 4;
    const unsigned grid = (unsigned)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
    moek_combine_f32x4_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const float4*>(rows), m, N / 4, top_k,
                                                    reinterpret_cast<uint2*>(out));
    return cudaGetLastError();
  }
  moek_combine_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, m, N, top_k, out);
  return cudaGetLastError();
}

cudaError_t launch_combine_routed(const float* rows, const int32_t* ids, int E, int m, int N, int top_k,
                                  __nv_bfloat16* out, cudaStream_t st) {
  const int64_t n = (int64_t)m * N;
  if (n == 0) return cudaSuccess;
  if (N % 4 == 0 && ((reinterpret_cast<uintptr_t>(rows) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
    const int64_t n4 = n / 4;
    const unsigned grid = (unsigned)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
    moek_combine_routed_f32x4_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const float4*>(rows), ids, E, m, N / 4,
                                                           top_k, reinterpret_cast<uint2*>(out));
    return cudaGetLastError();
  }
  moek_combine_routed_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, ids, E, m, N, top_k, out);
  return cudaGetLastError();
}

cudaError_t launch_combine_bf16(const __nv_bfloat16* rows, int m, int N, int top_k, __nv_bfloat16* out,
                                cudaStream_t st) {
  const int64_t n = (int64_t)m * N;
  if (n == 0) return cudaSuccess;
  moek_combine_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, m, N, top_k, out);
  return cudaGetLastError();
}

}  // namespace moek
