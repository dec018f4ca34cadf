"""Benchmark of the routed-expert NVFP4 (W4A16) MoE layer on B200.

Workloads (the reference's configs; synthetic seeded data of those shapes):

- decode8  (config 2, the headline): a decode verify step, M = 8 tokens per GPU, uniform routing (softmax of N(0,1)
           logits -> top-5 -> renormalise);
- decode32 (config 3): M = 32 tokens (4 streams x 8), Zipf(1.1) routing over a seeded permutation of the experts;
- prefill  (config 4): M = 6912 tokens, uniform routing; prefill_zipf: the same with Zipf(1.1) routing.
- block8   the whole MoE block at M = 8 (the routed layer's neighbours): the router gate GEMM, its
           softmax / top-5 routing, the routed experts and the MXFP8 shared expert (Is = 512) with its sigmoid gate,
           through ``ops.moe_block``; GB/s over the touched experts' bytes plus the gate's and the shared expert's.

Every workload runs on the same 48 layers of 512 experts (hidden 2048, expert intermediate 512, top-5) with
independent seeded NVFP4 weights (bf16 N(0, 0.02) quantised; 857 MB per layer, 41 GB in HBM). A step runs the 48
layers back to back through ``ops.fused_moe``, replayed as one CUDA graph; the weights the 48 layers touch exceed the
126 MB L2, so each layer streams its experts from HBM (the layer rotation is the L2 flush).

Units: decode = algorithmic HBM GB/s (touched experts' packed codes + packed scales + exception lists + x + output +
routing); prefill = algorithmic TFLOP/s (2 * M * 5 * 3 * 2048 * 512, real rows only). ``value`` is the chosen
workload's (``--workload``, default decode8); by default the other two are measured as well and reported under
``workloads``. ``e2e`` = the same metric through the public API with each step's inputs copied from pinned host
memory and its outputs read back inside the timed region. ``roofline`` = the gate_up GEMM launches replayed alone
(CUDA events on the replaying stream) against MEASURED_PEAKS.json.

``--impl reference`` times the reference's CPU path (the fp32 dequantise-then-matmul oracle of
bench/moek/problem.py:51-67, restated in oracle/moe_ref.py) on the host cores, same metric and unit.
Multi-GPU (torchrun, N > 1): the expert-parallel stack (the reference's config 5). The 512 experts of every layer are
split contiguously over the ranks (each GPU holds 1/N of the 41 GB), each rank brings its own tokens (weak scaling),
and ``ep.ep_moe`` moves them: decode M=8 per GPU (the headline, same metric as N=1) and M=64 Zipf with the
fixed-capacity exchange over peer memory, prefill M=6912 Zipf per GPU with exact counts over NCCL, and one M=6912
chunk split over the GPUs (strong scaling). Each EP workload also reports the load-balance ceiling of the contiguous
expert split (mean over max of the routed rows each rank owns), and before any timing every rank checks its tokens'
EP output against the one-GPU layer (``parity`` in the line; the run fails outside the gate). value = the bytes of the
experts the step touched (each streamed once, by its owner) plus every rank's x / output / routing (or the FLOPs of
all ranks' rows) over the slowest rank's time (CUDA events, max over ranks). The roofline is the local gate_up GEMM on
the rows one step delivered.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "routed-MoE layer µs & HBM GB/s (M=8,32); TFLOP/s (M=6912); 1/2/4/8 GPU"
H, I, E, TOPK = 2048, 512, 512, 5
FLOPS_PER_ROW = 2 * 3 * H * I  # gate + up + down per (token, slot) row

# DRAM bytes (read + write) of one launch of the roofline kernel: dram__bytes_read.sum + dram__bytes_write.sum of one
# launch in an ncu capture of this file's own command (given with each figure as "traffic_source"); not measured by
# the run that prints them.
TRAFFIC = {
    "decode8": (68_361_728, "ncu capture of one moek_layer_kernel<8> launch (stream-K plan, 8-row blocks), "
                            "bench.py --only --workload decode8 --layers 4"),
    "decode32": (141_612_800, "ncu capture of one moek_layer_kernel<8> launch (stream-K plan, 8-row blocks), "
                              "bench.py --only --workload decode32 --layers 4"),
    "prefill": (695_998_464, "ncu capture of one moek_prefill_kernel gate_up launch, "
                             "bench.py --only --workload prefill --layers 2"),
}

WORKLOADS = {
    "decode8": dict(m=8, route="uniform", unit="GB/s", desc="decode verify M=8 (1 stream x block 8), uniform routing"),
    "decode32": dict(m=32, route="zipf", unit="GB/s", desc="multi-stream decode M=32 (4 x 8), Zipf(1.1) routing"),
    "prefill": dict(m=6912, route="uniform", unit="TFLOP/s", desc="prefill chunk M=6912, uniform routing"),
    "prefill_zipf": dict(m=6912, route="zipf", unit="TFLOP/s", desc="prefill chunk M=6912, Zipf(1.1) routing"),
    "block8": dict(m=8, route="gate", unit="GB/s",
                   desc="whole MoE block M=8: router gate GEMM -> softmax top-5 -> routed experts, plus the MXFP8 "
                        "shared expert (Is = 512) with its sigmoid gate"),
}
SHARED_INTER = 512  # the block workload's shared-expert width


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode8", choices=list(WORKLOADS))
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", action="store_true", help="measure the chosen workload only")
    ap.add_argument("--ep-exchange", default="peer", choices=["peer", "nccl"],
                    help="N > 1, fixed-capacity workloads: exchange over peer memory or NCCL all-to-all")
    return ap.parse_args()


def route(m, seed, kind, device):
    from qwen38_flash_coder_b200 import synth

    if kind == "zipf":
        return synth.route_zipf(m, E, TOPK, seed, device=device)
    return synth.route_softmax(m, E, TOPK, seed, device=device)


def pack_inputs(x, ids, w):
    """One layer's inputs as one byte tensor x | ids | weights (x first, so that it stays 16-byte aligned), so that
    they cross between host and GPU in one copy."""
    import torch

    return torch.cat([t.contiguous().view(torch.uint8).reshape(-1) for t in (x, ids, w)])


def unpack_inputs(buf, m):
    """Views (x bf16 [m, H], ids int32 [m, TOPK], weights fp32 [m, TOPK]) of a ``pack_inputs`` buffer."""
    import torch

    xb, ib = m * H * 2, m * TOPK * 4
    return (buf[:xb].view(torch.bfloat16).view(m, H), buf[xb:xb + ib].view(torch.int32).view(m, TOPK),
            buf[xb + ib:xb + 2 * ib].view(torch.float32).view(m, TOPK))


def touched_bytes(layer, ids, m):
    """Algorithmic bytes of one layer call: touched experts' streamed bytes + x + out + routing."""
    import torch

    touched = torch.unique(ids.long())
    per = layer.expert_bytes().to(ids.device)
    return int(per[touched].sum()) + m * H * 2 * 2 + m * TOPK * 8, int(touched.numel())


def gate_bytes(layer, ids, m):
    """Algorithmic bytes of one gate_up GEMM launch: touched experts' w13 codes, packed scales, exceptions, and x."""
    import torch

    touched = torch.unique(ids.long()).cpu()
    w = layer.w13
    nkeys = (w.exc_off.numel() - 1) // w.E
    off = w.exc_off.to(torch.int64).cpu()
    n_exc = off[(touched + 1) * nkeys] - off[touched * nkeys]
    per = w.w[0].numel() * 4 + w.sp[0].numel() + 4 * (nkeys + 1)
    return int(touched.numel() * per + 4 * n_exc.sum()) + m * H * 2


class Clocks:
    """SM clock, power and clock-event reasons sampled during the timed region: NVML every ~2 ms from a thread
    (timed regions of a few milliseconds still get samples), nvidia-smi every 100 ms if NVML is not available."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, dev):
        import threading

        self.samples, self.h, self.p = [], None, None
        self.done = threading.Event()
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(dev).uuid)
                self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(dev.index)
            self.nv = pynvml
            self.mx = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            self.h = None
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            try:
                self.p = subprocess.Popen(["nvidia-smi", f"--id={dev.index}", f"--query-gpu={q}", "--format=csv,noheader",
                                           "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
            except OSError:
                self.p = None

    def _run(self):
        nv = self.nv
        while not self.done.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((sm, rs, pw))
            except Exception:
                pass
            time.sleep(0.002)

    def stop(self):
        if self.h is not None:
            self.done.set()
            self.t.join(timeout=5)
            sm = [x[0] for x in self.samples]
            reasons = sorted({n for _, rs, _ in self.samples for n, bit in self.REASONS.items() if rs & bit})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.mx, "samples": len(sm),
                    "power_w_max": max((x[2] for x in self.samples), default=None), "reasons": reasons,
                    "source": "nvml"}
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait(timeout=10)
        self.f.seek(0)
        sm, mx, reasons, power = [], None, set(), []
        for line in self.f.read().splitlines():
            c = [x.strip() for x in line.split(",")]
            if len(c) < 7:
                continue
            try:
                sm.append(float(c[0].split()[0]))
                mx = float(c[1].split()[0])
                power.append(float(c[2].split()[0]))
            except ValueError:
                continue
            for n, v in zip(list(self.REASONS), c[3:7]):
                if "Active" in v and "Not" not in v:
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "power_w_max": max(power) if power else None, "reasons": sorted(reasons), "source": "nvidia-smi"}


def make_graph(fn, warmup):
    """Warm up on a side stream, then capture one call of fn in a CUDA graph."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(max(3, warmup)):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def timed(fn, steps, barrier):
    """ms per call of fn over ``steps`` calls: barrier + synchronize on both sides, CUDA events on the stream."""
    import torch

    fn()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1) / steps


def gate_stats(out, ref):
    """(rel-L2, net max-abs / rms) of a bf16 result against a reference: the parity gate's two figures, the max-abs
    taken beyond half a bf16 ulp of the reference (the rounding of the output itself)."""
    import torch

    o, r = out.float(), ref.float()
    rel = float((o - r).norm() / r.norm().clamp_min(1e-30))
    rms = float(r.pow(2).mean().sqrt().clamp_min(1e-30))
    half_ulp = torch.pow(2.0, torch.floor(torch.log2(r.abs().clamp_min(2.0 ** -126))) - 8)
    net = float(((o - r).abs() - half_ulp).clamp_min(0).max()) / rms if o.numel() else 0.0
    return rel, net


def over_ranks(v, world, dev, op="max"):
    """The max (or sum) of a per-rank number over all ranks."""
    import torch

    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX if op == "max" else torch.distributed.ReduceOp.SUM)
    return float(t)


def cpu_baseline(layers, name, budget_s=12.0):
    """The oracle (fp32 dequantise-then-matmul, torch CPU, all host threads) on a bounded sample of the workload:
    whole decode layers, or the first 256 tokens of prefill layers; copying the touched experts to the host is not
    timed. Same unit as the workload."""
    import torch

    from oracle import moe_ref

    from qwen38_flash_coder_b200 import ops

    torch.set_num_threads(os.cpu_count())
    wl = WORKLOADS[name]
    sample_m = min(wl["m"], 256)
    amount, tot, n, checks = 0.0, 0.0, 0, []
    while n < len(layers) and (tot < budget_s or n == 0):
        w13, w2 = layers[n]["ckpt"]
        x = layers[n]["x"][name][:sample_m]
        ids, wts = (t[:sample_m] for t in layers[n]["route"][name])
        touched = torch.unique(ids.long())
        remap = torch.full((E,), -1, dtype=torch.long, device=ids.device)
        remap[touched] = torch.arange(touched.numel(), device=ids.device)
        cpu = lambda mm: (mm[0][touched].cpu().numpy(), mm[1][touched].view(torch.uint8).cpu().numpy(),
                          mm[2][touched].cpu().numpy())
        c13, c2, cid = cpu(w13), cpu(w2), remap[ids.long()].cpu().numpy()
        xc, wc = x.cpu(), wts.cpu().numpy()
        t1 = time.perf_counter()
        ref = moe_ref.reference(xc, cid, wc, c13, c2)
        tot += time.perf_counter() - t1
        # the oracle as the checker: this build's output for the same tokens must be inside the gate
        got = ops.fused_moe(x, layers[n]["prep"], wts, ids)
        checks.append(moe_ref.check(got.cpu(), ref))
        if wl["unit"] == "GB/s":
            amount += touched_bytes(layers[n]["prep"], ids, sample_m)[0] / 1e9
        else:
            amount += sample_m * TOPK * FLOPS_PER_ROW / 1e12
        n += 1
    rel, net = max(c[0] for c in checks), max(c[2] for c in checks)
    parity = {"vs": "the fp32 oracle (oracle/moe_ref.py) on the sampled tokens", "rel_l2": rel, "net_maxabs": net,
              "gate": "rel-L2 <= 5e-3, net max-abs <= 2e-2 * rms", "ok": bool(rel <= 5e-3 and net <= 2e-2)}
    return {"value": round(amount / tot, 6), "unit": wl["unit"], "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} layer(s) x {sample_m} tokens of this workload (touched experts only), torch-CPU oracle "
                      f"(oracle/moe_ref.py), {tot:.1f} s of compute"}, parity


def measure(name, layers, a, dev, world, barrier, headline):
    """One workload over all layers: device step time, value, the gate_up roofline and, for the headline, e2e."""
    import torch

    from qwen38_flash_coder_b200 import ops

    wl = WORKLOADS[name]
    m, nl = wl["m"], len(layers)
    out_all = torch.empty((nl, m, H), dtype=torch.bfloat16, device=dev)  # every layer's output, one buffer
    outs = list(out_all.unbind(0))

    block = wl["route"] == "gate"

    def step():
        for l in range(nl):
            ids, wts = layers[l]["route"][name]
            if block:
                ops.moe_block(layers[l]["x"][name], layers[l]["gate"], layers[l]["prep"], layers[l]["shared"], TOPK,
                              output=outs[l])
            else:
                ops.fused_moe(layers[l]["x"][name], layers[l]["prep"], wts, ids, output=outs[l])

    graph = make_graph(step, a.warmup)
    ops.check_device_errors(dev)
    clocks = Clocks(dev)
    ms = timed(graph.replay, a.steps, barrier)
    clk = clocks.stop()
    extra = 0  # the block's gate and shared-expert bytes per layer (weights, scales, the expert gate)
    if block:
        extra = E * H * 2 + 3 * SHARED_INTER * H * (1 + 1 / 32) + H * 2
    if wl["unit"] == "GB/s":
        amount = sum(touched_bytes(L["prep"], L["route"][name][0], m)[0] + extra for L in layers) / 1e9
    else:
        amount = nl * m * TOPK * FLOPS_PER_ROW / 1e12
    ms = over_ranks(ms, world, dev)
    amount = over_ranks(amount, world, dev, op="sum")
    value = amount / (ms / 1e3)

    # roofline of the dominant kernel: the step's gate_up GEMM launches alone, replayed as a graph
    rec = ops.record_launches(step)
    kern_us = {}
    for kname in ("layer", "gate_gemm", "down_gemm"):
        fns = [f for n, f in rec if n == kname]
        if not fns:
            continue
        g = make_graph(lambda: [f() for f in fns], 2)
        kern_us[kname] = over_ranks(timed(g.replay, a.steps, barrier) * 1e3 / len(fns), world, dev)
        del g
    peaks = {}
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        peaks = json.load(open(pp))
    traffic, traffic_src = TRAFFIC.get(name, (None, None))
    if block:  # the block's three kernels together: the step's own time per layer
        kern_us["layer"] = ms * 1e3 / nl
    if wl["unit"] == "GB/s":  # the whole-layer kernel: every touched expert's gate_up and down bytes, x, out
        gb = sum(touched_bytes(L["prep"], L["route"][name][0], m)[0] + extra for L in layers) / nl
        peak = peaks.get("hbm_gbs", 6650.0)
        achieved = gb / (kern_us["layer"] / 1e6) / 1e9
        roof = {"kernel": "moek_layer_kernel (whole decode layer, one launch)" if not block else
                "moek_moe_block (router gate, shared expert, whole layer: three launches, timed together)",
                "bound": "hbm",
                "achieved": round(achieved, 1), "peak": peak,
                "peak_source": "of measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "of fallback",
                "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_source": traffic_src,
                "bytes_per_launch": int(gb), "avg_launch_us": round(kern_us["layer"], 2)}
    else:
        flops = m * TOPK * 2 * H * 2 * I  # gate + up rows of real tokens
        peak = peaks.get("bf16_tflops_sustained", 1400.0)
        achieved = flops / (kern_us["gate_gemm"] / 1e6) / 1e12
        roof = {"kernel": "moek_prefill_kernel (gate_up, tcgen05)", "bound": "tensor", "achieved": round(achieved, 1),
                "peak": peak, "peak_source": "of measured sustained (MEASURED_PEAKS.json bf16_tflops_sustained)"
                if "bf16_tflops_sustained" in peaks else "of fallback", "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_source": traffic_src,
                "flops_per_launch": flops}
    if "gate_gemm" in kern_us:
        roof["avg_launch_us"] = round(kern_us["gate_gemm"], 2)
        roof["down_gemm_avg_us"] = round(kern_us["down_gemm"], 2)
    res = {"workload": wl["desc"], "value": round(value, 3), "unit": wl["unit"], "ms_per_step": round(ms, 4),
           "us_per_layer": round(ms * 1e3 / nl, 2), "roofline": roof, "clocks": clk,
           "gpu_launches_per_step": (4 if block else ops.launches_per_layer(m, TOPK)) * nl}
    if wl["unit"] == "GB/s":
        res["touched_experts_per_layer"] = round(
            sum(touched_bytes(L["prep"], L["route"][name][0], m)[1] for L in layers) / nl, 1)
    if headline:
        # e2e: the public API with each step's inputs copied from pinned host memory and its outputs read back
        # one pinned staging buffer per layer holding x | ids | weights, so that a layer's inputs cross to the GPU in
        # one copy (and its output back in one): x (16-byte aligned) at 0, then the int32 ids and the fp32 weights.
        # The step's staging buffers sit back to back in one pinned block, and a copy stream moves them in two
        # copies: the first layer's inputs, then all the others, which cross while the first layer computes. Only
        # the first two layers wait for a copy; the rest follow each other directly.
        packed = [pack_inputs(L["x"][name], *L["route"][name]) for L in layers]
        seg = (packed[0].numel() + 15) // 16 * 16
        hall = torch.zeros((nl, seg), dtype=torch.uint8).pin_memory()
        for l in range(nl):
            hall[l, :packed[l].numel()].copy_(packed[l])
        hout = torch.empty((nl, m, H), dtype=torch.bfloat16).pin_memory()
        dall = torch.empty_like(hall, device=dev)
        din = [dall[l, :packed[l].numel()] for l in range(nl)]
        dx, did, dw = zip(*[unpack_inputs(d, m) for d in din])
        copy_stream = torch.cuda.Stream(dev)
        copied = [torch.cuda.Event() for _ in range(2)]

        def e2e_step():
            cur = torch.cuda.current_stream(dev)
            copy_stream.wait_stream(cur)  # this step's copies start after the previous step's layers read them
            with torch.cuda.stream(copy_stream):
                dall[:1].copy_(hall[:1], non_blocking=True)  # the first layer's inputs
                copied[0].record(copy_stream)
                dall[1:].copy_(hall[1:], non_blocking=True)  # every other layer's, in one copy
                copied[1].record(copy_stream)
            for l in range(nl):
                if l < 2:
                    cur.wait_event(copied[l])
                if block:  # the block routes itself: x in, its output out (ids and weights are copied all the same)
                    ops.moe_block(dx[l], layers[l]["gate"], layers[l]["prep"], layers[l]["shared"], TOPK,
                                  output=outs[l])
                else:
                    ops.fused_moe(dx[l], layers[l]["prep"], dw[l], did[l], output=outs[l])
            hout.copy_(out_all, non_blocking=True)  # the step's results: every layer's output, one copy back

        device_out = out_all.clone()  # the device-resident step's results, to check the copied path against
        eg = make_graph(e2e_step, 2)
        ems = over_ranks(timed(eg.replay, a.steps, barrier), world, dev)
        del eg
        torch.cuda.synchronize()
        res["e2e"] = {"value": round(amount / (ems / 1e3), 3), "unit": wl["unit"],
                      "h2d_bytes_per_step": hall.numel(),
                      "d2h_bytes_per_step": hout.numel() * 2, "ms_per_step": round(ems, 4),
                      "api": ("ops.moe_block" if block else "ops.fused_moe") + " with host copies (the step's "
                             "pinned staging buffers in two copies on a copy stream, the first layer's inputs, then "
                             "the other layers' while the first computes; every layer's output back in one copy at "
                             "the step's end), one CUDA graph per step",
                      "output_equals_device_step": bool(torch.equal(hout, device_out.cpu()))}
        res["eager_ms_per_step"] = round(over_ranks(timed(step, max(2, a.steps // 4), barrier), world, dev), 4)
    del graph
    return res


def main():
    a = parse()
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        return reference_arm(a, rank, world)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        try:
            return ep_main(a, rank, world, dev)
        finally:
            dist.destroy_process_group()
    from qwen38_flash_coder_b200 import prep, synth

    names = [a.workload] + ([] if a.only else [n for n in ("decode8", "decode32", "prefill", "prefill_zipf", "block8")
                                               if n != a.workload])
    layers = []
    for l in range(a.layers):
        w13, w2 = synth.make_layer(E, H, I, l, device=dev)
        # checkpoint tensors are kept only for the layers the CPU baseline may sample
        L = {"prep": prep.PreparedLayer(w13, w2), "ckpt": (w13, w2) if l < 3 else None, "x": {}, "route": {}}
        del w13, w2
        for j, n in enumerate(names):
            seed = 100000 * rank + 100 * l + j
            L["x"][n] = synth.activations(WORKLOADS[n]["m"], H, seed, device=dev)
            if WORKLOADS[n]["route"] == "gate":  # the block routes itself: its gate and shared expert per layer
                from qwen38_flash_coder_b200 import ops

                L["gate"] = synth.make_router_gate(E, H, l, device=dev)
                L["shared"] = ops.SharedExpert(*synth.make_shared(H, SHARED_INTER, l, device=dev))
                w, ids = ops.router_topk(ops.router_gate(L["x"][n], L["gate"]), TOPK, True)
                L["route"][n] = (ids, w)
            else:
                L["route"][n] = route(WORKLOADS[n]["m"], seed, WORKLOADS[n]["route"], dev)
        layers.append(L)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    results = {n: measure(n, layers, a, dev, world, barrier, headline=(n == a.workload)) for n in names}
    head = results.pop(a.workload)
    cpu, parity = None, None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu, parity = cpu_baseline(layers[:3], a.workload)
    if world > 1:
        torch.distributed.barrier()
    if rank == 0:
        wl = WORKLOADS[a.workload]
        line = {
            "metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world, "steps": a.steps,
            "warmup": max(3, a.warmup), "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": wl["desc"], "layers_per_step": a.layers, "experts": E, "hidden": H, "inter": I,
                       "top_k": TOPK, "tokens_per_gpu": wl["m"],
                       "weights": "NVFP4 (E2M1 + E4M3/16 + fp32 global), bf16 activations",
                       "l2": f"{a.layers} distinct layers per step rotate; touched weights >> 126 MB L2",
                       "parallelism": "single GPU" if world == 1 else f"{world} independent replicas"},
            "us_per_layer": head["us_per_layer"], "roofline": head["roofline"], "cpu_baseline": cpu,
            "e2e": head["e2e"], "clocks": head["clocks"],
            "gpu_launches": head["gpu_launches_per_step"] * a.steps,
            "eager_ms_per_step": head["eager_ms_per_step"],
            "workloads": results, "parity": parity,
        }
        if "touched_experts_per_layer" in head:
            line["touched_experts_per_layer"] = head["touched_experts_per_layer"]
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


EP_WORKLOADS = {
    "decode8": dict(m=8, route="uniform", unit="GB/s", capacity=True,
                    desc="EP decode verify, M=8 tokens per GPU, uniform routing, fixed-capacity exchange"),
    "decode64": dict(m=64, route="zipf", unit="GB/s", capacity=True,
                     desc="EP decode, M=64 tokens per GPU (8 streams x 8), Zipf(1.1), fixed-capacity exchange"),
    "prefill": dict(m=6912, route="zipf", unit="TFLOP/s", capacity=False,
                    desc="EP prefill chunk, M=6912 tokens per GPU, Zipf(1.1), all-to-allv exchange"),
    "prefill_strong": dict(m=None, route="zipf", unit="TFLOP/s", capacity=False,
                           desc="EP prefill, strong scaling: one M=6912 chunk split over the GPUs (6912 / N tokens "
                                "each), Zipf(1.1), all-to-allv exchange"),
}


def ep_tokens(name, world):
    """Tokens per rank of an EP workload (the strong-scaling one splits one 6912-token chunk)."""
    m = EP_WORKLOADS[name]["m"]
    return m if m is not None else 6912 // world


def ep_main(a, rank, world, dev):
    """N > 1: the expert-parallel stack (experts split contiguously over the ranks, tokens per rank, NCCL
    all-to-all dispatch and combine). Weak scaling: every rank brings its own M tokens per layer."""
    import torch
    import torch.distributed as dist

    from qwen38_flash_coder_b200 import ep, ops, prep, synth

    names = ["decode8"] if a.only else ["decode8", "decode64", "prefill", "prefill_strong"]
    layers, touched_bytes_all = [], []
    for l in range(a.layers):
        w13, w2 = synth.make_layer(E, H, I, l, device=dev)
        L = ep.EPLayer(ep.shard_checkpoint(w13, E, world, rank), ep.shard_checkpoint(w2, E, world, rank), E, world,
                       rank)
        del w13, w2
        entry = {"layer": L, "x": {}, "route": {}}
        for j, n in enumerate(names):
            seed = 100000 * rank + 100 * l + j
            m = ep_tokens(n, world)
            entry["x"][n] = synth.activations(m, H, seed, device=dev)
            entry["route"][n] = route(m, seed, EP_WORKLOADS[n]["route"], dev)
        layers.append(entry)
    # parity: one more seeded layer, held whole (all 512 experts) on every rank besides its EP shard, so that every
    # rank can compare its tokens' expert-parallel output with the one-GPU layer before anything is timed
    pw13, pw2 = synth.make_layer(E, H, I, 977, device=dev)
    par_full = prep.PreparedLayer(pw13, pw2)
    par_ep = ep.EPLayer(ep.shard_checkpoint(pw13, E, world, rank), ep.shard_checkpoint(pw2, E, world, rank), E,
                        world, rank)
    del pw13, pw2
    torch.cuda.empty_cache()
    parity = {}

    def barrier():
        dist.barrier()

    def check_parity(name, wl, px):
        """ep.ep_moe on this rank's seeded tokens against ops.fused_moe of the same tokens on this GPU with every
        expert; the worst rank's figures."""
        seed = 100000 * rank + 99
        m = ep_tokens(name, world)
        x = synth.activations(m, H, seed, device=dev)
        ids, wts = route(m, seed, wl["route"], dev)
        got = ep.ep_moe(x, par_ep, wts, ids, capacity=wl["capacity"], peer=px)
        ref = ops.fused_moe(x, par_full, wts, ids)
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        rel, net = gate_stats(got, ref)
        rel, net = over_ranks(rel, world, dev), over_ranks(net, world, dev)
        parity[name] = {"rel_l2": rel, "net_maxabs": net, "ok": bool(rel <= 5e-3 and net <= 2e-2),
                        "exchange": "peer memory" if px is not None else "NCCL"}

    def load_balance(entry, name):
        """Mean over max of the routed rows each rank owns in this layer (all ranks' tokens): the most that the
        expert-compute side of a contiguous expert split lets the ranks reach of ideal scaling."""
        ids = entry["route"][name][0].to(torch.int32)
        allids = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(allids, ids)
        g = torch.cat([t.reshape(-1) for t in allids]).long()
        rows = torch.bincount(g[(g >= 0) & (g < E)] // (E // world), minlength=world).double()
        return float(rows.mean() / rows.max().clamp_min(1))

    def local_touched_bytes(entry, name):
        """Bytes of this rank's experts that any rank's tokens touch in this layer (each streamed once by its
        owner), plus this rank's x, output and routing."""
        L = entry["layer"]
        ids = entry["route"][name][0].to(torch.int32)
        allids = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(allids, ids)
        g = torch.cat([t.reshape(-1) for t in allids]).long()
        loc = g[(g >= L.lo) & (g < L.hi)] - L.lo
        touched = torch.unique(loc)
        m = ids.shape[0]
        return int(L.prep.expert_bytes().to(dev)[touched].sum()) + m * H * 2 * 2 + m * TOPK * 8

    results = {}
    for name in names:
        wl = EP_WORKLOADS[name]
        m = ep_tokens(name, world)

        # fixed-capacity workloads exchange over peer memory (CUDA IPC blocks, this build's kernels) unless asked
        # for NCCL; exact-count workloads use NCCL all-to-allv
        px = ep.PeerExchange(None, m, H, TOPK, dev) if wl["capacity"] and a.ep_exchange == "peer" else None

        def step(be=None, name=name, wl=wl, px=px):
            for e in layers:
                ids, wts = e["route"][name]
                ep.ep_moe(e["x"][name], e["layer"], wts, ids, backend=be, capacity=wl["capacity"], peer=px)

        check_parity(name, wl, px)

        for _ in range(max(3, a.warmup)):
            step()
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        run, how = step, "eager (exact-count exchange synchronises the host every layer)"
        if wl["capacity"]:  # no host synchronisation: the whole step, NCCL included, as one CUDA graph
            graph, err = None, None
            try:
                graph = make_graph(step, 1)
            except Exception as exc:  # every rank must take the same path: agree before timing
                err = f"{type(exc).__name__}: {str(exc)[:120]}"
            ok = torch.tensor([0 if err else 1], dtype=torch.int32, device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if int(ok) == 1:
                run, how = graph.replay, "one CUDA graph per step (NCCL all-to-alls captured)"
            else:
                how = f"eager (graph capture failed on a rank: {err})"
        clocks = Clocks(dev)
        ms = over_ranks(timed(run, a.steps, barrier), world, dev)
        clk = clocks.stop()
        if wl["unit"] == "GB/s":
            amount = over_ranks(sum(local_touched_bytes(e, name) for e in layers) / 1e9, world, dev, op="sum")
        else:
            amount = world * len(layers) * m * TOPK * FLOPS_PER_ROW / 1e12
        res = {"workload": wl["desc"], "value": round(amount / (ms / 1e3), 3), "unit": wl["unit"],
               "tokens_per_gpu": m, "ms_per_step": round(ms, 4), "us_per_layer": round(ms * 1e3 / len(layers), 2),
               "load_balance_ceiling": round(sum(load_balance(e, name) for e in layers) / len(layers), 4),
               "clocks": clk,
               "launch": how}
        # the local kernels on the rows one step delivered, replayed alone (this rank): the whole-layer kernel when
        # the received batch is a decode batch, else the tcgen05 gate_up GEMM
        rec = []
        step(ep.CudaBackend(record=rec))
        torch.cuda.synchronize()
        be = ep.CudaBackend()
        launches = ops.record_launches(lambda: [be.local(xr, mr, e["layer"], TOPK, ms)
                                                for (xr, mr, ms), e in zip(rec, layers)])
        kind = "layer" if any(n == "layer" for n, _ in launches) else "gate_gemm"
        fns = [f for n, f in launches if n == kind]
        kus = 0.0
        if fns:
            g = make_graph(lambda: [f() for f in fns], 2)
            kus = timed(g.replay, a.steps, lambda: None) * 1e3 / len(fns)
            del g
        kus = over_ranks(kus, world, dev)  # every rank takes part, whatever it launched
        roof = None
        if fns and kus > 0:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
                os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
            if wl["unit"] == "GB/s":
                gb = []
                for (xr, mr, _), e in zip(rec, layers):
                    lid = mr[:, :TOPK]
                    valid = lid[(lid >= 0) & (lid < e["layer"].local_experts)]
                    if valid.numel():
                        r = int(xr.shape[0])
                        gb.append(touched_bytes(e["layer"].prep, valid, r)[0] if kind == "layer"
                                  else gate_bytes(e["layer"].prep, valid, r))
                gbpl = sum(gb) / max(1, len(gb))
                peak = peaks.get("hbm_gbs", 6650.0)
                ach = gbpl / (kus / 1e6) / 1e9
                roof = {"kernel": "moek_layer_kernel (the local experts' whole layer on the received rows; timed "
                                  "alone, writing the fp32 rows locally)"
                        if kind == "layer" else "moek_prefill_kernel (gate_up of the local experts on the received rows)",
                        "bound": "hbm", "achieved": round(ach, 1), "peak": peak,
                        "peak_source": "of measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks
                        else "of fallback", "unit": "GB/s", "frac": round(ach / peak, 4), "traffic": None,
                        "bytes_per_launch": int(gbpl), "avg_launch_us": round(kus, 2), "rank": "max over ranks"}
            else:
                rows = sum(int(((mr[:, :TOPK] >= 0) & (mr[:, :TOPK] < e["layer"].local_experts)).sum())
                           for (xr, mr, _), e in zip(rec, layers)) / len(layers)
                flops = rows * 2 * H * 2 * I
                peak = peaks.get("bf16_tflops_sustained", 1400.0)
                ach = flops / (kus / 1e6) / 1e12
                roof = {"kernel": "moek_prefill_kernel (gate_up of the local experts on the received rows)",
                        "bound": "tensor", "achieved": round(ach, 1), "peak": peak,
                        "peak_source": "of measured sustained (MEASURED_PEAKS.json bf16_tflops_sustained)"
                        if "bf16_tflops_sustained" in peaks else "of fallback", "unit": "TFLOP/s",
                        "frac": round(ach / peak, 4), "traffic": None, "flops_per_launch": int(flops),
                        "avg_launch_us": round(kus, 2), "rank": "this rank's gate launches, max over ranks"}
        res["roofline"] = roof
        del rec
        rows_local = world * m if wl["capacity"] else m  # received rows per rank (exact counts: about m)
        local = ops.launches_per_layer(rows_local, TOPK) - (0 if ops._decode_path(rows_local, TOPK) else 1)
        fused = px is not None and ops.layer_p2p_fits(rows_local, TOPK)
        one_launch = fused and os.environ.get("MOEK_B200_EP_FUSED", "1") != "0"
        if fused:  # the whole-layer kernel dispatching and unpacking itself, or dispatch, that kernel, unpack
            per_layer = 1 if one_launch else 3
        else:  # plan + pack or dispatch + wait, the local layer's kernels (no top-k sum), partial or combine, unpack
            per_layer = 4 + local
        res["gpu_launches_per_step"] = per_layer * len(layers)
        if name == names[0]:
            # e2e: inputs copied from pinned host memory and the outputs read back, every layer, every step
            # the step's inputs as on one GPU: one pinned block, copied in two on a copy stream (the first layer's,
            # then the others' while the first computes)
            packed = [pack_inputs(e["x"][name], *e["route"][name]) for e in layers]
            seg = (packed[0].numel() + 15) // 16 * 16
            hall = torch.zeros((len(layers), seg), dtype=torch.uint8).pin_memory()
            for l, t in enumerate(packed):
                hall[l, :t.numel()].copy_(t)
            hout = [torch.empty((m, H), dtype=torch.bfloat16).pin_memory() for _ in layers]
            dall = torch.empty_like(hall, device=dev)
            din = [dall[l, :t.numel()] for l, t in enumerate(packed)]
            copy_stream = torch.cuda.Stream(dev)
            copied = [torch.cuda.Event() for _ in range(2)]

            def e2e_step():
                cur = torch.cuda.current_stream(dev)
                copy_stream.wait_stream(cur)
                with torch.cuda.stream(copy_stream):
                    dall[:1].copy_(hall[:1], non_blocking=True)
                    copied[0].record(copy_stream)
                    dall[1:].copy_(hall[1:], non_blocking=True)
                    copied[1].record(copy_stream)
                for l, e in enumerate(layers):
                    if l < 2:
                        cur.wait_event(copied[l])
                    dx, did, dw = unpack_inputs(din[l], m)
                    o = ep.ep_moe(dx, e["layer"], dw, did, capacity=wl["capacity"], peer=px)
                    hout[l].copy_(o, non_blocking=True)

            e2e_step()
            ems = over_ranks(timed(e2e_step, a.steps, barrier), world, dev)
            res["e2e"] = {"value": round(amount / (ems / 1e3), 3), "unit": wl["unit"],
                          "h2d_bytes_per_step": hall.numel(),
                          "d2h_bytes_per_step": sum(o.numel() * 2 for o in hout), "ms_per_step": round(ems, 4),
                          "api": "ep.ep_moe with host copies (per rank: the inputs in two copies on a copy stream, "
                                 "each layer's output back after it; value over all ranks)"}
        res["exchange"] = ("peer memory (CUDA IPC; " + (
            "one whole-layer launch: dispatch, layer, partials over NVLink, unpack)" if one_launch else
            "dispatch, whole-layer kernel returning the partials, unpack)" if fused else "dispatch / combine kernels)")
            if px is not None else "NCCL")
        if px is not None:
            px.close()
        results[name] = res
    head = results.pop(names[0])
    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world, "steps": a.steps,
            "warmup": max(3, a.warmup), "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": EP_WORKLOADS[names[0]]["desc"], "layers_per_step": a.layers, "experts": E,
                       "hidden": H, "inter": I, "top_k": TOPK, "tokens_per_gpu": EP_WORKLOADS[names[0]]["m"],
                       "weights": "NVFP4 (E2M1 + E4M3/16 + fp32 global), bf16 activations",
                       "l2": f"{a.layers} distinct layers per step rotate; touched weights >> 126 MB L2",
                       "parallelism": f"ep{world}: experts split contiguously, tokens per rank, "
                                      f"{head['exchange']} exchange"},
            "us_per_layer": head["us_per_layer"], "roofline": head["roofline"], "cpu_baseline": None,
            "e2e": head["e2e"], "clocks": head["clocks"],
            "gpu_launches": head["gpu_launches_per_step"] * a.steps, "launch": head["launch"], "workloads": results,
            "parity": {"vs": "ops.fused_moe on one GPU holding all 512 experts, the same tokens (every rank its own; "
                             "worst rank)", "gate": "rel-L2 <= 5e-3, net max-abs <= 2e-2 * rms",
                       "ok": all(v["ok"] for v in parity.values()), "workloads": parity},
        }
        print(json.dumps(line), flush=True)
    if not all(v["ok"] for v in parity.values()):
        raise SystemExit(f"expert-parallel output outside the parity gate: {parity}")


def reference_arm(a, rank, world):
    """The reference's fp32 CPU oracle on the host cores (rank 0 only), a bounded sample of the workload per step."""
    if rank != 0:
        return
    import torch

    from oracle import moe_ref
    from qwen38_flash_coder_b200 import prep, synth

    torch.set_num_threads(os.cpu_count())
    wl = WORKLOADS[a.workload]
    m = min(wl["m"], 256)
    ids, wts = route(m, 0, wl["route"], "cpu")
    touched = torch.unique(ids.long())
    remap = torch.full((E,), -1, dtype=torch.long)
    remap[touched] = torch.arange(touched.numel())
    nt = touched.numel()
    w13 = synth.make_experts(nt, 2 * I, H, 0)
    w2 = synth.make_experts(nt, H, I, 1)
    to_np = lambda mm: (mm[0].numpy(), mm[1].view(torch.uint8).numpy(), mm[2].numpy())
    c13, c2 = to_np(w13), to_np(w2)
    if wl["unit"] == "GB/s":
        amount = (int(prep.PreparedLayer(w13, w2).expert_bytes().sum()) + m * H * 4 + m * TOPK * 8) / 1e9
    else:
        amount = m * TOPK * FLOPS_PER_ROW / 1e12
    x = synth.activations(m, H, 0)
    cid = remap[ids.long()].numpy()
    times = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        moe_ref.reference(x, cid, wts.numpy(), c13, c2)
        if i >= a.warmup:
            times.append(time.perf_counter() - t0)
    s = statistics.median(times)
    v = amount / s
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 6), "unit": wl["unit"], "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(s * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": wl["desc"], "experts": E, "hidden": H, "inter": I, "top_k": TOPK, "tokens": m},
        "cpu_baseline": {"value": round(v, 6), "unit": wl["unit"], "cores": os.cpu_count(), "kind": "port",
                         "sample": f"one layer of {m} tokens ({nt} touched experts) per step, the fp32 "
                                   "dequantise-then-matmul oracle (oracle/moe_ref.py), all host threads"},
        "e2e": {"value": round(v, 6), "unit": wl["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
        flush=True)


if __name__ == "__main__":
    main()
