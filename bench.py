"""Benchmark of the routed-expert NVFP4 (W4A16) MoE layer on B200.

Default workload (the one the headline metric is quoted on): a decode verify step, M = 8 tokens per
GPU, 512 experts, hidden 2048, expert intermediate 512, top-5, uniform routing (softmax of N(0,1) logits -> top-5 ->
renormalise); 48 layers with independent seeded NVFP4 weights (bf16 N(0, 0.02) quantised, 857 MB per layer, 41 GB
in HBM). A step runs the 48 layers back to back; the weights the 48 layers touch (~3 GB) far exceed the 126 MB L2, so
every layer streams its experts from HBM (the rotation is the L2 flush). Other workloads: --workload decode32
(config 3: M=32, Zipf(1.1)), --workload prefill (config 4: M=6912, one layer per step, 48 rotating layers).

value = algorithmic HBM bytes per second over all GPUs (touched experts' packed weights + packed scales + exception
lists + x + output + routing, SURVEY 8(d) formula); e2e = the same metric through the public API with the step's
inputs copied from pinned host memory and the outputs read back inside the timed region.

--impl reference times the reference's CPU restatement (the fp32 dequantise-then-matmul oracle of
bench/moek/problem.py:51-67, oracle/moe_ref.py) on the host cores, same metric and unit, a bounded sample per step.
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode8", choices=["decode8", "decode32", "prefill"])
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def workload(name):
    if name == "decode8":
        return dict(m=8, route="uniform", desc="decode verify M=8 (1 stream x block 8), uniform routing")
    if name == "decode32":
        return dict(m=32, route="zipf", desc="multi-stream decode M=32 (4 x 8), Zipf(1.1) routing")
    return dict(m=6912, route="uniform", desc="prefill chunk M=6912, uniform routing")


def route(m, seed, kind, device):
    from qwen38_flash_coder_b200 import synth

    if kind == "zipf":
        return synth.route_zipf(m, E, TOPK, seed, device=device)
    return synth.route_softmax(m, E, TOPK, seed, device=device)


def layer_bytes(layer, ids, m):
    """Algorithmic bytes of one layer call: touched experts' streamed bytes + x + out + routing."""
    import torch

    touched = torch.unique(ids.long())
    per = layer.expert_bytes().to(ids.device)
    return int(per[touched].sum()) + m * H * 2 * 2 + m * TOPK * 8, int(touched.numel())


def gate_bytes(layer, ids, m):
    import torch

    touched = torch.unique(ids.long()).cpu()
    w = layer.w13
    nkeys = (w.exc_off.numel() - 1) // w.E
    off = w.exc_off.to(torch.int64).cpu()
    n_exc = off[(touched + 1) * nkeys] - off[touched * nkeys]
    per = w.w[0].numel() * 4 + w.sp[0].numel() + 4 * (nkeys + 1)
    return int(touched.numel() * per + 4 * n_exc.sum()) + m * H * 2


class Clocks:
    """nvidia-smi samples during the timed region (started before, stopped after)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}", "--format=csv,noheader",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait(timeout=10)
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1].split()[0]))
                mx = float(c[2].split()[0])
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if "Active" in v and "Not" not in v:
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def cpu_baseline(layers, xs, routes, budget_s=12.0):
    """The oracle (fp32 dequantise-then-matmul, torch CPU, all host threads) on whole layers until ~budget_s of
    compute; copying the touched experts to the host is not timed."""
    import torch

    from oracle import moe_ref

    torch.set_num_threads(os.cpu_count())
    done_bytes, tot, n = 0, 0.0, 0
    while n < len(layers) and (tot < budget_s or n == 0):
        (w13, w2, layer), x, (ids, wts) = layers[n], xs[n], routes[n]
        touched = torch.unique(ids.long())
        remap = torch.full((E,), -1, dtype=torch.long, device=ids.device)
        remap[touched] = torch.arange(touched.numel(), device=ids.device)
        cpu = lambda mm: (mm[0][touched].cpu().numpy(), mm[1][touched].view(torch.uint8).cpu().numpy(),
                          mm[2][touched].cpu().numpy())
        c13, c2, cid = cpu(w13), cpu(w2), remap[ids.long()].cpu().numpy()
        xc, wc = x.cpu(), wts.cpu().numpy()
        t1 = time.perf_counter()
        moe_ref.reference(xc, cid, wc, c13, c2)
        tot += time.perf_counter() - t1
        done_bytes += layer_bytes(layer, ids, x.shape[0])[0]
        n += 1
    return {"value": round(done_bytes / tot / 1e9, 4), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} layer(s) of the same workload (M={xs[0].shape[0]}, touched experts only), "
                      f"torch-CPU oracle (oracle/moe_ref.py), {tot:.1f} s of compute"}


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


def main():
    a = parse()
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    wl = workload(a.workload)
    if a.impl == "reference":
        return reference_arm(a, wl, rank, world)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from qwen38_flash_coder_b200 import ops, prep, synth

    m = wl["m"]
    nl = a.layers
    layers, xs, routes = [], [], []
    for l in range(nl):
        seed = 1000 * rank + l
        w13, w2 = synth.make_layer(E, H, I, l, device=dev)
        keep = l < 3  # checkpoint tensors only for the layers the CPU baseline may sample
        layers.append((w13 if keep else None, w2 if keep else None, prep.PreparedLayer(w13, w2)))
        del w13, w2
        xs.append(synth.activations(m, H, seed, device=dev))
        routes.append(route(m, seed, wl["route"], dev))
    outs = [torch.empty((m, H), dtype=torch.bfloat16, device=dev) for _ in range(nl)]
    per_layer = [layer_bytes(layers[l][2], routes[l][0], m) for l in range(nl)]
    step_bytes = sum(b for b, _ in per_layer)

    def step():
        for l in range(nl):
            ops.fused_moe(xs[l], layers[l][2], routes[l][1], routes[l][0], output=outs[l])

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    graph = make_graph(step, a.warmup)
    ops.check_device_errors(dev)
    clocks = Clocks(local)
    ms = timed(graph.replay, a.steps, barrier)
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t)
        sb = torch.tensor([step_bytes], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(sb)
        total_bytes = float(sb)
    else:
        total_bytes = step_bytes
    value = total_bytes / (ms / 1e3) / 1e9

    # --- roofline of the dominant kernel (the gate_up grouped GEMM): a graph of the step's gate_up launches alone,
    # CUDA events on the stream that replays it
    rec = ops.record_launches(step)
    kern_us = {}
    for name in ("gate_gemm", "down_gemm"):
        fns = [f for n, f in rec if n == name]
        g = make_graph(lambda: [f() for f in fns], 2)
        kern_us[name] = timed(g.replay, a.steps, barrier) * 1e3 / len(fns)
        del g
    gb = sum(gate_bytes(layers[l][2], routes[l][0], m) for l in range(nl)) / nl
    peaks = {}
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        peaks = json.load(open(pp))
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = gb / (kern_us["gate_gemm"] / 1e6) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        traffic = json.load(open(tp)).get(f"gate_gemm_{a.workload}")
    roof = {"kernel": "moek_decode_kernel (gate_up)", "bound": "hbm", "achieved": round(achieved, 1),
            "peak": peak, "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks
            else "fallback 6650", "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
            "bytes_per_launch": int(gb), "avg_launch_us": round(kern_us["gate_gemm"], 2),
            "down_gemm_avg_us": round(kern_us["down_gemm"], 2)}

    # --- e2e: the public API (fused_moe) with each step's inputs copied from pinned host memory and its outputs
    # read back, all inside the timed region (one CUDA graph per step, as vLLM runs decode)
    hx = [x.cpu().pin_memory() for x in xs]
    hid = [r[0].cpu().pin_memory() for r in routes]
    hw = [r[1].cpu().pin_memory() for r in routes]
    hout = [torch.empty((m, H), dtype=torch.bfloat16).pin_memory() for _ in range(nl)]
    dx = [torch.empty_like(x) for x in xs]
    did = [torch.empty_like(r[0]) for r in routes]
    dw = [torch.empty_like(r[1]) for r in routes]

    def e2e_step():
        for l in range(nl):
            dx[l].copy_(hx[l], non_blocking=True)
            did[l].copy_(hid[l], non_blocking=True)
            dw[l].copy_(hw[l], non_blocking=True)
            ops.fused_moe(dx[l], layers[l][2], dw[l], did[l], output=outs[l])
            hout[l].copy_(outs[l], non_blocking=True)

    eg = make_graph(e2e_step, 2)
    ems = timed(eg.replay, a.steps, barrier)
    if world > 1:
        t = torch.tensor([ems], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ems = float(t)
    h2d = sum(x.numel() * 2 + r.numel() * 4 + w.numel() * 4 for x, r, w in zip(hx, hid, hw))
    d2h = sum(o.numel() * 2 for o in hout)
    e2e = {"value": round(total_bytes / (ems / 1e3) / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "ms_per_step": round(ems, 4), "api": "ops.fused_moe, CUDA graph per step"}
    eager_ms = timed(step, max(2, a.steps // 4), barrier)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(layers[:3], xs[:3], routes[:3])
    if world > 1:
        torch.distributed.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": max(3, a.warmup), "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": wl["desc"], "layers_per_step": nl, "experts": E, "hidden": H, "inter": I,
                       "top_k": TOPK, "tokens_per_gpu": m, "weights": "NVFP4 (E2M1 + E4M3/16 + fp32), bf16 acts",
                       "l2": f"{nl} distinct layers per step (~{step_bytes / 1e9:.1f} GB touched) > 126 MB L2",
                       "parallelism": "single GPU" if world == 1 else f"{world} independent replicas"},
            "us_per_layer": round(ms * 1e3 / nl, 2),
            "touched_experts_per_layer": round(sum(t for _, t in per_layer) / nl, 1),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": ops.LAUNCHES_PER_LAYER * nl * a.steps,
            "eager_ms_per_step": round(eager_ms, 4),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def reference_arm(a, wl, rank, world):
    """The reference's fp32 CPU oracle on the host cores (rank 0 only)."""
    if rank != 0:
        return
    import torch

    from qwen38_flash_coder_b200 import prep, synth
    from oracle import moe_ref

    torch.set_num_threads(os.cpu_count())
    m = wl["m"]
    # a bounded sample of the same workload: one layer's touched experts (CPU-generated weights)
    ids, wts = route(m, 0, wl["route"], "cpu")
    touched = torch.unique(ids.long())
    remap = torch.full((E,), -1, dtype=torch.long)
    remap[touched] = torch.arange(touched.numel())
    nt = touched.numel()
    w13 = synth.make_experts(nt, 2 * I, H, 0)
    w2 = synth.make_experts(nt, H, I, 1)
    to_np = lambda mm: (mm[0].numpy(), mm[1].view(torch.uint8).numpy(), mm[2].numpy())
    c13, c2 = to_np(w13), to_np(w2)
    layer = prep.PreparedLayer(w13, w2)
    nbytes = int(layer.expert_bytes().sum()) + m * H * 4 + m * TOPK * 8
    x = synth.activations(m, H, 0)
    cid = remap[ids.long()].numpy()
    times = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        moe_ref.reference(x, cid, wts.numpy(), c13, c2)
        if i >= a.warmup:
            times.append(time.perf_counter() - t0)
    s = statistics.median(times)
    v = nbytes / s / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(s * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": wl["desc"], "experts": E, "hidden": H, "inter": I, "top_k": TOPK, "tokens": m},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"one layer (M={m}, {nt} touched experts) per step, fp32 dequantise-then-matmul"},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
        flush=True)


if __name__ == "__main__":
    main()
