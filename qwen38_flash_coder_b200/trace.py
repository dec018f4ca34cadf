"""Per-CTA timeline of one layer from the MOEK_TRACE build (``libmoek_b200_trace.so``).

    MOEK_B200_LIB=trace python -m qwen38_flash_coder_b200.trace [decode8|decode32|prefill] [--layers N]
    MOEK_B200_LIB=trace torchrun --nproc-per-node N -m qwen38_flash_coder_b200.trace ep_decode8

The ``ep_decode8`` form runs the expert-parallel decode layer (M = 8 tokens per rank, peer-memory exchange) on N
ranks and prints, per rank, the dispatch, whole-layer and unpack kernels' stamps of one layer call on one time axis
(the rank's %globaltimer): when each kernel started, when its cross-GPU waits ended and when it finished.

runs the benchmark's layer geometry (E = 512, hidden 2048, expert intermediate 512, top-5; seeded NVFP4 weights and
routing as bench.py) through ``ops.fused_moe`` eagerly, then reads the %globaltimer stamps of the last launch
(``moek_trace_read``; the stamp slots are listed in include/moek_b200.h) and prints, in microseconds from the
earliest CTA start, the median and maximum over CTAs of every phase, and per unit ordinal the stamps of the units'
first ready stage, last stage and end. The stamps are written by the kernels themselves, so the times are those of
a plain launch (no profiler replay).
"""
import argparse
import ctypes
import json
import os
import statistics

import numpy as np

CTAS, SLOTS = 1024, 128
CLOCK_GHZ = 1.965  # SM clock the cycle stamps are converted at (the B200's maximum, the clock the bench runs at)

LAYER_PHASES = {0: "start", 1: "after dependent-launch wait", 2: "EP flags seen", 3: "routing done",
                4: "first weight copy issued", 5: "consumers done", 47: "every role done (barrier arrival)",
                51: "grid barrier passed",
                52: "top-k sums written", 6: "end"}
GEMM_PHASES = {0: "start", 1: "after dependent-launch wait", 6: "end"}


def read(kind: int) -> np.ndarray:
    from ._lib import call

    buf = np.zeros((CTAS, SLOTS), dtype=np.uint64)
    call("moek_trace_read", kind, buf.ctypes.data_as(ctypes.c_void_p), buf.nbytes)
    return buf


def clear() -> None:
    from ._lib import call

    call("moek_trace_clear")


def summarize(t: np.ndarray, kind: int) -> dict:
    """Times in us relative to the earliest start stamp: per phase (median, max over CTAs); per unit ordinal u:
    (median, max) of its first-ready / last-stage / end stamps; act waits (median, max duration)."""
    live = t[:, 0] > 0
    t = t[live].astype(np.int64)
    t0 = t[:, 0].min()
    us = lambda v: (v - t0) / 1e3
    out = {"ctas": int(live.sum()), "phases": {}, "units": []}
    for slot, name in (LAYER_PHASES if kind == 0 else GEMM_PHASES).items():
        v = t[:, slot]
        v = v[v > 0]
        if v.size:
            out["phases"][name] = (round(float(np.median(us(v))), 2), round(float(us(v).max()), 2))
    nunit = 8 if kind == 0 else 16
    for u in range(nunit):
        cols = [t[:, 8 + 3 * u + j] for j in range(3)]
        have = cols[0] > 0
        if not have.any():
            break
        row = []
        for c in cols:
            c = c[have & (c > 0)]
            row.append((round(float(np.median(us(c))), 2), round(float(us(c).max()), 2)) if c.size else None)
        out["units"].append({"unit": u, "ctas": int(have.sum()), "first_ready": row[0], "last_stage": row[1],
                             "end": row[2]})
    if kind == 0:
        out["units_per_cta"] = (int(np.median(t[:, 7])), int(t[:, 7].max()))
        stages = []  # the first unit's stages, SM cycles relative to consumer warp 0's wait for stage 0
        base = t[:, 64]
        for s_ in range(8):
            cols = {k: t[:, off + s_] for k, off in (("begin", 64), ("scales", 80), ("done", 88),
                                                    ("scale_warp_in", 96), ("scale_warp_out", 104),
                                                    ("producer_issue", 112), ("act_issue", 120))}
            ok = (cols["begin"] > 0) & (cols["done"] > 0) & (base > 0)
            if not ok.any():
                break
            med = lambda v: round(float(np.median(v)) / CLOCK_GHZ / 1e3, 2)
            row = {"stage": s_, "ctas": int(ok.sum())}
            for k_, v in cols.items():
                okk = ok & (v > 0)
                row[k_] = med(v[okk] - base[okk]) if okk.any() else None
            stages.append(row)
        out["unit0_stages"] = stages
        # routing, SM cycles from the dependent-launch wait: keys built, counted, ranked, blocks cut, plans, published
        r0 = t[:, 39]
        rt = {}
        for name, sl in (("keys", 40), ("counted", 41), ("ranked", 42), ("blocks", 43), ("plans", 44), ("published", 45),
                         ("units counted", 53), ("producer: units decoded", 54), ("unit rows published", 55),
                         ("first copy", 112)):
            ok = (r0 > 0) & (t[:, sl] > 0)
            if ok.any():
                rt[name] = round(float(np.median(t[ok, sl] - r0[ok])) / CLOCK_GHZ / 1e3, 2)
        out["routing_us"] = rt
        ends = t[:, 6]
        order = np.argsort(-ends)[:4]
        slow = []
        for ci in order:
            units = []
            for u in range(8):
                if t[ci, 8 + 3 * u] == 0:
                    break
                v = int(t[ci, 32 + u])
                units.append({"unit": f"{'gd'[v >> 28]}/{(v >> 16) & 0xFFF}/{(v >> 8) & 0xFF}/{v & 0xFF}",
                              "ready": float(us(t[ci, 8 + 3 * u])), "end": float(us(t[ci, 10 + 3 * u]))
                              if t[ci, 10 + 3 * u] else float("nan")})
            slow.append({"cta": int(np.nonzero(live)[0][ci]), "end": float(us(ends[ci])), "units": units})
        out["slowest"] = slow
        waits = []
        for j in range(4):
            a, b = t[:, 56 + 2 * j], t[:, 57 + 2 * j]
            ok = (a > 0) & (b > 0)
            waits += list((b[ok] - a[ok]) / 1e3)
        if waits:
            out["act_wait_us"] = (round(statistics.median(waits), 2), round(max(waits), 2), len(waits))
    return out


EP_DISPATCH = {0: "start", 1: "-", 2: "rows written", 3: "flag raised"}


def ep_main(a):
    """The expert-parallel decode layer's kernels on every rank (see the module docstring)."""
    import datetime

    import torch
    import torch.distributed as dist

    from . import ep, ops, synth

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        m, E = 8, 512
        layers = []
        for l in range(a.layers):
            w13, w2 = synth.make_layer(E, 2048, 512, l, device=dev)
            L = ep.EPLayer(ep.shard_checkpoint(w13, E, world, rank), ep.shard_checkpoint(w2, E, world, rank), E,
                           world, rank)
            x = synth.activations(m, 2048, 1000 * rank + l, device=dev)
            ids, w = synth.route_softmax(m, E, 5, 1000 * rank + l, device=dev)
            layers.append((L, x, ids, w))
            del w13, w2
        px = ep.PeerExchange(None, m, 2048, 5, dev)
        for _ in range(3):
            for L, x, ids, w in layers:
                ep.ep_moe(x, L, w, ids, capacity=True, peer=px)
        torch.cuda.synchronize()
        dist.barrier()
        clear()
        torch.cuda.synchronize()
        dist.barrier()
        for L, x, ids, w in layers:  # the stamps keep the last layer's launches
            ep.ep_moe(x, L, w, ids, capacity=True, peer=px)
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        lay, epk = read(0), read(2)
        px.close()
        res = {"rank": rank}
        live = lay[:, 0] > 0
        d0 = epk[:, 0][epk[:, 0] > 0]
        t0 = int(min(d0.min() if d0.size else 2 ** 63, lay[live, 0].min() if live.any() else 2 ** 63))
        us = lambda v: round((float(v) - t0) / 1e3, 2)
        pick = lambda col: col[col > 0]
        stats = lambda col: (us(np.median(pick(col))), us(pick(col).max())) if pick(col).size else None
        res["dispatch"] = {"start": stats(epk[:, 0]), "rows written": stats(epk[:, 2]), "flag raised": stats(epk[:, 3])}
        res["layer"] = {"start": stats(lay[:, 0]), "flags seen": stats(lay[:, 2]), "routing done": stats(lay[:, 3]),
                        "end": stats(lay[:, 6])}
        res["unpack"] = {"start": stats(epk[:, 8]), "partials ready": stats(epk[:, 9]), "done": stats(epk[:, 10])}
        out = [None] * world
        dist.all_gather_object(out, res)
        if rank == 0:
            if a.json:
                print(json.dumps(out))
            else:
                for r in out:
                    print(f"rank {r['rank']} (us after its first kernel start; median / max over CTAs):")
                    for k in ("dispatch", "layer", "unpack"):
                        print(f"  {k:<9s} " + "; ".join(f"{n} {v[0]}/{v[1]}" for n, v in r[k].items() if v))
    finally:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("workload", nargs="?", default="decode8", choices=["decode8", "decode32", "prefill",
                                                                       "ep_decode8"])
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--dump", default=None, help="also save every layer's raw stamps [CTA][slot] to this .npy file")
    a = ap.parse_args()
    os.environ.setdefault("MOEK_B200_LIB", "trace")
    import torch

    from . import ops, prep, synth
    from ._lib import lib

    if not lib().moek_build_flags() & 1:
        raise SystemExit("moek_b200: load the trace build (MOEK_B200_LIB=trace)")
    if a.workload == "ep_decode8":
        return ep_main(a)
    m, kind = {"decode8": (8, "u"), "decode32": (32, "z"), "prefill": (6912, "u")}[a.workload]
    dev = torch.device("cuda", 0)
    layers = []
    for l in range(a.layers):
        w13, w2 = synth.make_layer(512, 2048, 512, l, device=dev)
        x = synth.activations(m, 2048, 100 * l, device=dev)
        ids, w = (synth.route_softmax if kind == "u" else synth.route_zipf)(m, 512, 5, 100 * l, device=dev)
        layers.append((prep.PreparedLayer(w13, w2), x, ids, w))
        del w13, w2
    for _ in range(3):
        for L, x, ids, w in layers:
            ops.fused_moe(x, L, w, ids)
    torch.cuda.synchronize()
    res, raw = [], []
    for L, x, ids, w in layers:
        clear()
        torch.cuda.synchronize()
        ops.fused_moe(x, L, w, ids)
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        k = 0 if a.workload != "prefill" else 1
        raw.append(read(k))
        res.append(summarize(raw[-1], k))
    if a.dump:
        np.save(a.dump, np.stack(raw))
    if a.json:
        print(json.dumps(res))
        return
    for i, r in enumerate(res):
        print(f"layer {i}: {r['ctas']} CTAs" + (f", units per CTA median {r['units_per_cta'][0]} max "
                                                 f"{r['units_per_cta'][1]}" if "units_per_cta" in r else ""))
        for name, (med, mx) in r["phases"].items():
            print(f"  {name:<28s} median {med:8.2f} us  max {mx:8.2f} us")
        for u in r["units"]:
            f = lambda v: f"{v[0]:7.2f}/{v[1]:7.2f}" if v else "      -"
            print(f"  unit {u['unit']:2d} ({u['ctas']:4d} CTAs): first ready {f(u['first_ready'])}  last stage "
                  f"{f(u['last_stage'])}  end {f(u['end'])}  (median/max us)")
        if r.get("unit0_stages"):
            keys = ["begin", "scales", "done", "scale_warp_in", "scale_warp_out", "producer_issue",
                    "act_issue"]
            print("  first unit, per stage (us after consumer warp 0 began waiting for stage 0; median over CTAs):")
            print("    stage " + " ".join(f"{k:>14s}" for k in keys))
            for s_ in r["unit0_stages"]:
                print(f"    {s_['stage']:5d} " + " ".join(f"{(s_[k] if s_[k] is not None else float('nan')):14.2f}"
                                                      for k in keys))
        if r.get("routing_us"):
            print("  routing (us after the dependent-launch wait, median): " +
                  ", ".join(f"{k} {v}" for k, v in r["routing_us"].items()))
        slow = r.get("slowest")
        if slow:
            print("  slowest CTAs (end us; units as phase/block/item/split: first ready, end):")
            for cta in slow:
                print(f"    CTA {cta['cta']:3d} end {cta['end']:7.2f}: " + "; ".join(
                    f"{u['unit']} {u['ready']:.1f}-{u['end']:.1f}" for u in cta["units"]))
        if "act_wait_us" in r:
            print(f"  act waits: median {r['act_wait_us'][0]} us, max {r['act_wait_us'][1]} us ({r['act_wait_us'][2]})")


if __name__ == "__main__":
    main()
