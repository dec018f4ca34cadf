"""Per-CTA timeline of one layer from the MOEK_TRACE build (``libmoek_b200_trace.so``).

    MOEK_B200_LIB=trace python -m qwen38_flash_coder_b200.trace [decode8|decode32|prefill] [--layers N]

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

LAYER_PHASES = {0: "start", 1: "after dependent-launch wait", 2: "EP flags seen", 3: "routing done",
                4: "first weight copy issued", 5: "consumers done", 6: "end"}
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
    for u in range(16):
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
        stages = []  # the first unit's stages (consumer warp 0): data wait, compute, and when the scale warp got them
        for s in range(16):
            w0, w1, sc, end = t[:, 64 + 2 * s], t[:, 65 + 2 * s], t[:, 96 + s], t[:, 112 + s]
            ok = (w0 > 0) & (w1 > 0) & (end > 0)
            if not ok.any():
                break
            med = lambda v: round(float(np.median(v)) / 1e3, 2)
            sok = ok & (sc > 0)
            stages.append({"stage": s, "ctas": int(ok.sum()), "ready_at": med(w1[ok] - t0),
                           "wait": med(w1[ok] - w0[ok]), "compute": med(end[ok] - w1[ok]),
                           "scale_lead": med(w1[sok] - sc[sok]) if sok.any() else None})
        out["unit0_stages"] = stages
        waits = []
        for j in range(4):
            a, b = t[:, 56 + 2 * j], t[:, 57 + 2 * j]
            ok = (a > 0) & (b > 0)
            waits += list((b[ok] - a[ok]) / 1e3)
        if waits:
            out["act_wait_us"] = (round(statistics.median(waits), 2), round(max(waits), 2), len(waits))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("workload", nargs="?", default="decode8", choices=["decode8", "decode32", "prefill"])
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    os.environ.setdefault("MOEK_B200_LIB", "trace")
    import torch

    from . import ops, prep, synth
    from ._lib import lib

    if not lib().moek_build_flags() & 1:
        raise SystemExit("moek_b200: load the trace build (MOEK_B200_LIB=trace)")
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
    res = []
    for L, x, ids, w in layers:
        clear()
        torch.cuda.synchronize()
        ops.fused_moe(x, L, w, ids)
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        k = 0 if a.workload != "prefill" else 1
        res.append(summarize(read(k), k))
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
        for s in r.get("unit0_stages", []):
            print(f"  unit 0 stage {s['stage']:2d}: ready at {s['ready_at']:7.2f} us (waited {s['wait']:5.2f}), compute "
                  f"{s['compute']:5.2f} us, scale warp had the data {s['scale_lead']} us before (median over CTAs)")
        if "act_wait_us" in r:
            print(f"  act waits: median {r['act_wait_us'][0]} us, max {r['act_wait_us'][1]} us ({r['act_wait_us'][2]})")


if __name__ == "__main__":
    main()
