"""The instrumented library builds on the GPU: the debug-check build (every input index range-checked) and the
trace build (timeline stamps) give the same bits as the product build on valid inputs, record no device error, and
the trace build's stamps are ordered. Each variant runs in its own process (MOEK_B200_LIB selects the library)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys, torch
sys.path.insert(0, {root!r})
from qwen38_flash_coder_b200 import ops, prep, synth
dev = torch.device("cuda", 0)
outs = []
for m, e in ((8, 512), (300, 64)):
    w13, w2 = synth.make_layer(e, 2048, 512, 50 + m, device=dev)
    L = prep.PreparedLayer(w13, w2)
    x = synth.activations(m, 2048, m, device=dev)
    ids, w = synth.route_zipf(m, e, 5, m, device=dev)
    outs.append(ops.fused_moe(x, L, w, ids))
torch.cuda.synchronize()
ops.check_device_errors(dev)
extra = None
if {trace}:
    from qwen38_flash_coder_b200 import trace
    extra = trace.read(0)
torch.save({{"outs": [o.cpu() for o in outs], "trace": None if extra is None else torch.from_numpy(extra.view("int64"))}},
           {path!r})
"""


def _run(variant, path):
    env = dict(os.environ)
    env["MOEK_B200_LIB"] = variant
    code = CHILD.format(root=ROOT, trace=variant == "trace", path=path)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return torch.load(path)


def test_debug_and_trace_builds_match_product(tmp_path):
    from qwen38_flash_coder_b200 import build

    for v in ("", "debug", "trace"):
        if not os.path.exists(build.lib_path(v)):
            pytest.fail(f"library variant {v!r} is not built (python -m qwen38_flash_coder_b200.build --all)")
    base = _run("", str(tmp_path / "base.pt"))
    for v in ("debug", "trace"):
        got = _run(v, str(tmp_path / f"{v}.pt"))
        for a, b in zip(base["outs"], got["outs"]):
            assert torch.equal(a, b), v
    t = got["trace"]  # the trace build's last whole-layer launch (M = 8): start <= routed <= consumers done <= end
    live = t[:, 0] > 0
    assert int(live.sum()) > 0
    t = t[live]
    assert bool((t[:, 3] >= t[:, 0]).all() and (t[:, 6] >= t[:, 3]).all())
