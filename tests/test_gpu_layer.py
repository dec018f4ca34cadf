"""The whole-layer decode kernel (moek_moe_layer) on the GPU: against the CPU oracle for batch sizes, k-split
settings, unrouted slots and the fp32 row output; and repeated calls across layer geometries, which exercise the
kernel's self-resetting counters and epoch-stamped ready flags (every call must give the same bits)."""
import numpy as np
import pytest
import torch

from oracle import moe_ref
from qwen38_flash_coder_b200 import ops, prep, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ckpt(mat):
    codes, scales, gs = mat
    return codes.cpu().numpy(), scales.view(torch.uint8).cpu().numpy(), gs.cpu().numpy()


def _oracle(w13, w2, x, ids, wts):
    return moe_ref.reference(x.cpu(), ids.cpu().numpy(), wts.cpu().numpy(), _ckpt(w13), _ckpt(w2))


@pytest.mark.parametrize("splits", ["1,1", "4,2", "16,4", "2,1", "8,2"])
@pytest.mark.parametrize("m,route,e", [(1, "u", 64), (8, "u", 64), (13, "z", 64), (32, "z", 64), (2, "u", 8),
                                       (64, "z", 512)])
def test_layer_kernel_vs_oracle(monkeypatch, splits, m, route, e):
    monkeypatch.setenv("MOEK_B200_LAYER_SPLITS", splits)
    w13, w2 = synth.make_layer(e, 2048, 512, m, device=DEV)
    x = synth.activations(m, 2048, m, device=DEV)
    ids, wts = (synth.route_softmax if route == "u" else synth.route_zipf)(m, e, 5, m, device=DEV)
    out = ops.fused_moe(x, prep.PreparedLayer(w13, w2), wts, ids)
    ops.check_device_errors(DEV)
    ok, stats = moe_ref.within_gate(out.cpu(), _oracle(w13, w2, x, ids, wts))
    assert ok, stats


def test_layer_kernel_unrouted_slots():
    """Ids outside [0, E) are not routed; a token whose slots are all unrouted gets a zero row."""
    w13, w2 = synth.make_layer(64, 2048, 512, 3, device=DEV)
    m = 12
    x = synth.activations(m, 2048, 3, device=DEV)
    ids, wts = synth.route_softmax(m, 64, 5, 3, device=DEV)
    ids = ids.clone()
    ids[1, 2] = -1
    ids[4, 0] = 64 + 7
    ids[7, :] = -1  # nothing routed for token 7
    out = ops.fused_moe(x, prep.PreparedLayer(w13, w2), wts, ids)
    ops.check_device_errors(DEV)
    assert torch.count_nonzero(out[7]) == 0
    ok, stats = moe_ref.within_gate(out.cpu(), _oracle(w13, w2, x, ids, wts))
    assert ok, stats


def test_layer_kernel_rows_output():
    """moe_rows through the whole-layer kernel: the fp32 weighted slot rows, before the top-k sum."""
    w13, w2 = synth.make_layer(64, 2048, 512, 4, device=DEV)
    m = 9
    x = synth.activations(m, 2048, 4, device=DEV)
    ids, wts = synth.route_zipf(m, 64, 5, 4, device=DEV)
    rows = ops.moe_rows(x, prep.PreparedLayer(w13, w2), wts, ids)
    ops.check_device_errors(DEV)
    ref = moe_ref.slot_rows(x.cpu(), ids.cpu().numpy(), wts.cpu().numpy(), _ckpt(w13), _ckpt(w2))
    rel = float((rows.cpu() - ref).norm() / ref.norm())
    assert rel < 5e-3, rel


def test_layer_kernel_repeat_across_geometries():
    """Alternating geometries and batch sizes on one stream: each call's result is bit-identical to its first run."""
    layers = [prep.PreparedLayer(*synth.make_layer(e, 2048, 512, e, device=DEV)) for e in (64, 512)]
    cases = []
    for li, e in enumerate((64, 512)):
        for m in (3, 8, 40):
            x = synth.activations(m, 2048, 100 + m, device=DEV)
            ids, wts = synth.route_zipf(m, e, 5, 100 + m, device=DEV)
            cases.append((layers[li], x, ids, wts))
    first = [ops.fused_moe(c[1], c[0], c[3], c[2]) for c in cases]
    for _ in range(3):
        for c, f in zip(cases, first):
            assert torch.equal(ops.fused_moe(c[1], c[0], c[3], c[2]), f)
    ops.check_device_errors(DEV)


def test_layer_kernel_matches_split_path(monkeypatch):
    """The whole-layer kernel and the separate split-k launches (moek_gemm mode 2 + epilogues) agree."""
    w13, w2 = synth.make_layer(512, 2048, 512, 6, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    x = synth.activations(32, 2048, 6, device=DEV)
    ids, wts = synth.route_zipf(32, 512, 5, 6, device=DEV)
    a = ops.fused_moe(x, layer, wts, ids)
    monkeypatch.setenv("MOEK_B200_DECODE_PATH", "split")
    b = ops.fused_moe(x, layer, wts, ids)
    ops.check_device_errors(DEV)
    rel = float((a.float() - b.float()).norm() / b.float().norm())
    assert rel < 1e-3, rel
    assert np.isfinite(a.float().cpu().numpy()).all()


@pytest.mark.parametrize("m,e", [(32, 8), (96, 64), (40, 512)])
def test_layer_kernel_sub_blocks(monkeypatch, m, e):
    """Experts with more routed slots than a block holds are cut into several blocks: every block size (8, 16, 32
    rows) gives a result within the gate of the oracle (8 experts: about 20 slots per expert at M = 32), the same
    bits on a repeated call, and results that agree with each other to fp32 summation order (the number of blocks
    sets how many CTAs share a gate_up item, which changes only the order of its fp32 partial sums)."""
    from qwen38_flash_coder_b200 import _lib

    monkeypatch.setattr(ops, "DECODE_MAX_M", 128)  # the whole-layer kernel up to 102 tokens of 5 slots
    w13, w2 = synth.make_layer(e, 2048, 512, 50 + m, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    x = synth.activations(m, 2048, 50 + m, device=DEV)
    ids, wts = synth.route_zipf(m, e, 5, 50 + m, device=DEV)
    outs, again = [], []
    try:
        for rows in (8, 16, 32):
            _lib.call("moek_set_layer_block_rows", rows)
            outs.append(ops.fused_moe(x, layer, wts, ids))
            again.append(ops.fused_moe(x, layer, wts, ids))
        ops.check_device_errors(DEV)
    finally:
        _lib.call("moek_set_layer_block_rows", 0)
    assert all(torch.equal(o, a) for o, a in zip(outs, again))
    for o in outs[1:]:
        rel, _, _ = moe_ref.check(o.cpu(), outs[0].float().cpu())
        assert rel < 2e-3, rel
    ref = _oracle(w13, w2, x, ids, wts)
    for o in outs:
        ok, stats = moe_ref.within_gate(o.cpu(), ref)
        assert ok, stats


def test_layer_kernel_beside_other_streams():
    """The whole-layer kernel's CTAs wait on one another, so it is launched as a cooperative grid: with large GEMMs
    occupying the GPU from another stream, every call still completes within the default 2 s wait bound and gives the
    same bits as a call on an idle GPU."""
    w13, w2 = synth.make_layer(64, 2048, 512, 31, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    m = 8
    x = synth.activations(m, 2048, 31, device=DEV)
    ids, wts = synth.route_softmax(m, 64, 5, 31, device=DEV)
    ref = ops.fused_moe(x, layer, wts, ids)
    torch.cuda.synchronize()
    a = torch.randn((8192, 8192), device=DEV, dtype=torch.bfloat16)
    side, main = torch.cuda.Stream(), torch.cuda.Stream()
    outs = []
    with torch.cuda.stream(side):
        for _ in range(8):
            a = a @ a
            a = a / a.abs().amax().clamp_min(1.0)
    with torch.cuda.stream(main):
        for _ in range(20):
            outs.append(ops.fused_moe(x, layer, wts, ids))
    torch.cuda.synchronize()
    ops.check_device_errors(DEV)
    for o in outs:
        assert torch.equal(o, ref)
