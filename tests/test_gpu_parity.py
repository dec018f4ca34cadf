"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and the reference's own golden outputs.

Mirrors the reference's GPU checks: layer vs the fp32 oracle (bench/moek/test_cuda.py:41-50), a sweep over sizes and
skews (bench/moek/correct_sweep.py:9-23), bitwise repeat determinism (bench/moek/determinism.py:5-10). The gate is
BASELINE's: rel-L2 <= 5e-3 and max-abs <= 2e-2 * rms against the oracle; routing permutations bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import align as oalign
from oracle import moe_ref
from qwen38_flash_coder_b200 import ops, prep, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"
REL, MAXABS = 5e-3, 2e-2  # rel-L2, and max-abs / rms beyond the bf16 rounding of the output (oracle.moe_ref.check)


def _np(t):
    return t.detach().cpu().numpy()


def _ckpt(mat):
    codes, scales, gs = mat
    return _np(codes), _np(scales.view(torch.uint8)), _np(gs)


def _compact(w13, w2, ids):
    """Checkpoint tensors of the touched experts only (ids remapped), for the CPU oracle."""
    touched = torch.unique(ids.long())
    remap = torch.full((int(w13[0].shape[0]),), -1, dtype=torch.long, device=ids.device)
    remap[touched] = torch.arange(touched.numel(), device=ids.device)
    sub = lambda m: tuple(t[touched] for t in m)
    return _ckpt(sub(w13)), _ckpt(sub(w2)), _np(remap[ids.long()])


def _run_and_check(w13, w2, x, ids, wts, rel_gate=REL, max_gate=MAXABS):
    layer = prep.PreparedLayer(w13, w2)
    out = ops.fused_moe(x, layer, wts, ids)
    ops.check_device_errors(x.device)
    c13, c2, cids = _compact(w13, w2, ids)
    ref = moe_ref.reference(x.cpu(), cids, _np(wts), c13, c2)
    ok, stats = moe_ref.within_gate(out.cpu(), ref, rel_gate, max_gate)
    assert torch.isfinite(out).all()
    assert ok, stats
    return out, layer


# --------------------------------------------------------------------------------------------------- moe_align
@pytest.mark.parametrize("m,e,bs,route", [(1, 512, 96, "u"), (8, 512, 96, "u"), (32, 512, 96, "z"), (6, 8, 4, "u"),
                                          (3, 4, 16, "u"), (300, 64, 96, "z"), (6912, 512, 96, "u"),
                                          (6912, 512, 96, "z"), (2000, 64, 16, "u"), (205, 512, 96, "u")])
def test_align_bit_exact(m, e, bs, route):
    k = 5 if e >= 5 else e
    ids, _ = (synth.route_softmax if route == "u" else synth.route_zipf)(m, e, k, seed=m + e)
    sid, eid, npad = ops.moe_align_block_size(ids.to(DEV), bs, e)
    rs, re_, rn = oalign.moe_align(_np(ids), e, bs)
    assert np.array_equal(_np(sid), rs)
    assert np.array_equal(_np(eid), re_)
    assert int(npad[0]) == int(rn[0])


def test_align_docstring_example(golden):
    ids = torch.from_numpy(golden["align_ids"]).to(DEV)
    sid, eid, npad = ops.moe_align_block_size(ids, 4, 4)
    assert int(npad[0]) == 16 and np.array_equal(_np(sid)[:16], golden["align_sorted"])


def test_align_skips_invalid_ids_and_empty():
    ids = torch.tensor([[0, 7, -1], [9, 3, 0]], dtype=torch.int32)
    sid, eid, npad = ops.moe_align_block_size(ids.to(DEV), 4, 8)
    rs, re_, rn = oalign.moe_align(_np(ids), 8, 4)
    assert np.array_equal(_np(sid), rs) and np.array_equal(_np(eid), re_) and int(npad[0]) == int(rn[0])
    sid, eid, npad = ops.moe_align_block_size(torch.zeros((0, 5), dtype=torch.int32, device=DEV), 96, 512)
    assert sid.numel() == 0 and int(npad[0]) == 0


# ----------------------------------------------------------------------------------------------------- layer
def test_layer_matches_reference_golden(golden):
    """The reference's own oracle output (problem.reference on make_weights' layer: 17 % exception scales)."""
    w13 = tuple(torch.from_numpy(golden[f"mw13_{k}"]).to(DEV) for k in ("codes", "scales", "gs"))
    w2 = tuple(torch.from_numpy(golden[f"mw2_{k}"]).to(DEV) for k in ("codes", "scales", "gs"))
    w13 = (w13[0], w13[1].view(torch.float8_e4m3fn), w13[2])
    w2 = (w2[0], w2[1].view(torch.float8_e4m3fn), w2[2])
    x = torch.from_numpy(golden["moe_x"]).view(torch.bfloat16).to(DEV)
    ids = torch.from_numpy(golden["moe_ids"]).to(DEV)
    wts = torch.from_numpy(golden["moe_wts"]).to(DEV)
    out = ops.fused_moe(x, prep.PreparedLayer(w13, w2), wts, ids)
    ops.check_device_errors(DEV)
    ok, stats = moe_ref.within_gate(out.cpu(), torch.from_numpy(golden["moe_out"]))
    assert ok, stats


def test_config1_cpu_reference_case():
    """E=64, hidden 2048, intermediate 512, top-5, M=8, softmax routing, seed 0."""
    w13, w2 = synth.make_layer(64, 2048, 512, 0, device=DEV)
    x = synth.activations(8, 2048, 0, device=DEV)
    ids, wts = synth.route_softmax(8, 64, 5, 0, device=DEV)
    _run_and_check(w13, w2, x, ids, wts)


@pytest.mark.parametrize("m,route,seed", [(8, "u", 1), (32, "z", 2), (1, "u", 3), (13, "z", 4), (64, "z", 5)])
def test_decode_sizes_512_experts(m, route, seed):
    w13, w2 = synth.make_layer(512, 2048, 512, seed, device=DEV)
    x = synth.activations(m, 2048, seed, device=DEV)
    ids, wts = (synth.route_softmax if route == "u" else synth.route_zipf)(m, 512, 5, seed, device=DEV)
    _run_and_check(w13, w2, x, ids, wts)


@pytest.mark.parametrize("m,e,route", [(65, 64, "u"), (200, 64, "z"), (700, 512, "z"), (2000, 64, "u")])
def test_prefill_path(m, e, route):
    """Batches above the decode threshold run the tcgen05 kernels (moe_align blocks of 128 rows)."""
    w13, w2 = synth.make_layer(e, 2048, 512, 7, device=DEV)
    x = synth.activations(m, 2048, 7, device=DEV)
    ids, wts = (synth.route_softmax if route == "u" else synth.route_zipf)(m, e, 5, 7, device=DEV)
    _run_and_check(w13, w2, x, ids, wts)


@pytest.mark.parametrize("route", ["u", "z"])
def test_prefill_config4_full_size(route):
    """M=6912, 512 experts, uniform and Zipf(1.1) routing, against the oracle on every row."""
    w13, w2 = synth.make_layer(512, 2048, 512, 21, device=DEV)
    x = synth.activations(6912, 2048, 21, device=DEV)
    ids, wts = (synth.route_softmax if route == "u" else synth.route_zipf)(6912, 512, 5, 21, device=DEV)
    _run_and_check(w13, w2, x, ids, wts)


def test_decode_and_prefill_paths_agree(monkeypatch):
    """The same 64-token batch through the split-k mma.sync path and the tcgen05 path."""
    w13, w2 = synth.make_layer(64, 2048, 512, 13, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    x = synth.activations(64, 2048, 13, device=DEV)
    ids, wts = synth.route_zipf(64, 64, 5, 13, device=DEV)
    a = ops.fused_moe(x, layer, wts, ids)
    monkeypatch.setattr(ops, "DECODE_MAX_M", 0)
    b = ops.fused_moe(x, layer, wts, ids)
    ops.check_device_errors(DEV)
    rel = float((a.float() - b.float()).norm() / b.float().norm())
    assert rel < 2e-3, rel


def test_bitwise_repeat():
    w13, w2 = synth.make_layer(64, 2048, 512, 9, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    for m in (8, 100):
        x = synth.activations(m, 2048, m, device=DEV)
        ids, wts = synth.route_zipf(m, 64, 5, m, device=DEV)
        a = ops.fused_moe(x, layer, wts, ids)
        b = ops.fused_moe(x, layer, wts, ids)
        assert torch.equal(a, b)


def test_reference_signature_ops():
    """moe_gemm / moe_split_epilogue with the kit's argument lists, gate_up act vs the oracle's act."""
    w13, w2 = synth.make_layer(16, 2048, 512, 11, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    m, k = 4, 5
    x = synth.activations(m, 2048, 11, device=DEV)
    ids, wts = synth.route_softmax(m, 16, k, 11, device=DEV)
    sid, eid, npad = ops.moe_align_block_size(ids, ops.BM, 16)
    a = layer.w13
    act = torch.empty((m * k, 512), dtype=torch.bfloat16, device=DEV)
    part = torch.empty(4 * m * k * 1024, dtype=torch.float32, device=DEV)
    cnt = torch.zeros(4, dtype=torch.int32, device=DEV)
    ops.moe_gemm(x, a.w, torch.empty(0, device=DEV), a.g, sid, eid, npad, a.g, act, k, True, a.sp, a.exc_off,
                 a.exc_ent, None, cnt, 2, 4, part, 0, True)
    ops.moe_split_epilogue(part, 4, ids, a.g, a.g, act, True, 1024)
    assert int(cnt[0]) == 0
    # oracle act: bf16(silu(h_g) * h_u) with the oracle's bf16 weights
    codes, scales, gs = _ckpt(w13)
    xf = x.float().cpu()
    flat = _np(ids).reshape(-1)
    for r in range(m * k):
        e = int(flat[r])
        wdq = torch.from_numpy(__import__("oracle.nvfp4", fromlist=["x"]).dequant_expert(codes[e], scales[e], gs[e]))
        h = xf[r // k] @ wdq.T
        ref = (torch.nn.functional.silu(h[:512]) * h[512:]).to(torch.bfloat16).float()
        got = act[r].float().cpu()
        assert float((got - ref).norm() / ref.norm()) < 2e-3
    with pytest.raises(ops.MoekError):
        ops.moe_gemm(x, a.w, torch.ones(3, device=DEV), a.g, sid, eid, npad, a.g, act, k, True, a.sp, a.exc_off,
                     a.exc_ent, None, cnt, 2, 4, part, 0, True)
    with pytest.raises(ops.MoekError):  # 5 splits do not cut 16 runs into whole runs
        ops.moe_gemm(x, a.w, None, a.g, sid, eid, npad, a.g, act, k, True, a.sp, a.exc_off, a.exc_ent, None, cnt, 2,
                     5, part, 0, True)


def test_empty_batch():
    w13, w2 = synth.make_layer(8, 2048, 512, 12, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    out = ops.fused_moe(torch.empty((0, 2048), dtype=torch.bfloat16, device=DEV), layer,
                        torch.empty((0, 5), device=DEV), torch.empty((0, 5), dtype=torch.int32, device=DEV))
    assert out.shape == (0, 2048)


@pytest.mark.parametrize("m", [17, 300])
def test_kit_prefill_call_mode0(m):
    """The kit's prefill sequence with its own argument lists (files/mbx_moek.py:266-289, ``split = False``): moe_align
    with block 96, moe_gemm mode 0 for gate_up (act into ``out``) and for down (dout = bf16(topk_w * sum) rows into
    ``out``), then torch.sum over the top-k slots. Mode 1 (the reference's stream-k schedule) writes the same bits;
    dout is exactly the bf16 rounding of mode 4's fp32 rows (the same sums); dout rows and the summed output are
    within rel-L2 5e-3 of the oracle (the max-abs bound is the layer output's, not a per-slot row's: rows with a large
    router weight sit far above the rms of all rows)."""
    e, k, hid, inter = 64, 5, 2048, 512
    w13, w2 = synth.make_layer(e, hid, inter, 21, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    x = synth.activations(m, hid, 21, device=DEV)
    ids, wts = synth.route_softmax(m, e, k, 21, device=DEV)
    sid, eid, npad = ops.moe_align_block_size(ids, 96, e, None, ignore_invalid_experts=True)
    a, b = layer.w13, layer.w2
    none = torch.empty(0, dtype=torch.uint8, device=DEV)
    ws = torch.empty(2 * 148 * 96 * 256, dtype=torch.float32, device=DEV)
    cnt = torch.zeros(1 << 16, dtype=torch.int32, device=DEV)
    part = torch.empty(5 * 12 * 8 * 2560, dtype=torch.float32, device=DEV)  # the kit's split buffer, unused here
    tw = wts.reshape(-1)
    douts = []
    for mode in (0, 1):
        act = torch.empty((m * k, inter), dtype=torch.bfloat16, device=DEV)
        dout = torch.empty((m * k, hid), dtype=torch.bfloat16, device=DEV)
        ops.moe_gemm(x, a.w, none, a.g, sid, eid, npad, a.g, act, k, True, a.sp, a.exc_off, a.exc_ent, ws, cnt, mode,
                     1, part, 0, True)
        ops.moe_gemm(act, b.w, none, b.g, sid, eid, npad, tw, dout, 1, False, b.sp, b.exc_off, b.exc_ent, ws, cnt,
                     mode, 1, part, 0, True)
        torch.cuda.synchronize()
        assert int(cnt[0]) == 0
        douts.append(dout)
    assert torch.equal(douts[0], douts[1])
    dout = douts[0]
    act = torch.empty((m * k, inter), dtype=torch.bfloat16, device=DEV)
    rows32 = torch.empty((m * k, hid), dtype=torch.float32, device=DEV)
    ops.moe_gemm(x, a.w, none, a.g, sid, eid, npad, a.g, act, k, True, a.sp, a.exc_off, a.exc_ent, ws, cnt, 4, 1,
                 rows32, 0, True)
    ops.moe_gemm(act, b.w, none, b.g, sid, eid, npad, tw, dout.clone(), 1, False, b.sp, b.exc_off, b.exc_ent, ws, cnt,
                 4, 1, rows32, 0, True)
    torch.cuda.synchronize()
    assert torch.equal(rows32.to(torch.bfloat16), dout)
    rows = moe_ref.slot_rows(x.cpu(), _np(ids), _np(wts), _ckpt(w13), _ckpt(w2))
    rel, _, _ = moe_ref.check(dout.float().cpu(), rows)
    assert rel <= REL, rel
    out = torch.sum(dout.view(-1, k, hid), dim=1)
    ref = moe_ref.reference(x.cpu(), _np(ids), _np(wts), _ckpt(w13), _ckpt(w2))
    rel, _, _ = moe_ref.check(out.cpu(), ref)
    assert rel <= REL, rel


def test_gemm_mode_errors():
    """Modes outside 0-5 and split-k requests on the whole-K tcgen05 modes are rejected before any launch."""
    w13, w2 = synth.make_layer(8, 2048, 512, 22, device=DEV)
    a = prep.PreparedLayer(w13, w2).w13
    m, k = 4, 5
    x = synth.activations(m, 2048, 22, device=DEV)
    ids, _ = synth.route_softmax(m, 8, k, 22, device=DEV)
    sid, eid, npad = ops.moe_align_block_size(ids, 96, 8)
    act = torch.empty((m * k, 512), dtype=torch.bfloat16, device=DEV)
    part = torch.empty(8 * m * k * 1024, dtype=torch.float32, device=DEV)
    cnt = torch.zeros(8, dtype=torch.int32, device=DEV)
    for mode, nsplit in ((6, 1), (-1, 1), (0, 2), (1, 4)):
        with pytest.raises(ops.MoekError):
            ops.moe_gemm(x, a.w, None, a.g, sid, eid, npad, a.g, act, k, True, a.sp, a.exc_off, a.exc_ent, None,
                         cnt, mode, nsplit, part, 0, True)
