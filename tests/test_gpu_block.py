"""The rest of the MoE block on the GPU (moek_router_gate, moek_shared_expert, moek_moe_block) against the CPU
oracle (oracle/shared.py): the router logits within fp32 summation error, the routing bit-exact from those logits,
the shared expert's rows and the block output within the parity gate, every call repeatable bit for bit."""
import numpy as np
import pytest
import torch

from oracle import moe_ref, router
from oracle import shared as shared_ref
from qwen38_flash_coder_b200 import ops, prep, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("m,e", [(1, 64), (8, 512), (33, 512), (64, 256), (200, 512)])
def test_router_gate_matches_oracle(m, e):
    x = synth.activations(m, 2048, m, device=DEV)
    wg = synth.make_router_gate(e, 2048, m, device=DEV)
    logits = ops.router_gate(x, wg)
    ref = shared_ref.gate_logits(x.cpu(), wg.cpu())
    err = (logits.cpu() - ref).abs().max() / ref.abs().max()
    assert err < 2e-6, err
    assert torch.equal(ops.router_gate(x, wg), logits)  # the same bits on every call


@pytest.mark.parametrize("m", [1, 8, 64, 300])
def test_shared_expert_matches_oracle(m):
    sh = synth.make_shared(2048, 512, m, device=DEV)
    x = synth.activations(m, 2048, 100 + m, device=DEV)
    rows = ops.shared_expert(x, ops.SharedExpert(*sh))
    ref = shared_ref.shared_rows(x.cpu(), *[_np(t) if t.dtype == torch.uint8 else t.cpu() for t in sh])
    rel = float((rows.cpu() - ref).norm() / ref.norm())
    assert rel < 1e-3, rel  # fp32 rows: only the bf16 act roundings of near-midpoint sums may differ
    assert torch.equal(ops.shared_expert(x, ops.SharedExpert(*sh)), rows)


def test_mxfp8_scale_range_is_checked():
    sh = list(synth.make_shared(256, 128, 0, device=DEV))
    sh[1] = sh[1].clone()
    sh[1][0, 0] = 135
    with pytest.raises(ops.MoekError):
        ops.SharedExpert(*sh)


@pytest.mark.parametrize("m,e,kind", [(1, 512, "u"), (8, 512, "u"), (32, 512, "u"), (64, 256, "u"), (300, 512, "u"),
                                      (8, 100, "u")])  # E % 16 != 0: the gate as a library GEMM, the layer from logits
@pytest.mark.parametrize("with_shared", [True, False])
def test_moe_block_matches_oracle(m, e, kind, with_shared):
    w13, w2 = synth.make_layer(e, 2048, 512, m, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    wg = synth.make_router_gate(e, 2048, m, device=DEV)
    sh = synth.make_shared(2048, 512, m, device=DEV)
    x = synth.activations(m, 2048, 200 + m, device=DEV)
    she = ops.SharedExpert(*sh) if with_shared else None
    out, (w, ids) = ops.moe_block(x, wg, layer, she, 5, return_routing=True)
    ops.check_device_errors(DEV)
    # the routing, bit-exact from the GPU's own logits
    logits = ops.router_gate(x, wg)
    rids, rw, _ = router.topk_softmax(_np(logits), 5, True)
    assert np.array_equal(_np(ids), rids)
    assert np.allclose(_np(w), rw, rtol=4e-6, atol=1e-9)
    cpu = lambda t: (_np(t[0]), _np(t[1].view(torch.uint8)), _np(t[2]))
    shc = [_np(t) if t.dtype == torch.uint8 else t.cpu() for t in sh]
    if with_shared:
        ref = shared_ref.block(x.cpu(), rids, rw, cpu(w13), cpu(w2), shc)
    else:
        ref = moe_ref.reference(x.cpu(), rids, rw, cpu(w13), cpu(w2))
    ok, (rel, raw, net) = moe_ref.within_gate(out.cpu(), ref)
    assert ok, (rel, raw, net)
    again = ops.moe_block(x, wg, layer, she, 5)
    assert torch.equal(again, out)


def test_moe_block_without_shared_equals_router_plus_layer():
    """With no shared expert the block is the gate followed by the fused router + layer, bit for bit."""
    w13, w2 = synth.make_layer(512, 2048, 512, 5, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    wg = synth.make_router_gate(512, 2048, 5, device=DEV)
    x = synth.activations(8, 2048, 5, device=DEV)
    out = ops.moe_block(x, wg, layer, None, 5)
    want = ops.fused_moe_from_logits(x, layer, ops.router_gate(x, wg), 5)
    assert torch.equal(out, want)
