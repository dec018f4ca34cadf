"""The router kernel (moek_router_topk) on the GPU against the CPU oracle: ids bit-exact (ties to the lowest
expert), weights to fp32 rounding, for fp32 and bf16 logits, with and without renormalisation; vLLM's fused_topk
signature; and the router + layer chain against the oracle chain."""
import numpy as np
import pytest
import torch

from oracle import moe_ref, router
from qwen38_flash_coder_b200 import ops, prep, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("m,e,k", [(1, 64, 5), (8, 512, 5), (64, 512, 5), (6912, 512, 5), (37, 100, 8), (5, 1024, 32)])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_matches_oracle(m, e, k, renorm):
    g = torch.Generator().manual_seed(m * 7 + e)
    logits = torch.randn((m, e), generator=g)
    w, ids = ops.router_topk(logits.to(DEV), k, renorm)
    rids, rw, _ = router.topk_softmax(logits.numpy(), k, renorm)
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert np.allclose(w.cpu().numpy(), rw, rtol=4e-6, atol=1e-9)


def test_router_bf16_logits_and_ties():
    g = torch.Generator().manual_seed(3)
    logits = torch.randn((16, 512), generator=g).to(torch.bfloat16)  # bf16 values repeat: many exact ties
    logits[4, :] = 0.5
    w, ids = ops.router_topk(logits.to(DEV), 5, True)
    rids, rw, _ = router.topk_softmax(logits.float().numpy(), 5, True)
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert ids[4].tolist() == [0, 1, 2, 3, 4]
    assert np.allclose(w.cpu().numpy(), rw, rtol=4e-6, atol=1e-9)


def test_fused_topk_signature():
    x = torch.zeros((8, 2048), dtype=torch.bfloat16, device=DEV)
    logits = torch.randn((8, 512), generator=torch.Generator().manual_seed(1)).to(DEV)
    w, ids, tei = ops.fused_topk(x, logits, 5, True)
    assert w.dtype == torch.float32 and ids.dtype == torch.int32 and tei.dtype == torch.int32
    assert tei.cpu().tolist()[2] == [2 + 8 * j for j in range(5)]
    w2, ids2, _ = ops.fused_topk(x, logits, 5, True, indices_type=torch.int64)
    assert ids2.dtype == torch.int64 and torch.equal(ids2.int(), ids)


def test_router_then_layer_matches_oracle_chain():
    m, e = 8, 64
    w13, w2 = synth.make_layer(e, 2048, 512, 2, device=DEV)
    x = synth.activations(m, 2048, 2, device=DEV)
    logits = torch.randn((m, e), generator=torch.Generator().manual_seed(2))
    out = ops.fused_moe_from_logits(x, prep.PreparedLayer(w13, w2), logits.to(DEV), 5)
    ops.check_device_errors(DEV)
    rids, rw, _ = router.topk_softmax(logits.numpy(), 5, True)
    cpu = lambda mm: (mm[0].cpu().numpy(), mm[1].view(torch.uint8).cpu().numpy(), mm[2].cpu().numpy())
    ref = moe_ref.reference(x.cpu(), rids, rw, cpu(w13), cpu(w2))
    ok, stats = moe_ref.within_gate(out.cpu(), ref)
    assert ok, stats


def test_router_matches_vllm_golden():
    """The router kernel against vLLM's own grouped_topk (one group, softmax) on the golden's seeded logits
    (tests/golden/make_router_golden.py): ids exact, weights to fp32 rounding."""
    import os

    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "router_golden.npz")))
    for n in sorted({k[: -len("_meta")] for k in g if k.endswith("_meta")}):
        m, e, k, renorm = (int(v) for v in g[f"{n}_meta"])
        w, ids = ops.router_topk(torch.from_numpy(g[f"{n}_logits"]).to(DEV), k, bool(renorm))
        order = np.argsort(-g[f"{n}_w"], axis=1, kind="stable")
        assert np.array_equal(ids.cpu().numpy(), np.take_along_axis(g[f"{n}_ids"], order, 1)), n
        assert np.allclose(w.cpu().numpy(), np.take_along_axis(g[f"{n}_w"], order, 1), rtol=4e-6, atol=1e-9), n


@pytest.mark.parametrize("m,e,dtype", [(8, 512, torch.float32), (32, 512, torch.bfloat16), (1, 64, torch.float32),
                                       (64, 256, torch.float32)])
def test_layer_with_fused_router(m, e, dtype):
    """The router fused into the whole-layer kernel (one launch): the routing it reports equals the router kernel's
    bit for bit, and the output equals router kernel + layer kernel bit for bit and is within the gate of the oracle
    chain."""
    w13, w2 = synth.make_layer(e, 2048, 512, 3 + m, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    x = synth.activations(m, 2048, 3 + m, device=DEV)
    logits = torch.randn((m, e), generator=torch.Generator().manual_seed(m + e)).to(dtype).to(DEV)
    out, (w, ids) = ops.fused_moe_from_logits(x, layer, logits, 5, return_routing=True)
    rw, rids = ops.router_topk(logits, 5, True)
    ref = ops.fused_moe(x, layer, rw, rids)
    ops.check_device_errors(DEV)
    assert torch.equal(ids, rids) and torch.equal(w, rw)
    assert torch.equal(out, ref)
    oids, ow, _ = router.topk_softmax(logits.float().cpu().numpy(), 5, True)
    cpu = lambda mm: (mm[0].cpu().numpy(), mm[1].view(torch.uint8).cpu().numpy(), mm[2].cpu().numpy())
    ok, stats = moe_ref.within_gate(out.cpu(), moe_ref.reference(x.cpu(), oids, ow, cpu(w13), cpu(w2)))
    assert ok, stats
