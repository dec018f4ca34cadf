"""The router oracle (oracle/router.py) against the synthetic router's torch computation, its tie rule, and the
router C entry point's host-side argument checks (no GPU needed)."""
import numpy as np
import torch

from oracle import router
from qwen38_flash_coder_b200 import _lib


def test_oracle_matches_torch_softmax_topk():
    g = torch.Generator().manual_seed(5)
    logits = torch.randn((64, 512), generator=g)
    ids, w, tei = router.topk_softmax(logits.numpy(), 5, True)
    p = torch.softmax(logits, dim=-1)
    tw, tids = torch.topk(p, 5, dim=-1)
    tw = tw / tw.sum(-1, keepdim=True)
    assert np.array_equal(ids, tids.numpy().astype(np.int32))
    assert np.allclose(w, tw.numpy(), rtol=2e-6, atol=0)
    assert tei[3, 2] == 2 * 64 + 3


def test_oracle_ties_take_the_lowest_expert():
    logits = np.zeros((2, 16), dtype=np.float32)
    logits[0, [3, 9, 12]] = 2.0  # three equal maxima, then thirteen equal values
    logits[1, :] = 1.0
    ids, w, _ = router.topk_softmax(logits, 5, False)
    assert ids[0].tolist() == [3, 9, 12, 0, 1]
    assert ids[1].tolist() == [0, 1, 2, 3, 4]
    assert np.allclose(w[1], 1.0 / 16)


def test_router_entry_rejects_bad_arguments():
    lib = _lib.lib()
    assert lib.moek_router_topk(None, 0, 4, 2048, 5, 1, None, None, None, None) == 1  # E > 1024
    assert b"E <= 1024" in lib.moek_last_error()
    assert lib.moek_router_topk(None, 0, 4, 64, 33, 1, None, None, None, None) == 1  # top_k > 32
    assert lib.moek_router_topk(None, 0, 4, 64, 5, 1, None, None, None, None) == 1  # null pointers
    assert lib.moek_router_topk(None, 0, 0, 64, 5, 1, None, None, None, None) == 0  # empty batch


def _golden_cases():
    import os

    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "router_golden.npz")))
    names = sorted({k[: -len("_meta")] for k in g if k.endswith("_meta")})
    for n in names:
        m, e, k, renorm = (int(v) for v in g[f"{n}_meta"])
        order = np.argsort(-g[f"{n}_w"], axis=1, kind="stable")  # vLLM's torch path leaves the top_k unsorted
        yield n, g[f"{n}_logits"], k, bool(renorm), np.take_along_axis(g[f"{n}_ids"], order, 1), \
            np.take_along_axis(g[f"{n}_w"], order, 1)


def test_oracle_matches_vllm_golden():
    """The router oracle against vLLM's own grouped_topk (one group, softmax) run on seeded logits
    (tests/golden/make_router_golden.py): ids exact, weights to fp32 rounding."""
    cases = list(_golden_cases())
    assert len(cases) == 6
    for name, logits, k, renorm, gids, gw in cases:
        ids, w, _ = router.topk_softmax(logits, k, renorm)
        assert np.array_equal(ids, gids), name
        assert np.allclose(w, gw, rtol=4e-6, atol=1e-9), name
