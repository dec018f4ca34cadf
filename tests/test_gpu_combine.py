"""The top-k combine over routed slots (moek_combine_routed) and the prefill path that uses it: slots whose expert
id lies outside [0, E) are skipped by moe_align, so their fp32 rows are never written and must not reach the sum."""
import ctypes

import pytest
import torch

from oracle import moe_ref
from qwen38_flash_coder_b200 import _lib, ops, prep, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ckpt(mat):
    codes, scales, gs = mat
    return codes.cpu().numpy(), scales.view(torch.uint8).cpu().numpy(), gs.cpu().numpy()


def _routed(rows, ids, e, m, n, k):
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.call("moek_combine_routed", ctypes.c_void_p(rows.data_ptr()), ctypes.c_void_p(ids.data_ptr()), e,
              ctypes.c_void_p(out.data_ptr()), m, n, k, stream)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("n", [2048, 1002])  # the vectorised form (N % 4 == 0) and the scalar one
def test_routed_combine_vs_torch(n):
    """Every slot routed: bit-equal to moek_combine (ops.combine). Unrouted slots (-1, >= E) holding NaN are left out;
    a token with none routed gets a zero row. The reference sum is fp32 in slot order, rounded once."""
    m, k, e = 37, 5, 64
    g = torch.Generator(device="cpu").manual_seed(5)
    rows = torch.randn((m * k, n), generator=g).to(DEV)
    ids = torch.randint(0, e, (m, k), generator=g, dtype=torch.int32).to(DEV)
    plain = ops.combine(rows, k)
    assert torch.equal(_routed(rows, ids, e, m, n, k), plain)

    ids[3, 1] = -1
    ids[5, 4] = e + 3
    ids[9, :] = -1
    for t, j in ((3, 1), (5, 4)):
        rows[t * k + j] = float("nan")
    rows.view(m, k, n)[9] = float("nan")
    got = _routed(rows, ids, e, m, n, k)
    valid = ((ids >= 0) & (ids < e)).cpu()
    r = rows.view(m, k, n).cpu()
    want = torch.zeros((m, n), dtype=torch.float32)
    for j in range(k):
        want += torch.where(valid[:, j:j + 1], r[:, j], torch.zeros(()))
    assert torch.equal(got.cpu(), want.to(torch.bfloat16))
    assert torch.count_nonzero(got[9]) == 0


def test_prefill_unrouted_slots_vs_oracle():
    """The prefill path (M > 64) with unrouted slots, after the row scratch was filled with NaN: the output equals
    the oracle within the gate and a token with no routed slot gets a zero row."""
    e, m = 64, 150
    w13, w2 = synth.make_layer(e, 2048, 512, 11, device=DEV)
    layer = prep.PreparedLayer(w13, w2)
    x = synth.activations(m, 2048, 11, device=DEV)
    ids, wts = synth.route_softmax(m, e, 5, 11, device=DEV)
    ops.fused_moe(x, layer, wts, ids)  # sizes the row scratch
    for key, t in ops._BUF.items():
        if key[0] == "part":
            t.fill_(float("nan"))
    ids = ids.clone()
    ids[2, 1] = -1
    ids[40, 0] = e + 9
    ids[77, :] = -1
    out = ops.fused_moe(x, layer, wts, ids)
    ops.check_device_errors(DEV)
    assert not torch.isnan(out).any()
    assert torch.count_nonzero(out[77]) == 0
    ref = moe_ref.reference(x.cpu(), ids.cpu().numpy(), wts.cpu().numpy(), _ckpt(w13), _ckpt(w2))
    ok, stats = moe_ref.within_gate(out.cpu(), ref)
    assert ok, stats
