"""moek_align_noalloc: the moe_align entry point that takes no workspace, for callers that cannot allocate device
memory on the calling path. Called through the C ABI and checked bit for bit against moek_align (which takes a
caller-allocated workspace) on two calls in a row, so that the second call also shows the fixed scratch array left
by the first does no harm. Named to be collected last: if it fails, every other test has already run."""
import ctypes

import numpy as np
import pytest
import torch

from qwen38_flash_coder_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _outs(numel, e, bs):
    n = numel + e * (bs - 1)
    if numel < e:
        n = min(numel * bs, n)
    nb = (n + bs - 1) // bs
    return (torch.full((n,), -7, dtype=torch.int32, device="cuda"),
            torch.full((nb,), -7, dtype=torch.int32, device="cuda"),
            torch.full((1,), -7, dtype=torch.int32, device="cuda"))


def _ptr(t):
    return t.data_ptr() if t is not None and t.numel() else None


def _with_workspace(ids, e, bs, stream):
    lib = _lib.lib()
    numel = ids.numel()
    sid, eid, npad = _outs(numel, e, bs)
    wsb = ctypes.c_size_t(0)
    assert lib.moek_align_workspace_bytes(numel, e, ctypes.byref(wsb)) == 0
    ws = torch.empty(max(1, wsb.value), dtype=torch.uint8, device="cuda")
    rc = lib.moek_align(_ptr(ids), numel, e, bs, _ptr(sid), sid.numel(), _ptr(eid), eid.numel(), _ptr(npad),
                        _ptr(ws) if wsb.value else None, wsb.value, stream)
    assert rc == 0, lib.moek_last_error()
    return sid, eid, npad


def _no_alloc(ids, e, bs, stream):
    lib = _lib.lib()
    numel = ids.numel()
    sid, eid, npad = _outs(numel, e, bs)
    rc = lib.moek_align_noalloc(_ptr(ids), numel, e, bs, _ptr(sid), sid.numel(), _ptr(eid), eid.numel(), _ptr(npad),
                                stream)
    assert rc == 0, lib.moek_last_error()
    return sid, eid, npad


@pytest.mark.parametrize("m,e,route", [(6912, 512, "zipf"), (8, 512, "uniform"), (13000, 64, "uniform")])
def test_no_alloc_matches_workspace_entry_point_twice(m, e, route):
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row: the fixed scratch keeps the first call's contents
        gen = synth.route_zipf if route == "zipf" else synth.route_softmax
        ids, _ = gen(m, e, 5, seed=100 * call + m, device="cuda")
        ids = ids.reshape(-1).contiguous()
        ref = _with_workspace(ids, e, 96, stream)
        got = _no_alloc(ids, e, 96, stream)
        torch.cuda.synchronize()
        for a, b in zip(ref, got):
            assert torch.equal(a, b)
        assert int(got[2][0]) > 0


def test_no_alloc_rejects_sizes_beyond_its_limit():
    lib = _lib.lib()
    ids = torch.zeros(65537, dtype=torch.int32, device="cuda")
    sid, eid, npad = _outs(65537, 512, 96)
    rc = lib.moek_align_noalloc(_ptr(ids), 65537, 512, 96, _ptr(sid), sid.numel(), _ptr(eid), eid.numel(),
                                _ptr(npad), torch.cuda.current_stream().cuda_stream)
    assert rc == 1 and b"65536" in lib.moek_last_error()
    rc = lib.moek_align_noalloc(_ptr(ids), 100, 2048, 96, _ptr(sid), sid.numel(), _ptr(eid), eid.numel(),
                                _ptr(npad), torch.cuda.current_stream().cuda_stream)
    assert rc == 1
