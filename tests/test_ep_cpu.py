"""Expert parallelism on CPU ranks (gloo): the dispatch / combine orchestration of ``ep.ep_moe`` with the oracle as
the backend, against the one-process oracle; host-side fault injection (a rank that fails before the exchange).
No GPU is involved: the CUDA backend's kernels are checked against the same oracle in test_gpu_ep.py."""
import datetime
import multiprocessing as pymp
import os
import socket
import traceback

import numpy as np
import pytest
import torch

from oracle import ep as oep
from oracle import moe_ref

E, H, I, K, M = 8, 256, 256, 5, 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plan_hand_example():
    # 4 experts over 2 ranks: rank 0 owns {0, 1}, rank 1 owns {2, 3}; -1 and 9 go nowhere
    ids = np.array([[0, 2], [1, 1], [3, -1], [9, -1]])
    pos, counts, offsets = oep.plan(ids, 4, 2)
    assert pos.tolist() == [[0, 0], [1, -1], [-1, 1], [-1, -1]]
    assert counts.tolist() == [2, 2] and offsets.tolist() == [0, 2, 4]
    x = torch.arange(4 * 8, dtype=torch.float32).view(4, 8).to(torch.bfloat16)
    w = np.array([[0.75, 0.25], [0.5, 0.5], [1.0, 0.0], [1.0, 0.0]], dtype=np.float32)
    sx, meta = oep.pack(x, ids, w, pos, offsets, 4, 2)
    assert torch.equal(sx, x[[0, 1, 0, 2]])
    m = meta.numpy()
    # rows: rank 0 gets tokens 0, 1; rank 1 gets tokens 0, 2 (slots owned elsewhere: id -1, weight 0)
    assert m[0, :2].tolist() == [0, -1] and m[1, :2].tolist() == [1, 1]
    assert m[2, :2].tolist() == [-1, 0] and m[3, :2].tolist() == [1, -1]
    assert m[0, 2:].view(np.float32).tolist() == [0.75, 0.0] and m[2, 2:].view(np.float32).tolist() == [0.0, 0.25]


class OracleBackend:
    """``ep.ep_moe``'s backend interface restated on the CPU with the oracle (test infrastructure)."""

    def plan(self, ids32, num_experts, world):
        pos, counts, offsets = oep.plan(ids32.numpy(), num_experts, world)
        self._pos = pos
        return torch.from_numpy(pos), torch.from_numpy(counts), torch.from_numpy(offsets)

    def pack(self, x, ids32, w, pos, offsets, num_experts, world, rows, counts=None, fill=False):
        sx, meta = oep.pack(x, ids32.numpy(), w.numpy(), pos.numpy(), offsets.numpy(), num_experts, world)
        assert sx.shape[0] == rows
        return sx, meta

    def local(self, x_recv, meta, layer, k):
        w13, w2 = layer.ckpt
        np_mat = lambda mm: (mm[0].numpy(), mm[1].view(torch.uint8).numpy(), mm[2].numpy())
        return oep.partial(x_recv, meta.numpy(), np_mat(w13), np_mat(w2), k)

    def unpack(self, back, pos, offsets, m, world):
        return oep.unpack(back, pos.numpy(), offsets.numpy(), m, world)


def _layer():
    from qwen38_flash_coder_b200 import synth

    return synth.make_layer(E, H, I, 3)


def _tokens(rank):
    from qwen38_flash_coder_b200 import synth

    x = synth.activations(M, H, 100 + rank)
    ids, w = synth.route_softmax(M, E, K, 100 + rank)
    return x, ids, w


def _rank_main(rank, world, port, fail_rank, q):
    import torch.distributed as dist

    from qwen38_flash_coder_b200 import ep

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=8))
        w13, w2 = _layer()
        layer = ep.EPLayer(ep.shard_checkpoint(w13, E, world, rank), ep.shard_checkpoint(w2, E, world, rank), E,
                           world, rank, ckpt=True)
        x, ids, w = _tokens(rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the exchange")
        out = ep.ep_moe(x, layer, w, ids, backend=OracleBackend())
        q.put((rank, "ok", out.numpy()))
    except Exception as exc:  # reported to the parent, which decides what was expected
        q.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()[-400:]}"))


def _run(world, fail_rank=-1, limit=120):
    ctx = pymp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=limit)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("world", [2, 4])
def test_ep_gloo_matches_one_process_oracle(world):
    res = _run(world)
    w13, w2 = _layer()
    np_mat = lambda mm: (mm[0].numpy(), mm[1].view(torch.uint8).numpy(), mm[2].numpy())
    for rank in range(world):
        status, out = res[rank]
        assert status == "ok", out
        x, ids, w = _tokens(rank)
        ref = moe_ref.reference(x, ids.numpy(), w.numpy(), np_mat(w13), np_mat(w2))
        # the same slot rows, added per rank and then over ranks. The CPU matmuls run over different row subsets
        # (fp32 sums in another order), so an act value can land on the other side of a bf16 rounding now and then
        d = torch.from_numpy(out) - ref
        err = float(d.abs().max()) / float(ref.abs().max())
        rel = float(d.norm() / ref.norm())
        assert err < 1e-3 and rel < 1e-4, (rank, err, rel)


def test_ep_gloo_rank_failure_is_reported_not_hung():
    res = _run(2, fail_rank=1, limit=90)
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    # the surviving rank's first collective ends with an error once the group's timeout expires
    assert res[0][0] == "error", res[0]


def test_owned_experts_and_errors():
    from qwen38_flash_coder_b200 import ep
    from qwen38_flash_coder_b200._lib import MoekError

    assert ep.owned_experts(512, 8, 3) == (192, 256)
    with pytest.raises(MoekError):
        ep.owned_experts(10, 4, 0)


def test_peer_exchange_call_checks_on_host():
    """ep_moe's peer-memory path rejects, before any device call, an exchange built for another process group,
    hidden states that are not bf16, and a batch beyond the exchange's capacity (one gloo rank on the CPU)."""
    import types

    import torch.distributed as dist

    from qwen38_flash_coder_b200 import ep
    from qwen38_flash_coder_b200._lib import MoekError

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=30))
    try:
        layer = types.SimpleNamespace(world=1, num_experts=8, local_experts=8, prep=None)
        ids = torch.zeros((4, 2), dtype=torch.int32)
        w = torch.full((4, 2), 0.5)
        x = torch.zeros((4, 64), dtype=torch.bfloat16)
        other = types.SimpleNamespace(world=2, rank=0, mcap=8, top_k=2, hidden=64)
        with pytest.raises(MoekError, match="built for rank 0 of 2"):
            ep.ep_moe(x, layer, w, ids, capacity=True, peer=other)
        px = types.SimpleNamespace(world=1, rank=0, mcap=2, top_k=2, hidden=64)
        with pytest.raises(MoekError, match="bf16"):
            ep.ep_moe(x.float(), layer, w, ids, capacity=True, peer=px)
        with pytest.raises(MoekError, match="holds 2 tokens"):
            ep.ep_moe(x, layer, w, ids, capacity=True, peer=px)
    finally:
        dist.destroy_process_group()
