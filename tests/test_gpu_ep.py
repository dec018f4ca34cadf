"""Expert parallelism on the GPU: the dispatch / combine kernels against the CPU restatement (bit-exact), the whole
EP layer on a one-rank NCCL group against ops.fused_moe, and, when 2, 4 or 8 GPUs are visible, that many NCCL ranks
against the one-GPU layer. The EP layer adds the same fp32 slot terms as the one-GPU layer, but the one-GPU decode epilogue
fuses each router-weight product into its running sum (one rounding) where EP rounds the weighted row first, so the
two agree to fp32 rounding, not bitwise."""
import datetime
import multiprocessing as pymp
import os
import socket

import numpy as np
import pytest
import torch

from oracle import ep as oep

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("m", [1, 37, 1500])
def test_ep_kernels_match_oracle(world, m):
    from qwen38_flash_coder_b200 import ep

    E, k, H = 64, 5, 256
    g = torch.Generator().manual_seed(world * 1000 + m)
    ids = torch.randint(-2, E + 3, (m, k), generator=g, dtype=torch.int32)  # a few invalid ids on purpose
    w = torch.rand((m, k), generator=g)
    x = torch.randn((m, H), generator=g).to(torch.bfloat16)
    be = ep.CudaBackend()
    pos, counts, offsets = be.plan(ids.to(DEV), E, world)
    rpos, rcounts, roff = oep.plan(ids.numpy(), E, world)
    assert np.array_equal(pos.cpu().numpy(), rpos)
    assert np.array_equal(counts.cpu().numpy(), rcounts) and np.array_equal(offsets.cpu().numpy(), roff)
    sx, meta = be.pack(x.to(DEV), ids.to(DEV), w.to(DEV), pos, offsets, E, world, int(roff[-1]))
    rsx, rmeta = oep.pack(x, ids.numpy(), w.numpy(), rpos, roff, E, world)
    assert torch.equal(sx.cpu(), rsx) and torch.equal(meta.cpu(), rmeta)
    # partial: fp32 sum of the valid slots' rows in slot order
    R = int(roff[-1])
    rows = torch.randn((R * k, H), generator=g)
    el = E // world
    out = torch.empty((R, H), dtype=torch.float32, device=DEV)
    from qwen38_flash_coder_b200 import ops
    from qwen38_flash_coder_b200._lib import call

    call("moek_ep_partial", ops._ptr(rows.to(DEV)) if R else None, ops._ptr(meta), 2 * k, el, R, H, k,
         ops._ptr(out), ops._stream(DEV))
    exp = torch.zeros((R, H))
    lid = rmeta[:, :k]
    for j in range(k):
        valid = ((lid[:, j] >= 0) & (lid[:, j] < el))[:, None]
        exp += torch.where(valid, rows.view(R, k, H)[:, j], torch.zeros(()))
    assert torch.equal(out.cpu(), exp)
    # merged fixed-capacity layout: segment d = rows [d*m, (d+1)*m), metadata in each row's tail, unused rows marked
    cap_off = torch.arange(world + 1, dtype=torch.int32, device=DEV) * m
    buf = be.pack(x.to(DEV), ids.to(DEV), w.to(DEV), pos, cap_off, E, world, world * m, counts=counts, merged=True)
    mc = ep.meta_columns(k)
    bx, bm = buf[:, :H].cpu(), buf[:, H:].contiguous().view(torch.int32).cpu()[:, :2 * k]
    for d in range(world):
        n = int(rcounts[d])
        assert torch.equal(bx[d * m:d * m + n], rsx[roff[d]:roff[d] + n])
        assert torch.equal(bm[d * m:d * m + n], rmeta[roff[d]:roff[d] + n])
        assert (bm[d * m + n:(d + 1) * m, :k] == -1).all() and (bm[d * m + n:(d + 1) * m, k:] == 0).all()
    assert buf.shape[1] == H + mc
    # unpack: returned partials added in rank order, one bf16 rounding
    back = torch.randn((R, H), generator=g)
    res = be.unpack(back.to(DEV), pos, offsets, m, world)
    assert torch.equal(res.cpu(), oep.unpack(back, rpos, roff, m, world).to(torch.bfloat16))


def _single_rank_group():
    import torch.distributed as dist

    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=DEV)


@pytest.mark.parametrize("m,capacity", [(8, True), (8, False), (300, False), (300, True)])
def test_ep_one_rank_equals_fused_moe(m, capacity):
    import torch.distributed as dist

    from qwen38_flash_coder_b200 import ep, ops, synth

    E = 64
    w13, w2 = synth.make_layer(E, 2048, 512, 21, device=DEV)
    layer = ep.EPLayer(w13, w2, E, 1, 0)
    x = synth.activations(m, 2048, 21, device=DEV)
    ids, wts = synth.route_zipf(m, E, 5, 21, device=DEV)
    ref = ops.fused_moe(x, layer.prep, wts, ids)
    _single_rank_group()
    try:
        out = ep.ep_moe(x, layer, wts, ids, capacity=capacity)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    ops.check_device_errors(DEV)
    from oracle import moe_ref

    rel, raw, net = moe_ref.check(out.cpu(), ref.float().cpu())
    assert rel < 1e-3 and net < 1e-2, (rel, net)
    assert (out != ref).float().mean() < 0.01  # only the odd output lands on the other side of a bf16 rounding


@pytest.mark.parametrize("m,mcap", [(8, 8), (5, 8), (100, 128)])
def test_ep_peer_exchange_one_rank(m, mcap):
    """The peer-memory exchange on a one-rank group (the block shared with itself): equal to the NCCL fixed-capacity
    path bit for bit, repeatable (the flags carry the call number), also when replayed as a CUDA graph. mcap 8: the
    whole-layer kernel dispatches, reads the receive segment, returns the partials and unpacks them itself (one
    launch; the three-launch sequence, dispatch, layer, unpack, gives the same bits); mcap 128: more slots than it
    takes, so the local layer's kernels run between a wait and the combine kernel."""
    import torch.distributed as dist

    from qwen38_flash_coder_b200 import ep, ops, synth

    E = 64
    w13, w2 = synth.make_layer(E, 2048, 512, 23, device=DEV)
    layer = ep.EPLayer(w13, w2, E, 1, 0)
    x = synth.activations(m, 2048, 23, device=DEV)
    ids, wts = synth.route_zipf(m, E, 5, 23, device=DEV)
    _single_rank_group()
    try:
        px = ep.PeerExchange(None, mcap, 2048, 5, DEV)
        assert ops.layer_p2p_fits(mcap, 5) == (mcap * 5 <= 512)
        ref = ep.ep_moe(x, layer, wts, ids, capacity=True)
        outs = [ep.ep_moe(x, layer, wts, ids, capacity=True, peer=px) for _ in range(3)]
        os.environ["MOEK_B200_EP_FUSED"] = "0"
        try:
            outs += [ep.ep_moe(x, layer, wts, ids, capacity=True, peer=px) for _ in range(2)]
        finally:
            del os.environ["MOEK_B200_EP_FUSED"]
        outs.append(ep.ep_moe(x, layer, wts, ids, capacity=True, peer=px))
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ep.ep_moe(x, layer, wts, ids, capacity=True, peer=px)
        torch.cuda.current_stream().wait_stream(s)
        with torch.cuda.graph(g):
            gout = ep.ep_moe(x, layer, wts, ids, capacity=True, peer=px)
        for _ in range(3):
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(gout, ref)
        del g
        px.close()
    finally:
        dist.destroy_process_group()
    ops.check_device_errors(DEV)
    for o in outs:
        assert torch.equal(o, ref)


def test_ep_peer_layer_wait_expires():
    """The whole-layer kernel on a receive segment that no sender fills: its bounded wait on the receive flag runs
    out, it records MOEK_DEV_TIMEOUT, writes nothing and returns (the context stays usable); after the error is
    cleared the exchange works again."""
    import torch.distributed as dist

    from qwen38_flash_coder_b200 import _lib, ep, ops, synth

    E, m = 64, 8
    w13, w2 = synth.make_layer(E, 2048, 512, 29, device=DEV)
    layer = ep.EPLayer(w13, w2, E, 1, 0)
    x = synth.activations(m, 2048, 29, device=DEV)
    ids, wts = synth.route_zipf(m, E, 5, 29, device=DEV)
    _single_rank_group()
    try:
        px = ep.PeerExchange(None, m, 2048, 5, DEV)
        ref = ep.ep_moe(x, layer, wts, ids, capacity=True, peer=px)
        torch.cuda.synchronize()
        back = px.back.clone()
        _lib.call("moek_set_wait_timeout_ns", 20_000_000)  # 20 ms
        try:
            ops.layer_p2p(px, layer.prep)  # no dispatch raised the receive flag to this call's number
            torch.cuda.synchronize()
        finally:
            _lib.call("moek_set_wait_timeout_ns", 2_000_000_000)
        with pytest.raises(ops.MoekError, match="timed out"):
            ops.check_device_errors(DEV)
        assert torch.equal(px.back, back)  # nothing was returned
        again = ep.ep_moe(x, layer, wts, ids, capacity=True, peer=px)
        torch.cuda.synchronize()
        ops.check_device_errors(DEV)
        assert torch.equal(again, ref)
        px.close()
    finally:
        dist.destroy_process_group()


def _ep_rank(rank, world, port, q):
    import torch.distributed as dist

    from oracle import moe_ref
    from qwen38_flash_coder_b200 import ep, ops, synth

    try:
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        E, m = 64, (40 if rank % 2 == 0 else 700)  # ranks on the decode path and on the tcgen05 path
        w13, w2 = synth.make_layer(E, 2048, 512, 31, device=dev)
        layer = ep.EPLayer(ep.shard_checkpoint(w13, E, world, rank), ep.shard_checkpoint(w2, E, world, rank), E,
                           world, rank)
        full = ep.EPLayer(w13, w2, E, 1, 0)
        x = synth.activations(m, 2048, 40 + rank, device=dev)
        ids, wts = synth.route_zipf(m, E, 5, 40 + rank, device=dev)
        out = ep.ep_moe(x, layer, wts, ids)
        # fixed-capacity mode: both ranks pass the same M
        m2 = 48
        x2 = synth.activations(m2, 2048, 60 + rank, device=dev)
        ids2, wts2 = synth.route_zipf(m2, E, 5, 60 + rank, device=dev)
        out2 = ep.ep_moe(x2, layer, wts2, ids2, capacity=True)
        # the same fixed-capacity batch over peer memory: world x 48 received rows (the whole-layer kernel takes up
        # to 102, so at 2 ranks it reads them in place and returns the partials over NVLink; with more ranks the local
        # layer's kernels run between a wait and the combine kernel); the same bits call after call, and the same gate
        # against the one-GPU layer
        px = ep.PeerExchange(None, m2, 2048, 5, dev)
        peer_outs = [ep.ep_moe(x2, layer, wts2, ids2, capacity=True, peer=px) for _ in range(3)]
        # a decode batch of 8 tokens a rank: the one-launch layer (dispatch, layer and unpack in the whole-layer
        # kernel) at every world size here, against the three-launch sequence, which must give the same bits
        m3 = 8
        x3 = synth.activations(m3, 2048, 80 + rank, device=dev)
        ids3, wts3 = synth.route_zipf(m3, E, 5, 80 + rank, device=dev)
        px3 = ep.PeerExchange(None, m3, 2048, 5, dev)
        fused3 = [ep.ep_moe(x3, layer, wts3, ids3, capacity=True, peer=px3) for _ in range(3)]
        os.environ["MOEK_B200_EP_FUSED"] = "0"
        try:
            three3 = [ep.ep_moe(x3, layer, wts3, ids3, capacity=True, peer=px3) for _ in range(2)]
        finally:
            del os.environ["MOEK_B200_EP_FUSED"]
        fused3.append(ep.ep_moe(x3, layer, wts3, ids3, capacity=True, peer=px3))
        ref = ops.fused_moe(x, full.prep, wts, ids)
        ref2 = ops.fused_moe(x2, full.prep, wts2, ids2)
        ref3 = ops.fused_moe(x3, full.prep, wts3, ids3)
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        px.close()
        px3.close()
        if not all(torch.equal(o, peer_outs[0]) for o in peer_outs[1:]):
            raise AssertionError("peer-memory exchange not repeatable")
        if not all(torch.equal(o, fused3[0]) for o in fused3[1:] + three3):
            raise AssertionError("one-launch EP layer differs from the three-launch sequence or between calls")
        rel4, _, net4 = moe_ref.check(fused3[0].cpu(), ref3.float().cpu())
        rel_pn, _, _ = moe_ref.check(peer_outs[0].cpu(), out2.float().cpu())
        if rel_pn > 2e-3:
            raise AssertionError(f"peer-memory exchange differs from the NCCL exchange: rel {rel_pn:.2e}")
        rel, raw, net = moe_ref.check(out.cpu(), ref.float().cpu())
        rel2, raw2, net2 = moe_ref.check(out2.cpu(), ref2.float().cpu())
        rel3, raw3, net3 = moe_ref.check(peer_outs[0].cpu(), ref2.float().cpu())
        q.put((rank, "ok", (max(rel, rel2, rel3, rel4), max(net, net2, net3, net4))))
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, "error", repr(exc)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_ranks_match_one_gpu_layer(world):
    """world NCCL ranks on world GPUs (NVLS off): exact-count and fixed-capacity NCCL exchanges and the peer-memory
    exchange, every rank's tokens against the one-GPU layer of the same experts."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = pymp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        procs = [ctx.Process(target=_ep_rank, args=(r, world, port, q)) for r in range(world)]
        for p in procs:
            p.start()
        res = dict((r, (s, v)) for r, s, v in (q.get(timeout=300) for _ in range(world)))
        for p in procs:
            p.join(timeout=60)
    finally:
        os.environ.clear()
        os.environ.update(env)
    for r in range(world):
        status, val = res[r]
        assert status == "ok", val
        rel, net = val
        # against the one-GPU result (itself bf16): the fp32 partials are added per rank, then over ranks
        assert rel < 2e-3 and net < 2e-2, (r, rel, net)
