"""Expert parallelism: the routed experts split over the ranks of a process group, tokens exchanged with NCCL or,
for fixed-capacity decode batches, over peer memory by this build's own kernels (``PeerExchange``).

The reference runs on one GPU and rejects vLLM's ``expert_map`` (files/mbx_moek.py:248-255). This module adds the
expert-parallel form of the same layer for 2/4/8 GPUs of one node, one process per GPU:

- **sharding**: the E experts are split contiguously, rank d owns [d * E / world, (d + 1) * E / world) and holds
  only those experts' prepared weights (``EPLayer``); every rank keeps its own tokens (data-parallel tokens,
  expert-parallel weights);
- **dispatch**: ``moek_ep_plan`` places every token in the send segment of each rank owning one of its top-k
  experts (ascending token order), an int32 all-to-all exchanges the row counts, ``moek_ep_pack`` copies the rows and
  their slot metadata (local expert ids, -1 for slots owned elsewhere, and router weights), and two all-to-allv
  (``torch.distributed.all_to_all_single`` on NCCL) move rows and metadata;
- **local experts**: the received rows go through the same align / gate_up / SwiGLU / down kernels
  (``ops.moe_rows``), and ``moek_ep_partial`` sums each row's local slots in fp32;
- **combine**: an all-to-allv returns the fp32 partial rows and ``moek_ep_unpack`` adds them in rank order and
  rounds once to bf16, so the result differs from the one-GPU layer only by the order of fp32 additions.

With exact row counts (the default) the counts cross to the host between the count exchange and the row exchange
(the receive buffers are sized from them), so one EP layer call synchronises its stream once; the fixed-capacity
mode (``capacity=True``, for decode batches) reserves M rows per destination instead and never synchronises.

Failure handling is the process group's: create it with a short ``timeout``; a rank that fails or never arrives
makes the others' next collective raise instead of hanging (tested with gloo ranks on the CPU). The backend is
pluggable so that the orchestration can be tested on CPU ranks against the oracle (``tests/test_ep_cpu.py``); the
default backend is the CUDA kernels, and there is no CPU fallback in it.
"""
import os

import torch
import torch.distributed as dist

from . import ops, prep
from ._lib import MoekError, call


def owned_experts(num_experts: int, world: int, rank: int):
    """[lo, hi) of the experts rank ``rank`` owns."""
    if num_experts % world:
        raise MoekError(f"moek_b200: {num_experts} experts do not split evenly over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


def shard_checkpoint(mat, num_experts: int, world: int, rank: int):
    """The local slice of a checkpoint matrix (codes, scales, global scales), each indexed by expert first."""
    lo, hi = owned_experts(num_experts, world, rank)
    return tuple(t[lo:hi] for t in mat)


class EPLayer:
    """The experts of one layer owned by this rank, prepared for the kernels, plus the global geometry."""

    def __init__(self, w13_local, w2_local, num_experts: int, world: int, rank: int, ckpt: bool = False):
        lo, hi = owned_experts(num_experts, world, rank)
        if w13_local[0].shape[0] != hi - lo or w2_local[0].shape[0] != hi - lo:
            raise MoekError("moek_b200: the local checkpoint slice does not match the rank's expert range")
        self.num_experts, self.world, self.rank, self.lo, self.hi = num_experts, world, rank, lo, hi
        self.prep = prep.PreparedLayer(w13_local, w2_local) if w13_local[0].is_cuda else None
        self.ckpt = (w13_local, w2_local) if ckpt or self.prep is None else None
        self.hidden = w2_local[0].shape[1]

    @property
    def local_experts(self) -> int:
        return self.hi - self.lo


class CudaBackend:
    """The build's kernels (C ABI) for the index work, the row copies and the local experts. With ``record`` a list,
    every received batch (rows, slot metadata, metadata row stride in int32) is appended to it."""

    def __init__(self, record=None):
        self.record = record

    def plan(self, ids32, num_experts, world):
        m, k = ids32.shape
        dev = ids32.device
        pos = torch.empty((m, world), dtype=torch.int32, device=dev)
        counts = torch.empty(world, dtype=torch.int32, device=dev)
        offsets = torch.empty(world + 1, dtype=torch.int32, device=dev)
        call("moek_ep_plan", ops._ptr(ids32), m, k, num_experts, world, ops._ptr(pos), ops._ptr(counts),
             ops._ptr(offsets), ops._stream(dev))
        return pos, counts, offsets

    def pack(self, x, ids32, w, pos, offsets, num_experts, world, rows, counts=None, merged=False):
        """Send rows and slot metadata. merged=False: (rows bf16 [rows, H], meta int32 [rows, 2k]); merged=True: one
        bf16 buffer [rows, H + mc] with each row's metadata in its last mc columns (one all-to-all moves both), and
        the rows no token uses (fixed-capacity segments, given ``counts``) marked as having no valid slot."""
        m, hid = x.shape
        k = ids32.shape[1]
        dev = x.device
        if merged:
            mc = meta_columns(k)
            buf = torch.empty((rows, hid + mc), dtype=torch.bfloat16, device=dev)
            call("moek_ep_pack", ops._ptr(x), ops._ptr(ids32), ops._ptr(w), ops._ptr(pos), ops._ptr(offsets),
                 ops._ptr(counts), 1, m, hid, k, num_experts, world, buf.data_ptr(), hid + mc,
                 buf.data_ptr() + 2 * hid, (hid + mc) // 2, ops._stream(dev))
            return buf
        send_x = torch.empty((rows, hid), dtype=torch.bfloat16, device=dev)
        meta = torch.empty((rows, 2 * k), dtype=torch.int32, device=dev)
        call("moek_ep_pack", ops._ptr(x), ops._ptr(ids32), ops._ptr(w), ops._ptr(pos), ops._ptr(offsets), None, 0, m,
             hid, k, num_experts, world, ops._ptr(send_x), hid, ops._ptr(meta), 2 * k, ops._stream(dev))
        return send_x, meta

    def local(self, x_recv, meta, layer: EPLayer, k, meta_stride=None):
        """fp32 partial rows [R, H] of the received rows' local slots. ``meta`` int32 rows (stride ``meta_stride``
        int32, default 2k)."""
        if self.record is not None:
            self.record.append((x_recv, meta, meta_stride or 2 * k))
        r, hid = x_recv.shape
        out = torch.empty((r, hid), dtype=torch.float32, device=x_recv.device)
        if r == 0:
            return out
        ids = meta[:, :k].contiguous()
        w = meta[:, k:2 * k].contiguous().view(torch.float32)
        rows = ops.moe_rows(x_recv, layer.prep, w, ids)
        call("moek_ep_partial", ops._ptr(rows), meta.data_ptr(), meta_stride or 2 * k, layer.local_experts, r, hid,
             k, ops._ptr(out), ops._stream(x_recv.device))
        return out

    def local_merged(self, recv, layer: EPLayer, k):
        """``local`` on a merged receive buffer [R, H + mc] (rows, then each row's metadata)."""
        hid = layer.hidden
        meta = recv[:, hid:].view(torch.int32)
        return self.local(recv[:, :hid].contiguous(), meta, layer, k, meta_stride=recv.shape[1] // 2)

    def unpack(self, back, pos, offsets, m, world):
        hid = back.shape[1]
        out = torch.empty((m, hid), dtype=torch.bfloat16, device=pos.device)
        call("moek_ep_unpack", ops._ptr(back), ops._ptr(pos), ops._ptr(offsets), m, hid, world, ops._ptr(out),
             ops._stream(pos.device))
        return out


class _DeviceBuffer:
    """A raw device range seen by torch (``__cuda_array_interface__``), without copying or owning it."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2}


class PeerExchange:
    """Fixed-capacity exchange blocks in every rank's memory, shared by CUDA IPC (plain peer loads and stores over
    NVLink, no multicast objects), for ``ep_moe(..., capacity=True, peer=...)``: each rank's rows, slot ids and router
    weights are written straight into the owners' receive segments (``moek_ep_dispatch_p2p``), the owners' fp32
    partial rows into their own back buffers, where the senders read them over NVLink (by the whole-layer kernel itself,
    ``moek_moe_layer_p2p``, or by ``moek_ep_combine_p2p`` after the multi-launch path), and flags hand each segment
    over. Every rank of ``group`` builds it together (one all_gather of the IPC handles) for up to ``mcap`` tokens per
    call of ``top_k`` slots and hidden size ``hidden``; ``close()`` (collective) releases it."""

    def __init__(self, group, mcap: int, hidden: int, top_k: int, device):
        import ctypes

        self.group, self.mcap, self.hidden, self.top_k = group, mcap, hidden, top_k
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        offs = (ctypes.c_int64 * 7)()
        call("moek_ep_p2p_layout", self.world, mcap, hidden, top_k, offs)
        self.layout = dict(zip(("x", "ids", "w", "back", "flags", "ctr", "total"), list(offs)))
        own = ctypes.c_void_p()
        with torch.cuda.device(device):
            call("moek_ipc_malloc", self.layout["total"], ctypes.byref(own))
            handle = (ctypes.c_char * 64)()
            call("moek_ipc_handle", own, handle)
        self.own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        bases, self.opened = [], []
        with torch.cuda.device(device):
            for r in range(self.world):
                if r == self.rank:
                    bases.append(self.own)
                    continue
                ptr = ctypes.c_void_p()
                call("moek_ipc_open", (ctypes.c_char * 64).from_buffer_copy(handles[r]), ctypes.byref(ptr))
                self.opened.append(ptr.value)
                bases.append(ptr.value)
        self.peer = torch.tensor(bases, dtype=torch.int64, device=device)
        rows, lay = self.world * mcap, self.layout
        view = lambda off, shape, typestr: torch.as_tensor(_DeviceBuffer(self.own + off, shape, typestr),
                                                           device=device)
        self.recv_x = view(lay["x"], (rows, hidden), "<i2").view(torch.bfloat16)
        self.recv_ids = view(lay["ids"], (rows, top_k), "<i4")
        self.recv_w = view(lay["w"], (rows, top_k), "<f4")
        self.back = view(lay["back"], (rows, hidden), "<f4")
        self.flags = self.own + lay["flags"]
        self.err = ops.error_word(device)
        self.device = device

    def close(self):
        """Collective: every rank unmaps its peers' blocks, then frees its own once all ranks have unmapped."""
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for ptr in self.opened:
                call("moek_ipc_close", ptr)
            dist.barrier(group=self.group)
            call("moek_ipc_free", self.own)
        self.own, self.opened = None, []


def _ep_moe_peer(x, layer: EPLayer, w, ids32, px: PeerExchange, be) -> torch.Tensor:
    """The fixed-capacity layer over peer memory (``PeerExchange``): no collective library call. One launch when the
    received rows fit the whole-layer kernel (it dispatches, computes and unpacks itself; three launches, dispatch,
    layer, unpack, with ``MOEK_B200_EP_FUSED=0`` or ``be.record``), else dispatch, wait, the local layer's kernels,
    combine, unpack. With ``be.record`` a list, a copy of the received batch (rows, slot metadata as in
    ``CudaBackend.local``, metadata row stride) is appended to it, taken before the unpack lets the senders write
    again."""
    m, hid = x.shape
    k = ids32.shape[1]
    dev = x.device
    if x.dtype != torch.bfloat16:
        raise MoekError(f"moek_b200: hidden states must be bf16 (got {x.dtype})")
    if m > px.mcap or k != px.top_k or hid != px.hidden:
        raise MoekError(f"moek_b200: the peer exchange holds {px.mcap} tokens of {px.top_k} slots and width "
                        f"{px.hidden} (call: {m}, {k}, {hid})")
    st = ops._stream(dev)
    head = (ops._ptr(px.peer), px.world, px.rank, px.mcap, hid, k)
    pos = torch.empty((m, px.world), dtype=torch.int32, device=dev)
    fits = ops.layer_p2p_fits(px.world * px.mcap, k)
    if fits and getattr(be, "record", None) is None and os.environ.get("MOEK_B200_EP_FUSED", "1") != "0":
        out = torch.empty((m, hid), dtype=torch.bfloat16, device=dev)
        ops.layer_ep(px, layer.prep, x, ids32, w, layer.num_experts, pos, out)
        return out
    call("moek_ep_dispatch_p2p", *head, ops._ptr(x), ops._ptr(ids32), ops._ptr(w), m, layer.num_experts,
         ops._ptr(pos), ops._ptr(px.err), st)
    if getattr(be, "record", None) is not None:
        call("moek_ep_wait", px.flags, px.world, ops._ptr(px.err), st)
        be.record.append((px.recv_x.clone(), torch.cat([px.recv_ids, px.recv_w.view(torch.int32)], 1), 2 * k))
    if fits:
        ops.layer_p2p(px, layer.prep)
    else:
        call("moek_ep_wait", px.flags, px.world, ops._ptr(px.err), st)
        rows = ops.moe_rows(px.recv_x, layer.prep, px.recv_w, px.recv_ids)
        call("moek_ep_combine_p2p", *head, ops._ptr(rows), layer.local_experts, ops._ptr(px.err), st)
    out = torch.empty((m, hid), dtype=torch.bfloat16, device=dev)
    call("moek_ep_unpack_p2p", *head, ops._ptr(pos), m, ops._ptr(out), ops._ptr(px.err), st)
    return out


def meta_columns(top_k: int) -> int:
    """bf16 columns that hold a row's 2 * top_k int32 of slot metadata in a merged send buffer (a multiple of 8, so
    rows stay 16-byte aligned)."""
    return (4 * top_k + 7) // 8 * 8


_OFFSETS: dict = {}


def ep_moe(hidden_states: torch.Tensor, layer: EPLayer, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
           group=None, backend=None, capacity: bool = False, peer: PeerExchange = None) -> torch.Tensor:
    """This rank's tokens through the expert-parallel layer: bf16 [M, H], the same result as ``ops.fused_moe`` on
    one GPU holding all experts (up to the order of fp32 additions). ``topk_ids`` are global expert ids.

    ``capacity=False``: all-to-allv with exact row counts (the counts cross to the host once per call).
    ``capacity=True``: every rank reserves M rows for every destination (M = this call's token count, the same on
    all ranks), so the exchange has fixed sizes and no host synchronisation; unused rows carry invalid slot ids and
    are skipped by the kernels. Suited to decode batches, where the rows are few and the latency matters. With
    ``peer`` (a ``PeerExchange`` of this group), the fixed-capacity exchange runs over peer memory instead of NCCL:
    rows, ids, weights and partials are written straight into the other ranks' blocks by this build's kernels.

    Every rank of ``group`` must call this for the same layer with the same mode (the collectives pair up in call
    order)."""
    be = backend or CudaBackend()
    world = dist.get_world_size(group)
    if world != layer.world:
        raise MoekError(f"moek_b200: layer sharded for {layer.world} ranks, process group has {world}")
    x = hidden_states.contiguous()
    m, hid = x.shape
    k = topk_ids.shape[1]
    ids32 = topk_ids.to(torch.int32).contiguous()
    w = topk_weights.float().contiguous()
    if capacity and peer is not None:
        if peer.world != world or peer.rank != dist.get_rank(group):
            raise MoekError(f"moek_b200: the peer exchange was built for rank {peer.rank} of {peer.world}, this call "
                            f"is rank {dist.get_rank(group)} of {world}")
        return _ep_moe_peer(x, layer, w, ids32, peer, be)
    pos, counts, offsets = be.plan(ids32, layer.num_experts, world)
    if capacity:
        key = (m, world, pos.device)
        offsets = _OFFSETS.get(key)
        if offsets is None:
            offsets = _OFFSETS[key] = torch.arange(world + 1, dtype=torch.int32, device=pos.device) * m
        if hasattr(be, "local_merged"):  # rows and metadata in one buffer: one all-to-all each way
            send = be.pack(x, ids32, w, pos, offsets, layer.num_experts, world, world * m, counts=counts,
                           merged=True)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=group)
            partial = be.local_merged(recv, layer, k)
        else:
            send_x, send_meta = be.pack(x, ids32, w, pos, offsets, layer.num_experts, world, world * m,
                                        counts=counts, fill=True)
            recv_x, recv_meta = torch.empty_like(send_x), torch.empty_like(send_meta)
            dist.all_to_all_single(recv_x, send_x, group=group)
            dist.all_to_all_single(recv_meta, send_meta, group=group)
            partial = be.local(recv_x, recv_meta, layer, k)
        back = torch.empty_like(partial)
        dist.all_to_all_single(back, partial, group=group)
        return be.unpack(back, pos, offsets, m, world)
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    send = [int(c) for c in counts.tolist()]
    recv = [int(c) for c in recv_counts.tolist()]
    send_x, send_meta = be.pack(x, ids32, w, pos, offsets, layer.num_experts, world, sum(send))
    recv_x = torch.empty((sum(recv), hid), dtype=send_x.dtype, device=send_x.device)
    recv_meta = torch.empty((sum(recv), 2 * k), dtype=torch.int32, device=send_meta.device)
    dist.all_to_all_single(recv_x, send_x, recv, send, group=group)
    dist.all_to_all_single(recv_meta, send_meta, recv, send, group=group)
    partial = be.local(recv_x, recv_meta, layer, k)
    back = torch.empty((sum(send), hid), dtype=torch.float32, device=partial.device)
    dist.all_to_all_single(back, partial, send, recv, group=group)
    return be.unpack(back, pos, offsets, m, world)
