"""CPU restatement of the expert-parallel dispatch / combine index work (test infrastructure only).

The reference has no expert parallelism (its hook rejects ``expert_map``, files/mbx_moek.py:248-255); this is the
specification the build's EP kernels (``moek_ep_plan`` / ``moek_ep_pack`` / ``moek_ep_partial`` / ``moek_ep_unpack``)
are checked against, written as plain loops and numpy:

- experts split contiguously: rank d owns [d * E / world, (d + 1) * E / world);
- a token goes once to every rank owning at least one of its top-k experts; within a destination's segment tokens
  are in ascending order; ids outside [0, E) go nowhere;
- a sent row carries k local ids (-1 for slots owned elsewhere) and k router weights (0 for those slots);
- the receiving rank sums its slots' rows (the oracle's per-slot rows) in slot order, in fp32;
- the source rank adds the returned partials in rank order, in fp32, and the caller rounds once to bf16.
"""
import numpy as np
import torch

from . import moe_ref


def plan(topk_ids, num_experts: int, world: int):
    """(pos int32 [M, world], counts int32 [world], offsets int32 [world + 1])."""
    ids = np.asarray(topk_ids, dtype=np.int64)
    m = ids.shape[0]
    per = num_experts // world
    pos = np.full((m, world), -1, dtype=np.int32)
    counts = np.zeros(world, dtype=np.int32)
    for t in range(m):
        dests = set()
        for e in ids[t]:
            if 0 <= e < num_experts:
                dests.add(int(e) // per)
        for d in sorted(dests):
            pos[t, d] = counts[d]
            counts[d] += 1
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return pos, counts, offsets


def pack(x, topk_ids, topk_w, pos, offsets, num_experts: int, world: int):
    """(send_x [S, H] same dtype as x, send_meta int32 [S, 2k])."""
    ids = np.asarray(topk_ids, dtype=np.int64)
    w = np.asarray(topk_w, dtype=np.float32)
    m, k = ids.shape
    per = num_experts // world
    s = int(offsets[-1])
    send_x = torch.empty((s, x.shape[1]), dtype=x.dtype)
    meta = np.zeros((s, 2 * k), dtype=np.int32)
    for t in range(m):
        for d in range(world):
            p = pos[t, d]
            if p < 0:
                continue
            row = int(offsets[d]) + int(p)
            send_x[row] = x[t]
            for j in range(k):
                e = ids[t, j]
                mine = 0 <= e < num_experts and e // per == d
                meta[row, j] = e - d * per if mine else -1
                meta[row, k + j] = np.float32(w[t, j] if mine else 0.0).view(np.int32)
    return send_x, torch.from_numpy(meta)


def partial(x_recv, meta, w13_local, w2_local, k: int) -> torch.Tensor:
    """fp32 [R, H]: the received rows' local slots (the oracle's slot rows), summed in slot order."""
    r, hid = x_recv.shape
    meta = np.asarray(meta, dtype=np.int32).reshape(r, 2 * k)
    ids = meta[:, :k]
    w = meta[:, k:].copy().view(np.float32)
    y = moe_ref.slot_rows(x_recv, ids, w, w13_local, w2_local).view(r, k, hid)
    out = torch.zeros((r, hid), dtype=torch.float32)
    for j in range(k):
        out += y[:, j]
    return out


def unpack(back, pos, offsets, m: int, world: int) -> torch.Tensor:
    """fp32 [M, H]: per token, the returned partials added in rank order."""
    hid = back.shape[1]
    out = torch.zeros((m, hid), dtype=torch.float32)
    for t in range(m):
        for d in range(world):
            p = pos[t, d]
            if p >= 0:
                out[t] += back[int(offsets[d]) + int(p)]
    return out
