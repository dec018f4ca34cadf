"""bench.py's host-side helpers, on the CPU: the packed staging layout of one layer's inputs (x | ids | weights) that
the end-to-end measurement copies in one piece, and the step's block of such segments (16-byte aligned rows)."""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_pack_unpack_round_trip_in_a_step_block():
    m, k = 8, bench.TOPK
    g = torch.Generator().manual_seed(3)
    xs = [torch.randn((m, bench.H), generator=g).to(torch.bfloat16) for _ in range(3)]
    ids = [torch.randint(-1, 512, (m, k), generator=g, dtype=torch.int32) for _ in range(3)]
    ws = [torch.rand((m, k), generator=g) for _ in range(3)]
    packed = [bench.pack_inputs(x, i, w) for x, i, w in zip(xs, ids, ws)]
    assert packed[0].numel() == m * bench.H * 2 + 2 * m * k * 4
    seg = (packed[0].numel() + 15) // 16 * 16
    block = torch.zeros((3, seg), dtype=torch.uint8)
    for l, t in enumerate(packed):
        block[l, :t.numel()].copy_(t)
    for l in range(3):
        row = block[l, :packed[l].numel()]
        assert row.storage_offset() % 16 == 0  # x starts 16-byte aligned in every segment
        x, i, w = bench.unpack_inputs(row, m)
        assert torch.equal(x, xs[l]) and torch.equal(i, ids[l]) and torch.equal(w, ws[l])
