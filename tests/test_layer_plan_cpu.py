"""The whole-layer decode kernel's stream-K plan (``SKPlan`` in csrc/moek_layer.cu), restated on the CPU with exact
integer division, and checked for the properties the kernel relies on:

- the gate_up stages of every (block, gate_up item) pair are cut into contiguous non-empty ranges, one per CTA below
  C1 = min(C, S1), and every stage is streamed by exactly one CTA;
- a CTA's gate_up units are the pairs its range meets, in order, each writing one record; record indices
  (CTA + pair) are unique and below grid + pairs, the records the workspace holds;
- the down items of every pair are cut the same way over all C CTAs, each (pair, item) streamed once;
- a down unit's contributors [c0, c1] are exactly the CTAs whose gate_up ranges meet its pair (at most H / 128 of
  them), found by ``owner1``'s float estimate plus one correction each way;
- ``div_small``'s quotient estimate (v times an approximate reciprocal of d) is within one of the exact quotient over
  its stated range, so its single correction step gives the exact result.
"""
import itertools

import numpy as np
import pytest


class Plan:
    """SKPlan with exact division (div_small's contract)."""

    def __init__(self, nblk, nt1, nst1, nt2, C):
        self.npairs, self.nt1, self.nst1, self.nt2, self.C = nblk * nt1, nt1, nst1, nt2, C
        self.s1 = self.npairs * nst1
        self.c1n = min(C, self.s1)
        self.q1, self.r1 = divmod(self.s1, self.c1n) if self.c1n else (0, 0)
        self.s2 = self.npairs * nt2
        self.q2, self.r2 = divmod(self.s2, C)

    def lo1(self, c):
        c = min(c, self.c1n)
        return c * self.q1 + (c * self.r1) // self.c1n if self.c1n else 0

    def lo2(self, c):
        return c * self.q2 + (c * self.r2) // self.C

    def owner1(self, q):
        est = int(np.float32(np.float32(q + 1) * np.float32(self.c1n)) / np.float32(self.s1))
        c = min(max(est, 0), self.c1n - 1)
        if c + 1 < self.c1n and self.lo1(c + 1) <= q:
            c += 1
        if self.lo1(c) > q:
            c -= 1
        return c

    def n_gate(self, c):
        a, b = self.lo1(c), self.lo1(c + 1)
        return (b - 1) // self.nst1 - a // self.nst1 + 1 if b > a else 0

    def n_down(self, c):
        a, b = self.lo2(c), self.lo2(c + 1)
        return (b - 1) // self.nt2 - a // self.nt2 + 1 if b > a else 0

    def unit(self, c, j):
        ng = self.n_gate(c)
        if j < ng:
            a, b = self.lo1(c), self.lo1(c + 1)
            pr = a // self.nst1 + j
            s0 = pr * self.nst1
            st0 = max(a - s0, 0)
            return dict(ph=0, pair=pr, st0=st0, nst=min(b - s0, self.nst1) - st0, rec=c + pr)
        a, b = self.lo2(c), self.lo2(c + 1)
        pr = a // self.nt2 + (j - ng)
        i0 = pr * self.nt2
        item = max(a - i0, 0)
        return dict(ph=1, pair=pr, item=item, nst=min(b - i0, self.nt2) - item,
                    c0=self.owner1(pr * self.nst1), c1=self.owner1(pr * self.nst1 + self.nst1 - 1))


GEOMETRIES = [(2048, 512), (2048, 256), (4096, 512), (1024, 768)]  # (H, I)
BLOCKS = [1, 2, 3, 5, 8, 13, 39, 40, 77, 100, 200, 512]  # decode batches: at most 512 routed slots
GRIDS = [1, 2, 7, 148, 296, 1000]


@pytest.mark.parametrize("H,I", GEOMETRIES)
def test_plan_covers_every_stage_once(H, I):
    nt1, nst1, nt2 = 2 * I // 256, H // 128, H // 256
    for nblk, C in itertools.product(BLOCKS, GRIDS):
        p = Plan(nblk, nt1, nst1, nt2, C)
        # gate_up ranges: contiguous, non-empty below C1, empty from C1 on
        assert p.lo1(0) == 0 and p.lo1(C) == p.s1
        for c in range(C):
            if c < p.c1n:
                assert p.lo1(c + 1) > p.lo1(c)
            else:
                assert p.lo1(c + 1) == p.lo1(c) == p.s1
        gate_seen = np.zeros(p.s1, dtype=np.int32)
        down_seen = np.zeros(p.s2, dtype=np.int32)
        recs = set()
        meets = {}  # pair -> CTAs whose gate_up range meets it
        for c in range(C):
            prev_pair = -1
            for j in range(p.n_gate(c) + p.n_down(c)):
                u = p.unit(c, j)
                assert u["nst"] >= 1
                if u["ph"] == 0:
                    assert u["pair"] > prev_pair
                    prev_pair = u["pair"]
                    s = u["pair"] * nst1 + u["st0"]
                    assert 0 <= u["st0"] and u["st0"] + u["nst"] <= nst1
                    gate_seen[s:s + u["nst"]] += 1
                    assert u["rec"] not in recs and u["rec"] < C + p.npairs
                    recs.add(u["rec"])
                    meets.setdefault(u["pair"], []).append(c)
                else:
                    s = u["pair"] * nt2 + u["item"]
                    assert 0 <= u["item"] and u["item"] + u["nst"] <= nt2
                    down_seen[s:s + u["nst"]] += 1
        assert (gate_seen == 1).all(), (nblk, C)
        assert (down_seen == 1).all(), (nblk, C)
        # down units wait for exactly the CTAs that wrote the pair's records: a contiguous run of at most H/128
        for c in range(C):
            for j in range(p.n_gate(c), p.n_gate(c) + p.n_down(c)):
                u = p.unit(c, j)
                writers = meets[u["pair"]]
                assert writers == list(range(u["c0"], u["c1"] + 1)), (nblk, C, u)
                assert len(writers) <= nst1


@pytest.mark.parametrize("H,I", GEOMETRIES)
def test_owner_estimate_is_corrected(H, I):
    """owner1 returns the CTA whose range holds stage q for every q (the float estimate may be off by one)."""
    nt1, nst1, nt2 = 2 * I // 256, H // 128, H // 256
    for nblk, C in itertools.product(BLOCKS, GRIDS):
        p = Plan(nblk, nt1, nst1, nt2, C)
        for q in range(0, p.s1, max(1, p.s1 // 2000)):
            c = p.owner1(q)
            assert p.lo1(c) <= q < p.lo1(c + 1), (nblk, C, q)


def test_plan_arithmetic_stays_in_div_small_range():
    """The kernel evaluates lo1/lo2 as c q + floor(c r / C) with div_small, valid for v < 2^22 and d <= 2^10: the
    largest decode batch (512 slots, so at most 512 blocks) on the largest grid keeps every operand in range."""
    for H, I in GEOMETRIES:
        nt1, nst1, nt2 = 2 * I // 256, H // 128, H // 256
        for C in (1024,):
            p = Plan(512, nt1, nst1, nt2, C)
            assert C * max(p.r1, p.r2) < 2 ** 22
            assert p.s1 < 2 ** 22 and p.s2 < 2 ** 22
            assert max(nst1, nt1, nt2) <= 2 ** 10


def test_div_small_estimate_within_one():
    """div_small: q = trunc(v * rcp(d)) with the approximate reciprocal (modelled as the correctly rounded fp32 1/d
    perturbed by up to 2 ulp either way), then one correction each way, equals v // d for 0 <= v < 2^22, 1 <= d <=
    2^10."""
    rng = np.random.default_rng(7)
    v = np.concatenate([np.arange(0, 4096), rng.integers(0, 2 ** 22, 200_000), [2 ** 22 - 1]]).astype(np.int64)
    for d in list(range(1, 1025, 7)) + [16, 32, 64, 256, 296, 1000, 1024]:
        exact = v // d
        r = np.float32(1.0) / np.float32(d)
        for ulp in (-2, -1, 0, 1, 2):
            rr = np.float32(r * np.float32(1.0 + ulp * 2.0 ** -23))
            q = np.trunc(v.astype(np.float32) * rr).astype(np.int64)
            assert np.abs(q - exact).max() <= 1, (d, ulp)
            rem = v - q * d
            q = q + (rem >= d) - (rem < 0)
            assert (q == exact).all(), (d, ulp)
