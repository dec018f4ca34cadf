"""A model check of the flag protocol of the peer-memory EP exchange, on the CPU.

The protocol lives in csrc/moek_ep.cu (ep_dispatch_p2p_kernel, ep_wait_kernel, ep_combine_p2p_kernel,
ep_unpack_p2p_kernel) and csrc/moek_layer.cu (the whole-layer kernel's receive-flag wait and ep_signal). Per layer, on
every rank's stream: dispatch, then either the whole-layer kernel (fused) or wait + local layer + combine, then
unpack. The kernels of one rank run in stream order; the CTAs of one kernel run concurrently. This test models each
kernel as concurrent sub-tasks made of the protocol's waits and actions on the flags and on generation-tagged
segments, runs every rank's program under many random schedules (sequentially consistent interleavings), and checks:

- progress: some step is always runnable until every rank has finished its layers (no deadlock);
- freshness: every read of a receive or back segment sees the data of the current layer;
- no overwrite: nobody writes a segment before its reader has consumed the previous layer's data.

It checks the protocol's logic, not the memory ordering of the CUDA code (the kernels publish with fences and
system-scope release stores and read after acquire loads). Planted mistakes (a missing wait, a missing reset, a flag
raised before its data is written) must be caught, so the checker is known to bite. Clearing the receive flags at the
start of unpack is safe: unpack starts only after the layer's readers have completed (stream order), and a sender
cannot dispatch the next layer before its own unpack has seen this rank's back flag anyway.
"""
import random

import pytest


class Violation(AssertionError):
    pass


class State:
    def __init__(self, world):
        w = range(world)
        self.world = world
        self.recv_flag = [[0] * world for _ in w]  # [owner][sender]
        self.back_flag = [[0] * world for _ in w]  # [owner][returner]
        self.recv_gen = [[0] * world for _ in w]
        self.recv_read = [[0] * world for _ in w]
        self.back_gen = [[0] * world for _ in w]
        self.back_read = [[0] * world for _ in w]


def _program(st: State, r: int, layers: int, fused: bool, plant: str):
    """Rank r's kernels, each a list of sub-tasks (concurrent CTAs), each a list of steps. A step is ("wait", cond)
    or ("do", action)."""
    W = st.world
    kernels = []
    for L in range(1, layers + 1):
        # dispatch: CTA d resets my back flag d, waits for d's receive flag for me to be 0, writes, raises it
        dispatch = []
        for d in range(W):
            steps = []
            if plant != "dispatch_no_reset":
                steps.append(("do", lambda d=d: st.back_flag[r].__setitem__(d, 0)))
            if plant != "dispatch_no_wait":
                steps.append(("wait", lambda d=d: st.recv_flag[d][r] == 0))

            def write(d=d, L=L):
                if st.recv_read[d][r] != L - 1:
                    raise Violation(f"rank {r} overwrote rank {d}'s receive segment before layer {L - 1} was read")
                st.recv_gen[d][r] = L

            steps.append(("do", write))
            steps.append(("do", lambda d=d: st.recv_flag[d].__setitem__(r, 1)))
            dispatch.append(steps)
        kernels.append(dispatch)

        def read_all(L=L):
            for s in range(W):
                if st.recv_gen[r][s] != L:
                    raise Violation(f"rank {r} read a stale receive segment {s} in layer {L}")
                st.recv_read[r][s] = L

        def return_to(s, L=L):
            if st.back_read[s][r] != L - 1:
                raise Violation(f"rank {r} overwrote rank {s}'s back segment before layer {L - 1} was read")
            st.back_gen[s][r] = L

        recv_ready = ("wait", lambda: all(st.recv_flag[r][s] == 1 for s in range(W)))
        if fused:
            # the whole-layer kernel: wait, route + compute (reads every segment), return every row, then raise
            # every sender's back flag (the arrival that completes the last row)
            steps = [recv_ready, ("do", read_all)]
            returns = [("do", lambda s=s, f=return_to: f(s)) for s in range(W)]
            raises = [("do", lambda s=s: st.back_flag[s].__setitem__(r, 1)) for s in range(W)]
            steps += raises + returns if plant == "layer_signals_before_return" else returns + raises
            kernels.append([steps])
        else:
            kernels.append([[recv_ready]])  # ep_wait
            kernels.append([[("do", read_all)]])  # the local layer's kernels
            raise_back = lambda s: ("do", lambda: st.back_flag[s].__setitem__(r, 1))
            # combine: CTA s returns segment s and raises s's back flag
            kernels.append([[("do", lambda s=s, f=return_to: f(s)), raise_back(s)] for s in range(W)])

        # unpack: wait for every back flag, clear my receive flags (CTA 0), read the back segments (other CTAs)
        def read_back(L=L):
            for d in range(W):
                if st.back_gen[r][d] != L:
                    raise Violation(f"rank {r} read a stale back segment {d} in layer {L}")
                st.back_read[r][d] = L

        back_ready = ("wait", lambda: all(st.back_flag[r][d] == 1 for d in range(W)))
        clear = [("do", lambda s=s: st.recv_flag[r].__setitem__(s, 0)) for s in range(W)]
        unpack = [[back_ready] + clear, ([] if plant == "unpack_no_wait" else [back_ready]) + [("do", read_back)]]
        kernels.append(unpack)
    return kernels


def run_schedule(world, layers, fused, seed, plant=""):
    st = State(world)
    rng = random.Random(seed)
    progs = [_program(st, r, layers, fused, plant) for r in range(world)]
    kidx = [0] * world
    pcs = [[0] * len(progs[r][0]) for r in range(world)]
    steps = 0
    while True:
        runnable = []
        for r in range(world):
            if kidx[r] >= len(progs[r]):
                continue
            for t, task in enumerate(progs[r][kidx[r]]):
                pc = pcs[r][t]
                if pc < len(task) and (task[pc][0] == "do" or task[pc][1]()):
                    runnable.append((r, t))
        if not runnable:
            if all(kidx[r] >= len(progs[r]) for r in range(world)):
                return steps
            raise Violation(f"deadlock after {steps} steps (kernels at {kidx})")
        r, t = rng.choice(runnable)
        kind, fn = progs[r][kidx[r]][t][pcs[r][t]]
        if kind == "do":
            fn()
        pcs[r][t] += 1
        steps += 1
        if all(pc >= len(task) for pc, task in zip(pcs[r], progs[r][kidx[r]])):  # kernel complete: next in stream
            kidx[r] += 1
            if kidx[r] < len(progs[r]):
                pcs[r] = [0] * len(progs[r][kidx[r]])


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_protocol_progress_and_freshness(world, fused):
    for seed in range(300 if world <= 4 else 60):
        run_schedule(world, layers=6, fused=fused, seed=1000 * world + seed)


@pytest.mark.parametrize("plant", ["dispatch_no_wait", "dispatch_no_reset", "layer_signals_before_return",
                                   "unpack_no_wait"])
def test_planted_mistakes_are_caught(plant):
    """Each planted mistake leads, in some schedule, to a stale read, an overwrite or a deadlock."""
    caught = 0
    for seed in range(400):
        try:
            run_schedule(2, layers=4, fused=True, seed=seed, plant=plant)
        except Violation:
            caught += 1
    assert caught > 0, plant
