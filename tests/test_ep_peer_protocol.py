"""A model check of the flag protocol of the peer-memory EP exchange, on the CPU.

The protocol lives in csrc/moek_ep.cuh and csrc/moek_ep.cu (dispatch, ep_wait_kernel, ep_combine_p2p_kernel,
unpack) and csrc/moek_layer.cu (the whole-layer kernel's receive-flag wait and ep_signal). Per layer, on every rank's
stream: dispatch, then either the whole-layer kernel (fused) or wait + local layer + combine, then unpack; or one
launch of the whole-layer kernel whose CTAs dispatch, compute and unpack (one). The kernels of one rank run in stream
order; the CTAs of one kernel run concurrently. This test models each
kernel as concurrent sub-tasks made of the protocol's waits and actions on the flags and on generation-tagged
segments, runs every rank's program under many random schedules (sequentially consistent interleavings), and checks:

- progress: some step is always runnable until every rank has finished its layers (no deadlock);
- freshness: every read of a receive or back segment sees the data of the current layer;
- no overwrite: nobody writes a segment before its reader has consumed the previous layer's data.

The flags carry the call (layer) number L instead of 0/1, so nothing resets them and dispatch writes without
waiting: a sender dispatches call L only after its own unpack of call L - 1 has seen every owner's back flag for
L - 1, which each owner raised after it had read the sender's rows of L - 1.

It checks the protocol's logic, not the memory ordering of the CUDA code (the kernels publish with fences and
system-scope release stores and read after acquire loads). Planted mistakes (a flag raised before its data is
written, a back flag raised before the partials, an unpack that does not wait or that accepts the previous call's
flag, a 0/1 flag that is never reset) must be caught, so the checker is known to bite.
"""
import random

import pytest


class Violation(AssertionError):
    pass


class State:
    """Flags, arrival counters and the generation (layer number) of each part of each segment: part g of receive
    segment s on rank r is what CTA g of rank s's dispatch wrote; part j of back segment d is what piece j of rank
    d's layer (or CTA j of its combine) returned."""

    def __init__(self, world, parts):
        w = range(world)
        self.world, self.parts = world, parts
        grid = lambda: [[0] * world for _ in w]
        self.recv_flag, self.back_flag = grid(), grid()  # [owner][sender], [owner][returner]
        self.disp_ctr, self.comb_ctr, self.piece_ctr = grid(), grid(), [0] * world
        seg = lambda: [[[0] * parts for _ in w] for _ in w]
        self.recv_gen, self.recv_read, self.back_gen, self.back_read = seg(), seg(), seg(), seg()


def _program(st: State, r: int, layers: int, fused, plant: str):
    """Rank r's kernels, each a list of sub-tasks (concurrent CTAs or warps), each a list of steps. A step is
    ("wait", cond) or ("do", action). fused: False (wait, local layer, combine), True (the whole-layer kernel
    between dispatch and unpack) or "one" (dispatch, layer and unpack as the CTAs of one kernel)."""
    W, G = st.world, st.parts
    do = lambda f: ("do", f)
    kernels = []
    for L in range(1, layers + 1):
        # dispatch: CTA (d, g) writes its part of d's receive segment for me; the last of the G arrivals (a
        # self-resetting counter) sets d's receive flag for me to this call's number
        dispatch = []
        mark = (lambda L: 1) if plant == "binary_flags" else (lambda L: L)
        for d in range(W):
            for g in range(G):
                def write(d=d, g=g, L=L):
                    if st.recv_read[d][r][g] != L - 1:
                        raise Violation(f"rank {r} overwrote rank {d}'s receive segment before layer {L - 1} was read")
                    st.recv_gen[d][r][g] = L

                def arrive(d=d, L=L):
                    st.disp_ctr[r][d] += 1
                    if st.disp_ctr[r][d] == G:
                        st.disp_ctr[r][d] = 0
                        st.recv_flag[d][r] = mark(L)

                dispatch.append([do(arrive), do(write)] if plant == "flag_before_data" else [do(write), do(arrive)])
        kernels.append(dispatch)

        def read(s, g, L=L):
            if st.recv_gen[r][s][g] != L:
                raise Violation(f"rank {r} read a stale receive segment {s} in layer {L}")
            st.recv_read[r][s][g] = L

        def return_part(s, j, L=L):
            if st.back_read[s][r][j] != L - 1:
                raise Violation(f"rank {r} overwrote rank {s}'s back segment before layer {L - 1} was read")
            st.back_gen[s][r][j] = L

        def raise_all(L=L):
            for s in range(W):
                st.back_flag[s][r] = mark(L)

        recv_ready = ("wait", lambda L=L: all(st.recv_flag[r][s] == mark(L) for s in range(W)))
        read_all = [do(lambda s=s, g=g, f=read: f(s, g)) for s in range(W) for g in range(G)]
        if fused:
            # the whole-layer kernel: every CTA waits for the receive flags and routes (reads every segment); each
            # piece (a row's sum for one item) goes back to its sender; the arrival that completes the last piece
            # raises every sender's back flag (the kernel's other case, nothing to return, raises them right after
            # the wait and is not modelled)
            def piece_arrive(raise_all=raise_all):
                st.piece_ctr[r] += 1
                if st.piece_ctr[r] == W * G:
                    st.piece_ctr[r] = 0
                    raise_all()

            pieces = []
            for s in range(W):
                for j in range(G):
                    steps = [recv_ready] + read_all + [do(lambda s=s, j=j, f=return_part: f(s, j))]
                    pieces.append(steps + ([] if plant == "layer_signals_before_return" else [do(piece_arrive)]))
            if plant == "layer_signals_before_return":
                pieces.append([recv_ready, do(raise_all)])
            kernels.append(pieces)
        else:
            kernels.append([[recv_ready]])  # ep_wait
            kernels.append([read_all])  # the local layer's kernels

            def comb_arrive(s, L=L):
                st.comb_ctr[r][s] += 1
                if st.comb_ctr[r][s] == G:
                    st.comb_ctr[r][s] = 0
                    st.back_flag[s][r] = mark(L)

            # combine: CTA (s, j) returns part j of segment s; the last of the G arrivals raises s's back flag
            kernels.append([[do(lambda s=s, j=j, f=return_part: f(s, j)), do(lambda s=s, c=comb_arrive: c(s))]
                            for s in range(W) for j in range(G)])

        # unpack: every CTA waits until the back flags carry this call's number, then reads the back segments (the
        # last CTA advancing the completed-call count is the L + 1 of the next call's closures)
        def read_back(d, j, L=L):
            if st.back_gen[r][d][j] != L:
                raise Violation(f"rank {r} read a stale back segment {d} in layer {L}")
            st.back_read[r][d][j] = L

        if plant == "unpack_no_wait":
            back_ready = []
        elif plant == "unpack_accepts_previous":
            back_ready = [("wait", lambda L=L: all(st.back_flag[r][d] >= L - 1 for d in range(W)))]
        else:
            back_ready = [("wait", lambda L=L: all(st.back_flag[r][d] == mark(L) for d in range(W)))]
        unpack = [back_ready + [do(lambda d=d, j=j, f=read_back: f(d, j))] for d in range(W) for j in range(G)]
        kernels.append(unpack)
        if fused == "one":  # dispatch, layer and unpack: the concurrent CTAs of one launch
            kernels[-3:] = [kernels[-3] + kernels[-2] + kernels[-1]]
    return kernels


def run_schedule(world, layers, fused, seed, plant="", parts=1):
    st = State(world, parts)
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


@pytest.mark.parametrize("parts", [1, 3])
@pytest.mark.parametrize("fused", [True, False, "one"])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_protocol_progress_and_freshness(world, fused, parts):
    """parts: CTAs per peer in dispatch and combine, and pieces per sender in the whole-layer kernel."""
    n = (200 if world <= 4 else 30) // parts
    for seed in range(n):
        run_schedule(world, layers=5, fused=fused, seed=1000 * world + seed, parts=parts)


@pytest.mark.parametrize("fused", [True, "one"])
@pytest.mark.parametrize("plant", ["flag_before_data", "binary_flags", "layer_signals_before_return",
                                   "unpack_no_wait", "unpack_accepts_previous"])
def test_planted_mistakes_are_caught(plant, fused):
    """Each planted mistake leads, in some schedule, to a stale read, an overwrite or a deadlock."""
    caught = 0
    for seed in range(400):
        try:
            run_schedule(2, layers=4, fused=fused, seed=seed, plant=plant, parts=2)
        except Violation:
            caught += 1
    assert caught > 0, plant
