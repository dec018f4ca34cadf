"""Torch-facing operators over the C ABI, with the reference's names and argument lists.

- ``moe_align_block_size``: vLLM's wrapper signature (vllm/model_executor/layers/fused_moe/moe_align_block_size.py:
  11-18, buffer sizes :74-88), backed by this build's kernel instead of ``torch.ops._moe_C``.
- ``moe_gemm`` / ``moe_split_epilogue``: the kit's extension functions (files/mbx_moek.cu:717-721,835-836).
- ``fused_moe``: the body of the kit's forward wrap (files/mbx_moek.py:236-289): align -> gate_up -> epilogue -> down
  -> epilogue fused with the top-k sum.

Every tensor must already live on a CUDA device; there is no CPU path. Errors raise ``MoekError`` (a RuntimeError),
like the reference's TORCH_CHECK failures.
"""
import os

import torch

from . import _lib
from ._lib import MoekError, call
from .prep import PreparedLayer

BM = 96  # moe_align block size (rows per block) of the decode path, as the kit (files/mbx_moek.py:33)
BM_PREFILL = 128  # block size of the tcgen05 path (the MMA's N, at most)
LAUNCHES_PER_LAYER = 1  # decode: the whole layer (routing, gate_up + SwiGLU, down, top-k sum) is one kernel
_BUF: dict = {}
_PROF = None  # when a list, fused_moe appends (name, launch closure) for each of its GEMM launches


def _ptr(t):
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise MoekError("moek_b200: tensors must be on a CUDA device (no CPU implementation)")


def error_word(dev) -> torch.Tensor:
    """Per-device int32 [65536], zero-filled (the size of the kit's cnt buffer, files/mbx_moek.py:179): [0] is the
    kernels' device error word (MOEK_DEV_*), [1..] the split-k arrival counters, which every launch leaves at 0."""
    key = ("cnt", torch.device(dev))
    if key not in _BUF:
        _BUF[key] = torch.zeros(1 << 16, dtype=torch.int32, device=dev)
    return _BUF[key]


def check_device_errors(dev) -> None:
    """Synchronises and raises if a kernel recorded a device-side error (timeout, bad expert id, too many rows)."""
    w = error_word(dev)
    code = int(w[0].item())
    if code:
        w.zero_()  # an aborted launch may also have left split counters behind
        for key, t in _BUF.items():  # and the whole-layer kernel's counters and record flags
            if key[0] == "layer_state" and key[1] == torch.device(dev):
                t.zero_()
        names = {1: "a bounded wait timed out", 2: "an expert id out of range", 3: "a block with more rows than "
                 "max_rows", 4: "an input index out of range (debug checks)"}
        raise MoekError(f"moek_b200: device error {code}: {names.get(code, 'unknown')}")


def _scratch(name: str, numel: int, dtype, dev) -> torch.Tensor:
    key = (name, torch.device(dev), dtype)
    t = _BUF.get(key)
    if t is None or t.numel() < numel:
        t = _BUF[key] = torch.empty(max(numel, 1), dtype=dtype, device=dev)
    return t


# ---------------------------------------------------------------------------------------------------- moe_align
def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int, expert_map=None,
                         pad_sorted_ids: bool = False, ignore_invalid_experts: bool = False):
    """(sorted_ids, expert_ids, num_tokens_post_pad) with vLLM's contract; ids outside [0, E) are always skipped."""
    if expert_map is not None:
        raise MoekError("moek_b200: expert_map is not supported by moe_align (use qwen38_flash_coder_b200.ep)")
    _need_cuda(topk_ids)
    ids = topk_ids.reshape(-1)
    if ids.dtype != torch.int32:
        ids = ids.to(torch.int32)
    ids = ids.contiguous()
    numel = ids.numel()
    n = numel + num_experts * (block_size - 1)
    if pad_sorted_ids:
        n = (n + block_size - 1) // block_size * block_size
    if numel < num_experts:
        n = min(numel * block_size, n)
    dev = ids.device
    sorted_ids = torch.empty(n, dtype=torch.int32, device=dev)
    expert_ids = torch.empty((n + block_size - 1) // block_size, dtype=torch.int32, device=dev)
    npad = torch.empty(1, dtype=torch.int32, device=dev)
    import ctypes

    wsb = ctypes.c_size_t(0)
    call("moek_align_workspace_bytes", numel, num_experts, ctypes.byref(wsb))
    ws = _scratch("align_ws", (wsb.value + 3) // 4, torch.int32, dev) if wsb.value else None
    call("moek_align", _ptr(ids), numel, num_experts, block_size, _ptr(sorted_ids), sorted_ids.numel(),
         _ptr(expert_ids), expert_ids.numel(), _ptr(npad), _ptr(ws), wsb.value, _stream(dev))
    return sorted_ids, expert_ids, npad


# ------------------------------------------------------------------------------------------------------ moe_gemm
def moe_gemm(A, W, S, G, sorted_ids, expert_ids, num_post_pad, topk_w, out, top_k: int, gate_up: bool, SP, exc_off,
             exc_ent, ws, cnt, mode: int, nsplit: int, part, order: int = 0, tiled: bool = True, *,
             block_m: int = BM, max_rows: int = 0) -> None:
    """The kit's moe_gemm argument list (files/mbx_moek.cu:717-721). ``ws`` and ``order`` are accepted and unused;
    ``S`` must be empty (packed scales only); ``cnt``'s first int32 receives device error codes.

    Modes with the reference's meaning: 0 and 1 (the kit's prefill call, files/mbx_moek.py:276-283; the reference's
    item counter and stream-k schedules are one tcgen05 schedule here): gate_up writes act bf16 [num_ids, N/2] to
    ``out``, down writes dout bf16 [num_ids, N] = bf16(topk_w * sum) to ``out``; 2 (the kit's decode call): split-k
    fp32 partials into ``part``, finished by ``moe_split_epilogue``. This build's own modes: 3 (split-k with fused
    epilogues), 4 (tcgen05, down writes fp32 rows topk_w * sum to ``part`` for ``combine``), 5 (as 4, act rows in
    moe_align's sorted order)."""
    _need_cuda(A, W, G, sorted_ids, SP, part)
    if S is not None and S.numel():
        raise MoekError("moek_b200: plain Marlin scales are not supported; pass the packed SP")
    k = A.shape[1]
    n = W.shape[2] // 2
    num_ids = out.shape[0]  # act [num_ids, N/2] or dout [num_ids, N], as the reference sizes the call
    if max_rows <= 0:
        m_tok = num_ids // top_k if gate_up else num_ids
        max_rows = min(block_m, max(1, m_tok))
    call("moek_gemm", _ptr(A), _ptr(W), None, _ptr(G), _ptr(sorted_ids), sorted_ids.numel(), _ptr(expert_ids),
         _ptr(num_post_pad), _ptr(topk_w), _ptr(out), num_ids, n, k, W.shape[0], top_k, int(bool(gate_up)), _ptr(SP),
         _ptr(exc_off), _ptr(exc_ent), _ptr(cnt), cnt.numel(), mode, nsplit, _ptr(part), part.numel(), int(tiled),
         block_m, min(max_rows, 96), None, 0, _stream(A.device))


def moe_split_epilogue(part, nsplit: int, topk_ids, G, topk_w, out, gate_up: bool, N: int) -> None:
    """The kit's moe_split_epilogue argument list (files/mbx_moek.cu:835-836). ``G`` is accepted and unused (the
    global scale is already inside the dequantised weights). Down: ``out`` fp32 [num_ids, N] receives the weighted
    rows; ``out`` bf16 [num_ids / top_k, N] the rows already summed over each token's top_k slots."""
    _need_cuda(part, out)
    num_ids = topk_ids.numel()
    top_k = topk_ids.shape[-1] if topk_ids.dim() > 1 else 1
    if gate_up:
        call("moek_split_epilogue", _ptr(part), nsplit, num_ids, N, 1, None, top_k, _ptr(out), 0, _stream(out.device))
        return
    if out.dtype == torch.float32 and out.shape[0] == num_ids:
        kind = 1
    elif out.dtype == torch.bfloat16 and out.shape[0] * top_k == num_ids:
        kind = 2
    else:
        raise MoekError("moek_b200: down epilogue writes fp32 [num_ids, N] rows or the bf16 [M, N] top-k sum")
    call("moek_split_epilogue", _ptr(part), nsplit, num_ids, N, 0, _ptr(topk_w), top_k, _ptr(out), kind,
         _stream(out.device))


def combine(rows: torch.Tensor, top_k: int, out: torch.Tensor = None) -> torch.Tensor:
    """Top-k sum of per-slot rows [M * top_k, N] (fp32 or bf16) -> bf16 [M, N] (files/mbx_moek.py:284-289)."""
    _need_cuda(rows)
    m = rows.shape[0] // top_k
    n = rows.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=rows.device)
    call("moek_combine", _ptr(rows), int(rows.dtype == torch.float32), _ptr(out), m, n, top_k, _stream(rows.device))
    return out


# ------------------------------------------------------------------------------------------------------ router
def fused_topk(hidden_states: torch.Tensor, gating_output: torch.Tensor, topk: int, renormalize: bool,
               indices_type=None, scoring_func: str = "softmax"):
    """vLLM's ``fused_topk`` (vllm/.../router/fused_topk_router.py:69-108) on this build's router kernel:
    (topk_weights fp32 [M, k], topk_ids int32 (or ``indices_type``) [M, k], token_expert_indices int32 [M, k])."""
    if scoring_func != "softmax":
        raise MoekError(f"moek_b200: router scoring {scoring_func!r} is not supported (softmax only)")
    if hidden_states.shape[0] != gating_output.shape[0]:
        raise MoekError("moek_b200: number of tokens mismatch between hidden states and router logits")
    w, ids, tei = router_topk(gating_output, topk, renormalize, with_indices=True)
    if indices_type is not None and indices_type != torch.int32:
        ids = ids.to(indices_type)
    return w, ids, tei


def router_topk(logits: torch.Tensor, top_k: int, renormalize: bool = True, with_indices: bool = False):
    """softmax -> top-k -> renormalise on the GPU: (weights fp32 [M, k], ids int32 [M, k][, token_expert_indices])."""
    _need_cuda(logits)
    if logits.dtype not in (torch.float32, torch.bfloat16):
        logits = logits.float()
    logits = logits.contiguous()
    m, e = logits.shape
    dev = logits.device
    ids = torch.empty((m, top_k), dtype=torch.int32, device=dev)
    w = torch.empty((m, top_k), dtype=torch.float32, device=dev)
    tei = torch.empty((m, top_k), dtype=torch.int32, device=dev) if with_indices else None
    call("moek_router_topk", _ptr(logits), int(logits.dtype == torch.bfloat16), m, e, top_k, int(renormalize),
         _ptr(ids), _ptr(w), _ptr(tei), _stream(dev))
    return (w, ids, tei) if with_indices else (w, ids)


def fused_moe_from_logits(hidden_states: torch.Tensor, layer: PreparedLayer, router_logits: torch.Tensor,
                          top_k: int, renormalize: bool = True, output: torch.Tensor = None,
                          return_routing: bool = False):
    """Router + routed-expert layer. Decode batches (the whole-layer kernel's sizes, E <= 512): one launch, the
    router fused into the layer kernel's routing (moek_moe_layer_logits, the same bits as the router kernel); larger
    batches: the router kernel, then ``fused_moe`` (two launches). With ``return_routing`` also returns the
    (weights fp32 [M, k], ids int32 [M, k]) the layer used."""
    x = hidden_states
    _need_cuda(x, router_logits)
    m, hid = x.shape
    e = router_logits.shape[1]
    if output is None:
        output = torch.empty((m, hid), dtype=torch.bfloat16, device=x.device)
    if (m == 0 or not _decode_path(m, top_k) or e > 512 or x.dtype != torch.bfloat16
            or os.environ.get("MOEK_B200_DECODE_PATH", "layer") != "layer"):
        w, ids = router_topk(router_logits, top_k, renormalize)
        out = fused_moe(x, layer, w, ids, output=output)
        return (out, (w, ids)) if return_routing else out
    import ctypes

    _layer_rows_knob()
    logits = router_logits if router_logits.dtype in (torch.float32, torch.bfloat16) else router_logits.float()
    logits = logits.contiguous()
    x = x.contiguous()
    dev = x.device
    ids = torch.empty((m, top_k), dtype=torch.int32, device=dev) if return_routing else None
    w = torch.empty((m, top_k), dtype=torch.float32, device=dev) if return_routing else None
    a, b = layer.w13, layer.w2
    hidden, inter = a.K, b.K
    ns1, ns2 = _layer_splits(hidden, inter)
    wsb = ctypes.c_size_t(0)
    call("moek_layer_workspace_bytes", m, top_k, hidden, inter, ns1, ns2, 0, ctypes.byref(wsb))
    ws = _scratch("layer_ws", wsb.value, torch.uint8, dev)
    st = _layer_state(dev, layer.E, hidden, inter)
    _timed("layer", lambda: call(
        "moek_moe_layer_logits", _ptr(x), m, hidden, inter, layer.E, _ptr(logits), int(logits.dtype == torch.bfloat16),
        top_k, int(renormalize), _ptr(ids), _ptr(w), _ptr(a.w), _ptr(a.sp), _ptr(a.g), _ptr(a.exc_off),
        _ptr(a.exc_ent), _ptr(b.w), _ptr(b.sp), _ptr(b.g), _ptr(b.exc_off), _ptr(b.exc_ent), ns1, ns2, _ptr(ws),
        ws.numel(), _ptr(st), st.numel(), _ptr(error_word(dev)), _ptr(output), _stream(dev)))
    return (output, (w, ids)) if return_routing else output


# ----------------------------------------------------------------------------------------------------- forward
DECODE_MAX_M = int(os.environ.get("MOEK_B200_DECODE_MAX_M", "64"))  # split-k with fused epilogues up to this M


def launches_per_layer(m: int, top_k: int) -> int:
    """Kernels of this library one fused_moe call launches: decode = one (moek_moe_layer); prefill = align (one
    kernel up to 1024 indices, else count/offsets/scatter), gate_up GEMM, down GEMM, top-k combine."""
    if _decode_path(m, top_k):
        return LAUNCHES_PER_LAYER
    return (1 if m * top_k <= 1024 else 3) + 3


LAYER_MAXIDS = 512  # routed slots per whole-layer call (moek_layer.cu)


def _decode_path(m: int, top_k: int) -> bool:
    return m <= DECODE_MAX_M and m * top_k <= LAYER_MAXIDS


def _layer_splits(hidden: int, inter: int):
    """The (gate_up, down) k-split arguments passed to the whole-layer kernel: 2 and 1 where they cut K into whole
    128-k runs (MOEK_B200_LAYER_SPLITS="g,d" overrides). The kernel checks them and otherwise plans its own split
    (stream-K ranges over the CTAs), so they do not change the results."""
    env = os.environ.get("MOEK_B200_LAYER_SPLITS")
    if env:
        g, d = (int(v) for v in env.split(","))
        return g, d
    pick = lambda k, want: max(d for d in range(1, want + 1) if (k // 128) % d == 0)
    return pick(hidden, 2), pick(inter, 1)


def _layer_state(dev, E: int, hidden: int, inter: int) -> torch.Tensor:
    """Persistent zero-initialised int32 state of the whole-layer kernel (counters and record flags) for one layer
    geometry on one device; calls in one stream share it (concurrent calls on other streams would race)."""
    import ctypes

    key = ("layer_state", torch.device(dev), E, hidden, inter)
    if key not in _BUF:
        n = ctypes.c_int64(0)
        call("moek_layer_state_ints", E, hidden, inter, ctypes.byref(n))
        _BUF[key] = torch.zeros(n.value, dtype=torch.int32, device=dev)
    return _BUF[key]


_ROWS_SET = False


def _layer_rows_knob():
    """MOEK_B200_LAYER_ROWS (8, 16 or 32): rows per block of the whole-layer kernel instead of the automatic 8
    (moek_set_layer_block_rows); MOEK_B200_LAYER_TAIL: accepted for the earlier plan, no effect
    (moek_set_layer_tail_split); MOEK_B200_LAYER_COOP=0: a plain launch instead of a cooperative one
    (moek_set_layer_cooperative). Read once."""
    global _ROWS_SET
    if not _ROWS_SET:
        env = os.environ.get("MOEK_B200_LAYER_ROWS")
        if env:
            call("moek_set_layer_block_rows", int(env))
        env = os.environ.get("MOEK_B200_LAYER_TAIL")
        if env:
            call("moek_set_layer_tail_split", int(env))
        env = os.environ.get("MOEK_B200_LAYER_COOP")
        if env:
            call("moek_set_layer_cooperative", int(env))
        _ROWS_SET = True


def _layer_kernel(x, layer, tw, ids32, m, top_k, output, rows):
    import ctypes

    _layer_rows_knob()

    a, b = layer.w13, layer.w2
    hidden, inter = a.K, b.K
    dev = x.device
    ns1, ns2 = _layer_splits(hidden, inter)
    wsb = ctypes.c_size_t(0)
    call("moek_layer_workspace_bytes", m, top_k, hidden, inter, ns1, ns2, int(rows is not None), ctypes.byref(wsb))
    ws = _scratch("layer_ws", wsb.value, torch.uint8, dev)
    st = _layer_state(dev, layer.E, hidden, inter)
    call("moek_moe_layer", _ptr(x), m, hidden, inter, layer.E, _ptr(ids32), _ptr(tw), top_k, _ptr(a.w), _ptr(a.sp),
         _ptr(a.g), _ptr(a.exc_off), _ptr(a.exc_ent), _ptr(b.w), _ptr(b.sp), _ptr(b.g), _ptr(b.exc_off),
         _ptr(b.exc_ent), ns1, ns2, _ptr(ws), ws.numel(), _ptr(st), st.numel(), _ptr(error_word(dev)),
         _ptr(output), _ptr(rows), _stream(dev))


def layer_p2p_fits(rows: int, top_k: int) -> bool:
    """Whether ``rows`` received rows of ``top_k`` slots fit the whole-layer kernel (``layer_p2p``)."""
    return 0 < rows and rows * top_k <= LAYER_MAXIDS


def layer_p2p(px, layer: PreparedLayer):
    """The whole-layer kernel on a peer exchange's receive segments (``ep.PeerExchange``): waits for the senders'
    flags, and writes each row's fp32 partial straight into its sender's back segment (moek_moe_layer_p2p)."""
    import ctypes

    _layer_rows_knob()
    a, b = layer.w13, layer.w2
    hidden, inter = a.K, b.K
    dev = px.recv_x.device
    rows, k = px.world * px.mcap, px.top_k
    ns1, ns2 = _layer_splits(hidden, inter)
    wsb = ctypes.c_size_t(0)
    call("moek_layer_workspace_bytes", rows, k, hidden, inter, ns1, ns2, 0, ctypes.byref(wsb))
    ws = _scratch("layer_ws", wsb.value, torch.uint8, dev)
    st = _layer_state(dev, layer.E, hidden, inter)
    call("moek_moe_layer_p2p", _ptr(px.peer), px.own, px.world, px.rank, px.mcap, hidden, inter, layer.E, k,
         _ptr(a.w), _ptr(a.sp), _ptr(a.g), _ptr(a.exc_off), _ptr(a.exc_ent), _ptr(b.w), _ptr(b.sp), _ptr(b.g),
         _ptr(b.exc_off), _ptr(b.exc_ent), ns1, ns2, _ptr(ws), ws.numel(), _ptr(st), st.numel(), _ptr(px.err),
         _stream(dev))


def layer_ep(px, layer: PreparedLayer, x: torch.Tensor, ids32: torch.Tensor, w: torch.Tensor, num_experts: int,
             pos: torch.Tensor, out: torch.Tensor):
    """The whole expert-parallel decode layer in one launch (moek_moe_layer_ep): the whole-layer kernel dispatches this
    rank's tokens ``x`` (global expert ids ``ids32``, router weights ``w``) into the owners' receive segments, runs
    the layer on its own receive segments as ``layer_p2p`` does, and sums the owners' partials into ``out`` bf16
    [M, H]; ``pos`` [M, world] receives each token's row in each owner's segment."""
    import ctypes

    _layer_rows_knob()
    a, b = layer.w13, layer.w2
    hidden, inter = a.K, b.K
    dev = x.device
    rows, k = px.world * px.mcap, px.top_k
    ns1, ns2 = _layer_splits(hidden, inter)
    wsb = ctypes.c_size_t(0)
    call("moek_layer_workspace_bytes", rows, k, hidden, inter, ns1, ns2, 0, ctypes.byref(wsb))
    ws = _scratch("layer_ws", wsb.value, torch.uint8, dev)
    st = _layer_state(dev, layer.E, hidden, inter)
    call("moek_moe_layer_ep", _ptr(px.peer), px.own, px.world, px.rank, px.mcap, hidden, inter, num_experts, k,
         _ptr(x), _ptr(ids32), _ptr(w), x.shape[0], _ptr(pos), _ptr(out), _ptr(a.w), _ptr(a.sp), _ptr(a.g),
         _ptr(a.exc_off), _ptr(a.exc_ent), _ptr(b.w), _ptr(b.sp), _ptr(b.g), _ptr(b.exc_off), _ptr(b.exc_ent), ns1,
         ns2, _ptr(ws), ws.numel(), _ptr(st), st.numel(), _ptr(px.err), _stream(dev))


def _splits(k: int, units_per_split: int, grid: int) -> int:
    """k-split (whole 128-k runs per unit) that balances units over the grid best: the split whose busiest CTA has the
    least work (in stages), preferring fewer splits on ties."""
    nstage = k // 64
    best, best_cost = 1, None
    for d in range(1, nstage + 1):
        if nstage % d or (nstage // d) % 2:
            continue
        units = units_per_split * d
        cost = -(-units // grid) * (nstage // d)  # stages of the busiest CTA
        if best_cost is None or cost < best_cost:
            best, best_cost = d, cost
    return best


def _sms(dev) -> int:
    key = ("sms", torch.device(dev))
    if key not in _BUF:
        _BUF[key] = torch.cuda.get_device_properties(dev).multi_processor_count
    return _BUF[key]


def fused_moe(hidden_states: torch.Tensor, layer: PreparedLayer, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
              output: torch.Tensor = None) -> torch.Tensor:
    """One routed-expert layer: out[t] = sum_j w[t, j] * down_e(silu(gate_e(x_t)) * up_e(x_t)), e = topk_ids[t, j].
    Slots whose expert id lies outside [0, E) (an expert map's -1) are not routed and add nothing; a token with no
    routed slot gets a zero row."""
    x = hidden_states
    _need_cuda(x, topk_ids, topk_weights)
    m, hid = x.shape
    if output is None:
        output = torch.empty((m, hid), dtype=torch.bfloat16, device=x.device)
    if m == 0:
        return output
    _layer_call(x, layer, topk_weights, topk_ids, output, None)
    return output


def moe_rows(hidden_states: torch.Tensor, layer: PreparedLayer, topk_weights: torch.Tensor,
             topk_ids: torch.Tensor) -> torch.Tensor:
    """The same layer without the top-k sum: fp32 rows [M * top_k, H], row t * top_k + j = w[t, j] *
    down_e(silu(gate_e(x_t)) * up_e(x_t)) for e = topk_ids[t, j] in [0, E). Rows of slots whose expert is outside
    [0, E) are not computed and hold arbitrary values (the expert-parallel partial sum leaves them out)."""
    x = hidden_states
    _need_cuda(x, topk_ids, topk_weights)
    m, hid = x.shape
    top_k = topk_ids.shape[1]
    if m == 0:
        return torch.empty((0, hid), dtype=torch.float32, device=x.device)
    return _layer_call(x, layer, topk_weights, topk_ids, None, top_k)


def _layer_call(x, layer, topk_weights, topk_ids, output, rows_k):
    """Align + gate_up + SwiGLU + down. ``output`` bf16 [M, H] gets the top-k sums; with ``rows_k`` set instead,
    the fp32 weighted rows [M * top_k, H] are returned."""
    if x.dtype != torch.bfloat16:
        raise MoekError("moek_b200: hidden states must be bf16")
    x = x.contiguous()
    m = x.shape[0]
    top_k = topk_ids.shape[1]
    num_ids = m * top_k
    dev = x.device
    a, b = layer.w13, layer.w2
    ids32 = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
    ids32 = ids32.reshape(-1).contiguous()
    tw = topk_weights.reshape(-1).float().contiguous()
    cnt = error_word(dev)
    rows = min(BM, m)
    if _decode_path(m, top_k) and os.environ.get("MOEK_B200_DECODE_PATH", "layer") == "layer":
        # the whole layer in one persistent kernel: routing, gate_up + SwiGLU, down x router weight, top-k sum
        out_rows = None if rows_k is None else torch.empty((num_ids, b.N), dtype=torch.float32, device=dev)
        _timed("layer", lambda: _layer_kernel(x, layer, tw, ids32, m, top_k, output if rows_k is None else None,
                                              out_rows))
        return output if rows_k is None else out_rows
    act = torch.empty((num_ids, a.N // 2), dtype=torch.bfloat16, device=dev)
    if m <= DECODE_MAX_M:
        # split-k GEMM launches (moek_gemm mode 2) and their two epilogue kernels (MOEK_B200_DECODE_PATH=split); like
        # the kit's own split epilogue, this path adds every slot's partials, so it expects every id in [0, E)
        sid, eid, npad = moe_align_block_size(ids32, BM, layer.E)
        # split-k with fp32 partials (no cross-CTA synchronisation in the GEMMs), finished by two small
        # deterministic epilogue kernels: SwiGLU -> act, and router weight + top-k sum -> output
        grid = (2 if rows <= 32 else 1) * _sms(dev)
        blocks = min(layer.E, num_ids)
        ns1 = _splits(a.K, blocks * (a.N // 256), grid)
        ns2 = _splits(b.K, blocks * (b.N // 256), grid)
        part = _scratch("part", max(ns1 * num_ids * a.N, ns2 * num_ids * b.N), torch.float32, dev)
        st = _stream(dev)
        _timed("gate_gemm", lambda: _gemm(x, a, sid, eid, npad, num_ids, top_k, True, cnt, ns1, part, rows, None,
                                          None, None, 0, mode=2))
        call("moek_split_epilogue", _ptr(part), ns1, num_ids, a.N, 1, None, top_k, _ptr(act), 0, st)
        _timed("down_gemm", lambda: _gemm(act, b, sid, eid, npad, num_ids, 1, False, cnt, ns2, part, rows, None,
                                          None, None, 0, mode=2))
        if rows_k is None:
            call("moek_split_epilogue", _ptr(part), ns2, num_ids, b.N, 0, _ptr(tw), top_k, _ptr(output), 2, st)
            return output
        dout = torch.empty((num_ids, b.N), dtype=torch.float32, device=dev)
        call("moek_split_epilogue", _ptr(part), ns2, num_ids, b.N, 0, _ptr(tw), top_k, _ptr(dout), 1, st)
        return dout
    # prefill: tcgen05 GEMMs over moe_align blocks of <= 128 rows (the MMA's N), SwiGLU and router weight in their
    # epilogues, the top-k sum of the routed slots' fp32 rows in one more kernel
    sid, eid, npad = moe_align_block_size(ids32, BM_PREFILL, layer.E)
    part = _scratch("part", num_ids * b.N, torch.float32, dev) if rows_k is None else \
        torch.empty((num_ids, b.N), dtype=torch.float32, device=dev)
    # mode 5: act rows in moe_align's sorted order (row = position in sorted_ids), so the down GEMM reads each block's
    # rows as one tile instead of gathering them
    act = torch.empty((sid.numel(), a.N // 2), dtype=torch.bfloat16, device=dev)
    _timed("gate_gemm", lambda: _gemm(x, a, sid, eid, npad, num_ids, top_k, True, cnt, 1, part, rows, act, tw, ids32,
                                      top_k, mode=5, block_m=BM_PREFILL))
    _timed("down_gemm", lambda: _gemm(act, b, sid, eid, npad, num_ids, 1, False, cnt, 1, part, rows, None, tw, ids32,
                                      top_k, mode=5, block_m=BM_PREFILL))
    if rows_k is not None:
        return part
    # the top-k sum over the routed slots: rows of slots outside [0, E) were never written (moe_align skips them)
    call("moek_combine_routed", _ptr(part), _ptr(ids32), layer.E, _ptr(output), m, b.N, top_k, _stream(dev))
    return output


def _gemm(a_in, mat, sid, eid, npad, num_ids, a_div, gate_up, cnt, nsplit, part, rows, out, tw, ids32, combine_k,
          mode=3, block_m=None):
    block_m = block_m or BM
    call("moek_gemm", _ptr(a_in), _ptr(mat.w), None, _ptr(mat.g), _ptr(sid), sid.numel(), _ptr(eid), _ptr(npad),
         _ptr(tw), _ptr(out), num_ids, mat.N, mat.K, mat.E, a_div, int(gate_up), _ptr(mat.sp), _ptr(mat.exc_off),
         _ptr(mat.exc_ent), _ptr(cnt), cnt.numel(), mode, nsplit, _ptr(part), part.numel(), 1, block_m, rows,
         _ptr(ids32), combine_k, _stream(a_in.device))


def _timed(name, fn):
    if _PROF is not None:
        _PROF.append((name, fn))
    return fn()


def record_launches(fn) -> list:
    """Run ``fn`` once and return the (name, closure) of every GEMM launch fused_moe made: replaying a closure
    re-launches that kernel with the same arguments (bench.py times the GEMMs alone this way)."""
    global _PROF
    _PROF = []
    try:
        fn()
        return list(_PROF)
    finally:
        _PROF = None


# ------------------------------------------------------------------------------- the rest of the MoE block
SHARED_MAXM = 64  # decode sizes of the router gate and shared-expert kernels (moek_shared.cu)


class SharedExpert:
    """The block's shared expert in the kit's checkpoint format (MXFP8): w_gu uint8 [2 Is, H] float8_e4m3fn bytes
    (gate rows, then up rows), s_gu uint8 [2 Is, H / 32] E8M0 exponents, w_d uint8 [H, Is], s_d uint8 [H, Is / 32],
    and the expert gate w_sg bf16 [H] (vllm/model_executor/models/qwen2_moe.py:114-122). Used as is: the kernels read
    the checkpoint layout."""

    def __init__(self, w_gu, s_gu, w_d, s_d, w_sg):
        self.w_gu, self.s_gu = w_gu.contiguous().view(torch.uint8), s_gu.contiguous().view(torch.uint8)
        self.w_d, self.s_d = w_d.contiguous().view(torch.uint8), s_d.contiguous().view(torch.uint8)
        self.w_sg = w_sg.contiguous().reshape(-1).to(torch.bfloat16)
        self.inter = self.w_gu.shape[0] // 2
        self.hidden = self.w_gu.shape[1]
        lo = min(int(self.s_gu.min()), int(self.s_d.min()))
        hi = max(int(self.s_gu.max()), int(self.s_d.max()))
        if lo < 10 or hi > 134:  # outside, an e4m3 x 2^(s - 127) weight may not be a normal bf16 (see moek_shared.cu)
            raise MoekError(f"moek_b200: MXFP8 scale exponents must lie in [10, 134] (got [{lo}, {hi}])")

    def dequant(self):
        """bf16 (exact) weights (W_gu [2 Is, H], W_d [H, Is]) for batches past the decode kernels."""
        f = lambda q, s: (q.view(torch.float8_e4m3fn).float().view(q.shape[0], -1, 32)
                          * torch.exp2(s.float() - 127.0)[..., None]).view(q.shape[0], -1).to(torch.bfloat16)
        return f(self.w_gu, self.s_gu), f(self.w_d, self.s_d)


def router_gate(hidden_states: torch.Tensor, w_gate: torch.Tensor) -> torch.Tensor:
    """Router logits fp32 [M, E] = x @ w_gate^T (the block's gate, vllm/.../qwen3_next.py:125-131,193): this build's
    kernel for decode batches (M <= 64), a library fp32 GEMM for larger ones."""
    x = hidden_states
    _need_cuda(x, w_gate)
    m, hid = x.shape
    e = w_gate.shape[0]
    if m > SHARED_MAXM or e % 16 or hid % 128:
        return x.float() @ w_gate.float().t()
    x, w_gate = x.contiguous(), w_gate.contiguous()
    logits = torch.empty((m, e), dtype=torch.float32, device=x.device)
    call("moek_router_gate", _ptr(x), m, hid, _ptr(w_gate), e, _ptr(logits), _ptr(error_word(x.device)),
         _stream(x.device))
    return logits


def shared_expert(hidden_states: torch.Tensor, shared: SharedExpert) -> torch.Tensor:
    """fp32 rows [M, H] = sigmoid(x @ w_sg) * down(bf16(silu(gate) * up)) of the MXFP8 shared expert: this build's
    kernels for decode batches (M <= 64), exact bf16 weights and library fp32 GEMMs for larger ones."""
    x = hidden_states
    _need_cuda(x, shared.w_gu)
    m, hid = x.shape
    if m > SHARED_MAXM:
        a, b = shared.dequant()
        h = x.float() @ a.float().t()
        act = (torch.nn.functional.silu(h[:, :shared.inter]) * h[:, shared.inter:]).to(torch.bfloat16)
        return torch.sigmoid(x.float() @ shared.w_sg.float()[:, None]) * (act.float() @ b.float().t())
    import ctypes

    x = x.contiguous()
    wsb = ctypes.c_size_t(0)
    call("moek_shared_workspace_bytes", m, shared.inter, ctypes.byref(wsb))
    ws = _scratch("shared_ws", wsb.value, torch.uint8, x.device)
    rows = torch.empty((m, hid), dtype=torch.float32, device=x.device)
    call("moek_shared_expert", _ptr(x), m, hid, shared.inter, _ptr(shared.w_gu), _ptr(shared.s_gu), _ptr(shared.w_d),
         _ptr(shared.s_d), _ptr(shared.w_sg), _ptr(ws), ws.numel(), _ptr(rows), _ptr(error_word(x.device)),
         _stream(x.device))
    return rows


def moe_block(hidden_states: torch.Tensor, w_gate: torch.Tensor, layer: PreparedLayer, shared: SharedExpert,
              top_k: int, renormalize: bool = True, output: torch.Tensor = None, return_routing: bool = False):
    """The MoE block (vllm/model_executor/models/qwen3_next.py:177-204, which the kit's files/v54/model.py:193-210
    subclasses): router gate -> softmax / top-k -> routed experts, plus the shared expert (``shared`` may be None),
    out = bf16(sum of the routed slots in slot order + the shared row). Decode batches (M <= 64, E <= 512): one call
    of moek_moe_block (the gate, the shared expert and the whole-layer kernel, chained on the GPU). Larger batches: the
    gate and the shared expert as library GEMMs, the routed experts' fp32 slot rows from this build's prefill kernels,
    added in slot order. With ``return_routing`` also returns (weights fp32 [M, k], ids int32 [M, k])."""
    x = hidden_states
    _need_cuda(x, w_gate)
    m, hid = x.shape
    e = w_gate.shape[0]
    if output is None:
        output = torch.empty((m, hid), dtype=torch.bfloat16, device=x.device)
    if m == 0:
        return (output, (None, None)) if return_routing else output
    if m <= SHARED_MAXM and e <= 512 and e % 16 == 0 and hid % 128 == 0 and top_k <= 32 and _decode_path(m, top_k) and \
            x.dtype == torch.bfloat16 and (shared is None or shared.inter % 128 == 0):
        import ctypes

        _layer_rows_knob()
        x = x.contiguous()
        a, b = layer.w13, layer.w2
        hidden, inter = a.K, b.K
        ns1, ns2 = _layer_splits(hidden, inter)
        is_ = shared.inter if shared is not None else 0
        wsb = ctypes.c_size_t(0)
        call("moek_block_workspace_bytes", m, top_k, hidden, inter, e, is_, ctypes.byref(wsb))
        ws = _scratch("block_ws", wsb.value, torch.uint8, x.device)
        st = _layer_state(x.device, layer.E, hidden, inter)
        ids = torch.empty((m, top_k), dtype=torch.int32, device=x.device) if return_routing else None
        w = torch.empty((m, top_k), dtype=torch.float32, device=x.device) if return_routing else None
        sh = [None] * 5 if shared is None else [shared.w_gu, shared.s_gu, shared.w_d, shared.s_d, shared.w_sg]
        call("moek_moe_block", _ptr(x), m, hidden, inter, e, _ptr(w_gate.contiguous()), top_k, int(renormalize),
             _ptr(ids), _ptr(w), _ptr(a.w), _ptr(a.sp), _ptr(a.g), _ptr(a.exc_off), _ptr(a.exc_ent), _ptr(b.w),
             _ptr(b.sp), _ptr(b.g), _ptr(b.exc_off), _ptr(b.exc_ent), ns1, ns2, is_, *[_ptr(t) for t in sh], _ptr(ws),
             ws.numel(), _ptr(st), st.numel(), _ptr(error_word(x.device)), _ptr(output), _stream(x.device))
        return (output, (w, ids)) if return_routing else output
    logits = router_gate(x, w_gate)
    w, ids = router_topk(logits, top_k, renormalize)
    rows = moe_rows(x, layer, w, ids).view(m, top_k, hid)
    valid = ((ids >= 0) & (ids < layer.E)).unsqueeze(-1)
    acc = torch.zeros((m, hid), dtype=torch.float32, device=x.device)
    for j in range(top_k):  # slot order, as the oracle (invalid slots' rows hold arbitrary values: left out)
        acc = acc + torch.where(valid[:, j], rows[:, j], 0.0)
    if shared is not None:
        acc = acc + shared_expert(x, shared)
    output.copy_(acc.to(torch.bfloat16))
    return (output, (w, ids)) if return_routing else output
