"""ctypes binding of libmoek_b200.so (include/moek_b200.h). Loading fails loudly: there is no fallback path.

``MOEK_B200_LIB=trace`` or ``=debug`` loads the instrumented build of the same kernels instead (``build.py``): the
timeline stamps of ``qwen38_flash_coder_b200.trace``, or the input-index checks."""
import ctypes
import os

from .build import lib_path

_P, _I32, _I64, _U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64

SIGNATURES = {
    "moek_last_error": (ctypes.c_char_p, []),
    "moek_version": (ctypes.c_int, []),
    "moek_set_wait_timeout_ns": (ctypes.c_int, [_U64]),
    "moek_set_layer_block_rows": (ctypes.c_int, [_I32]),
    "moek_set_layer_tail_split": (ctypes.c_int, [_I32]),
    "moek_set_layer_cooperative": (ctypes.c_int, [_I32]),
    "moek_align_workspace_bytes": (ctypes.c_int, [_I64, _I32, ctypes.POINTER(ctypes.c_size_t)]),
    "moek_align": (ctypes.c_int, [_P, _I64, _I32, _I32, _P, _I64, _P, _I64, _P, _P, ctypes.c_size_t, _P]),
    "moek_align_noalloc": (ctypes.c_int, [_P, _I64, _I32, _I32, _P, _I64, _P, _I64, _P, _P]),
    "moek_gemm": (ctypes.c_int, [_P, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                                 _P, _P, _P, _P, _I64, _I32, _I32, _P, _I64, _I32, _I32, _I32, _P, _I32, _P]),
    "moek_split_epilogue": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _P, _I32, _P, _I32, _P]),
    "moek_combine": (ctypes.c_int, [_P, _I32, _P, _I32, _I32, _I32, _P]),
    "moek_combine_routed": (ctypes.c_int, [_P, _P, _I32, _P, _I32, _I32, _I32, _P]),
    "moek_router_topk": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P]),
    "moek_router_gate": (ctypes.c_int, [_P, _I32, _I32, _P, _I32, _P, _P, _P]),
    "moek_prep_workspace_bytes": (ctypes.c_int, [_I32, _I32, _I32, ctypes.POINTER(ctypes.c_size_t)]),
    "moek_prep_weights": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _P, _P]),
    "moek_prep_scales": (ctypes.c_int, [_P, _P, _I32, _I32, _I32, _I32, _P, ctypes.c_size_t, _P, _P, _P,
                                        ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int64), _P]),
    "moek_prep_exceptions": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, ctypes.c_float, _P, _P, _P, _P]),
    "moek_shared_workspace_bytes": (ctypes.c_int, [_I32, _I32, ctypes.POINTER(ctypes.c_size_t)]),
    "moek_shared_expert": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P, _P,
                                          _P]),
    "moek_block_workspace_bytes": (ctypes.c_int, [_I32] * 6 + [ctypes.POINTER(ctypes.c_size_t)]),
    "moek_moe_block": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _P, _I32, _I32, _P, _P] + [_P] * 10 +
                       [_I32, _I32, _I32] + [_P] * 5 + [_P, ctypes.c_size_t, _P, _I64, _P, _P, _P]),
    "moek_layer_state_ints": (ctypes.c_int, [_I32, _I32, _I32, ctypes.POINTER(ctypes.c_int64)]),
    "moek_layer_workspace_bytes": (ctypes.c_int, [_I32] * 7 + [ctypes.POINTER(ctypes.c_size_t)]),
    "moek_moe_layer": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _P, _P, _I32] + [_P] * 10 + [_I32, _I32, _P,
                                     ctypes.c_size_t, _P, _I64, _P, _P, _P, _P]),
    "moek_moe_layer_logits": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _P, _I32, _I32, _I32, _P, _P] + [_P] * 10 +
                              [_I32, _I32, _P, ctypes.c_size_t, _P, _I64, _P, _P, _P]),
    "moek_ep_plan": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _P, _P, _P, _P]),
    "moek_ep_pack": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P, _I64, _P, _I64,
                                    _P]),
    "moek_ep_partial": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P]),
    "moek_ep_unpack": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I32, _P, _P]),
    "moek_ipc_malloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "moek_ipc_free": (ctypes.c_int, [_P]),
    "moek_ipc_handle": (ctypes.c_int, [_P, _P]),
    "moek_ipc_open": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "moek_ipc_close": (ctypes.c_int, [_P]),
    "moek_ep_p2p_layout": (ctypes.c_int, [_I32] * 4 + [_P]),
    "moek_ep_dispatch_p2p": (ctypes.c_int, [_P] + [_I32] * 5 + [_P] * 3 + [_I32, _I32, _P, _P, _P]),
    "moek_ep_wait": (ctypes.c_int, [_P, _I32, _P, _P]),
    "moek_ep_combine_p2p": (ctypes.c_int, [_P] + [_I32] * 5 + [_P, _I32, _P, _P]),
    "moek_ep_unpack_p2p": (ctypes.c_int, [_P] + [_I32] * 5 + [_P, _I32, _P, _P, _P]),
    "moek_moe_layer_p2p": (ctypes.c_int, [_P, _P] + [_I32] * 7 + [_P] * 10 + [_I32, _I32, _P, ctypes.c_size_t, _P,
                                                                              _I64, _P, _P]),
    "moek_moe_layer_ep": (ctypes.c_int, [_P, _P] + [_I32] * 7 + [_P] * 3 + [_I32] + [_P] * 12 +
                          [_I32, _I32, _P, ctypes.c_size_t, _P, _I64, _P, _P]),
    "moek_build_flags": (ctypes.c_int, []),
    "moek_trace_read": (ctypes.c_int, [_I32, _P, ctypes.c_size_t]),
    "moek_trace_clear": (ctypes.c_int, []),
}

_lib = None


class MoekError(RuntimeError):
    pass


def variant() -> str:
    v = os.environ.get("MOEK_B200_LIB", "")
    if v not in ("", "trace", "debug"):
        raise ImportError(f"moek_b200: MOEK_B200_LIB={v!r}: the variants are trace and debug")
    return v


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = lib_path(variant())
        if not os.path.exists(path):
            raise ImportError(f"moek_b200: {path} is missing; build it with `python -m qwen38_flash_coder_b200.build"
                              f"{' --variant=' + variant() if variant() else ''}` (nvcc, sm_100a). There is no "
                              "fallback implementation.")
        h = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(h, name)
            f.restype, f.argtypes = res, args
        _lib = h
    return _lib


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc:
        msg = lib().moek_last_error().decode(errors="replace")
        raise MoekError(f"{name} failed ({rc}): {msg}")
