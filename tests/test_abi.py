"""The C ABI library: it loads without a GPU, exports every function include/*.h declares, and rejects bad
arguments on the host (no kernel is launched for them)."""
import ctypes
import glob
import os
import re

import pytest

from qwen38_flash_coder_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names += re.findall(r"\b(moek_\w+)\s*\(", src)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared()
    for must in ("moek_align", "moek_gemm", "moek_split_epilogue", "moek_combine", "moek_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared()) <= set(_lib.SIGNATURES), "ctypes signatures out of date"


def test_version_and_errors_without_gpu():
    lib = _lib.lib()
    assert lib.moek_version() == 1
    # bad arguments are rejected before any CUDA call
    rc = lib.moek_align(None, 10, 0, 96, None, 0, None, 0, None, None, 0, None)
    assert rc == 1 and b"num_experts" in lib.moek_last_error()
    rc = lib.moek_gemm(*([None] * 4), None, 0, None, None, None, None, 5, 300, 2048, 8, 5, 1, None, None, None, None,
                       0, 2, 1, None, 0, 1, 96, 8, None, 0, None)
    assert rc == 1 and b"N % 256" in lib.moek_last_error()
    rc = lib.moek_set_wait_timeout_ns(0)
    assert rc == 1


def test_routed_combine_rejects_bad_arguments():
    lib = _lib.lib()
    fake = ctypes.c_void_p(256)  # never dereferenced: the argument checks fail first
    assert lib.moek_combine_routed(fake, fake, 64, fake, 0, 2048, 5, None) == 0  # empty batch: nothing to do
    assert lib.moek_combine_routed(fake, None, 64, fake, 4, 2048, 5, None) == 1
    assert b"routed combine" in lib.moek_last_error()
    assert lib.moek_combine_routed(fake, fake, 0, fake, 4, 2048, 5, None) == 1  # no experts
    assert lib.moek_combine_routed(fake, fake, 64, fake, 4, 2048, 0, None) == 1  # top_k 0


def test_align_workspace_query():
    lib = _lib.lib()
    b = ctypes.c_size_t(7)
    assert lib.moek_align_workspace_bytes(40, 512, ctypes.byref(b)) == 0 and b.value == 0
    assert lib.moek_align_workspace_bytes(34560, 512, ctypes.byref(b)) == 0
    assert b.value == 4 * (34 * 512 + 34560)


def test_call_raises_moek_error():
    with pytest.raises(_lib.MoekError):
        _lib.call("moek_set_wait_timeout_ns", 0)


def test_layer_entry_points_reject_bad_arguments():
    lib = _lib.lib()
    n = ctypes.c_int64(0)
    assert lib.moek_layer_state_ints(512, 2048, 512, ctypes.byref(n)) == 0 and n.value > 2
    b = ctypes.c_size_t(0)
    assert lib.moek_layer_workspace_bytes(8, 5, 2048, 512, 4, 2, 0, ctypes.byref(b)) == 0
    # the fp32 gate_up records (grid bound 2 x 148 CTAs -- no GPU here, so the SM count is B200's 148 -- plus 40 slots
    # x 4 gate_up items, each 8 block rows x 256 columns) + the down partials per 128-k slice [I / 128, 40, H] fp32
    assert b.value == (296 + 40 * 4) * 8 * 256 * 4 + 4 * 40 * 2048 * 4
    args = [None, 200, 2048, 512, 512, None, None, 5] + [None] * 10 + [4, 2, None, 0, None, 0, None, None, None, None]
    assert lib.moek_moe_layer(*args) == 3 and b"decode batches" in lib.moek_last_error()  # M = 200 too large
    args[1] = 8
    assert lib.moek_moe_layer(*args) == 1 and b"null pointer" in lib.moek_last_error()
    args[18] = 3  # 3 splits do not cut 16 runs
    assert lib.moek_moe_layer(*args) == 1 and b"k-splits" in lib.moek_last_error()


def test_peer_exchange_layout_and_argument_checks():
    """The exchange block layout (x, ids, w, back, flags, counters, total; 256-byte aligned sections) and the
    argument checks of the peer-exchange entry points (no device call is reached)."""
    lib = _lib.lib()
    offs = (ctypes.c_int64 * 7)()
    world, mcap, H, k = 2, 8, 2048, 5
    assert lib.moek_ep_p2p_layout(world, mcap, H, k, offs) == 0
    up = lambda b: (b + 255) // 256 * 256
    R = world * mcap
    want = [0]
    for size in (R * H * 2, R * k * 4, R * k * 4, R * H * 4, 2 * world * 4, 2 * world * 4):
        want.append(want[-1] + up(size))
    assert list(offs) == want
    assert lib.moek_ep_p2p_layout(world, 1025, H, k, offs) == 1  # more than 1024 tokens per rank
    assert lib.moek_ep_p2p_layout(33, mcap, H, k, offs) == 1  # more ranks than supported
    fake = ctypes.c_void_p(256)  # never dereferenced: every call below fails its argument checks first
    assert lib.moek_ep_dispatch_p2p(None, 2, 0, 8, H, k, fake, fake, fake, 4, 64, fake, fake, None) == 1
    assert lib.moek_ep_dispatch_p2p(fake, 2, 2, 8, H, k, fake, fake, fake, 4, 64, fake, fake, None) == 1  # rank
    assert lib.moek_ep_dispatch_p2p(fake, 2, 0, 8, H, k, fake, fake, fake, 9, 64, fake, fake, None) == 1  # M > mcap
    assert lib.moek_ep_dispatch_p2p(fake, 2, 0, 8, H, k, fake, fake, fake, 4, 63, fake, fake, None) == 1  # E % world
    assert lib.moek_ep_unpack_p2p(fake, 2, 0, 8, H, k, None, 4, fake, fake, None) == 1
    assert lib.moek_ep_combine_p2p(fake, 2, 0, 8, H, k, fake, 0, fake, None) == 1
    args = [fake, None, 2, 0, 8, H, 512, 256, k] + [fake] * 10 + [2, 1, fake, 1 << 30, fake, 1 << 20, fake, None]
    assert lib.moek_moe_layer_p2p(*args) == 1 and b"exchange block" in lib.moek_last_error()
    args[1], args[4] = fake, 60  # 120 received rows of 5 slots: more than the whole-layer kernel takes
    assert lib.moek_moe_layer_p2p(*args) == 3 and b"decode batches" in lib.moek_last_error()
    assert lib.moek_set_layer_block_rows(24) == 1 and lib.moek_set_layer_block_rows(0) == 0


@pytest.mark.parametrize("variant,flag", [("trace", 1), ("debug", 2)])
def test_instrumented_builds_export_the_same_symbols(variant, flag):
    """The trace and debug builds (build.py variants) export every declared function and report their flag; the
    product build reports none and refuses trace reads."""
    from qwen38_flash_coder_b200 import build

    path = build.lib_path(variant)
    if not os.path.exists(path):
        build.build(variant=variant)
    h = ctypes.CDLL(path)
    missing = [n for n in declared() if not hasattr(h, n)]
    assert not missing, missing
    assert h.moek_build_flags() == flag
    lib = _lib.lib()
    assert lib.moek_build_flags() == 0
    buf = ctypes.create_string_buffer(64)
    assert lib.moek_trace_read(0, buf, 64) == 3  # MOEK_ERR_UNSUPPORTED without MOEK_TRACE
