"""The MoE block's oracle pieces on the CPU (no GPU): the MXFP8 format and quantiser, and the shared-expert kernels'
exact dequantisation restated bit for bit (e4m3 bits at bf16 bits 4-10 with the sign at 15, times 2^(s - 7)); the
C ABI's argument checks of the new entry points."""
import ctypes

import numpy as np
import torch

from oracle import shared as shared_ref
from oracle.nvfp4 import E4M3
from qwen38_flash_coder_b200 import _lib, synth


def _bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def test_kernel_dequant_is_exact_for_every_code_and_scale():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint32)  # 0x7F / 0xFF are NaN
    pattern = ((codes & 0x7F) << 4) | ((codes & 0x80) << 8)  # the kernel's bf16 bits: e4m3 x 2^-120
    assert np.array_equal(_bf16_bits_to_f32(pattern).astype(np.float64) * 2.0 ** 120, E4M3[codes].astype(np.float64))
    for s in range(10, 135):  # the range the library accepts: every product a normal bf16
        factor = _bf16_bits_to_f32(np.uint32((s + 120) << 7))  # the kernel's bf16 2^(s - 7)
        prod = (_bf16_bits_to_f32(pattern) * factor).astype(np.float32)  # exact: <= 7 significant bits
        want = (E4M3[codes].astype(np.float64) * 2.0 ** (s - 127)).astype(np.float32)
        bf = torch.from_numpy(prod).to(torch.bfloat16).float().numpy()
        assert np.array_equal(bf, want) and np.array_equal(prod, want), s


def test_mxfp8_quantiser_round_trip():
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(64, 256, generator=g) * 0.02).to(torch.bfloat16)
    q, s = synth.quantize_mxfp8(w)
    assert q.dtype == torch.uint8 and s.shape == (64, 8)
    deq = shared_ref.mxfp8_dequant(q.numpy(), s.numpy())
    rel = np.abs(deq - w.float().numpy()).max(axis=1) / np.abs(w.float().numpy()).max(axis=1)
    assert rel.max() < 2 ** -4  # e4m3 keeps 3 mantissa bits and nothing saturates
    # every block's largest magnitude lands in (224, 448]: the smallest scale that needs no saturation
    blk = np.abs(deq.reshape(64, 8, 32)).max(-1) / np.ldexp(1.0, s.numpy().astype(np.int32) - 127)
    assert (blk > 224 - 16).all() and (blk <= 448).all()


def test_block_entry_points_reject_bad_arguments():
    lib = _lib.lib()
    b = ctypes.c_size_t(0)
    assert lib.moek_shared_workspace_bytes(8, 512, ctypes.byref(b)) == 0 and b.value == 8 * 512 * 2 + 256
    assert lib.moek_block_workspace_bytes(8, 5, 2048, 512, 512, 512, ctypes.byref(b)) == 0 and b.value > 8 * 2048 * 4
    fake = ctypes.c_void_p(256)  # never dereferenced: each call fails its argument checks first
    assert lib.moek_router_gate(fake, 65, 2048, fake, 512, fake, None, None) == 3  # M > 64: a library GEMM's job
    assert lib.moek_router_gate(fake, 8, 2048, fake, 100, fake, None, None) == 3  # E % 16
    assert lib.moek_router_gate(ctypes.c_void_p(264), 8, 2048, fake, 512, fake, None, None) == 1  # x not 16-aligned
    args = [fake, 8, 2048, 500, fake, fake, fake, fake, fake, fake, 1 << 20, fake, None, None]
    assert lib.moek_shared_expert(*args) == 3  # Is % 128
    args[3], args[10] = 512, 16
    assert lib.moek_shared_expert(*args) == 1  # workspace too small
