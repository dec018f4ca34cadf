"""The rest of the MoE block around the routed experts, restated on the CPU (test infrastructure only).

The kit's model (files/v54/model.py:193-210, ``Qwen4ExpSparseMoeBlock``) is vLLM's ``Qwen3NextSparseMoeBlock`` with
the kit's checks; its forward (vllm/model_executor/models/qwen3_next.py:177-204) computes, per token row x:

- the router gate GEMM ``logits = x @ W_gate^T`` (qwen3_next.py:125-131,193; a bf16 ``ReplicatedLinear`` with no
  quantisation), which feeds the routed experts' softmax / top-k (``oracle/router.py``);
- the shared expert (qwen2_moe.py:114-122, ``Qwen2MoeMLP.forward`` with ``expert_gate``):
  ``shared = sigmoid(x @ w_sg) * down(silu(gate) * up)``, ``[gate | up] = x @ W_gu^T``; in the kit's checkpoint its
  weights are MXFP8 (README.md:38: "MXFP8 as shipped (attention, shared expert)"): e4m3 values with one power-of-two
  scale (E8M0, 2^(s - 127)) per 32 inputs along K;
- the block output ``routed + shared`` (vLLM's FusedMoE with ``shared_experts``).

This oracle follows the routed layer's rounding points (``moe_ref``): weights dequantised exactly (an e4m3 value times
a power of two is exact in bf16 and fp32), sums in fp32, the SwiGLU output rounded to bf16, the shared expert's fp32
row times the fp32 sigmoid gate added to the fp32 sum of the routed slots (in slot order), then one bf16 rounding of
the block output.
"""
import numpy as np
import torch

from . import moe_ref
from .nvfp4 import E4M3


def mxfp8_dequant(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 [N, K] = e4m3(codes) * 2^(scales - 127), codes uint8 [N, K] (float8_e4m3fn bits), scales uint8
    [N, K / 32] (E8M0; 255 is not a scale)."""
    codes = np.asarray(codes, dtype=np.uint8)
    scales = np.asarray(scales, dtype=np.uint8)
    n, k = codes.shape
    assert scales.shape == (n, k // 32) and not (scales == 255).any()
    f = np.ldexp(np.float32(1.0), scales.astype(np.int32) - 127).astype(np.float32)
    return (E4M3[codes] * np.repeat(f, 32, axis=1)).astype(np.float32)


def gate_logits(x, w_gate) -> torch.Tensor:
    """fp32 [M, E] router logits from bf16 x [M, H] and bf16 W_gate [E, H] (an fp32 matmul; the GPU's order of fp32
    additions differs, so compare within an fp32 tolerance)."""
    return x.float() @ torch.as_tensor(w_gate).float().T


def shared_rows(x, w_gu, s_gu, w_d, s_d, w_sg) -> torch.Tensor:
    """fp32 [M, H]: sigmoid(x @ w_sg) * (bf16(silu(g) * u) @ W_d^T), (g, u) = x @ W_gu^T in fp32, MXFP8 weights
    (w_gu [2 Is, H] with the gate rows first, w_d [H, Is], scales per 32 along K), w_sg bf16 [H]."""
    xf = x.float()
    a = torch.from_numpy(mxfp8_dequant(w_gu, s_gu))
    b = torch.from_numpy(mxfp8_dequant(w_d, s_d))
    inter = a.shape[0] // 2
    h = xf @ a.T
    act = moe_ref._bf16(torch.nn.functional.silu(h[:, :inter]) * h[:, inter:])
    sg = torch.sigmoid(xf @ torch.as_tensor(w_sg).float().reshape(-1, 1))
    return sg * (act @ b.T)


def block(x, topk_ids, topk_w, w13, w2, shared) -> torch.Tensor:
    """fp32 [M, H] block output for a given routing: the routed slot rows (``moe_ref.slot_rows``) summed in slot
    order, plus ``shared_rows(x, *shared)``."""
    m, hid = x.shape
    k = topk_ids.shape[1]
    y = moe_ref.slot_rows(x, topk_ids, topk_w, w13, w2).view(m, k, hid)
    out = torch.zeros((m, hid), dtype=torch.float32)
    for j in range(k):
        out += y[:, j]
    return out + shared_rows(x, *shared)
