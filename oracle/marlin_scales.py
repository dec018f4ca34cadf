"""vLLM's Marlin preparation of NVFP4 block scales, restated in numpy (test infrastructure only).

The kit's packed-scale codec (files/mbx_moek.py:61-120) is defined over these bytes, so the oracle rebuilds them from
the checkpoint scales exactly as vLLM 0.22.0's ``prepare_nvfp4_moe_layer_for_marlin`` does for the scales
(vllm/model_executor/layers/quantization/utils/marlin_utils_fp4.py:355-386):

1. one power-of-two ``scale_factor`` shared by all experts of a matrix (``_nvfp4_compute_scale_factor``,
   marlin_utils_fp4.py:30-50): the largest 2^j with max(nonzero scale) * 2^7 * 2^j <= 448 * 2^7, else 1;
2. per expert the [N, K/16] scales are transposed to [K/16, N] and permuted within every 64 consecutive values with
   ``scale_perm`` (vllm/.../marlin_utils.py:296-316: new[8i + j] = old[i + 8j]);
3. ``nvfp4_marlin_process_scales`` (marlin_utils_fp4.py:53-114): to fp16, swap the middle pair of every 4
   ([0, 2, 1, 3]), multiply by scale_factor and 2^7, zero values below 2, shift the fp16 bits left by one and keep
   the high byte ("S0E5M3": 5 exponent bits, 3 mantissa bits);
4. the global scale becomes gs * 2^(126 - 7) / scale_factor for bf16 activations
   (``nvfp4_marlin_process_global_scale``, marlin_utils_fp4.py:134-146, and :385-386).
"""
import numpy as np

from .nvfp4 import E4M3

SCALE_PERM = np.array([i + 8 * j for i in range(8) for j in range(8)], dtype=np.int64)  # marlin_utils.py:296-303
PAIR_SWAP = np.array([0, 2, 1, 3], dtype=np.int64)  # marlin_utils_fp4.py:91-93


def scale_factor(scales_u8: np.ndarray) -> float:
    """Shared power-of-two factor for all experts of one matrix (marlin_utils_fp4.py:30-50), in exact arithmetic."""
    v = E4M3[scales_u8].astype(np.float64) * 2.0 ** 7
    nz = v[v > 0]
    if nz.size == 0:
        return 1.0
    mx = float(nz.max())
    lim = 448.0 * 2.0 ** 7
    if mx >= lim:
        return 1.0
    j = 0
    while mx * 2.0 ** (j + 1) <= lim:
        j += 1
    return float(2.0 ** j)


def process_expert(scales_u8: np.ndarray, sf: float) -> np.ndarray:
    """One expert's checkpoint scales [N, K/16] (E4M3 bits) -> Marlin S0E5M3 bytes [K/16, N]."""
    n, kg = scales_u8.shape
    s = E4M3[scales_u8].T.reshape(-1, 64)[:, SCALE_PERM].reshape(kg, n)  # marlin_permute_scales
    h = s.astype(np.float16)
    h = h.reshape(-1, 4)[:, PAIR_SWAP].reshape(kg, n)
    if sf > 1.0:
        h = (h.astype(np.float32) * np.float32(sf)).astype(np.float16)
    h = h * np.float16(2 ** 7)
    h[h < 2] = 0
    bits = (h.view(np.uint16).astype(np.uint32) << 1) & 0xFFFF
    return (bits >> 8).astype(np.uint8)


def process_scales(scales_u8: np.ndarray):
    """All experts [E, N, K/16] -> (bytes [E, K/16, N], scale_factor)."""
    sf = scale_factor(scales_u8)
    return np.stack([process_expert(scales_u8[e], sf) for e in range(scales_u8.shape[0])]), sf


def process_global(gs: np.ndarray, sf: float) -> np.ndarray:
    """weight_scale_2 [E] -> the kernel's global multiplier gs * 2^119 / scale_factor (fp32)."""
    return (gs.astype(np.float32) * np.float32(2.0 ** 119) / np.float32(sf)).astype(np.float32)


def logical_column(pos: np.ndarray) -> np.ndarray:
    """Column of the original scale row held at position ``pos`` of a processed row (the two permutations above)."""
    pos = np.asarray(pos)
    base, p = pos - pos % 64, pos % 64
    m = (p // 4) * 4 + PAIR_SWAP[p % 4]
    return base + m // 8 + 8 * (m % 8)
