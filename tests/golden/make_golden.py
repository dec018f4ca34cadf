"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's own Python code on the CPU.

Run in the build container (it needs the reference sources and vLLM 0.22.0's Python):

    python tests/golden/make_golden.py /path/to/reference

What runs, and what it pins:

- bench/moek/problem.py ``make_weights`` (the reference's own seeded NVFP4 fixture generator, with DEV set to "cpu")
  for the checkpoint tensors of a small layer (E=8, hidden 256, intermediate 256);
- vLLM's scale helpers ``_nvfp4_compute_scale_factor``, ``marlin_permute_scales``, ``nvfp4_marlin_process_scales``
  and ``nvfp4_marlin_process_global_scale`` in the order ``prepare_nvfp4_moe_layer_for_marlin`` calls them
  (vllm/.../marlin_utils_fp4.py:355-386) -> the Marlin scale bytes and global scales;
- files/mbx_moek.py ``pack_scales`` / ``tile_scales`` / ``unpack_scales`` -> the packed-scale fixtures;
- bench/moek/problem.py ``reference`` (module globals set to the small geometry) -> the layer output for every row;
- build/make_fp4_variant.py ``to_e2m1_codes`` -> E2M1 codes for a sweep of values (pins the quantiser's rounding).

The same is repeated for a realistic-statistics matrix (N(0, 0.02) weights quantised by this build's synthetic
quantiser, whose scales sit in a narrow band, unlike make_weights' U(30, 300)). The moe_align fixture is the
docstring example of vllm/.../moe_align_block_size.py:59-72 (experts renumbered from 0), because the compiled op
cannot run without a GPU.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main(ref_root: str):
    sys.path.insert(0, os.path.join(ref_root, "files"))
    sys.path.insert(0, os.path.join(ref_root, "bench", "moek"))
    sys.path.insert(0, os.path.join(ref_root, "build"))
    sys.path.insert(0, REPO)
    import mbx_moek as kit
    import problem as P
    import make_fp4_variant as Q
    from vllm.model_executor.layers.quantization.utils.marlin_utils import marlin_permute_scales
    from vllm.model_executor.layers.quantization.utils.marlin_utils_fp4 import (
        _nvfp4_compute_scale_factor, nvfp4_marlin_process_global_scale, nvfp4_marlin_process_scales)
    from qwen38_flash_coder_b200 import synth

    P.DEV = "cpu"
    E, HID, INTER, TOPK = 8, 256, 256, 5
    P.E, P.HID, P.INTER, P.TOPK = E, HID, INTER, TOPK

    def vllm_scales(s, size_n, size_k):
        """The scale half of prepare_nvfp4_moe_layer_for_marlin (marlin_utils_fp4.py:355-386)."""
        s = s.to(torch.bfloat16)
        sf = _nvfp4_compute_scale_factor(s, torch.bfloat16)
        out = []
        for i in range(s.shape[0]):
            ms = marlin_permute_scales(s=s[i].T, size_k=size_k, size_n=size_n, group_size=16, is_a_8bit=False)
            ms, _ = nvfp4_marlin_process_scales(ms, scale_factor=sf, a_dtype=torch.bfloat16)
            out.append(ms)
        return torch.stack(out).view(torch.uint8), sf

    fx = {}
    # ---- the reference's own fixture generator: make_weights (U(30,300) scales: many exceptions)
    w13 = P.make_weights(2 * INTER, HID, 1, e=E)
    w2 = P.make_weights(HID, INTER, 2, e=E)
    sets = {"mw13": (w13, 2 * INTER, HID, True), "mw2": (w2, HID, INTER, False)}
    # ---- realistic statistics: N(0, 0.02) weights through this build's quantiser
    r13 = synth.make_experts(E, 2 * INTER, HID, 11)
    r2 = synth.make_experts(E, HID, INTER, 12)
    sets["rw13"] = (r13, 2 * INTER, HID, True)
    sets["rw2"] = (r2, HID, INTER, False)
    # ---- tiny E4M3 scales (subnormals included): scale_factor > 1 and the "zero below 2" rule
    g = torch.Generator().manual_seed(5)
    tiny = torch.randint(1, 0x48, (E, HID, INTER // 16), generator=g, dtype=torch.uint8).view(torch.float8_e4m3fn)
    sets["tw2"] = ((w2[0], tiny, w2[2]), HID, INTER, False)
    for name, ((codes, scales, gs), n, k, gu) in sets.items():
        sb, sf = vllm_scales(scales, n, k)
        g = nvfp4_marlin_process_global_scale(gs.float(), torch.bfloat16) / sf
        packed, off, ent = kit.pack_scales(sb.contiguous(), gu)
        back = kit.unpack_scales(packed, off, ent, sb.shape[1], sb.shape[2])
        assert torch.equal(back, sb), name
        tiled = kit.tile_scales(packed, n, gu)
        fx[f"{name}_codes"] = codes.numpy()
        fx[f"{name}_scales"] = scales.view(torch.uint8).numpy()
        fx[f"{name}_gs"] = gs.float().numpy()
        fx[f"{name}_sbytes"] = sb.numpy()
        fx[f"{name}_sf"] = np.array([sf], dtype=np.float64)
        fx[f"{name}_g"] = g.float().numpy()
        fx[f"{name}_packed"] = packed.numpy()
        fx[f"{name}_exc_off"] = off.numpy()
        fx[f"{name}_exc_ent"] = ent.numpy()
        fx[f"{name}_tiled"] = tiled.numpy()
        print(f"{name}: N={n} K={k} sf={sf} exceptions={int(off[-1])} ({int(off[-1]) / sb.numel() * 100:.2f} %)")

    # ---- the reference's layer oracle on make_weights' layer, every row
    torch.manual_seed(0)
    M = 6
    x = (torch.randn((M, HID)) * 0.5).to(torch.bfloat16)
    ids, wts = P.routing(M, seed=3)
    out = P.reference(x, ids, wts, w13, w2)
    fx["moe_x"] = x.view(torch.int16).numpy()
    fx["moe_ids"] = ids.numpy()
    fx["moe_wts"] = wts.numpy()
    fx["moe_out"] = out.numpy()

    # ---- E2M1 rounding of the reference quantiser on a value sweep (ties included)
    sweep = torch.cat([torch.linspace(-7, 7, 2801), torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25,
                                                                  -0.75, -2.5, -5.0, 0.0, -0.0, 6.0, 8.0, -9.0])])
    codes, _ = Q.to_e2m1_codes(sweep)
    fx["e2m1_in"] = sweep.numpy()
    fx["e2m1_codes"] = codes.numpy()

    # ---- moe_align: vllm/.../moe_align_block_size.py:59-72 with experts renumbered 1..4 -> 0..3
    fx["align_ids"] = np.array([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]], dtype=np.int32) - 1
    fx["align_sorted"] = np.array([3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12, 2, 5, 8, 12], dtype=np.int32)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **fx)
    print("wrote", os.path.join(HERE, "golden.npz"))


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOEK_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: python tests/golden/make_golden.py <checkout of the reference project> "
                 "(or set MOEK_REFERENCE_ROOT)")
    main(root)
