"""The vLLM hook's host logic on the CPU: layers it cannot serve stay on the wrapped functions, unregistered calls
pass through, and install() rebinds vLLM's functions once (when vLLM imports here)."""
import pytest
import torch

from qwen38_flash_coder_b200 import moek, synth
from tests.hook_stubs import Reached, stub_fused, stub_prepare


def test_prepare_falls_back_for_cpu_or_non_nvfp4_layers():
    w13, w2 = synth.make_layer(4, 256, 256, 1)  # CPU tensors: the kernels need a GPU, so Marlin keeps the layer
    prep = moek._prep_wrap(stub_prepare)
    with pytest.raises(Reached):
        prep(None, w13[0], w13[1], w13[2], w2[0], w2[1], w2[2], True)
    with pytest.raises(Reached):  # not act-and-mul
        prep(None, w13[0], w13[1], w13[2], w2[0], w2[1], w2[2], is_act_and_mul=False)
    assert prep._moek_b200


def test_fused_passes_unregistered_weights_through():
    fused = moek._fused_wrap(stub_fused)
    w = torch.zeros((2, 4, 8), dtype=torch.int32)
    with pytest.raises(Reached):
        fused(torch.zeros((1, 8)), w, w, None, None, None, None, torch.ones((1, 1)), torch.zeros((1, 1)), 0)


def test_install_rebinds_vllm_once():
    mm = pytest.importorskip("vllm.model_executor.layers.fused_moe.experts.marlin_moe")
    import vllm.model_executor.layers.quantization.utils.marlin_utils_fp4 as mu

    before = mm.fused_marlin_moe
    moek.install()
    assert mm.fused_marlin_moe._moek_b200 and mu.prepare_nvfp4_moe_layer_for_marlin._moek_b200
    after = mm.fused_marlin_moe
    moek.install()  # idempotent
    assert mm.fused_marlin_moe is after and after is not before
