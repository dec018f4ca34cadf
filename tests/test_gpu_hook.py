"""The vLLM hook on the GPU: a layer prepared through the wrapped prepare_nvfp4_moe_layer_for_marlin and called
through the wrapped fused_marlin_moe (vLLM's argument lists) gives ops.fused_moe's output bit for bit; calls the
kernels cannot serve raise, as the kit's hook does; and, where vLLM imports, install() routes vLLM's own module
functions the same way."""
import pytest
import torch

from qwen38_flash_coder_b200 import moek, ops, synth
from tests.hook_stubs import stub_fused, stub_prepare

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def _layer():
    return synth.make_layer(64, 2048, 512, 5, device=DEV)


def _check(prepare, fused):
    w13, w2 = _layer()
    tw13, s13, g13, tw2, s2, g2 = prepare(None, w13[0], w13[1], w13[2], w2[0], w2[1], w2[2], True)
    layer = moek._REG[tw13.data_ptr()]
    for m in (8, 300):  # decode and tcgen05 paths
        x = synth.activations(m, 2048, m, device=DEV)
        ids, wts = synth.route_zipf(m, 64, 5, m, device=DEV)
        out = torch.empty_like(x)
        r = fused(x, tw13, tw2, None, None, s13, s2, wts, ids, 0, output=out, global_scale1=g13, global_scale2=g2)
        assert r is out
        assert torch.equal(out, ops.fused_moe(x, layer, wts, ids))
    x = synth.activations(4, 2048, 1, device=DEV)
    ids, wts = synth.route_zipf(4, 64, 5, 1, device=DEV)
    with pytest.raises(RuntimeError):
        fused(x, tw13, tw2, None, None, s13, s2, wts, ids, 0, expert_map=torch.arange(64, device=DEV))
    empty = torch.empty((0, 2048), dtype=torch.bfloat16, device=DEV)
    assert fused(empty, tw13, tw2, None, None, s13, s2, wts[:0], ids[:0], 0).shape == (0, 2048)
    ops.check_device_errors(DEV)


def test_hook_wrappers_match_fused_moe():
    _check(moek._prep_wrap(stub_prepare), moek._fused_wrap(stub_fused))


def test_install_routes_vllm_functions():
    mm = pytest.importorskip("vllm.model_executor.layers.fused_moe.experts.marlin_moe")
    import vllm.model_executor.layers.quantization.utils.marlin_utils_fp4 as mu

    moek.install()
    _check(mu.prepare_nvfp4_moe_layer_for_marlin, mm.fused_marlin_moe)


@pytest.mark.parametrize("t", [1, 5, 8, 12, 13, 31, 128, 700, 6912])
def test_serve_path_sweep(t):
    """The serving call path across batch sizes, as the reference's serve_path harness drives it
    (bench/moek/serve_path.py:19-27: T in {1, 5, 8, 12, 13, 31, 128, 700, 6912}, keyword arguments, vLLM's own
    prepare_nvfp4_moe_layer_for_marlin and fused_marlin_moe after install()): every size against the fp32 oracle
    within the parity gate (the reference compares with Marlin, which does not run here)."""
    from oracle import moe_ref

    mm = pytest.importorskip("vllm.model_executor.layers.fused_moe.experts.marlin_moe")
    import vllm.model_executor.layers.quantization.utils.marlin_utils_fp4 as mu

    moek.install()
    e = 128
    w13, w2 = synth.make_layer(e, 2048, 512, 40, device=DEV)
    out = mu.prepare_nvfp4_moe_layer_for_marlin(None, w13[0], w13[1], w13[2], w2[0], w2[1], w2[2], True)
    x = (synth.activations(t, 2048, t, device=DEV).float() * 0.5).to(torch.bfloat16)
    ids, wts = synth.route_softmax(t, e, 5, t, device=DEV)
    y = mm.fused_marlin_moe(hidden_states=x, w1=out[0], w2=out[3], bias1=None, bias2=None, w1_scale=out[1],
                            w2_scale=out[4], topk_weights=wts, topk_ids=ids, quant_type_id=0, global_scale1=out[2],
                            global_scale2=out[5])
    ops.check_device_errors(DEV)
    ck = lambda mat: (mat[0].cpu().numpy(), mat[1].view(torch.uint8).cpu().numpy(), mat[2].cpu().numpy())
    ref = moe_ref.reference(x.cpu(), ids.cpu().numpy(), wts.cpu().numpy(), ck(w13), ck(w2))
    ok, stats = moe_ref.within_gate(y.cpu(), ref)
    assert ok, (t, stats)
