"""vLLM hook: routes the NVFP4 routed-expert layers' Marlin MoE calls to this build's kernels.

The same two rebinds as the kit's hook (files/mbx_moek.py:296-330, ``install``):

- load time: ``prepare_nvfp4_moe_layer_for_marlin(layer, w13, w13_scale, w13_scale_2, w2, w2_scale, w2_scale_2,
  is_act_and_mul)`` (vllm/.../marlin_utils_fp4.py:288-298, also bound in ``fused_moe/oracle/nvfp4.py``) is wrapped.
  The kit's wrapper converts the Marlin-prepared tensors (files/mbx_moek.py:186-229); this one prepares the layer
  from the wrapped function's checkpoint inputs (``prep.PreparedLayer``: the kit's packed scales, this build's weight
  layout), registers it under the returned gate_up tensor's address and returns (tiled w13, placeholder scale, global
  scale, tiled w2, placeholder scale, global scale) in place of Marlin's tensors. A layer that is not plain NVFP4
  (not act-and-mul, other shapes or dtypes, not on a GPU) stays on the wrapped function, with a one-time warning;
- forward: ``fused_marlin_moe`` (vllm/.../fused_moe/experts/marlin_moe.py, signature at :225-258) is wrapped; a call
  whose ``w1`` is registered runs ``ops.fused_moe`` (align, gate_up + SwiGLU, down x router weight, top-k sum, one
  bf16 rounding) into ``output``, any other call goes to the original. Like the kit (files/mbx_moek.py:245-255) the
  wrapper raises ``RuntimeError`` for calls it cannot serve: biases, ``expert_map``, router weights applied on the
  input, a non-SiLU activation, a different ``global_num_experts`` or 8-bit inputs. The top-k sum is part of the
  kernels, so ``moe_sum`` is not called (it is vLLM's sum over the top-k slots).

``install()`` is idempotent; ``report()`` logs the converted layers and the scale bytes, as the kit's does.
"""
import inspect
import logging

import torch

from . import ops, prep
from ._lib import lib

_REG: dict = {}
_S = {"layers": 0, "bytes_plain": 0, "bytes_packed": 0, "warned": False}


def _log():
    return logging.getLogger("moek_b200")


def _plain_nvfp4(w13, s13, g13, w2, s2, g2, act_and_mul) -> bool:
    try:
        e, n13, k13 = w13.shape
        _, n2, k2 = w2.shape
        return (bool(act_and_mul) and w13.is_cuda and w13.dtype == torch.uint8 and w2.dtype == torch.uint8
                and s13.dtype == torch.float8_e4m3fn and s2.dtype == torch.float8_e4m3fn
                and tuple(s13.shape) == (e, n13, 2 * k13 // 16) and tuple(s2.shape) == (e, n2, 2 * k2 // 16)
                and w2.shape[0] == e and n13 % 256 == 0 and n2 % 256 == 0 and (2 * k13) % 128 == 0
                and (2 * k2) % 128 == 0 and g13.numel() in (e, 2 * e) and g2.numel() == e)
    except (AttributeError, ValueError, TypeError):
        return False


def _global(g, e):
    """Per-expert fp32 global scale; a [E, 2] gate / up pair must agree (the kernels take one per expert)."""
    g = g.float().reshape(e, -1)
    if g.shape[1] == 2 and not torch.equal(g[:, 0], g[:, 1]):
        raise RuntimeError("moek_b200: gate and up carry different global scales; the kernels take one per expert")
    return g[:, 0].contiguous()


def _prep_wrap(orig):
    sig = inspect.signature(orig)

    def prepare(*args, **kwargs):
        a = sig.bind(*args, **kwargs).arguments
        w13, s13, g13 = a["w13"], a["w13_scale"], a["w13_scale_2"]
        w2, s2, g2 = a["w2"], a["w2_scale"], a["w2_scale_2"]
        if not _plain_nvfp4(w13, s13, g13, w2, s2, g2, a.get("is_act_and_mul", True)):
            if not _S["warned"]:
                _S["warned"] = True
                _log().warning("moek_b200: a MoE layer is not plain NVFP4 on a GPU (weights %s, scales %s): it "
                               "stays on Marlin", getattr(w13, "dtype", None), getattr(s13, "dtype", None))
            return orig(*args, **kwargs)
        lib()
        e = w13.shape[0]
        layer = prep.PreparedLayer((w13, s13, _global(g13, e)), (w2, s2, _global(g2, e)))
        _S["bytes_plain"] += s13.numel() + s2.numel()
        _S["bytes_packed"] += sum(m.sp.numel() + 4 * (m.exc_off.numel() + m.exc_ent.numel())
                                  for m in (layer.w13, layer.w2))
        _REG[layer.w13.w.data_ptr()] = layer
        _S["layers"] += 1
        placeholder = torch.zeros(1, dtype=s13.dtype, device=w13.device)
        return layer.w13.w, placeholder, layer.w13.g, layer.w2.w, placeholder.clone(), layer.w2.g

    prepare._moek_b200 = True
    return prepare


def _fused_wrap(orig):
    sig = inspect.signature(orig)

    def fused(*args, **kwargs):
        a = sig.bind(*args, **kwargs).arguments
        w1 = a["w1"]
        layer = _REG.get(w1.data_ptr())
        if layer is None:
            return orig(*args, **kwargs)
        x, w2 = a["hidden_states"], a["w2"]
        act_kind = a.get("activation")
        if (a.get("bias1") is not None or a.get("bias2") is not None or a.get("expert_map") is not None
                or a.get("apply_router_weight_on_input") or w2.data_ptr() != layer.w2.w.data_ptr()
                or (act_kind is not None and "SILU" not in str(act_kind).upper())
                or a.get("global_num_experts", -1) not in (-1, layer.E)
                or (a.get("input_dtype") is not None and a["input_dtype"].itemsize == 1)):
            raise RuntimeError("moek_b200: unsupported fused_marlin_moe call for this build's weights: "
                               f"activation {act_kind}, expert_map {a.get('expert_map') is not None}, "
                               f"bias {a.get('bias1') is not None}, input_dtype {a.get('input_dtype')}")
        output = a.get("output")
        if x.shape[0] == 0:  # empty batch (vLLM dummy runs)
            return output if output is not None else torch.empty_like(x)
        return ops.fused_moe(x, layer, a["topk_weights"], a["topk_ids"], output=output)

    fused._moek_b200 = True
    return fused


def install() -> None:
    """Rebind vLLM's NVFP4 Marlin MoE preparation and forward to this build (once per process)."""
    import vllm.model_executor.layers.fused_moe.experts.marlin_moe as mm
    import vllm.model_executor.layers.quantization.utils.marlin_utils_fp4 as mu

    if getattr(mm.fused_marlin_moe, "_moek_b200", False):
        return
    wrapped = _prep_wrap(mu.prepare_nvfp4_moe_layer_for_marlin)
    mu.prepare_nvfp4_moe_layer_for_marlin = wrapped
    try:
        import vllm.model_executor.layers.fused_moe.oracle.nvfp4 as onv

        onv.prepare_nvfp4_moe_layer_for_marlin = wrapped
    except ImportError:
        pass
    mm.fused_marlin_moe = _fused_wrap(mm.fused_marlin_moe)
    lib()  # load the library now, not in the middle of the weight processing
    _log().info("moek_b200: routed experts on the B200 kernels (split-k decode up to %d tokens, tcgen05 above)",
                ops.DECODE_MAX_M)


def report() -> None:
    if _S["layers"]:
        _log().info("moek_b200: %d MoE layers converted; expert scales %.2f GB plain -> %.2f GB packed",
                    _S["layers"], _S["bytes_plain"] / 1e9, _S["bytes_packed"] / 1e9)
