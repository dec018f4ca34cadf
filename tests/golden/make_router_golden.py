"""Generate tests/golden/router_golden.npz by running vLLM's own torch routing code on the CPU.

Run in the build container (it needs vLLM 0.22.0's Python sources; no GPU):

    python tests/golden/make_router_golden.py

vLLM's fused_topk (vllm/model_executor/layers/fused_moe/router/fused_topk_router.py:69-108, the router in front of
the reference's MoE layer) calls the compiled topk_softmax op, which cannot run here. Its torch restatement in the
same package, ``grouped_topk`` (vllm/.../router/grouped_topk_router.py:81-153), with one expert group
(num_expert_group = topk_group = 1) and scoring "softmax" computes the same thing: softmax over the experts in
fp32, the top_k largest probabilities, renormalised by their sum when asked. This script runs the undecorated
function (``torch.compile`` skipped) on seeded fp32 logits and stores the logits, the chosen ids and the weights.

Ties. vLLM's torch path returns the members of a tie in no defined order (``torch.topk(..., sorted=False)``; with
all-equal logits it picked experts 41-46 of 64 here). The cases below therefore contain no ties among the chosen or
at the boundary of the top_k (checked at generation); the lowest-index rule for ties is this build's definition
(oracle/router.py) and is tested against the oracle on its own.
"""
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [  # (name, tokens, experts, top_k, renormalize, seed)
    ("m8_e512_k5", 8, 512, 5, True, 0),
    ("m64_e512_k5", 64, 512, 5, True, 1),
    ("m64_e512_k5_raw", 64, 512, 5, False, 2),
    ("m33_e64_k5", 33, 64, 5, True, 3),
    ("m16_e128_k8", 16, 128, 8, True, 4),
    ("m7_e1024_k32", 7, 1024, 32, False, 5),
]


def grouped_topk_fn():
    from vllm.model_executor.layers.fused_moe.router import grouped_topk_router as g

    f = g.grouped_topk
    return getattr(f, "_torchdynamo_orig_callable", None) or getattr(f, "__wrapped__", None) or f


def main():
    fn = grouped_topk_fn()
    out = {}
    for name, m, e, k, renorm, seed in CASES:
        logits = torch.randn((m, e), generator=torch.Generator().manual_seed(1000 + seed), dtype=torch.float32)
        w, ids = fn(torch.zeros((m, 8)), logits, k, renorm, num_expert_group=1, topk_group=1,
                    scoring_func="softmax")
        p = torch.softmax(logits, dim=-1)
        srt = torch.sort(p, dim=-1, descending=True).values
        assert bool((srt[:, : k + 1][:, 1:] < srt[:, : k + 1][:, :-1]).all()), f"{name}: tie among the top_k + 1"
        out[f"{name}_logits"] = logits.numpy()
        out[f"{name}_ids"] = ids.numpy().astype(np.int32)
        out[f"{name}_w"] = w.numpy().astype(np.float32)
        out[f"{name}_meta"] = np.array([m, e, k, int(renorm)], dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "router_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "router_golden.npz"), sorted(out)[:4], "...")


if __name__ == "__main__":
    main()
