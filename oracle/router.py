"""The MoE router restated on the CPU (test infrastructure only): vLLM's fused_topk with scoring "softmax"
(vllm/model_executor/layers/fused_moe/router/fused_topk_router.py:69-108; the compiled topk_softmax op it calls is not
in this container, so the definition below is this build's): p = softmax(logits) in fp32, the top_k largest p with the
lowest expert index first among equal p, weights = those p, divided by their sum when renormalising;
token_expert_indices = j * M + t for slot j of token t. The same computation as the synthetic router
(qwen38_flash_coder_b200/synth.py ``route_softmax``: torch.softmax, torch.topk, renormalise)."""
import numpy as np


def topk_softmax(logits: np.ndarray, top_k: int, renormalize: bool = True):
    """(ids int32 [M, k], weights fp32 [M, k], token_expert_indices int32 [M, k]) from fp32 logits [M, E]."""
    x = np.asarray(logits, dtype=np.float32)
    m, e = x.shape
    mx = x.max(axis=1, keepdims=True)
    ex = np.exp(x - mx, dtype=np.float32)
    p = (ex / ex.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    ids = np.empty((m, top_k), dtype=np.int32)
    w = np.empty((m, top_k), dtype=np.float32)
    idx = np.arange(e)
    for t in range(m):
        order = np.lexsort((idx, -p[t]))[:top_k]  # p descending, expert ascending on ties
        ids[t] = order
        w[t] = p[t, order]
    if renormalize:
        w = (w / w.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    tei = (np.arange(top_k)[None, :] * m + np.arange(m)[:, None]).astype(np.int32)
    return ids, w, tei
