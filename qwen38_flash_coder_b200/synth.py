"""Seeded synthetic inputs with the benchmark's shapes and distributions (torch, any device).

The reference ships no fixtures (its real layer-10 cache is not public); these generators stand in for it:

- NVFP4 experts in the checkpoint layout (bench/moek/problem.py:1-7): ``weight`` uint8 [E, N, K/2] with element 2i
  in the low nibble, ``weight_scale`` float8 E4M3 [E, N, K/16], ``weight_scale_2`` fp32 [E]. Weights are drawn
  bf16 ~ N(0, 0.02) and quantised the way the reference's own quantiser does with its first candidate
  (build/make_fp4_variant.py:52-81, ``to_e2m1_codes`` / ``quant_nvfp4`` with f = 1): per-expert global
  ``weight_scale_2 = amax / (6 * 448)`` (gate and up share one), block scale ``E4M3(amax16 / 6 / weight_scale_2)``
  clamped to [2^-9, 448], codes = the nearest E2M1 magnitude (ties to the smaller one) with the sign in bit 3.
- Routing: softmax of N(0, 1) fp32 logits, top-k, renormalised (vLLM fused_topk, the router of the reference's
  model), or Zipf(s) expert popularity over a seeded permutation of the expert ids with k distinct experts per token
  drawn without replacement and weights = softmax of N(0, 1) logits at those ids.
"""
import torch

E2M1_MAG = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
_MIDS = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])


def quantize_nvfp4(w: torch.Tensor):
    """w [E, N, K] (bf16/fp32) -> (codes uint8 [E, N, K/2], scales float8_e4m3fn [E, N, K/16], gs fp32 [E])."""
    e, n, k = w.shape
    wf = w.float()
    gs = wf.abs().amax(dim=(1, 2)) / (6.0 * 448.0)
    gs = torch.where(gs > 0, gs, torch.ones_like(gs))
    b = wf.view(e, n, k // 16, 16)
    amax = b.abs().amax(-1, keepdim=True)
    s = (amax / 6.0 / gs.view(e, 1, 1, 1)).clamp(min=2 ** -9, max=448.0).to(torch.float8_e4m3fn)
    sv = s.float() * gs.view(e, 1, 1, 1)
    x = b / sv.clamp(min=1e-30)
    mag = torch.bucketize(x.abs().clamp(max=6.0), _MIDS.to(x.device), right=False)  # ties -> smaller magnitude
    c = (mag | ((x < 0).to(mag.dtype) << 3)).to(torch.uint8).view(e, n, k)
    codes = (c[..., 0::2] | (c[..., 1::2] << 4)).contiguous()
    return codes, s.view(e, n, k // 16).contiguous(), gs.float()


def make_experts(num_experts: int, n: int, k: int, seed: int, device="cpu", chunk: int = 64):
    """Seeded bf16 N(0, 0.02) experts [E, N, K] quantised to NVFP4, generated in expert chunks on ``device``."""
    g = torch.Generator(device=device).manual_seed(seed)
    codes = torch.empty((num_experts, n, k // 2), dtype=torch.uint8, device=device)
    scales = torch.empty((num_experts, n, k // 16), dtype=torch.float8_e4m3fn, device=device)
    gs = torch.empty((num_experts,), dtype=torch.float32, device=device)
    for e0 in range(0, num_experts, chunk):
        e1 = min(num_experts, e0 + chunk)
        w = (torch.randn((e1 - e0, n, k), generator=g, device=device) * 0.02).to(torch.bfloat16)
        codes[e0:e1], scales[e0:e1], gs[e0:e1] = quantize_nvfp4(w)
    return codes, scales, gs


def make_layer(num_experts: int, hidden: int, inter: int, seed: int, device="cpu"):
    """One layer: (w13, w2) checkpoint tuples; w13 stacks the gate rows then the up rows of each expert."""
    w13 = make_experts(num_experts, 2 * inter, hidden, 2 * seed, device)
    w2 = make_experts(num_experts, hidden, inter, 2 * seed + 1, device)
    return w13, w2


def activations(m: int, hidden: int, seed: int, device="cpu") -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn((m, hidden), generator=g).to(torch.bfloat16).to(device)


def route_softmax(m: int, num_experts: int, top_k: int, seed: int, device="cpu"):
    """softmax(N(0,1) logits) -> top-k -> renormalise: (ids int32 [M, k], weights fp32 [M, k])."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    logits = torch.randn((m, num_experts), generator=g, dtype=torch.float32)
    p = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(p, top_k, dim=-1)
    w = w / w.sum(-1, keepdim=True)
    return ids.to(torch.int32).to(device), w.float().to(device)


def route_zipf(m: int, num_experts: int, top_k: int, seed: int, s: float = 1.1, device="cpu"):
    """Zipf(s) popularity over a seeded permutation of expert ids; k distinct experts per token."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    perm = torch.randperm(num_experts, generator=g)
    pr = torch.arange(1, num_experts + 1, dtype=torch.float64).pow(-s)
    p = torch.empty(num_experts, dtype=torch.float64)
    p[perm] = pr / pr.sum()
    ids = torch.multinomial(p.float().expand(m, -1), top_k, replacement=False, generator=g)
    w = torch.softmax(torch.randn((m, top_k), generator=g, dtype=torch.float32), dim=-1)
    return ids.to(torch.int32).to(device), w.float().to(device)


def quantize_mxfp8(w: torch.Tensor):
    """w [N, K] (bf16/fp32) -> (codes uint8 [N, K] = float8_e4m3fn bits, scales uint8 [N, K/32] = E8M0 exponents):
    per block of 32 along K the smallest power-of-two scale that keeps amax / scale <= 448 (e4m3's largest value, so
    nothing saturates), elements = w / scale rounded to the nearest e4m3; an all-zero block takes scale 2^0."""
    n, k = w.shape
    wf = w.float().reshape(n, k // 32, 32)
    amax = wf.abs().amax(-1)
    e = torch.where(amax > 0, torch.ceil(torch.log2(amax.clamp_min(2.0 ** -126) / 448.0)), torch.zeros_like(amax))
    e = e.clamp(-127, 127)
    q = (wf / torch.exp2(e)[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(torch.uint8).reshape(n, k), (e + 127).to(torch.uint8)


def make_shared(hidden: int, inter: int, seed: int, device="cpu"):
    """A seeded MXFP8 shared expert (the kit's checkpoint format for it): (w_gu codes [2 inter, hidden] with the gate
    rows first, its scales [2 inter, hidden / 32], w_d codes [hidden, inter], its scales [hidden, inter / 32],
    shared_expert_gate bf16 [hidden]); weights bf16 N(0, 0.02), the gate vector N(0, 0.02)."""
    g = torch.Generator(device="cpu").manual_seed(7_000_000 + seed)
    w_gu = (torch.randn(2 * inter, hidden, generator=g) * 0.02).to(torch.bfloat16)
    w_d = (torch.randn(hidden, inter, generator=g) * 0.02).to(torch.bfloat16)
    w_sg = (torch.randn(hidden, generator=g) * 0.02).to(torch.bfloat16)
    gu, sgu = quantize_mxfp8(w_gu)
    d, sd = quantize_mxfp8(w_d)
    return tuple(t.to(device) for t in (gu, sgu, d, sd, w_sg))


def make_router_gate(num_experts: int, hidden: int, seed: int, device="cpu") -> torch.Tensor:
    """The router gate's bf16 weight [E, hidden], N(0, 0.02) (vLLM's unquantised ReplicatedLinear)."""
    g = torch.Generator(device="cpu").manual_seed(8_000_000 + seed)
    return (torch.randn(num_experts, hidden, generator=g) * 0.02).to(torch.bfloat16).to(device)
