"""Seeded synthetic inputs and weights with the BASELINE shapes and distributions.

No checkpoints or datasets are used.  Distributions follow the benchmark
configs: activations N(0, 1) in bf16, router weight N(0, 0.02) in bf16,
correction bias N(0, 0.01), expert and shared weights N(0, 0.02).  Expert
weights are drawn per expert as full [2I, H] gate/up and [H, I] down
matrices, sliced to this rank's TP shard the way the reference shards them
(crates/glm-reference/src/manifest.rs:143-165: gate and up rows split
independently then concatenated gate-first; down split along K), and packed
to NVFP4 per shard (each shard has its own global scale, nvfp4.rs:142-149).
"""
from __future__ import annotations

import math

import torch

from .moe import Exl3Experts, MoEConfig, RankWeights, pack_nvfp4


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_input(tokens: int, hidden: int, seed: int, device) -> torch.Tensor:
    return torch.randn(tokens, hidden, generator=_gen(device, seed * 7919 + 11),
                       device=device).to(torch.bfloat16)


def zipf_bias(experts: int, seed: int, beta: float, s: float = 1.1, device="cpu") -> torch.Tensor:
    """Correction bias bias_e = beta * (-s * ln(1 + pi(e))) over a seeded permutation
    pi, which skews per-expert token counts towards a Zipf(s) profile."""
    g = torch.Generator()
    g.manual_seed(seed * 31 + 5)
    perm = torch.randperm(experts, generator=g).to(torch.float32)
    return (beta * (-s * torch.log1p(perm))).to(device)


def make_router(cfg: MoEConfig, seed: int, device, zipf_beta: float | None = None):
    """Router weight bf16 [E, H] ~ N(0, 0.02) and correction bias f32 [E] ~ N(0, 0.01),
    plus the Zipf skew term when zipf_beta is given (identical on every rank)."""
    E, H = cfg.experts, cfg.hidden
    router_w = (torch.randn(E, H, generator=_gen(device, seed * 1000 + 1), device=device) *
                0.02).to(torch.bfloat16)
    bias = torch.randn(E, generator=_gen(device, seed * 1000 + 2), device=device) * 0.01
    if zipf_beta is not None:
        bias = bias + zipf_bias(E, seed, zipf_beta, device=device)
    return router_w, bias


def make_shared(cfg: MoEConfig, seed: int, device):
    """bf16 shared-expert shard of rank cfg.rank: gate/up rows [2*Is_r, H] (rank
    gate rows then up rows) and down [H, Is_r], from full N(0, 0.02) matrices;
    (None, None) without a shared expert."""
    if not cfg.shared_intermediate:
        return None, None
    H, r = cfg.hidden, cfg.rank
    Is, Isr = cfg.shared_intermediate, cfg.local_shared
    gen = _gen(device, seed * 1000 + 7)
    f13 = torch.randn(2 * Is, H, generator=gen, device=device) * 0.02
    f2 = torch.randn(H, Is, generator=gen, device=device) * 0.02
    shared13 = torch.cat([f13[r * Isr:(r + 1) * Isr], f13[Is + r * Isr:Is + (r + 1) * Isr]]
                         ).to(torch.bfloat16).contiguous()
    shared2 = f2[:, r * Isr:(r + 1) * Isr].to(torch.bfloat16).contiguous()
    return shared13, shared2


def make_rank_weights(cfg: MoEConfig, seed: int, device, *, zipf_beta: float | None = None,
                      expert_chunk: int = 8, keep_masters: bool = False,
                      only_experts: torch.Tensor | None = None):
    """Router (replicated), NVFP4 expert shards and bf16 shared shard of rank cfg.rank.
    only_experts (bool [E]): generate and pack only those experts; the others are
    all-zero NVFP4 tensors (global scale 1), for layers that never route to them."""
    E, H, I, Ir, r = cfg.experts, cfg.hidden, cfg.intermediate, cfg.local_intermediate, cfg.rank
    router_w, bias = make_router(cfg, seed, device, zipf_beta)
    w13_parts, w2_parts = [], []
    masters = []
    for e0 in range(0, E, expert_chunk):
        ne = min(expert_chunk, E - e0)
        g13 = torch.empty((ne, 2 * Ir, H), dtype=torch.float32, device=device)
        g2 = torch.empty((ne, H, Ir), dtype=torch.float32, device=device)
        for j in range(ne):
            if only_experts is not None and not bool(only_experts[e0 + j]):
                g13[j].zero_()
                g2[j].zero_()
                continue
            gen = _gen(device, seed * 1000003 + 17 * (e0 + j) + 3)
            full13 = torch.randn(2 * I, H, generator=gen, device=device) * 0.02
            full2 = torch.randn(H, I, generator=gen, device=device) * 0.02
            g13[j, :Ir] = full13[r * Ir:(r + 1) * Ir]
            g13[j, Ir:] = full13[I + r * Ir:I + (r + 1) * Ir]
            g2[j] = full2[:, r * Ir:(r + 1) * Ir]
            if keep_masters:
                masters.append((g13[j].clone(), g2[j].clone()))
        w13_parts.append(pack_nvfp4(g13))
        w2_parts.append(pack_nvfp4(g2))
        del g13, g2

    def cat(parts):
        from .moe import PackedNvfp4
        return PackedNvfp4(torch.cat([p.values for p in parts]), torch.cat([p.scales for p in parts]),
                           torch.cat([p.global_scale for p in parts]),
                           torch.cat([p.global_amax for p in parts]), parts[0].n, parts[0].k)

    shared13, shared2 = make_shared(cfg, seed, device)
    w = RankWeights(router_w.contiguous(), bias.contiguous(), cat(w13_parts), cat(w2_parts),
                    shared13, shared2)
    return (w, masters) if keep_masters else w


def approx_route_counts(logits: torch.Tensor, bias: torch.Tensor, groups: int,
                        topk_groups: int, top_k: int) -> torch.Tensor:
    """Per-expert assignment counts of group-limited sigmoid top-k routing, computed
    with plain torch ops.  Input synthesis only (fitting the Zipf skew): tie order
    and summation order are not the layer's."""
    T, E = logits.shape
    gs = E // groups
    choice = torch.sigmoid(logits) + bias
    gscore = choice.view(T, groups, gs).topk(min(2, gs), dim=-1).values.sum(-1)
    keep = gscore.topk(topk_groups, dim=-1).indices
    mask = torch.zeros(T, groups, dtype=torch.bool, device=logits.device).scatter_(1, keep, True)
    masked = choice.masked_fill(~mask.repeat_interleave(gs, 1), float("-inf"))
    sel = masked.topk(top_k, dim=-1).indices
    return torch.bincount(sel.flatten(), minlength=E)


def zipf_slope(counts: torch.Tensor) -> float:
    """Least-squares slope of log(count) against log(rank) over the non-zero counts."""
    c = counts.double().sort(descending=True).values
    c = c[c > 0]
    lr = torch.arange(1, c.numel() + 1, dtype=torch.float64, device=c.device).log()
    lc = c.log()
    lr0, lc0 = lr - lr.mean(), lc - lc.mean()
    return float((lr0 * lc0).sum() / (lr0 * lr0).sum())


def fit_zipf_beta(cfg: MoEConfig, tokens: int, seed: int, device, s: float = 1.1,
                  iters: int = 30) -> tuple[float, float]:
    """Bisection on beta so that the log-log slope of the sorted per-expert token
    counts is -s under this seed's router and input.  Returns (beta, slope)."""
    x = make_input(tokens, cfg.hidden, seed, device).float()
    router_w, bias0 = make_router(cfg, seed, device, None)
    logits = x @ router_w.float().t()
    lo, hi = 0.0, 2.0
    best = (0.0, 0.0)
    for _ in range(iters):
        mid = 0.5 * (lo + hi)
        bias = bias0 + zipf_bias(cfg.experts, seed, mid, s=s, device=device)
        slope = zipf_slope(approx_route_counts(logits, bias, cfg.groups, cfg.topk_groups,
                                               cfg.top_k))
        best = (mid, slope)
        if -slope < s:
            lo = mid
        else:
            hi = mid
    return best


def exl3_decoded_std() -> float:
    """Standard deviation of the 3INST decoded weight over uniformly random 16-bit
    trellis windows (value = window * 0xCBAC1FED, (value & 0x8FFF8FFF) ^ 0x3B603B60
    read as two fp16 halves, summed; exl3.rs:471-477)."""
    import numpy as np
    w = np.arange(65536, dtype=np.uint64)
    v = ((w * 0xCBAC1FED) & 0xFFFFFFFF) & 0x8FFF8FFF ^ 0x3B603B60
    lo = (v & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
    hi = (v >> 16).astype(np.uint16).view(np.float16).astype(np.float32)
    return float(np.std((lo + hi).astype(np.float16).astype(np.float32)))


def make_exl3_experts(cfg: MoEConfig, seed: int, device, codec: torch.Tensor | None = None,
                      weight_std: float = 0.02) -> Exl3Experts:
    """Seeded EXL3 3-bit expert shards of rank cfg.rank.  The reference's CPU
    encoder is not part of the reference repository, so the trellis words are
    seeded random, as in its own fixtures (exl3.rs:667-684); suh holds random
    signs and svh random signs of magnitude weight_std / std(decoded weight),
    which gives the effective weights (H128-rotated on both sides) std weight_std."""
    E, H, Ir, r = cfg.experts, cfg.hidden, cfg.local_intermediate, cfg.rank
    g = _gen(device, seed * 7717 + 101 * r + 13)
    words_gu = (H // 16) * (Ir // 16) * 48

    def trellis():
        return torch.randint(-32768, 32768, (E, words_gu), generator=g, device=device,
                             dtype=torch.int32).to(torch.int16)

    def signs(n, mag):
        s = torch.randint(0, 2, (E, n), generator=g, device=device).to(torch.float32) * 2 - 1
        return (s * mag).to(torch.float16)

    mag = weight_std / exl3_decoded_std()
    return Exl3Experts(gate_trellis=trellis(), up_trellis=trellis(), down_trellis=trellis(),
                       gate_suh=signs(H, 1.0), gate_svh=signs(Ir, mag),
                       up_suh=signs(H, 1.0), up_svh=signs(Ir, mag),
                       down_suh=signs(Ir, 1.0), down_svh=signs(H, mag), codec=codec)


def make_exl3_rank_weights(cfg: MoEConfig, seed: int, device, *, zipf_beta: float | None = None,
                           nvfp4_experts: torch.Tensor | None = None) -> RankWeights:
    """Router, EXL3 experts and bf16 shared shard of rank cfg.rank.  With
    nvfp4_experts (a bool [E] mask) the layer is hybrid: those experts use NVFP4
    weights (generated as make_rank_weights does) and the rest EXL3."""
    if nvfp4_experts is None:
        router_w, bias = make_router(cfg, seed, device, zipf_beta)
        shared13, shared2 = make_shared(cfg, seed, device)
        return RankWeights(router_w.contiguous(), bias.contiguous(), None, None, shared13,
                           shared2, make_exl3_experts(cfg, seed, device))
    w = make_rank_weights(cfg, seed, device, zipf_beta=zipf_beta, only_experts=nvfp4_experts)
    codec = (~nvfp4_experts.to(device)).to(torch.uint8)
    w.exl3 = make_exl3_experts(cfg, seed, device, codec=codec)
    return w
