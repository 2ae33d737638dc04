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

from .moe import MoEConfig, RankWeights, pack_nvfp4


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


def make_rank_weights(cfg: MoEConfig, seed: int, device, *, zipf_beta: float | None = None,
                      expert_chunk: int = 8, keep_masters: bool = False):
    """Router (replicated), NVFP4 expert shards and bf16 shared shard of rank cfg.rank."""
    E, H, I, Ir, r = cfg.experts, cfg.hidden, cfg.intermediate, cfg.local_intermediate, cfg.rank
    router_w = (torch.randn(E, H, generator=_gen(device, seed * 1000 + 1), device=device) *
                0.02).to(torch.bfloat16)
    bias = torch.randn(E, generator=_gen(device, seed * 1000 + 2), device=device) * 0.01
    if zipf_beta is not None:
        bias = bias + zipf_bias(E, seed, zipf_beta, device=device)
    w13_parts, w2_parts = [], []
    masters = []
    for e0 in range(0, E, expert_chunk):
        ne = min(expert_chunk, E - e0)
        g13 = torch.empty((ne, 2 * Ir, H), dtype=torch.float32, device=device)
        g2 = torch.empty((ne, H, Ir), dtype=torch.float32, device=device)
        for j in range(ne):
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

    shared13 = shared2 = None
    if cfg.shared_intermediate:
        Is, Isr = cfg.shared_intermediate, cfg.local_shared
        gen = _gen(device, seed * 1000 + 7)
        f13 = torch.randn(2 * Is, H, generator=gen, device=device) * 0.02
        f2 = torch.randn(H, Is, generator=gen, device=device) * 0.02
        shared13 = torch.cat([f13[r * Isr:(r + 1) * Isr], f13[Is + r * Isr:Is + (r + 1) * Isr]]
                             ).to(torch.bfloat16).contiguous()
        shared2 = f2[:, r * Isr:(r + 1) * Isr].to(torch.bfloat16).contiguous()
    w = RankWeights(router_w.contiguous(), bias.contiguous(), cat(w13_parts), cat(w2_parts),
                    shared13, shared2)
    return (w, masters) if keep_masters else w


def fit_zipf_beta(cfg: MoEConfig, tokens: int, seed: int, device, s: float = 1.1) -> float:
    """Bisection on beta so that the log-log slope of sorted per-expert counts is ~ -s."""
    from .moe import RoutedMoE
    x = make_input(tokens, cfg.hidden, seed, device)
    lo, hi = 0.0, 1.0
    best = 0.0
    for _ in range(12):
        mid = 0.5 * (lo + hi)
        w = make_rank_weights(MoEConfig(**{**cfg.__dict__, "tp": 1, "rank": 0,
                                           "shared_intermediate": 0}), seed, device,
                              zipf_beta=mid, expert_chunk=cfg.experts)
        layer = RoutedMoE(MoEConfig(**{**cfg.__dict__, "shared_intermediate": 0}), w, tokens)
        layer(x)
        counts = torch.bincount(layer.route_experts[:tokens].long().flatten(),
                                minlength=cfg.experts).float().sort(descending=True).values
        counts = counts[counts > 0]
        ranks = torch.arange(1, counts.numel() + 1, device=counts.device, dtype=torch.float32)
        slope = float(torch.linalg.lstsq(torch.stack([ranks.log(), torch.ones_like(ranks)], 1),
                                         counts.log()[:, None]).solution[0])
        best = mid
        if -slope < s:
            lo = mid
        else:
            hi = mid
        if math.isclose(-slope, s, rel_tol=0.02):
            break
    return best
