"""Measurement harness, not library API: run a few routed-MoE layer steps of a
chosen shape (the target of ncu captures and single-GPU A/B timings).

    python -m glmaxx_b200.profile_case --experts 64 --tokens 64 --steps 3 [--tp 1] [--path 1]
        [--codec nvfp4|exl3|hybrid]

Per step the layer launches, in order: router_logits, router_select, compact,
quant_scatter, FC1 grouped GEMM, fc2_quant, shared FC1 GEMM, shared FC2 GEMM,
FC2 grouped GEMM, combine.  With --experts < 256 the expert weights of one
step stay a few GB, which keeps an `ncu --set full` capture small.  With
--codec exl3 the routed experts are EXL3 3-bit trellises (the decode-fused
projection for experts with few rows, the trellis-decoding tensor-core GEMM
for many); hybrid makes a quarter of them NVFP4.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import abi, synth
from .moe import MoEConfig, RoutedMoE


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--experts", type=int, default=64)
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--path", type=int, default=0)
    p.add_argument("--shared", type=int, default=2048)
    p.add_argument("--seed", type=int, default=7)
    p.add_argument("--codec", choices=["nvfp4", "exl3", "hybrid"], default="nvfp4")
    # the layer flag GLMAXX_MOE_DETERMINISTIC (slot plane + expert-order combine)
    p.add_argument("--deterministic", action="store_true")
    # after the steps, time this many more (CUDA events on the launch stream)
    p.add_argument("--time", type=int, default=0)
    a = p.parse_args()
    groups = 8 if a.experts % 8 == 0 and a.experts >= 64 else 1
    cfg = MoEConfig(experts=a.experts, groups=groups, topk_groups=min(4, groups),
                    shared_intermediate=a.shared, tp=a.tp)
    dev = torch.device("cuda:0")
    if a.codec == "nvfp4":
        w = synth.make_rank_weights(cfg, seed=a.seed, device=dev)
    else:
        mask = None
        if a.codec == "hybrid":
            g = torch.Generator().manual_seed(a.seed)
            mask = torch.zeros(a.experts, dtype=torch.bool)
            mask[torch.randperm(a.experts, generator=g)[:a.experts // 4]] = True
        w = synth.make_exl3_rank_weights(cfg, seed=a.seed, device=dev, nvfp4_experts=mask)
    x = synth.make_input(a.tokens, cfg.hidden, seed=a.seed, device=dev)
    layer = RoutedMoE(cfg, w, a.tokens, deterministic=a.deterministic)
    out = torch.empty((a.tokens, cfg.hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream()
    ms = None
    with torch.cuda.stream(stream):
        for _ in range(a.steps):
            layer(x, out, path=a.path)
        if a.time:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(a.time):
                layer(x, out, path=a.path)
            e1.record(stream)
    torch.cuda.synchronize()
    if a.time:
        ms = e0.elapsed_time(e1) / a.time
    status = layer.device_status()
    routed = layer.routes(a.tokens)[0].long().flatten()
    touched = int(torch.unique(routed).numel())
    info = {"experts": a.experts, "tokens": a.tokens, "tp": a.tp, "steps": a.steps,
            "codec": a.codec, "deterministic": a.deterministic, "ms_per_step": ms,
            "touched_experts": touched, "status": status, "abi": abi.abi_string()}
    if a.codec == "exl3":
        # weights the decode-fused projection decodes per projection of one step:
        # every work item (an expert's rows in blocks of 4; experts with 8 or
        # more rows take the tensor-core path) decodes its expert's whole matrix
        rows = torch.bincount(routed, minlength=a.experts).tolist()
        items = sum((r + 3) // 4 for r in rows if 0 < r < 8)
        info["gemv_items"] = items
        info["gemv_weights_per_projection"] = items * cfg.hidden * cfg.local_intermediate
    print(json.dumps(info))
    if status:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
