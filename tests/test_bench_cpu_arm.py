"""bench.py's CPU arm (the reference's CPU path restated in oracle/): on a reduced
layer its step reproduces the straightforward oracle layer bit for bit, with the
experts prepared once (held) and the timed part excluding the preparation."""
import numpy as np
import torch

import bench
import oracle as O
from glmaxx_b200.moe import MoEConfig, PackedNvfp4, RankWeights


def _weights(cfg, rng):
    E, H, I, IS = cfg.experts, cfg.hidden, cfg.intermediate, cfg.shared_intermediate
    p13 = [O.pack((rng.standard_normal((2 * I, H)) * 0.02).astype(np.float32)) for _ in range(E)]
    p2 = [O.pack((rng.standard_normal((H, I)) * 0.02).astype(np.float32)) for _ in range(E)]

    def packed(ps, n, k):
        return PackedNvfp4(torch.from_numpy(np.stack([p.values.reshape(n, k // 2) for p in ps])),
                           torch.from_numpy(np.stack([p.scales for p in ps])),
                           torch.tensor([p.global_scale for p in ps]), torch.zeros(E), n, k)
    wr = O.f32_to_bf16_bits((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    s13 = O.f32_to_bf16_bits((rng.standard_normal((2 * IS, H)) * 0.02).astype(np.float32))
    s2 = O.f32_to_bf16_bits((rng.standard_normal((H, IS)) * 0.02).astype(np.float32))
    t16 = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    return RankWeights(t16(wr), torch.from_numpy((rng.standard_normal(E) * 0.01).astype(np.float32)),
                       packed(p13, 2 * I, H), packed(p2, H, I), t16(s13), t16(s2))


def test_cpu_arm_step_matches_oracle_layer():
    cfg = MoEConfig(hidden=512, experts=8, intermediate=256, top_k=4, groups=1, topk_groups=1,
                    shared_intermediate=128)
    rng = np.random.default_rng(0)
    w = _weights(cfg, rng)
    xb = O.f32_to_bf16_bits(rng.standard_normal((6, cfg.hidden)).astype(np.float32))
    cl = bench.CpuLayer(w, cfg, None, xb)
    assert cl.prep.hold
    busy, touched, out = cl.step()
    assert busy > 0 and touched <= cfg.experts
    re, rw = O.router(xb, bench.host_u16(w.router_weight), w.router_bias.numpy(), 1, 1, 4, 2.5)
    routed, shared = O.moe_layer(xb, re, rw, w.w13.values.numpy(), w.w13.scales.numpy(),
                                 w.w13.global_scale.numpy(), w.w2.values.numpy(),
                                 w.w2.scales.numpy(), w.w2.global_scale.numpy(), cfg.intermediate,
                                 bench.host_u16(w.shared13), bench.host_u16(w.shared2))
    ref = O.finish_sparse_layer(None, None, routed[None], shared[None])
    assert np.array_equal(out.view(np.uint32), ref.reshape(out.shape).view(np.uint32))
    prep_once = cl.prep.prep_s
    cl.step()  # held experts are not prepared again
    assert cl.prep.prep_s == prep_once


def test_cpu_sample_rule():
    assert np.array_equal(bench.cpu_sample(64, "decode", 1), np.arange(64))
    s = bench.cpu_sample(8192, "prefill", 1)
    assert s.size == bench.CPU_PREFILL_SAMPLE_TOKENS and np.all(np.diff(s) > 0)


def test_bench_options_defaults_and_workload_tokens(monkeypatch):
    """The driver runs `bench.py` with no workload flags: decode at T=64, the
    peer finish, token-split routing where it pays, atomic prefill combine and
    an unchunked step; a workload flag picks that configuration's token count."""
    import sys
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    assert (a.workload, a.tokens, a.gpus, a.reduce, a.split_route, a.combine, a.chunks) == \
        ("decode", 64, 1, "peer", "auto", "atomic", 1)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--workload", "prefill", "--chunks", "2"])
    a = bench.parse()
    assert (a.tokens, a.chunks) == (8192, 2)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--workload", "exl3"])
    assert bench.parse().tokens == 32
