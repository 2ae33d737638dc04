"""Routed-MoE layer with EXL3 3-bit experts and with the
hybrid NVFP4/EXL3 per-expert codec.

The CPU reference composes the restated Exl3Trellis::matmul_reference_f16
(crates/glm-format/src/exl3.rs:404-453; bit-exact on the GPU by test_gpu_exl3)
per assignment: gate and up on the fp16 token row, h = fp16(silu(g) * u), down
on h, times the routing weight, summed over the token's slots in ascending
expert order (the reference FC2 order, routed_fc2.rs:20-89).  The SiLU between
the projections is not pinned by the reference; both sides use v / (1 + exp(-v))
in fp32, so they differ at most where an fp16 rounding of h flips.  Tolerance:
the layer bound of gpu_util (rel-L2 1e-3, max-abs 4 bf16 ulp).
"""
import numpy as np
import pytest
import torch

import oracle as O
from glmaxx_b200 import abi, synth
from glmaxx_b200.moe import MoEConfig, RankWeights, RoutedMoE

from gpu_util import assert_layer_close, cuda, rel_l2, to_np_bf16_bits

pytestmark = pytest.mark.gpu

# experts with at least this many rows use the tensor-core projection (exl3_gemm.cu)
EXL3_TC_MIN_ROWS = 8


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().numpy().view(np.uint16)


def _f16(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


def _exl3_reference(layer: RoutedMoE, x: torch.Tensor, cfg: MoEConfig, subset: np.ndarray):
    """Per-slot contributions [len(subset), K, H] and outputs [len(subset), H]."""
    T = x.shape[0]
    w = layer.w.exl3
    H, I, K = cfg.hidden, cfg.local_intermediate, cfg.top_k
    re, rw = layer.routes(T)
    re = re.cpu().numpy().astype(np.int64)
    rw = rw.cpu().numpy()
    xb = to_np_bf16_bits(x)
    x16 = (xb.astype(np.uint32) << 16).view(np.float32).astype(np.float16).view(np.uint16)
    tr = {n: _u16(getattr(w, n + "_trellis")) for n in ("gate", "up", "down")}
    sc = {n: _u16(getattr(w, n)) for n in ("gate_suh", "gate_svh", "up_suh", "up_svh",
                                            "down_suh", "down_svh")}
    contrib = np.zeros((len(subset), K, H), np.float32)
    for e in np.unique(re[subset]):
        rows = [(i, s) for i, t in enumerate(subset) for s in range(K) if re[t, s] == e]
        xin = np.stack([x16[subset[i]] for i, _ in rows])
        g = O.exl3_matmul_reference(tr["gate"][e], H, I, sc["gate_suh"][e], sc["gate_svh"][e], xin)
        u = O.exl3_matmul_reference(tr["up"][e], H, I, sc["up_suh"][e], sc["up_svh"][e], xin)
        gf, uf = _f16(g), _f16(u)
        silu = gf / (np.float32(1.0) + np.exp(-gf))
        h = (silu * uf).astype(np.float16).view(np.uint16)
        d = O.exl3_matmul_reference(tr["down"][e], I, H, sc["down_suh"][e], sc["down_svh"][e], h)
        df = _f16(d)
        for j, (i, s) in enumerate(rows):
            contrib[i, s] = np.float32(rw[subset[i], s]) * df[j]
    out = np.zeros((len(subset), H), np.float32)
    for i, t in enumerate(subset):
        order = np.argsort(re[t], kind="stable")
        acc = contrib[i, order[0]].copy()
        for s in order[1:]:
            acc = acc + contrib[i, s]
        out[i] = acc
    return contrib, out


def _plane(layer: RoutedMoE, T: int, cfg: MoEConfig) -> np.ndarray:
    raw = layer.plane("routed_f32")
    return raw.view(torch.float32).reshape(T, cfg.top_k, cfg.hidden).cpu().numpy()


def test_gpu_layer_exl3_reduced():
    cfg = MoEConfig(experts=16, groups=1, topk_groups=1, intermediate=512, shared_intermediate=0)
    dev = cuda()
    T = 8
    w = synth.make_exl3_rank_weights(cfg, seed=31, device=dev)
    x = synth.make_input(T, cfg.hidden, seed=31, device=dev)
    layer = RoutedMoE(cfg, w, T)
    out = layer(x).cpu().numpy()
    torch.cuda.synchronize()
    assert layer.device_status() == []
    subset = np.arange(T)
    contrib, ref = _exl3_reference(layer, x, cfg, subset)
    plane = _plane(layer, T, cfg)
    # experts with fewer than 8 rows run the bit-exact decode-fused GEMV chain
    re = layer.routes(T)[0].cpu().numpy().astype(np.int64)
    rows = np.bincount(re.ravel(), minlength=cfg.experts)
    gemv = rows[re] < EXL3_TC_MIN_ROWS
    assert gemv.any()
    exact = float(np.mean(plane[gemv] == contrib[gemv]))
    assert exact > 0.99, f"only {exact:.4f} of GEMV-path slot outputs bit-exact"
    assert_layer_close(out, ref, "exl3 layer")


def test_gpu_layer_exl3_tensor_core_rows():
    """Experts with >= 8 rows take the tensor-core projection (trellis decoded into
    shared memory, fp32 tensor-core accumulation): within the layer tolerance of
    the sequential reference composition."""
    cfg = MoEConfig(experts=16, groups=1, topk_groups=1, intermediate=512, shared_intermediate=0)
    dev = cuda()
    T = 64
    w = synth.make_exl3_rank_weights(cfg, seed=41, device=dev)
    x = synth.make_input(T, cfg.hidden, seed=41, device=dev)
    layer = RoutedMoE(cfg, w, T)
    out = layer(x).cpu().numpy()
    torch.cuda.synchronize()
    assert layer.device_status() == []
    counts = np.bincount(layer.routes(T)[0].cpu().numpy().astype(np.int64).ravel(),
                         minlength=cfg.experts)
    assert counts.max() >= 8  # the tensor-core path ran
    subset = np.arange(0, T, 3)
    contrib, ref = _exl3_reference(layer, x, cfg, subset)
    assert_layer_close(out[subset], ref, "exl3 tensor-core rows")
    plane = _plane(layer, T, cfg)[subset]
    assert rel_l2(plane, contrib) < 1e-3


def test_gpu_layer_exl3_decode_tp4_subset():
    """configs[3] geometry (T=32, 256 experts, top-8 of 8 groups / top-4) at TP4."""
    cfg = MoEConfig(tp=4, rank=1, shared_intermediate=0)
    dev = cuda()
    T = 32
    w = synth.make_exl3_rank_weights(cfg, seed=5, device=dev)
    x = synth.make_input(T, cfg.hidden, seed=5, device=dev)
    layer = RoutedMoE(cfg, w, T)
    out = layer(x).cpu().numpy()
    torch.cuda.synchronize()
    assert layer.device_status() == []
    subset = np.array([0, 13, 31])
    _, ref = _exl3_reference(layer, x, cfg, subset)
    assert_layer_close(out[subset], ref, "exl3 decode tp4")


@pytest.mark.parametrize("path", [abi.DECODE_PERSISTENT, abi.PREFILL_GROUPED])
def test_gpu_layer_hybrid_codec(path):
    """Experts with codec 0 take the NVFP4 path, the rest EXL3: every slot output
    equals the all-NVFP4 or the all-EXL3 layer's, and the output is their
    ascending-expert sum plus the shared expert."""
    cfg = MoEConfig(experts=16, groups=1, topk_groups=1, intermediate=512,
                    shared_intermediate=256)
    dev = cuda()
    T = 24
    g = torch.Generator().manual_seed(3)
    nvfp4_mask = torch.zeros(cfg.experts, dtype=torch.bool)
    nvfp4_mask[torch.randperm(cfg.experts, generator=g)[:cfg.experts // 2]] = True
    w = synth.make_exl3_rank_weights(cfg, seed=17, device=dev, nvfp4_experts=nvfp4_mask)
    x = synth.make_input(T, cfg.hidden, seed=17, device=dev)
    hyb = RoutedMoE(cfg, w, T)
    out = hyb(x, path=path).cpu().numpy()
    plane_h = _plane(hyb, T, cfg)
    w_n = RankWeights(w.router_weight, w.router_bias, w.w13, w.w2, w.shared13, w.shared2)
    w_x = RankWeights(w.router_weight, w.router_bias, None, None, w.shared13, w.shared2,
                      synth.Exl3Experts(**{**w.exl3.__dict__, "codec": None}))
    nv = RoutedMoE(cfg, w_n, T)
    nv(x, path=abi.DECODE_PERSISTENT)
    plane_n = _plane(nv, T, cfg)
    ex = RoutedMoE(cfg, w_x, T)
    ex(x, path=path)
    plane_x = _plane(ex, T, cfg)
    torch.cuda.synchronize()
    for layer in (hyb, nv, ex):
        assert layer.device_status() == []
    re = hyb.routes(T)[0].cpu().numpy().astype(np.int64)
    assert np.array_equal(re, nv.routes(T)[0].cpu().numpy().astype(np.int64))
    is_nv = nvfp4_mask.numpy()[re]  # [T, K]
    assert is_nv.any() and (~is_nv).any()
    assert np.array_equal(plane_h[~is_nv], plane_x[~is_nv])
    if path == abi.DECODE_PERSISTENT:
        assert np.array_equal(plane_h[is_nv], plane_n[is_nv])
    else:  # 128-row tiles against the decode path's 32-row tiles
        assert rel_l2(plane_h[is_nv], plane_n[is_nv]) < 1e-6
    shared = hyb.plane("shared_f32").view(torch.float32).reshape(T, cfg.hidden).cpu().numpy()
    for t in range(T):
        order = np.argsort(re[t], kind="stable")
        acc = plane_h[t, order[0]].copy()
        for s in order[1:]:
            acc = acc + plane_h[t, s]
        assert np.array_equal(out[t], acc + shared[t])
