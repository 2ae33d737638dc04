"""GPU parity at the stated shapes of the BASELINE configs (calls go through the C ABI).

- configs[2] (prefill): T=8192, 256 experts, Zipf(1.1)-skewed router bias, at TP1
  and on one TP8 shard.  Routes and compaction bit-exact for all 8192 tokens; the
  FC1 output of every row of the heaviest expert against the oracle FC1; the layer
  output on a seeded token subset that holds the first and last row of every
  128-row tile of the heaviest expert (rel-L2 <= 1e-3, max-abs <= 4 bf16 ulp).
- configs[3] (EXL3 decode) at TP1 (I = 2048), the benched shape.
- configs[4] (hybrid stack): 2048 tokens, 64 NVFP4 + 192 EXL3 experts, Zipf
  routing, shared expert, 4 stacked layers joined by the finish with a bf16
  residual and RMSNorm input, at TP4 (the four ranks run on one GPU).  Every layer:
  routes bit-exact on the subset, rank 1's partial against the oracle composition,
  and the finish against orc_finish_sparse_layer on the GPU's partials (bit-exact).
- configs[0] anchored to an fp64 evaluation of the same quantised arithmetic.

Per-token independence (an output row depends only on its token's row, routes
and the weights; crates/glm-reference/src/routed_fc1.rs:84-103) makes the token
subsets exact checks of the full-size launches.  The oracle runs in its
prepared-expert form (oracle.moe_layer_prepared), which is the same bits as
orc_moe_layer (tests/test_oracle_prepared.py).
"""
import numpy as np
import pytest
import torch

import oracle as O
from glmaxx_b200 import synth
from glmaxx_b200.moe import MoEConfig, RoutedMoE, finish

from gpu_util import (MAX_ABS_ULPS, REL_L2, assert_layer_close, bf16_ulp, cuda, rel_l2,
                      to_np_bf16_bits)

pytestmark = pytest.mark.gpu

SEED = 1234  # bench.py's default seed: the tests check the benched inputs


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().numpy().view(np.uint16)


def _prepare_fn(w, cfg):
    """prepare(e) for oracle.moe_layer_prepared: expert e's NVFP4 shard copied to the
    host and dequantised once (nvfp4.rs:279-301) into k-major planes."""
    H, I = cfg.hidden, cfg.local_intermediate

    def prep(e):
        return O.expert_prepare(w.w13.values[e].cpu().numpy(), w.w13.scales[e].cpu().numpy(),
                                float(w.w13.global_scale[e]), w.w2.values[e].cpu().numpy(),
                                w.w2.scales[e].cpu().numpy(), float(w.w2.global_scale[e]), H, I)
    return prep


def _shared_prep(w):
    if w.shared13 is None:
        return None
    return O.shared_prepare(to_np_bf16_bits(w.shared13), to_np_bf16_bits(w.shared2))


def _check_routes_all(layer, xb, cfg, tokens=None):
    """Routes of `tokens` (all by default) equal the oracle router's bits."""
    w = layer.w
    sel = slice(None) if tokens is None else tokens
    ref_e, ref_w = O.router(xb[sel], to_np_bf16_bits(w.router_weight),
                            w.router_bias.cpu().numpy(), cfg.groups, cfg.topk_groups,
                            cfg.top_k, cfg.route_scale)
    got_e, got_w = layer.routes(xb.shape[0])
    got_e = got_e.cpu().numpy().view(np.uint16)[sel]
    got_w = got_w.cpu().numpy()[sel]
    assert np.array_equal(got_e, ref_e)
    assert np.array_equal(got_w.view(np.uint32), ref_w.view(np.uint32))
    return ref_e, ref_w


# --------------------------------------------------------------------------- configs[2]
@pytest.mark.parametrize("tp,rank", [(1, 0), (8, 3)])
def test_gpu_prefill_config2_zipf(tp, rank):
    cfg = MoEConfig(tp=tp, rank=rank)
    dev = cuda()
    T = 8192
    beta, slope = synth.fit_zipf_beta(cfg, T, SEED, dev)
    assert abs(slope + 1.1) < 0.05, slope
    w = synth.make_rank_weights(cfg, seed=SEED, device=dev, zipf_beta=beta)
    x = synth.make_input(T, cfg.hidden, seed=SEED, device=dev)
    layer = RoutedMoE(cfg, w, T)
    out = layer(x)  # T > 256: the prefill path (N tile 128, atomic combine)
    torch.cuda.synchronize()
    assert layer.device_status() == []
    xb = to_np_bf16_bits(x)
    re, rw = _check_routes_all(layer, xb, cfg)

    # compaction: tokens, slots and offsets of the stable (expert, token, slot) order
    A = T * cfg.top_k
    routes = O.routes_array([(t, int(re[t, s]), s, float(rw[t, s]))
                             for t in range(T) for s in range(cfg.top_k)])
    comp = O.compact_routes(routes, T)
    tok = layer.plane("row_token_u32").view(torch.int32).cpu().numpy().astype(np.uint32)
    slot = layer.plane("row_slot_u32").view(torch.int32).cpu().numpy()
    off = layer.plane("expert_offsets_u32").view(torch.int32).cpu().numpy().astype(np.int64)
    assert np.array_equal(tok, comp["token"])
    assert np.array_equal(slot.astype(np.uint8), comp["slot"])
    counts = np.bincount(comp["expert"], minlength=cfg.experts)
    assert np.array_equal(off, np.concatenate([[0], np.cumsum(counts)]))

    # the Zipf skew puts many 128-row tiles on the heaviest expert
    hot = int(np.argmax(counts))
    n_hot = int(counts[hot])
    assert n_hot >= 8 * 128, n_hot
    prep = _prepare_fn(w, cfg)
    w13t, _ = prep(hot)
    hot_rows = tok[off[hot]:off[hot + 1]]
    I = cfg.local_intermediate
    h = layer.plane("fc1_output_bf16").view(torch.bfloat16).reshape(A, I)[off[hot]:off[hot + 1]]
    h_err = rel_l2(h.float().cpu().numpy(), O.moe_expert_h(xb, hot_rows, w13t))
    assert h_err <= REL_L2, f"FC1 of the heaviest expert ({n_hot} rows): rel-L2 {h_err:.3e}"
    del w13t

    # layer output on a subset holding the first and last row of every 128-row tile
    # of the heaviest expert, plus seeded random tokens
    tiles = [hot_rows[i:i + 128] for i in range(0, n_hot, 128)]
    subset = {int(t[0]) for t in tiles} | {int(t[-1]) for t in tiles}
    rng = np.random.default_rng(tp * 100 + rank)
    subset |= set(rng.choice(T, 48, replace=False).tolist())
    subset = np.array(sorted(subset), np.uint32)
    routed, shared, _ = O.moe_layer_prepared(xb, re, rw, prep, I, shared=_shared_prep(w),
                                             token_subset=subset)
    ref = O.finish_sparse_layer(None, None, routed[None], shared[None])
    assert_layer_close(out[torch.from_numpy(subset.astype(np.int64)).to(dev)].cpu().numpy(),
                       ref, f"prefill config2 tp{tp} r{rank}")


# --------------------------------------------------------------------------- EXL3 oracle
def _exl3_slot_contrib(w, cfg, x16, re, rw, tokens, nvfp4_mask=None):
    """Per (subset row, slot) EXL3 contributions w * down(fp16(silu(g) * u)) of the
    oracle composition (exl3.rs:404-453 per projection); slots whose expert is NVFP4
    (nvfp4_mask) are left zero."""
    H, I, K = cfg.hidden, cfg.local_intermediate, cfg.top_k
    x3 = w.exl3
    contrib = np.zeros((len(tokens), K, H), np.float32)
    tr = {n: getattr(x3, n + "_trellis") for n in ("gate", "up", "down")}
    for e in np.unique(re[tokens]):
        e = int(e)
        if nvfp4_mask is not None and nvfp4_mask[e]:
            continue
        rows = [(i, s) for i, t in enumerate(tokens) for s in range(K) if re[t, s] == e]
        xin = np.stack([x16[tokens[i]] for i, _ in rows])
        sc = {n: _u16(getattr(x3, n)[e]) for n in ("gate_suh", "gate_svh", "up_suh", "up_svh",
                                                     "down_suh", "down_svh")}
        g = O.exl3_matmul_reference(_u16(tr["gate"][e]), H, I, sc["gate_suh"], sc["gate_svh"], xin)
        u = O.exl3_matmul_reference(_u16(tr["up"][e]), H, I, sc["up_suh"], sc["up_svh"], xin)
        gf = g.view(np.float16).astype(np.float32)
        uf = u.view(np.float16).astype(np.float32)
        hh = (gf / (np.float32(1.0) + np.exp(-gf)) * uf).astype(np.float16).view(np.uint16)
        d = O.exl3_matmul_reference(_u16(tr["down"][e]), I, H, sc["down_suh"], sc["down_svh"], hh)
        df = d.view(np.float16).astype(np.float32)
        for j, (i, s) in enumerate(rows):
            contrib[i, s] = np.float32(rw[tokens[i], s]) * df[j]
    return contrib


def _nvfp4_slot_contrib(w, cfg, xb, re, rw, tokens, nvfp4_mask):
    """Per (subset row, slot) NVFP4 contributions w * FC2(FC1) of the oracle, for
    slots whose expert is NVFP4; each slot has its own zeroed output row, so it
    receives exactly the rounded product w * acc of routed_fc2.rs:60-86."""
    H, K = cfg.hidden, cfg.top_k
    contrib = np.zeros((len(tokens) * K, H), np.float32)
    prep = _prepare_fn(w, cfg)
    for e in np.unique(re[tokens]):
        e = int(e)
        if not nvfp4_mask[e]:
            continue
        pairs = [(i, s) for i, t in enumerate(tokens) for s in range(K) if re[t, s] == e]
        toks = np.array([tokens[i] for i, _ in pairs], np.uint32)
        wts = np.array([rw[tokens[i], s] for i, s in pairs], np.float32)
        rows = np.array([i * K + s for i, s in pairs], np.uint32)
        w13t, w2t = prep(e)
        O.moe_expert_rows(xb, toks, wts, rows, w13t, w2t, contrib)
    return contrib.reshape(len(tokens), K, H)


def _expert_order_sum(contrib, re_rows):
    """Slot contributions summed in ascending expert order (routed_fc2.rs:20-89)."""
    out = np.zeros((contrib.shape[0], contrib.shape[2]), np.float32)
    for i in range(contrib.shape[0]):
        order = np.argsort(re_rows[i], kind="stable")
        acc = contrib[i, order[0]].copy()
        for s in order[1:]:
            acc = acc + contrib[i, s]
        out[i] = acc
    return out


# --------------------------------------------------------------------------- configs[3]
def test_gpu_exl3_config3_tp1():
    """configs[3] at TP1 (I = 2048) as benched (bench.py --workload exl3: shared expert
    on), on a seeded 12-token subset; routes bit-exact for all 32 tokens."""
    cfg = MoEConfig()
    dev = cuda()
    T = 32
    w = synth.make_exl3_rank_weights(cfg, seed=SEED, device=dev)
    x = synth.make_input(T, cfg.hidden, seed=SEED, device=dev)
    layer = RoutedMoE(cfg, w, T)
    out = layer(x).cpu().numpy()
    torch.cuda.synchronize()
    assert layer.device_status() == []
    xb = to_np_bf16_bits(x)
    re, rw = _check_routes_all(layer, xb, cfg)
    subset = np.sort(np.random.default_rng(3).choice(T, 12, replace=False))
    x16 = (xb.astype(np.uint32) << 16).view(np.float32).astype(np.float16).view(np.uint16)
    contrib = _exl3_slot_contrib(w, cfg, x16, re.astype(np.int64), rw, subset)
    routed = _expert_order_sum(contrib, re[subset])
    shared = O.shared_rows(xb, subset, *_shared_prep(w))
    ref = O.finish_sparse_layer(None, None, routed[None], shared[None])
    assert_layer_close(out[subset], ref, "exl3 config3 tp1")


# --------------------------------------------------------------------------- configs[4]
def test_gpu_hybrid_config4_stack_tp4():
    """4 stacked hybrid layers at TP4, the four ranks on one GPU as
    bench.py --workload hybrid builds them (64 NVFP4 + 192 EXL3 experts by seeded
    permutation, Zipf routing, shared expert, bf16 residual, RMSNorm input)."""
    T, tp, n_layers, check_rank = 2048, 4, 4, 1
    dev = cuda()
    H, E = 6144, 256
    cfg0 = MoEConfig(tp=tp, rank=0)
    beta, _ = synth.fit_zipf_beta(cfg0, T, SEED, dev)
    g = torch.Generator().manual_seed(SEED * 13 + 1)
    mask = torch.zeros(E, dtype=torch.bool)
    mask[torch.randperm(E, generator=g)[:64]] = True
    nvfp4_mask = mask.numpy()
    x0 = synth.make_input(T, H, seed=SEED, device=dev)
    subset = np.sort(np.random.default_rng(4).choice(T, 12, replace=False)).astype(np.uint32)
    sub_t = torch.from_numpy(subset.astype(np.int64)).to(dev)
    rs, xs = x0, x0  # bf16 residual stream and this layer's normalised input
    for li in range(n_layers):
        seed = SEED + 7919 * li
        partials = []
        check = None
        for r in range(tp):
            cfg = MoEConfig(tp=tp, rank=r)
            w = synth.make_exl3_rank_weights(cfg, seed=seed, device=dev, zipf_beta=beta,
                                             nvfp4_experts=mask)
            layer = RoutedMoE(cfg, w, T)
            partials.append(layer(xs).clone())
            torch.cuda.synchronize()
            assert layer.device_status() == []
            if r == check_rank:
                check = (cfg, w, layer)
            else:
                del w, layer
        cfg, w, layer = check
        xb = to_np_bf16_bits(xs)
        re, rw = _check_routes_all(layer, xb, cfg, tokens=subset)
        re_sub = np.zeros((T, cfg.top_k), np.int64)
        rw_sub = np.zeros((T, cfg.top_k), np.float32)
        re_sub[subset], rw_sub[subset] = re, rw
        x16 = (xb.astype(np.uint32) << 16).view(np.float32).astype(np.float16).view(np.uint16)
        contrib = (_exl3_slot_contrib(w, cfg, x16, re_sub, rw_sub, subset, nvfp4_mask) +
                   _nvfp4_slot_contrib(w, cfg, xb, re_sub, rw_sub, subset, nvfp4_mask))
        routed = _expert_order_sum(contrib, re)
        shared = O.shared_rows(xb, subset, *_shared_prep(w))
        ref = O.finish_sparse_layer(None, None, routed[None], shared[None])
        got = partials[check_rank][sub_t].cpu().numpy()
        assert_layer_close(got, ref, f"hybrid layer {li} rank {check_rank} partial")
        del check, w, layer
        # the finish: bit-exact against orc_finish_sparse_layer on the GPU's partials
        out_f32 = torch.empty((T, H), dtype=torch.float32, device=dev)
        rs_next = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        xs_next = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        finish(partials, rs, out_f32=out_f32, out_bf16=rs_next, norm_bf16=xs_next, hidden=H)
        torch.cuda.synchronize()
        res = O.bf16_bits_to_f32(to_np_bf16_bits(rs[sub_t]))
        fin = O.finish_sparse_layer(res, None, np.stack([p[sub_t].cpu().numpy() for p in partials]),
                                    None)
        assert np.array_equal(out_f32[sub_t].cpu().numpy(), fin), f"finish of layer {li}"
        assert np.array_equal(to_np_bf16_bits(rs_next[sub_t]), O.f32_to_bf16_bits(fin))
        assert np.isfinite(out_f32.cpu().numpy()).all()
        rs, xs = rs_next, xs_next
        del partials


# --------------------------------------------------------------------------- configs[0]
def _fp64_layer(xb, re, rw, w, cfg):
    """The layer's quantised arithmetic evaluated with fp64 sums: the same rounding
    points (bf16 x, NVFP4 activations, bf16 h, NVFP4 h; routed_fc1.rs:84-103,
    routed_fc2.rs:60-86), every dot product and the weighted accumulation exact to
    fp64 instead of sequential fp32."""
    H, I = cfg.hidden, cfg.local_intermediate
    T, K = re.shape
    out = np.zeros((T, H), np.float64)
    deq = {}

    def weights(e):
        if e not in deq:
            p13 = O.Packed(w.w13.values[e].cpu().numpy().ravel(), w.w13.scales[e].cpu().numpy().ravel(),
                           float(w.w13.global_scale[e]), 0.0, 2 * I, H, "1d")
            p2 = O.Packed(w.w2.values[e].cpu().numpy().ravel(), w.w2.scales[e].cpu().numpy().ravel(),
                          float(w.w2.global_scale[e]), 0.0, H, I, "1d")
            deq[e] = (p13.dequantize().reshape(2 * I, H).astype(np.float64),
                      p2.dequantize().reshape(H, I).astype(np.float64))
        return deq[e]

    def roundtrip(row):
        return O.pack(row[None, :].astype(np.float32)).dequantize().reshape(-1)[:row.size]

    for t in range(T):
        act = roundtrip(O.bf16_round(O.bf16_bits_to_f32(xb[t]))).astype(np.float64)
        for s in range(K):
            w13, w2 = weights(int(re[t, s]))
            gate, up = w13[:I] @ act, w13[I:] @ act
            hh = O.bf16_round((gate / (1.0 + np.exp(-gate)) * up).astype(np.float32))
            src = roundtrip(hh).astype(np.float64)
            out[t] += np.float64(rw[t, s]) * (w2 @ src)
    return out


@pytest.mark.parametrize("seed", [3, 4, 5, 6])
def test_gpu_config0_against_fp64_evaluation(seed):
    """configs[0] (T=8, E=16, top-8, I=2048, no shared expert): the GPU and the
    sequential-fp32 oracle against an fp64 evaluation of the same quantised
    arithmetic.  The GPU's rel-L2 to it is no larger than the oracle's (plus an
    fp32-accumulation floor of 1e-5) and within the layer tolerance; so where GPU
    and oracle disagree by more than the tolerance, the oracle's sequential rounding,
    which moves a bf16 h value across an NVFP4 code step, is the one further from
    the exact result."""
    cfg = MoEConfig(experts=16, groups=1, topk_groups=1, shared_intermediate=0)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=seed, device=dev)
    x = synth.make_input(8, cfg.hidden, seed=seed, device=dev)
    layer = RoutedMoE(cfg, w, 8)
    out = layer(x)
    torch.cuda.synchronize()
    assert layer.device_status() == []
    xb = to_np_bf16_bits(x)
    re, rw = _check_routes_all(layer, xb, cfg)
    routed, _ = O.moe_layer(xb, re, rw, w.w13.values.cpu().numpy(), w.w13.scales.cpu().numpy(),
                            w.w13.global_scale.cpu().numpy(), w.w2.values.cpu().numpy(),
                            w.w2.scales.cpu().numpy(), w.w2.global_scale.cpu().numpy(),
                            cfg.local_intermediate)
    exact = _fp64_layer(xb, re, rw, w, cfg)
    got = out.cpu().numpy()
    e_gpu = rel_l2(got.astype(np.float64), exact)
    e_orc = rel_l2(routed.astype(np.float64), exact)
    print(f"seed {seed}: GPU vs fp64 {e_gpu:.3e}, oracle vs fp64 {e_orc:.3e}, "
          f"GPU vs oracle {rel_l2(got, routed):.3e}")
    assert e_gpu <= e_orc + 1e-5, (e_gpu, e_orc)
    assert e_gpu <= REL_L2
    err = float(np.abs(got - exact).max())
    assert err <= MAX_ABS_ULPS * bf16_ulp(float(np.abs(exact).max()))
