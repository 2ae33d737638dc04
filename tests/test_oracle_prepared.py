"""The prepared-expert oracle (experts dequantised once into k-major planes,
OpenMP over assignments, SIMD across output columns) is the same arithmetic as
the straightforward restatement orc_moe_layer: equal bits on a reduced layer,
for the whole token set and for a token subset, with a shared expert."""
import numpy as np

import oracle as O


def _layer(seed=1, T=12, H=1024, E=8, I=256, K=4, IS=128):
    rng = np.random.default_rng(seed)
    x = O.f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    re = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.uint16)
    rw = rng.random((T, K)).astype(np.float32)
    p13 = [O.pack((rng.standard_normal((2 * I, H)) * 0.02).astype(np.float32)) for _ in range(E)]
    p2 = [O.pack((rng.standard_normal((H, I)) * 0.02).astype(np.float32)) for _ in range(E)]
    w = (np.stack([p.values for p in p13]), np.stack([p.scales for p in p13]),
         np.array([p.global_scale for p in p13], np.float32), np.stack([p.values for p in p2]),
         np.stack([p.scales for p in p2]), np.array([p.global_scale for p in p2], np.float32))
    s13 = O.f32_to_bf16_bits((rng.standard_normal((2 * IS, H)) * 0.02).astype(np.float32))
    s2 = O.f32_to_bf16_bits((rng.standard_normal((H, IS)) * 0.02).astype(np.float32))
    return x, re, rw, w, s13, s2, H, I


def test_prepared_layer_equals_moe_layer_bits():
    x, re, rw, w, s13, s2, H, I = _layer()
    prep = lambda e: O.expert_prepare(w[0][e], w[1][e], w[2][e], w[3][e], w[4][e], w[5][e], H, I)
    shared = O.shared_prepare(s13, s2)
    for subset in (None, np.array([0, 5, 11], np.uint32)):
        r, s = O.moe_layer(x, re, rw, *w, I, s13, s2, token_subset=subset)
        r2, s2o, busy = O.moe_layer_prepared(x, re, rw, prep, I, shared=shared,
                                             token_subset=subset)
        assert busy > 0
        assert np.array_equal(r.view(np.uint32), r2.view(np.uint32))
        assert np.array_equal(s.view(np.uint32), s2o.view(np.uint32))


def test_prepared_fc1_equals_routed_fc1_bits():
    x, re, rw, w, s13, s2, H, I = _layer(seed=2)
    w13t, _ = O.expert_prepare(w[0][3], w[1][3], w[2][3], w[3][3], w[4][3], w[5][3], H, I)
    tokens = np.array([1, 4, 9], np.uint32)
    h = O.moe_expert_h(x, tokens, w13t)
    packed = O.Packed(w[0][3].ravel(), w[1][3].ravel(), float(w[2][3]), 0.0, 2 * I, H, "1d")
    ref = O.routed_fc1(O.bf16_bits_to_f32(x[tokens]), packed)
    assert np.array_equal(h.view(np.uint32), ref.view(np.uint32))
