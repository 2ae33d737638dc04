"""Pin the CPU oracle to the reference's own golden vectors (tests/golden/golden.json)."""
import hashlib

import numpy as np
import pytest

import oracle as O
from exl3_util import warp_activations


def test_actual_shape_packed_sha256(golden):
    g = golden["actual_shape"]
    p = O.pack(O.actual_shape_values(g["n"], g["k"]))
    assert p.values.size == g["value_bytes"] and p.scales.size == g["scale_bytes"]
    assert p.sha256() == g["packed_sha256"]


@pytest.mark.parametrize("case", O.NUMERICAL_CASES)
def test_matrix_proof_numerical_hashes(golden, case):
    mp = golden["matrix_proof"]
    n, k, _ = mp["model_shape"]
    entry = next(e for e in mp["numerical"] if e["case"] == case)
    act, w = O.generate_numerical_fixture(case, entry["activation_rows"], n, k)
    assert O.f32_hash(act) == entry["activation_sha256"]
    p = O.pack(w)
    assert p.values.size == entry["value_bytes"] and p.scales.size == entry["scale_bytes"]
    assert p.sha256() == entry["packed_weight_sha256"]


@pytest.mark.parametrize("case", O.ROUTING_CASES)
def test_matrix_proof_routing_counts(golden, case):
    entry = next(e for e in golden["matrix_proof"]["routing"] if e["case"] == case)
    for rows, expected in entry["assignments_by_rows"]:
        routes = O.generate_routes(case, rows)
        if entry["expected"] == "reject":
            with pytest.raises(O.OracleError):
                O.compact_routes(routes, rows)
            assert expected == 0
        else:
            assert len(O.compact_routes(routes, rows)) == expected


def test_fc1_fixed_shape_cancellation_bits(golden):
    g = golden["fc1_fixed_shape"]
    act, w = O.generate_numerical_fixture("deterministic-random-v1", g["rows"], g["n"], g["k"])
    p = O.pack(w)
    row = act[g["row"]: g["row"] + 1]
    seq = O.routed_fc1(row, p)[0, g["column"]]
    tree = O.routed_fc1_fixed_tree_at(row[0], p, g["column"])[0]
    assert int(np.float32(seq).view(np.uint32)) == g["sequential_bits"]
    assert int(np.float32(tree).view(np.uint32)) == g["fixed_tree_bits"]
    assert abs(float(seq) - float(tree)) == 5.0


def test_fc2_weight_after_projection(golden):
    g = golden["fc2_toy"]
    routes = O.routes_array([(0, 1, 0, 0.25), (0, 2, 1, 0.75)])
    w1 = O.pack(np.array([[1, 0], [0, 1]], np.float32))
    w2 = O.pack(np.array([[2, 0], [0, 2]], np.float32))
    out = O.routed_fc2(np.array([[1, 2], [1, 2]], np.float32), routes, 1, 2, 2, {1: w1, 2: w2})
    for got, exp, tol in zip(out[0], g["expected"], g["tolerance"]):
        assert abs(got - exp) < tol


def test_finish_rank_order(golden):
    r = np.arange(4, dtype=np.float32)[:, None] + 1.0
    att, routed, shared = np.repeat(r, 4, 1), np.repeat(10 * r, 4, 1), np.repeat(0.5 * r, 4, 1)
    out = O.finish_sparse_layer(np.ones(4, np.float32), att, routed, shared)
    assert np.all(out == golden["finish_rank_order"]["expected"])


def test_exl3_native_decode_digest(golden):
    g = golden["exl3_native"]
    tr = O.exl3_xorshift_trellis(g["seed"], O.exl3_trellis_words(g["k"], g["n"], g["bits"]))
    assert O.u16_hash(O.exl3_reconstruct_native(tr, g["k"], g["n"], g["bits"])) == g["sha256"]


@pytest.mark.parametrize("index", [0, 1])
def test_exl3_warp_proof_hashes(golden, index):
    g = golden["exl3_warp_proof"]["shapes"][index]
    k, n = g["k"], g["n"]
    tr = O.exl3_xorshift_trellis(g["seed"], O.exl3_trellis_words(k, n, 3))
    native = O.exl3_reconstruct_native(tr, k, n)
    # weight digest order: n-tile outer, k ascending, column in tile ascending (warp_proof.rs:118-150)
    wh = hashlib.sha256()
    for nt in range(n // 16):
        wh.update(np.ascontiguousarray(native[:, nt * 16:(nt + 1) * 16]).astype("<u2").tobytes())
    assert wh.hexdigest() == g["weight_sha256"]
    wf = O.bf16_bits_to_f32(np.zeros(1, np.uint16))  # dtype helper warm-up
    wf = np.array([O.f16_bits_to_f32(int(b)) for b in range(65536)], np.float32)[native]
    act = warp_activations(golden["exl3_warp_proof"]["rows"], k)
    acc = np.zeros((act.shape[0], n), np.float32)
    for kk in range(k):  # multiply_then_add, ascending k (warp_proof.rs:378-381)
        acc = acc + act[:, kk:kk + 1] * wf[kk:kk + 1, :]
    f16 = np.array([[O.f32_to_f16_bits(float(v)) for v in row] for row in acc], np.uint16)
    assert O.u16_hash(f16) == g["projection_f16_sha256"]


def test_scale_offset_closed_form(golden):
    assert O.scale_offset(0, 0, 128, 64) == 0
    for n, g, pn, pk, exp in golden["scale_offset_closed_form"]:
        assert O.scale_offset(n, g, pn, pk) == exp


def test_scale_layout_bijective():
    n, k = 256, 512
    seen = np.zeros(n * k // 16, bool)
    for row in range(n):
        for g in range(k // 16):
            off = O.scale_offset(row, g, n, k)
            assert not seen[off]
            seen[off] = True
    assert seen.all()


def test_e2m1_ties_even_and_roundtrip():
    for value, expected in [(0.25, 0), (0.75, 2), (1.25, 2), (1.75, 4), (2.5, 4), (3.5, 6), (5.0, 6)]:
        assert O.encode_e2m1(value) == expected
    for code in range(16):
        v = O.decode_e2m1(code)
        assert O.encode_e2m1(v) == (0 if v == 0 else code)


def test_e4m3_roundtrip():
    for code in range(0x7F):
        assert O.encode_e4m3(O.decode_e4m3(code)) == code
    for code in range(0x81, 0xFF):
        assert O.encode_e4m3(O.decode_e4m3(code)) == code
    assert O.decode_e4m3(0x7E) == 448.0


def test_nibble_order_low_then_high():
    x = np.zeros((128, 64), np.float32)
    x[0, 0], x[0, 1] = 6.0, -6.0
    p = O.pack(x)
    assert p.values[0] & 0x0F == 0x07 and p.values[0] >> 4 == 0x0F


def test_zero_tensor_canonical():
    p = O.pack(np.zeros((129, 65), np.float32))
    assert p.global_scale == 1.0 and not p.values.any() and not p.scales.any()
    assert not p.dequantize().any()


def test_crc32c_check_value():
    assert O.crc32c(b"123456789") == 0xE3069283
