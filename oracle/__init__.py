"""CPU oracle for the routed-MoE hot path -- TEST INFRASTRUCTURE ONLY.

numpy/ctypes front end of ``oracle/liboracle.so`` (plain C restatement of the
reference arithmetic in yatesdr/glmaxx's ``crates/glm-format`` and
``crates/glm-reference``; every C function cites the file:line it follows).
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package.  The product library (``glmaxx_b200``) never does.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"

ROUTING_CASES = [
    "one-hot-expert-0",
    "one-hot-expert-255",
    "uniform-all-experts",
    "zipf-skew",
    "empty-experts",
    "same-token-duplicate-expert-rejected",
    "route-slot-permutation",
    "tail-assignment-count",
]
NUMERICAL_CASES = [
    "all-zero",
    "all-e2m1-codes",
    "all-e4m3-finite-scale-classes",
    "bf16-extrema",
    "subnormal-block-scale",
    "single-outlier-per-block",
    "alternating-sign",
    "deterministic-random-v1",
]

ROUTE_DTYPE = np.dtype(
    [("token", "<u4"), ("expert", "<u2"), ("slot", "u1"), ("pad", "u1"), ("weight", "<f4")]
)
COMPACTED_DTYPE = np.dtype([("token", "<u4"), ("expert", "<u2"), ("slot", "u1"), ("pad", "u1")])


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
        _declare(_lib)
    return _lib


def _p(array: np.ndarray | None):
    if array is None:
        return None
    return array.ctypes.data_as(ctypes.c_void_p)


def _declare(L: ctypes.CDLL) -> None:
    c = ctypes
    vp, u8, u16, u32, u64, i32, f32 = (c.c_void_p, c.c_uint8, c.c_uint16, c.c_uint32,
                                       c.c_uint64, c.c_int, c.c_float)
    sig = {
        "orc_decode_e2m1": (f32, [u8]),
        "orc_encode_e2m1": (i32, [f32, vp]),
        "orc_decode_e4m3": (f32, [u8]),
        "orc_encode_e4m3": (i32, [f32, vp]),
        "orc_crc32c": (u32, [vp, u64]),
        "orc_scale_offset": (c.c_int64, [u64, u64, u64, u64]),
        "orc_nvfp4_pack": (i32, [vp, u64, u64, i32, vp, vp, vp, vp]),
        "orc_nvfp4_dequantize": (i32, [vp, vp, f32, u64, u64, vp]),
        "orc_nvfp4_metadata_encode": (None, [i32, u32, u32, u32, u32, f32, f32, u32, u32, vp]),
        "orc_bf16_round": (f32, [f32]),
        "orc_compact_routes": (i32, [vp, u64, u64, vp]),
        "orc_routed_fc1": (i32, [vp, u64, u64, vp, vp, f32, u64, vp]),
        "orc_routed_fc1_fixed_tree_at": (i32, [vp, u64, vp, vp, f32, u64, u64, vp]),
        "orc_routed_fc2": (i32, [vp, vp, u64, u64, u64, u64, vp, vp, vp, vp, u64, vp]),
        "orc_finish_sparse_layer": (i32, [vp, vp, vp, vp, u32, u64, vp]),
        "orc_generate_routes": (i32, [i32, u64, vp, vp]),
        "orc_generate_numerical_fixture": (i32, [i32, u64, u64, u64, vp, vp]),
        "orc_actual_shape_values": (None, [u64, u64, vp]),
        "orc_router_exp": (f32, [f32]),
        "orc_router_sigmoid": (f32, [f32]),
        "orc_router_logits": (None, [vp, u64, u64, vp, u64, vp, i32]),
        "orc_router_select": (i32, [vp, u64, u64, vp, u32, u32, u32, f32, vp, vp]),
        "orc_moe_layer": (i32, [u32, u32, u32, u32, u32, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                vp, vp, u32, vp, u32, vp, vp, i32]),
        "orc_expert_prepare": (i32, [vp, vp, f32, vp, vp, f32, u32, u32, vp, vp]),
        "orc_shared_prepare": (i32, [vp, vp, u32, u32, vp, vp]),
        "orc_moe_expert_h": (i32, [u32, u32, vp, vp, u32, vp, vp, i32]),
        "orc_moe_expert_rows": (i32, [u32, u32, vp, vp, vp, vp, u32, vp, vp, vp, i32]),
        "orc_shared_rows": (i32, [u32, u32, vp, vp, u32, vp, vp, vp, i32]),
        "orc_threads": (i32, []),
        "orc_f32_to_f16_bits": (u16, [f32]),
        "orc_f16_bits_to_f32": (f32, [u16]),
        "orc_exl3_xorshift_trellis": (None, [u64, u64, vp]),
        "orc_exl3_decode_native_at": (u16, [vp, u64, u32, u64, u64]),
        "orc_exl3_reconstruct_native": (None, [vp, u64, u64, u32, vp]),
        "orc_exl3_prepare": (i32, [vp, u64, u64, u32, vp]),
        "orc_exl3_project": (i32, [vp, u64, u64, vp, vp, vp, u64, vp, i32]),
        "orc_exl3_matmul_reference": (i32, [vp, u64, u64, u32, vp, vp, vp, u64, vp, i32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


class OracleError(RuntimeError):
    pass


def _check(status: int, what: str) -> None:
    if status != 0:
        raise OracleError(f"{what} failed with status {status}")


def threads() -> int:
    return int(os.environ.get("GLMAXX_ORACLE_THREADS", os.cpu_count() or 1))


# --------------------------------------------------------------------------- codecs
def decode_e2m1(code: int) -> float:
    return lib().orc_decode_e2m1(code)


def encode_e2m1(value: float) -> int:
    out = np.zeros(1, np.uint8)
    _check(lib().orc_encode_e2m1(value, _p(out)), "encode_e2m1")
    return int(out[0])


def decode_e4m3(code: int) -> float:
    return lib().orc_decode_e4m3(code)


def encode_e4m3(value: float) -> int:
    out = np.zeros(1, np.uint8)
    _check(lib().orc_encode_e4m3(value, _p(out)), "encode_e4m3")
    return int(out[0])


def crc32c(data: bytes) -> int:
    buf = np.frombuffer(data, np.uint8).copy()
    return int(lib().orc_crc32c(_p(buf), len(data)))


def scale_offset(n: int, group: int, padded_n: int, padded_k: int) -> int:
    return int(lib().orc_scale_offset(n, group, padded_n, padded_k))


def padded(n: int, k: int) -> tuple[int, int]:
    return (n + 127) // 128 * 128, (k + 63) // 64 * 64


class Packed:
    """PackedNvfp4 (nvfp4.rs:165-169): metadata fields + value and scale planes."""

    def __init__(self, values, scales, global_scale, global_amax, n, k, codec):
        self.values, self.scales = values, scales
        self.global_scale, self.global_amax = float(global_scale), float(global_amax)
        self.n, self.k, self.codec = n, k, codec

    def metadata(self) -> bytes:
        pn, pk = padded(self.n, self.k)
        out = np.zeros(128, np.uint8)
        lib().orc_nvfp4_metadata_encode(1 if self.codec == "1d" else 2, self.n, self.k, pn, pk,
                                        self.global_scale, self.global_amax, self.values.size,
                                        self.scales.size, _p(out))
        return out.tobytes()

    def sha256(self) -> str:
        """packed_hash (crates/glm-cli/src/main.rs:6080-6086)."""
        h = hashlib.sha256()
        h.update(self.metadata())
        h.update(self.values.tobytes())
        h.update(self.scales.tobytes())
        return h.hexdigest()

    def dequantize(self) -> np.ndarray:
        out = np.zeros(self.n * self.k, np.float32)
        _check(lib().orc_nvfp4_dequantize(_p(self.values), _p(self.scales), self.global_scale,
                                          self.n, self.k, _p(out)), "dequantize")
        return out.reshape(self.n, self.k)


def pack(x: np.ndarray, codec: str = "1d") -> Packed:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, k = x.shape
    pn, pk = padded(n, k)
    values = np.zeros(pn * pk // 2, np.uint8)
    scales = np.zeros(pn * pk // 16, np.uint8)
    gs = np.zeros(1, np.float32)
    ga = np.zeros(1, np.float32)
    _check(lib().orc_nvfp4_pack(_p(x), n, k, 1 if codec == "1d" else 2, _p(values), _p(scales),
                                _p(gs), _p(ga)), "pack")
    return Packed(values, scales, gs[0], ga[0], n, k, codec)


def f32_hash(values: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(values, dtype="<f4").tobytes()).hexdigest()


def u16_hash(values: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(values, dtype="<u2").tobytes()).hexdigest()


# ------------------------------------------------------------------- bf16 helpers
def bf16_round(x: np.ndarray) -> np.ndarray:
    """routed_fc1.rs:156-163, vectorised (RNE to bf16, non-finite passes through)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    bias = 0x7FFF + ((bits >> 16) & 1)
    out = ((bits + bias) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    return np.where(np.isfinite(x), out, x)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------ routes / fc1 / fc2
def routes_array(rows) -> np.ndarray:
    arr = np.zeros(len(rows), ROUTE_DTYPE)
    for i, (t, e, s, w) in enumerate(rows):
        arr[i] = (t, e, s, 0, w)
    return arr


def compact_routes(routes: np.ndarray, token_count: int) -> np.ndarray:
    routes = np.ascontiguousarray(routes, ROUTE_DTYPE)
    out = np.zeros(max(len(routes), 1), COMPACTED_DTYPE)
    _check(lib().orc_compact_routes(_p(routes), len(routes), token_count, _p(out)), "compact_routes")
    return out[: len(routes)]


def generate_routes(case: str, token_count: int) -> np.ndarray:
    routes = np.zeros(max(token_count * 8, 2), ROUTE_DTYPE)
    count = np.zeros(1, np.uint64)
    _check(lib().orc_generate_routes(ROUTING_CASES.index(case), token_count, _p(routes),
                                     _p(count)), "generate_routes")
    return routes[: int(count[0])]


def generate_numerical_fixture(case: str, rows: int, n: int, k: int):
    act = np.zeros(rows * k, np.float32)
    w = np.zeros(n * k, np.float32)
    _check(lib().orc_generate_numerical_fixture(NUMERICAL_CASES.index(case), rows, n, k,
                                                _p(act), _p(w)), "numerical fixture")
    return act.reshape(rows, k), w.reshape(n, k)


def actual_shape_values(n: int, k: int) -> np.ndarray:
    out = np.zeros(n * k, np.float32)
    lib().orc_actual_shape_values(n, k, _p(out))
    return out.reshape(n, k)


def routed_fc1(activations: np.ndarray, weights: Packed) -> np.ndarray:
    a = np.ascontiguousarray(activations, np.float32)
    rows, k = a.shape
    out = np.zeros(rows * (weights.n // 2), np.float32)
    _check(lib().orc_routed_fc1(_p(a), rows, k, _p(weights.values), _p(weights.scales),
                                weights.global_scale, weights.n, _p(out)), "routed_fc1")
    return out.reshape(rows, weights.n // 2)


def routed_fc1_fixed_tree_at(activation: np.ndarray, weights: Packed, column: int) -> float:
    a = np.ascontiguousarray(activation, np.float32)
    out = np.zeros(1, np.float32)
    _check(lib().orc_routed_fc1_fixed_tree_at(_p(a), a.size, _p(weights.values),
                                              _p(weights.scales), weights.global_scale,
                                              weights.n, column, _p(out)), "fixed_tree")
    return out


def routed_fc2(activated: np.ndarray, routes: np.ndarray, token_count: int,
               local_intermediate: int, hidden: int, weights: dict) -> np.ndarray:
    """weights: {expert: Packed down [hidden, local_intermediate]}"""
    act = np.ascontiguousarray(activated, np.float32)
    routes = np.ascontiguousarray(routes, ROUTE_DTYPE)
    experts = np.array(sorted(weights), np.uint16)
    vals = (ctypes.c_void_p * len(experts))(*[weights[e].values.ctypes.data for e in experts])
    scs = (ctypes.c_void_p * len(experts))(*[weights[e].scales.ctypes.data for e in experts])
    globs = np.array([weights[e].global_scale for e in experts], np.float32)
    out = np.zeros(token_count * hidden, np.float32)
    _check(lib().orc_routed_fc2(_p(act), _p(routes), len(routes), token_count,
                                local_intermediate, hidden, _p(experts),
                                ctypes.cast(vals, ctypes.c_void_p),
                                ctypes.cast(scs, ctypes.c_void_p), _p(globs), len(experts),
                                _p(out)), "routed_fc2")
    return out.reshape(token_count, hidden)


def finish_sparse_layer(residual, attention, routed, shared) -> np.ndarray:
    """Rank-order finish (routed_fc2.rs:214-258).  attention/routed/shared: [ranks, ...]."""
    routed = np.ascontiguousarray(routed, np.float32)
    ranks = routed.shape[0]
    elems = routed[0].size
    res = np.ascontiguousarray(residual, np.float32) if residual is not None else None
    att = np.ascontiguousarray(attention, np.float32) if attention is not None else None
    sh = np.ascontiguousarray(shared, np.float32) if shared is not None else None
    out = np.zeros(elems, np.float32)
    _check(lib().orc_finish_sparse_layer(_p(res), _p(att), _p(routed), _p(sh), ranks, elems,
                                         _p(out)), "finish")
    return out.reshape(routed.shape[1:])


# ------------------------------------------------------------------------ router
def router_exp(x: float) -> float:
    return lib().orc_router_exp(x)


def router_logits(x_bf16: np.ndarray, w_bf16: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16, np.uint16)
    w = np.ascontiguousarray(w_bf16, np.uint16)
    t, h = x.shape
    e = w.shape[0]
    out = np.zeros(t * e, np.float32)
    lib().orc_router_logits(_p(x), t, h, _p(w), e, _p(out), threads())
    return out.reshape(t, e)


def router_select(logits: np.ndarray, bias: np.ndarray, groups: int, topk_groups: int,
                  topk: int = 8, route_scale: float = 2.5):
    lg = np.ascontiguousarray(logits, np.float32)
    t, e = lg.shape
    b = np.ascontiguousarray(bias, np.float32)
    ex = np.zeros(t * topk, np.uint16)
    w = np.zeros(t * topk, np.float32)
    _check(lib().orc_router_select(_p(lg), t, e, _p(b), groups, topk_groups, topk, route_scale,
                                   _p(ex), _p(w)), "router_select")
    return ex.reshape(t, topk), w.reshape(t, topk)


def router(x_bf16, w_bf16, bias, groups, topk_groups, topk=8, route_scale=2.5):
    return router_select(router_logits(x_bf16, w_bf16), bias, groups, topk_groups, topk,
                         route_scale)


# ------------------------------------------------------------------------- layer
def moe_layer(x_bf16, route_experts, route_weights, w13_values, w13_scales, w13_global,
              w2_values, w2_scales, w2_global, local_inter, shared13_bf16=None,
              shared2_bf16=None, token_subset=None):
    """Rank-local routed + shared partials (fp32), each [tokens_or_subset, hidden]."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    t, h = x.shape
    re = np.ascontiguousarray(route_experts, np.uint16)
    rw = np.ascontiguousarray(route_weights, np.float32)
    topk = re.shape[1]
    experts = w13_global.shape[0]
    subset = None if token_subset is None else np.ascontiguousarray(token_subset, np.uint32)
    nsel = t if subset is None else subset.size
    routed = np.zeros(nsel * h, np.float32)
    shared = np.zeros(nsel * h, np.float32)
    arrs = [np.ascontiguousarray(a) for a in (w13_values, w13_scales, w13_global, w2_values,
                                               w2_scales, w2_global)]
    s13 = None if shared13_bf16 is None else np.ascontiguousarray(shared13_bf16, np.uint16)
    s2 = None if shared2_bf16 is None else np.ascontiguousarray(shared2_bf16, np.uint16)
    shared_inter = 0 if s2 is None else s2.shape[1]
    _check(lib().orc_moe_layer(t, h, experts, local_inter, topk, _p(x), _p(re), _p(rw),
                               *[_p(a) for a in arrs], _p(s13), _p(s2), shared_inter, _p(subset),
                               0 if subset is None else subset.size, _p(routed), _p(shared),
                               threads()), "moe_layer")
    return routed.reshape(nsel, h), shared.reshape(nsel, h)


def expert_prepare(w13_values, w13_scales, w13_global, w2_values, w2_scales, w2_global,
                   hidden, local_inter):
    """One expert dequantised once (nvfp4.rs:279-301) into k-major fp32 planes:
    (w13t [H, 2I], w2t [I, H])."""
    w13t = np.empty((hidden, 2 * local_inter), np.float32)
    w2t = np.empty((local_inter, hidden), np.float32)
    a = [np.ascontiguousarray(v) for v in (w13_values, w13_scales, w2_values, w2_scales)]
    _check(lib().orc_expert_prepare(_p(a[0]), _p(a[1]), float(w13_global), _p(a[2]), _p(a[3]),
                                    float(w2_global), hidden, local_inter, _p(w13t), _p(w2t)),
           "expert_prepare")
    return w13t, w2t


def shared_prepare(shared13_bf16, shared2_bf16):
    """The bf16 shared expert as k-major fp32 planes (s13t [H, 2Is], s2t [Is, H])."""
    s13 = np.ascontiguousarray(shared13_bf16, np.uint16)
    s2 = np.ascontiguousarray(shared2_bf16, np.uint16)
    hidden, inter = s2.shape
    s13t = np.empty((hidden, 2 * inter), np.float32)
    s2t = np.empty((inter, hidden), np.float32)
    _check(lib().orc_shared_prepare(_p(s13), _p(s2), hidden, inter, _p(s13t), _p(s2t)),
           "shared_prepare")
    return s13t, s2t


def moe_expert_rows(x_bf16, tokens, weights, out_rows, w13t, w2t, out):
    """Adds one expert's weighted FC1 -> SwiGLU -> FC2 rows into out[out_rows]."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    tok = np.ascontiguousarray(tokens, np.uint32)
    wt = np.ascontiguousarray(weights, np.float32)
    rows = np.ascontiguousarray(out_rows, np.uint32)
    hidden, inter = x.shape[1], w2t.shape[0]
    assert out.dtype == np.float32 and out.flags.c_contiguous
    _check(lib().orc_moe_expert_rows(hidden, inter, _p(x), _p(tok), _p(wt), _p(rows), tok.size,
                                     _p(w13t), _p(w2t), _p(out), threads()), "moe_expert_rows")


def moe_expert_h(x_bf16, tokens, w13t):
    """FC1 + SwiGLU (routed_fc1.rs:84-103) of one expert's rows: h [rows, I],
    bf16-valued fp32."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    tok = np.ascontiguousarray(tokens, np.uint32)
    inter = w13t.shape[1] // 2
    h = np.zeros((tok.size, inter), np.float32)
    _check(lib().orc_moe_expert_h(x.shape[1], inter, _p(x), _p(tok), tok.size, _p(w13t), _p(h),
                                  threads()), "moe_expert_h")
    return h


def shared_rows(x_bf16, tokens, s13t, s2t):
    x = np.ascontiguousarray(x_bf16, np.uint16)
    tok = np.ascontiguousarray(tokens, np.uint32)
    out = np.zeros((tok.size, x.shape[1]), np.float32)
    _check(lib().orc_shared_rows(x.shape[1], s2t.shape[0], _p(x), _p(tok), tok.size, _p(s13t),
                                 _p(s2t), _p(out), threads()), "shared_rows")
    return out


def expert_rows_plan(route_experts, token_subset=None):
    """Compacted order (routed_fc1.rs:20-58) of the routes of the selected tokens:
    {expert: (tokens ascending, slots, output rows)} in ascending expert order."""
    re = np.asarray(route_experts).astype(np.int64)
    t_all = np.arange(re.shape[0]) if token_subset is None else np.asarray(token_subset, np.int64)
    out_row = np.arange(t_all.size)
    tok = np.repeat(t_all, re.shape[1])
    slot = np.tile(np.arange(re.shape[1]), t_all.size)
    row = np.repeat(out_row, re.shape[1])
    exp = re[tok, slot]
    order = np.lexsort((slot, tok, exp))
    plan = {}
    exp, tok, slot, row = exp[order], tok[order], slot[order], row[order]
    bounds = np.flatnonzero(np.diff(exp)) + 1
    for a, b in zip(np.r_[0, bounds], np.r_[bounds, exp.size]):
        if b > a:
            plan[int(exp[a])] = (tok[a:b], slot[a:b], row[a:b])
    return plan


def moe_layer_prepared(x_bf16, route_experts, route_weights, prepare, local_inter,
                       shared=None, token_subset=None):
    """orc_moe_layer, bit for bit, on experts dequantised once: prepare(e) returns
    expert e's (w13t, w2t) (expert_prepare) and is called once per routed expert in
    ascending order, outside the timed part; shared is (s13t, s2t) or None.
    Returns (routed, shared_out, compute seconds excluding prepare)."""
    import time
    x = np.ascontiguousarray(x_bf16, np.uint16)
    rw = np.asarray(route_weights, np.float32)
    hidden = x.shape[1]
    plan = expert_rows_plan(route_experts, token_subset)
    nsel = x.shape[0] if token_subset is None else len(token_subset)
    routed = np.zeros((nsel, hidden), np.float32)
    busy = 0.0
    for e in sorted(plan):
        tok, slot, row = plan[e]
        w13t, w2t = prepare(e)
        t0 = time.perf_counter()
        moe_expert_rows(x, tok, rw[tok, slot], row, w13t, w2t, routed)
        busy += time.perf_counter() - t0
    shared_out = np.zeros((nsel, hidden), np.float32)
    if shared is not None:
        toks = np.arange(x.shape[0]) if token_subset is None else np.asarray(token_subset)
        t0 = time.perf_counter()
        shared_out = shared_rows(x, toks, *shared)
        busy += time.perf_counter() - t0
    return routed, shared_out, busy


# -------------------------------------------------------------------------- exl3
def f32_to_f16_bits(x: float) -> int:
    return int(lib().orc_f32_to_f16_bits(x))


def f16_bits_to_f32(b: int) -> float:
    return lib().orc_f16_bits_to_f32(b)


def exl3_trellis_words(k: int, n: int, bits: int) -> int:
    return (k // 16) * (n // 16) * 16 * bits


def exl3_xorshift_trellis(seed: int, words: int) -> np.ndarray:
    out = np.zeros(words, np.uint16)
    lib().orc_exl3_xorshift_trellis(seed, words, _p(out))
    return out


def exl3_reconstruct_native(trellis: np.ndarray, k: int, n: int, bits: int = 3) -> np.ndarray:
    out = np.zeros(k * n, np.uint16)
    tr = np.ascontiguousarray(trellis, np.uint16)
    lib().orc_exl3_reconstruct_native(_p(tr), k, n, bits, _p(out))
    return out.reshape(k, n)


def exl3_matmul_reference(trellis, k, n, suh, svh, activations_f16, bits=3) -> np.ndarray:
    tr = np.ascontiguousarray(trellis, np.uint16)
    su = np.ascontiguousarray(suh, np.uint16)
    sv = np.ascontiguousarray(svh, np.uint16)
    a = np.ascontiguousarray(activations_f16, np.uint16)
    rows = a.shape[0]
    out = np.zeros(rows * n, np.uint16)
    _check(lib().orc_exl3_matmul_reference(_p(tr), k, n, bits, _p(su), _p(sv), _p(a), rows,
                                           _p(out), threads()), "exl3 matmul")
    return out.reshape(rows, n)


def exl3_prepare(trellis, k: int, n: int, bits: int = 3) -> np.ndarray:
    """One trellis decoded once (exl3.rs:490-513) to fp32 [k, n]."""
    tr = np.ascontiguousarray(trellis, np.uint16)
    out = np.empty((k, n), np.float32)
    _check(lib().orc_exl3_prepare(_p(tr), k, n, bits, _p(out)), "exl3_prepare")
    return out


def exl3_project(weights_f32, suh, svh, activations_f16) -> np.ndarray:
    """matmul_reference_f16 (exl3.rs:404-453) on weights from exl3_prepare: same bits."""
    k, n = weights_f32.shape
    x = np.ascontiguousarray(activations_f16, np.uint16).reshape(-1, k)
    out = np.zeros((x.shape[0], n), np.uint16)
    _check(lib().orc_exl3_project(_p(weights_f32), k, n, _p(np.ascontiguousarray(suh, np.uint16)),
                                  _p(np.ascontiguousarray(svh, np.uint16)), _p(x), x.shape[0],
                                  _p(out), threads()), "exl3_project")
    return out

