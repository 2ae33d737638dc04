"""Reference-ABI entry points (glmaxx_nvfp4_routed_fc1_launch / _fc2_launch) against
the CPU oracle's routed_fc1 / routed_fc2 (crates/glm-reference/src/routed_fc1.rs:66-105,
routed_fc2.rs:20-89), on the reference TP4 geometry (hidden 6144, local
intermediate 512, 256 experts) and on the TP1 geometry (intermediate 2048)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from glmaxx_b200 import abi
from glmaxx_b200.moe import pack_nvfp4

from gpu_util import cuda, rel_l2

pytestmark = pytest.mark.gpu


_STREAM = None


def _stream():
    """The reference ABI rejects a null stream (nvfp4_routed_fc1.cu:542-553), so the
    tests run on a created stream rather than torch's legacy default stream."""
    global _STREAM
    if _STREAM is None:
        _STREAM = torch.cuda.Stream()
    torch.cuda.current_stream().synchronize()
    return ctypes.c_void_p(_STREAM.cuda_stream)


class Case:
    """Routes of a seeded token batch over `experts`, with packed random weights."""

    def __init__(self, rows, experts, inter, hidden=6144, seed=0, routing="random"):
        dev = cuda()
        self.rows, self.E, self.I, self.H = rows, experts, inter, hidden
        rng = np.random.default_rng(seed)
        x = O.bf16_round(rng.standard_normal((rows, hidden)).astype(np.float32))
        self.x = x
        if routing == "random":
            routes = []
            for t in range(rows):
                ex = rng.choice(experts, size=min(8, experts), replace=False)
                for s, e in enumerate(ex):
                    routes.append((t, int(e), s, float(rng.uniform(0.05, 1.0))))
            self.routes = O.routes_array(routes)
        else:
            self.routes = O.generate_routes(routing, rows)
            self.routes["weight"] = rng.uniform(0.05, 1.0, len(self.routes)).astype(np.float32)
        self.comp = O.compact_routes(self.routes, rows)
        self.A = len(self.comp)
        g = torch.Generator(device=dev)
        g.manual_seed(seed + 1)
        self.w13 = pack_nvfp4(torch.randn(experts, 2 * inter, hidden, generator=g, device=dev) * 0.02)
        self.w2 = pack_nvfp4(torch.randn(experts, hidden, inter, generator=g, device=dev) * 0.02)
        counts = np.bincount(self.comp["expert"], minlength=experts)
        self.offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint32)
        wmap = {(int(r["token"]), int(r["expert"]), int(r["slot"])): float(r["weight"])
                for r in self.routes}
        self.comp_w = np.array([wmap[(int(c["token"]), int(c["expert"]), int(c["slot"]))]
                                for c in self.comp], np.float32)

    def packed(self, p, e):
        return O.Packed(p.values[e].cpu().numpy().ravel(), p.scales[e].cpu().numpy().ravel(),
                        float(p.global_scale[e]), float(p.global_amax[e]), p.n, p.k, "1d")

    def t(self, a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a)).to(cuda()).view(dtype)


def run_fc1(c: Case, path):
    dev = cuda()
    A, H, I = c.A, c.H, c.I
    L = abi.load()
    need = int(L.glmaxx_nvfp4_routed_fc1_workspace_bytes_v3(c.rows, A, H, I, c.E, 8))
    bufs = {
        "input": c.t(O.f32_to_bf16_bits(c.x).view(np.int16), torch.int16),
        "re": c.t(c.comp["expert"].astype(np.int16), torch.int16),
        "rt": c.t(c.comp["token"].astype(np.int32), torch.int32),
        "rs": c.t(c.comp["slot"].astype(np.uint8), torch.uint8),
        "rw": c.t(c.comp_w, torch.float32),
        "off": c.t(c.offsets.astype(np.int32), torch.int32),
        "compacted": torch.zeros(A * H * 2, dtype=torch.uint8, device=dev),
        "values": torch.zeros((A + 127) // 128 * 128 * H // 2, dtype=torch.uint8, device=dev),
        "scales": torch.zeros((A + 127 * min(A, c.E)) * H // 16 + 4096, dtype=torch.uint8, device=dev),
        "globals": torch.zeros(A, dtype=torch.float32, device=dev),
        "gate_up": torch.zeros(A * 2 * I, dtype=torch.float32, device=dev),
        "out": torch.zeros((A, I), dtype=torch.bfloat16, device=dev),
    }
    d = abi.Fc1Descriptor.new(
        abi_version=1, path=path, rows=c.rows, assignments=A, hidden=H, local_gate_up=2 * I,
        local_intermediate=I, experts=c.E, top_k=8, input_bf16=bufs["input"].data_ptr(),
        expert_value_base=c.w13.values.data_ptr(), expert_scale_base=c.w13.scales.data_ptr(),
        expert_global_scales=c.w13.global_scale.data_ptr(), route_experts_u16=bufs["re"].data_ptr(),
        route_tokens_u32=bufs["rt"].data_ptr(), route_slots_u8=bufs["rs"].data_ptr(),
        route_weights_f32=bufs["rw"].data_ptr(), expert_offsets_u32=bufs["off"].data_ptr(),
        compacted_input_bf16=bufs["compacted"].data_ptr(), activation_values=bufs["values"].data_ptr(),
        activation_scales=bufs["scales"].data_ptr(),
        activation_global_scales=bufs["globals"].data_ptr(),
        gate_up_accum_f32=bufs["gate_up"].data_ptr(), output_bf16=bufs["out"].data_ptr(),
        workspace_bytes=need, sequence=1)
    err = ctypes.c_int32(0)
    abi.check(L.glmaxx_nvfp4_routed_fc1_launch(ctypes.byref(d), _stream(), ctypes.byref(err)),
              "fc1")
    torch.cuda.synchronize()
    return bufs["out"].float().cpu().numpy()


def oracle_fc1(c: Case):
    out = np.zeros((c.A, c.I), np.float32)
    for e in range(c.E):
        b0, b1 = c.offsets[e], c.offsets[e + 1]
        if b1 > b0:
            rows = c.x[c.comp["token"][b0:b1]]
            out[b0:b1] = O.routed_fc1(rows, c.packed(c.w13, e))
    return out


def run_fc2(c: Case, h: np.ndarray, path):
    dev = cuda()
    A, H, I, R = c.A, c.H, c.I, c.rows
    L = abi.load()
    need = int(L.glmaxx_nvfp4_routed_fc2_workspace_bytes_v3(R, A, H, I, c.E, 8))
    b = {
        "input": torch.from_numpy(O.bf16_round(h)).to(dev).to(torch.bfloat16),
        "re": c.t(c.comp["expert"].astype(np.int16), torch.int16),
        "rt": c.t(c.comp["token"].astype(np.int32), torch.int32),
        "rs": c.t(c.comp["slot"].astype(np.uint8), torch.uint8),
        "rw": c.t(c.comp_w, torch.float32),
        "off": c.t(c.offsets.astype(np.int32), torch.int32),
        "values": torch.zeros((A + 127) // 128 * 128 * I // 2, dtype=torch.uint8, device=dev),
        "scales": torch.zeros((A + 127 * min(A, c.E)) * I // 16 + 4096, dtype=torch.uint8, device=dev),
        "globals": torch.zeros(A, dtype=torch.float32, device=dev),
        "down": torch.zeros((A, H), dtype=torch.float32, device=dev),
        "tok": torch.zeros((R, H), dtype=torch.float32, device=dev),
        "slots": torch.zeros(R * 8, dtype=torch.int32, device=dev),
        "status": torch.zeros(1, dtype=torch.int32, device=dev),
    }
    d = abi.Fc2Descriptor.new(
        abi_version=1, path=path, rows=R, assignments=A, hidden=H, local_intermediate=I,
        experts=c.E, top_k=8, input_bf16=b["input"].data_ptr(),
        expert_value_base=c.w2.values.data_ptr(), expert_scale_base=c.w2.scales.data_ptr(),
        expert_global_scales=c.w2.global_scale.data_ptr(), route_experts_u16=b["re"].data_ptr(),
        route_tokens_u32=b["rt"].data_ptr(), route_slots_u8=b["rs"].data_ptr(),
        route_weights_f32=b["rw"].data_ptr(), expert_offsets_u32=b["off"].data_ptr(),
        activation_values=b["values"].data_ptr(), activation_scales=b["scales"].data_ptr(),
        activation_global_scales=b["globals"].data_ptr(), assignment_down_f32=b["down"].data_ptr(),
        token_output_f32=b["tok"].data_ptr(), slot_assignment_u32=b["slots"].data_ptr(),
        validation_error_u32=b["status"].data_ptr(), workspace_bytes=need, sequence=1)
    err = ctypes.c_int32(0)
    abi.check(L.glmaxx_nvfp4_routed_fc2_launch(ctypes.byref(d), _stream(), ctypes.byref(err)),
              "fc2")
    torch.cuda.synchronize()
    assert int(b["status"].item()) == 0
    return b["tok"].cpu().numpy(), b["down"].cpu().numpy()


def oracle_fc2(c: Case, h: np.ndarray):
    weights = {e: c.packed(c.w2, e) for e in np.unique(c.comp["expert"])}
    return O.routed_fc2(O.bf16_round(h), c.routes, c.rows, c.I, c.H, weights)


def _report(got, ref, what):
    diff = got != ref
    print(f"{what}: rel-L2 {rel_l2(got, ref):.3e}, mismatched elements {diff.mean():.4%}, "
          f"max |d| {np.abs(got - ref).max():.3e} (ref max {np.abs(ref).max():.3e})")


@pytest.mark.parametrize("inter,experts,path", [(512, 256, 1), (512, 256, 2), (2048, 16, 1)])
def test_gpu_reference_fc1_abi(inter, experts, path):
    c = Case(rows=16, experts=experts, inter=inter, seed=inter + experts + path)
    got = run_fc1(c, path)
    ref = oracle_fc1(c)
    _report(got, ref, "fc1")
    # FC1 tolerance of the reference harness (crates/glm-cli/src/main.rs:3518):
    # |got - ref| <= 0.5 + 0.02 |ref|, plus rel-L2 <= 1e-3
    assert np.all(np.abs(got - ref) <= 0.5 + 0.02 * np.abs(ref))
    assert rel_l2(got, ref) <= 1e-3


@pytest.mark.parametrize("inter,experts,path", [(512, 256, 1), (512, 256, 2), (2048, 16, 1)])
def test_gpu_reference_fc2_abi(inter, experts, path):
    c = Case(rows=16, experts=experts, inter=inter, seed=7 + inter + experts + path)
    rng = np.random.default_rng(3)
    h = O.bf16_round(rng.standard_normal((c.A, c.I)).astype(np.float32) * 0.05)
    tok, _ = run_fc2(c, h, path)
    ref = oracle_fc2(c, h)
    _report(tok, ref, "fc2")
    # FC2 tolerance of the reference harness (main.rs:3672): 0.5 + 0.03 |ref|, plus rel-L2
    assert np.all(np.abs(tok - ref) <= 0.5 + 0.03 * np.abs(ref))
    assert rel_l2(tok, ref) <= 1e-3
