"""The allocation-free router entry point (glmaxx_router_compact_launch_static).

Callers that cannot allocate -- an engine with a fixed up-front HBM plan, or code
that must not call cudaMalloc (it can synchronise the device) -- use this
variant, whose scratch is a device array inside the library.  This file sorts last so that a
run stopping at its first failure has already run every other test; it also
passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from glmaxx_b200 import abi

pytestmark = pytest.mark.gpu

H, E, K = 6144, 256, 8


def _bufs(T, seed):
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    b = torch.randn(E, generator=g, device=dev) * 0.01
    return x, w, b


def _outputs(T, dev):
    return {
        "re": torch.full((T, K), -1, dtype=torch.int16, device=dev),
        "rw": torch.full((T, K), float("nan"), dtype=torch.float32, device=dev),
        "ct": torch.full((T * K,), -1, dtype=torch.int32, device=dev),
        "ce": torch.full((T * K,), -1, dtype=torch.int16, device=dev),
        "cs": torch.full((T * K,), 255, dtype=torch.uint8, device=dev),
        "cw": torch.full((T * K,), float("nan"), dtype=torch.float32, device=dev),
        "off": torch.full((E + 1,), -1, dtype=torch.int32, device=dev),
        "st": torch.full((1,), -1, dtype=torch.int32, device=dev),
    }


def _launch(fn, T, x, w, b, o, ws=None):
    d = abi.RouterDescriptor.new(
        abi_version=abi.ROUTER_ABI_VERSION, tokens=T, hidden=H, experts=E, top_k=K, groups=8,
        topk_groups=4, route_scale=2.5, input_bf16=x.data_ptr(), router_weight_bf16=w.data_ptr(),
        router_bias_f32=b.data_ptr(), route_experts_u16=o["re"].data_ptr(),
        route_weights_f32=o["rw"].data_ptr(), compacted_tokens_u32=o["ct"].data_ptr(),
        compacted_experts_u16=o["ce"].data_ptr(), compacted_slots_u8=o["cs"].data_ptr(),
        compacted_weights_f32=o["cw"].data_ptr(), expert_offsets_u32=o["off"].data_ptr(),
        validation_error_u32=o["st"].data_ptr(),
        workspace=0 if ws is None else ws.data_ptr(),
        workspace_bytes=0 if ws is None else ws.numel())
    err = ctypes.c_int32(0)
    status = fn(ctypes.byref(d), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                ctypes.byref(err))
    return status


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_static_router_matches_workspace_router_twice():
    """Calls in a row on different shapes: T=64 and T=200 take the small-T logits
    kernel, T=507 (the largest shape whose scratch fits) the tiled one.  Every
    output equals the workspace router's, and the routes equal the oracle
    router's bits."""
    assert torch.cuda.is_available()
    dev = torch.device("cuda:0")
    L = abi.load()
    for T, seed in [(64, 1), (200, 2), (507, 4)]:
        x, w, b = _bufs(T, seed)
        ref = _outputs(T, dev)
        ws = torch.empty(int(L.glmaxx_router_workspace_bytes(T, H, E, K)), dtype=torch.uint8,
                         device=dev)
        assert _launch(L.glmaxx_router_compact_launch, T, x, w, b, ref, ws) == 0
        got = _outputs(T, dev)
        assert _launch(L.glmaxx_router_compact_launch_static, T, x, w, b, got) == 0
        torch.cuda.synchronize()
        assert int(got["st"].item()) == 0
        for k in ref:
            assert torch.equal(got[k], ref[k]), k
        ref_e, ref_w = O.router(_bits(x), _bits(w), b.cpu().numpy(), 8, 4, K, 2.5)
        assert np.array_equal(_bits(got["re"]), ref_e)
        assert np.array_equal(got["rw"].cpu().numpy().view(np.uint32), ref_w.view(np.uint32))


def test_static_router_rejects_shapes_beyond_its_scratch():
    L = abi.load()
    dev = torch.device("cuda:0")
    T = 508  # the first token count whose scratch exceeds the array (T = 507 fits)
    assert int(L.glmaxx_router_workspace_bytes(T, H, E, K)) > abi.ROUTER_STATIC_SCRATCH_BYTES
    assert int(L.glmaxx_router_workspace_bytes(T - 1, H, E, K)) <= abi.ROUTER_STATIC_SCRATCH_BYTES
    x, w, b = _bufs(T, 3)
    o = _outputs(T, dev)
    assert _launch(L.glmaxx_router_compact_launch_static, T, x, w, b, o) == -2  # GLMAXX_ERR_DESCRIPTOR
    torch.cuda.synchronize()
    assert int(o["st"].item()) == -1  # nothing ran: the status word is untouched
