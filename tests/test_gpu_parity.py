"""GPU parity of the sm_100a path against the CPU oracle (calls go through the C ABI).

Bit-exact: NVFP4 packing (against the reference golden hashes and the oracle),
routing indices/weights and compaction.  Layer outputs: rel-L2 <= 1e-3 and
max-abs <= 4 bf16 ulp of the output scale (tests/gpu_util.py).
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from glmaxx_b200 import abi, synth
from glmaxx_b200.moe import MoEConfig, RoutedMoE, pack_nvfp4

from gpu_util import (MAX_ABS_ULPS, assert_layer_close, bf16_ulp, cuda, rel_l2,
                      to_np_bf16_bits)

pytestmark = pytest.mark.gpu


def _packed_to_oracle(p, b=0):
    return O.Packed(p.values[b].cpu().numpy().ravel(), p.scales[b].cpu().numpy().ravel(),
                    float(p.global_scale[b]), float(p.global_amax[b]), p.n, p.k, "1d")


def test_gpu_packer_actual_shape_golden(golden):
    g = golden["actual_shape"]
    w = torch.from_numpy(O.actual_shape_values(g["n"], g["k"])).to(cuda())
    p = pack_nvfp4(w)
    torch.cuda.synchronize()
    assert _packed_to_oracle(p).sha256() == g["packed_sha256"]


@pytest.mark.parametrize("case", O.NUMERICAL_CASES)
def test_gpu_packer_matrix_golden(golden, case):
    mp = golden["matrix_proof"]
    n, k, _ = mp["model_shape"]
    entry = next(e for e in mp["numerical"] if e["case"] == case)
    _, w = O.generate_numerical_fixture(case, 1, n, k)
    p = pack_nvfp4(torch.from_numpy(w).to(cuda()))
    assert _packed_to_oracle(p).sha256() == entry["packed_weight_sha256"]


def test_gpu_packer_random_bf16_matches_oracle():
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((3, 256, 512)) * rng.choice([1e-3, 1.0, 300.0], (3, 1, 1)))
    wb = O.bf16_round(w.astype(np.float32))
    t = torch.from_numpy(wb).to(cuda()).to(torch.bfloat16)
    p = pack_nvfp4(t)
    for b in range(3):
        ref = O.pack(wb[b])
        got = _packed_to_oracle(p, b)
        assert np.array_equal(got.values, ref.values)
        assert np.array_equal(got.scales, ref.scales)
        assert got.global_scale == ref.global_scale


def _router_case(T, H, E, groups, topk_groups, seed):
    rng = np.random.default_rng(seed)
    x = O.f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    w = O.f32_to_bf16_bits((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    return x, w, bias


# (40, 40, 10, 3): groups of 4 experts, which are not whole lane runs, take the
# general selection kernel; the others take the lane-run kernel (groups of 8, 16,
# 32 experts).
@pytest.mark.parametrize("T,E,groups,topk_groups", [(64, 256, 8, 4), (8, 16, 1, 1), (333, 256, 8, 4),
                                                    (40, 40, 10, 3), (24, 96, 3, 2)])
def test_gpu_router_compact_bit_exact(T, E, groups, topk_groups):
    H, K = 6144, 8
    dev = cuda()
    x, w, bias = _router_case(T, H, E, groups, topk_groups, seed=T + E)
    ref_e, ref_w = O.router(x, w, bias, groups, topk_groups, K, 2.5)
    xd = torch.from_numpy(x.view(np.int16)).to(dev)
    wd = torch.from_numpy(w.view(np.int16)).to(dev)
    bd = torch.from_numpy(bias).to(dev)
    re = torch.empty((T, K), dtype=torch.int16, device=dev)
    rw = torch.empty((T, K), dtype=torch.float32, device=dev)
    ct = torch.empty(T * K, dtype=torch.int32, device=dev)
    ce = torch.empty(T * K, dtype=torch.int16, device=dev)
    cs = torch.empty(T * K, dtype=torch.uint8, device=dev)
    cw = torch.empty(T * K, dtype=torch.float32, device=dev)
    off = torch.empty(E + 1, dtype=torch.int32, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    L = abi.load()
    wsb = int(L.glmaxx_router_workspace_bytes(T, H, E, K))
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    d = abi.RouterDescriptor.new(
        abi_version=abi.ROUTER_ABI_VERSION, tokens=T, hidden=H, experts=E, top_k=K, groups=groups,
        topk_groups=topk_groups, route_scale=2.5, input_bf16=xd.data_ptr(),
        router_weight_bf16=wd.data_ptr(), router_bias_f32=bd.data_ptr(),
        route_experts_u16=re.data_ptr(), route_weights_f32=rw.data_ptr(),
        compacted_tokens_u32=ct.data_ptr(), compacted_experts_u16=ce.data_ptr(),
        compacted_slots_u8=cs.data_ptr(), compacted_weights_f32=cw.data_ptr(),
        expert_offsets_u32=off.data_ptr(), validation_error_u32=st.data_ptr(),
        workspace=ws.data_ptr(), workspace_bytes=wsb)
    err = ctypes.c_int32(0)
    abi.check(L.glmaxx_router_compact_launch(
        ctypes.byref(d), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
        ctypes.byref(err)), "router")
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    got_e = re.cpu().numpy().view(np.uint16)
    got_w = rw.cpu().numpy()
    assert np.array_equal(got_e, ref_e)
    assert np.array_equal(got_w.view(np.uint32), ref_w.view(np.uint32))
    routes = O.routes_array([(t, int(ref_e[t, s]), s, float(ref_w[t, s]))
                             for t in range(T) for s in range(K)])
    comp = O.compact_routes(routes, T)
    assert np.array_equal(ct.cpu().numpy().view(np.uint32), comp["token"])
    assert np.array_equal(ce.cpu().numpy().view(np.uint16), comp["expert"])
    assert np.array_equal(cs.cpu().numpy(), comp["slot"])
    counts = np.bincount(comp["expert"], minlength=E)
    assert np.array_equal(off.cpu().numpy().view(np.uint32), np.concatenate([[0], np.cumsum(counts)]))


def _oracle_layer(layer: RoutedMoE, x: torch.Tensor, cfg: MoEConfig, subset=None):
    w = layer.w
    xb = to_np_bf16_bits(x)
    re, rw = layer.routes(x.shape[0])
    re = re.cpu().numpy().view(np.uint16)
    rw = rw.cpu().numpy()
    routed, shared = O.moe_layer(
        xb, re, rw, w.w13.values.cpu().numpy(), w.w13.scales.cpu().numpy(),
        w.w13.global_scale.cpu().numpy(), w.w2.values.cpu().numpy(), w.w2.scales.cpu().numpy(),
        w.w2.global_scale.cpu().numpy(), cfg.local_intermediate,
        None if w.shared13 is None else to_np_bf16_bits(w.shared13),
        None if w.shared2 is None else to_np_bf16_bits(w.shared2), token_subset=subset)
    return O.finish_sparse_layer(None, None, routed[None], shared[None])


def _check_routes(layer, x, cfg):
    xb = to_np_bf16_bits(x)
    ref_e, ref_w = O.router(xb, to_np_bf16_bits(layer.w.router_weight),
                            layer.w.router_bias.cpu().numpy(), cfg.groups, cfg.topk_groups,
                            cfg.top_k, cfg.route_scale)
    got_e, got_w = layer.routes(x.shape[0])
    assert np.array_equal(got_e.cpu().numpy().view(np.uint16), ref_e)
    assert np.array_equal(got_w.cpu().numpy().view(np.uint32), ref_w.view(np.uint32))


def _stage_pins(layer: RoutedMoE, x: torch.Tensor, cfg: MoEConfig, out: np.ndarray):
    """Pin each stage of the real layer run: the FC1 output h read back from the
    workspace against the oracle FC1 on the same compacted rows, and FC2 + combine
    against the oracle FC2 evaluated on the GPU's own h.  Returns (h rel-L2,
    routed rel-L2 given h)."""
    T, I, H = x.shape[0], cfg.local_intermediate, cfg.hidden
    A = T * cfg.top_k
    h = layer.plane("fc1_output_bf16").view(torch.bfloat16).reshape(A, I).float().cpu().numpy()
    tok = layer.plane("row_token_u32").view(torch.int32).cpu().numpy()
    slot = layer.plane("row_slot_u32").view(torch.int32).cpu().numpy()
    off = layer.plane("expert_offsets_u32").view(torch.int32).cpu().numpy()
    xf = O.bf16_bits_to_f32(to_np_bf16_bits(x))
    w = layer.w
    packed13 = lambda e: O.Packed(w.w13.values[e].cpu().numpy().ravel(),
                                  w.w13.scales[e].cpu().numpy().ravel(),
                                  float(w.w13.global_scale[e]), 0.0, 2 * I, H, "1d")
    packed2 = lambda e: O.Packed(w.w2.values[e].cpu().numpy().ravel(),
                                 w.w2.scales[e].cpu().numpy().ravel(),
                                 float(w.w2.global_scale[e]), 0.0, H, I, "1d")
    h_ref = np.zeros_like(h)
    experts = []
    for e in range(cfg.experts):
        if off[e + 1] > off[e]:
            experts.append(e)
            h_ref[off[e]:off[e + 1]] = O.routed_fc1(xf[tok[off[e]:off[e + 1]]], packed13(e))
    re, rw = layer.routes(T)
    re, rw = re.cpu().numpy().view(np.uint16), rw.cpu().numpy()
    routes = O.routes_array([(t, int(re[t, s]), s, float(rw[t, s]))
                             for t in range(T) for s in range(cfg.top_k)])
    comp = O.compact_routes(routes, T)
    assert np.array_equal(comp["token"], tok.astype(np.uint32))
    assert np.array_equal(comp["slot"], slot.astype(np.uint8))
    routed_on_gpu_h = O.routed_fc2(h, routes, T, I, H, {e: packed2(e) for e in experts})
    shared = 0.0
    if w.shared13 is not None:
        shared = layer.plane("shared_f32").view(torch.float32).reshape(T, H).cpu().numpy()
    return rel_l2(h, h_ref), rel_l2(out - shared, routed_on_gpu_h)


def test_gpu_layer_reduced_config0():
    """T=8, E=16, top-8 (no groups), I=2048, NVFP4 W4A4, no shared expert.

    Checks: routes bit-exact; end-to-end max-abs <= 4 bf16 ulp of the output scale;
    FC1 output h within rel-L2 1e-3 of the oracle FC1; FC2 + combine within rel-L2
    1e-5 of the oracle FC2 applied to the same h.  The end-to-end rel-L2 against
    the sequential-fp32 oracle is not asserted at 1e-3 for this 8-token case: the
    oracle's own rounding moves ~0.15% of the bf16 h values by one ulp relative to
    the tensor-core sum, and NVFP4 re-quantisation of h turns an isolated one-ulp
    move into a whole code step (measured across seeds: 6e-7 to 2.3e-3); with
    64 tokens or a shared expert the same path measures 2e-4 to 8e-4."""
    cfg = MoEConfig(experts=16, groups=1, topk_groups=1, shared_intermediate=0)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=3, device=dev)
    x = synth.make_input(8, cfg.hidden, seed=3, device=dev)
    layer = RoutedMoE(cfg, w, 8)
    out = layer(x)
    torch.cuda.synchronize()
    assert layer.device_status() == []
    _check_routes(layer, x, cfg)
    got = out.cpu().numpy()
    ref = _oracle_layer(layer, x, cfg)
    err = float(np.abs(got - ref).max())
    assert err <= MAX_ABS_ULPS * bf16_ulp(float(np.abs(ref).max()))
    h_err, fc2_err = _stage_pins(layer, x, cfg, got)
    assert h_err <= 1e-3, h_err
    assert fc2_err <= 1e-5, fc2_err


@pytest.mark.parametrize("tp,rank", [(1, 0), (4, 3)])
def test_gpu_layer_decode_config1(tp, rank):
    """BASELINE configs[1] shapes: T=64, E=256, 8 groups/top-4, shared expert, TP shard."""
    cfg = MoEConfig(tp=tp, rank=rank)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=11, device=dev)
    x = synth.make_input(64, cfg.hidden, seed=11, device=dev)
    layer = RoutedMoE(cfg, w, 64)
    out = layer(x)
    torch.cuda.synchronize()
    assert layer.device_status() == []
    _check_routes(layer, x, cfg)
    ref = _oracle_layer(layer, x, cfg)
    got = out.cpu().numpy()
    assert_layer_close(got, ref, f"decode tp{tp} r{rank}")
    h_err, fc2_err = _stage_pins(layer, x, cfg, got)
    assert h_err <= 1e-3, h_err
    assert fc2_err <= 1e-5, fc2_err


def test_gpu_layer_prefill_path_subset():
    """Prefill path (N tile 128, atomic combine) on T=1024, checked on a token subset."""
    cfg = MoEConfig(tp=2, rank=1)
    dev = cuda()
    T = 1024
    w = synth.make_rank_weights(cfg, seed=5, device=dev)
    x = synth.make_input(T, cfg.hidden, seed=5, device=dev)
    layer = RoutedMoE(cfg, w, T)
    out = layer(x, path=abi.PREFILL_GROUPED)
    torch.cuda.synchronize()
    assert layer.device_status() == []
    subset = np.arange(0, T, 37, dtype=np.uint32)
    ref = _oracle_layer(layer, x, cfg, subset=subset)
    assert_layer_close(out.cpu().numpy()[subset], ref, "prefill subset")


def test_gpu_layer_decode_and_prefill_paths_agree():
    """The routed experts compute the same rows on both paths (only the order of the
    prefill path's atomic combine differs).  The shared expert is split along K on the
    decode path and not on the prefill path, so with it the two paths agree to the
    layer tolerance rather than to fp32 reassociation."""
    cfg = MoEConfig(tp=8, rank=0)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=9, device=dev)
    x = synth.make_input(96, cfg.hidden, seed=9, device=dev)
    routed_only = RoutedMoE(MoEConfig(**{**cfg.__dict__, "shared_intermediate": 0}), w, 96)
    a = routed_only(x, path=abi.DECODE_PERSISTENT).clone()
    b = routed_only(x, path=abi.PREFILL_GROUPED).clone()
    torch.cuda.synchronize()
    assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < 1e-5
    layer = RoutedMoE(cfg, w, 96)
    a = layer(x, path=abi.DECODE_PERSISTENT).clone()
    b = layer(x, path=abi.PREFILL_GROUPED).clone()
    torch.cuda.synchronize()
    assert_layer_close(a.cpu().numpy(), b.cpu().numpy(), "decode vs prefill")


def test_gpu_layer_deterministic_decode():
    cfg = MoEConfig(tp=4, rank=0)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=2, device=dev)
    x = synth.make_input(64, cfg.hidden, seed=2, device=dev)
    layer = RoutedMoE(cfg, w, 64)
    outs = [layer(x).clone() for _ in range(5)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_gpu_layer_prefill_deterministic_flag():
    """GLMAXX_MOE_DETERMINISTIC on a prefill-size step (T=1024, TP2 shard): the
    routed rows go through the slot plane and the expert-order combine, so five
    runs give the same bits; the output is within the layer tolerance of the
    oracle on a token subset, and within fp32 reassociation of the atomic path."""
    cfg = MoEConfig(tp=2, rank=0)
    dev = cuda()
    T = 1024
    w = synth.make_rank_weights(cfg, seed=6, device=dev)
    x = synth.make_input(T, cfg.hidden, seed=6, device=dev)
    det = RoutedMoE(cfg, w, T, deterministic=True)
    outs = [det(x, path=abi.PREFILL_GROUPED).clone() for _ in range(5)]
    torch.cuda.synchronize()
    assert det.device_status() == []
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    subset = np.arange(3, T, 41, dtype=np.uint32)
    ref = _oracle_layer(det, x, cfg, subset=subset)
    assert_layer_close(outs[0].cpu().numpy()[subset], ref, "deterministic prefill subset")
    atomic = RoutedMoE(cfg, w, T)(x, path=abi.PREFILL_GROUPED)
    torch.cuda.synchronize()
    assert rel_l2(outs[0].cpu().numpy(), atomic.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("path,T", [(abi.DECODE_PERSISTENT, 64), (abi.PREFILL_GROUPED, 512)])
def test_gpu_layer_in_cuda_graph_matches_eager(path, T):
    """The shared expert runs on a side stream forked from the launch stream and
    joined before its consumer; captured in a CUDA graph the fork and join become
    graph edges.  Replays on new inputs equal eager launches (bit for bit on the
    deterministic decode path, to the layer tolerance on the atomic prefill path)."""
    cfg = MoEConfig(tp=4, rank=1)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=11, device=dev)
    layer = RoutedMoE(cfg, w, T)
    x = synth.make_input(T, cfg.hidden, seed=11, device=dev)
    out = torch.empty((T, cfg.hidden), dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer(x, out, path=path)  # eager warm-up on the capture stream
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            layer(x, out, path=path)
    for seed in (12, 13):
        x.copy_(synth.make_input(T, cfg.hidden, seed=seed, device=dev))
        g.replay()
        torch.cuda.synchronize()
        got = out.clone()
        ref = layer(x, path=path).clone()
        torch.cuda.synchronize()
        assert layer.device_status() == []
        if path == abi.DECODE_PERSISTENT:
            assert torch.equal(got, ref)
        else:
            assert_layer_close(got.cpu().numpy(), ref.cpu().numpy(), "graph vs eager")


def test_gpu_layer_first_launch_under_capture():
    """The side stream of the shared expert is created by an uncaptured launch;
    a thread whose first layer launch is captured runs the shared expert in order
    on the launch stream instead, with the same results."""
    import threading

    cfg = MoEConfig(tp=4, rank=2)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=21, device=dev)
    T = 64
    layer = RoutedMoE(cfg, w, T)
    x = synth.make_input(T, cfg.hidden, seed=21, device=dev)
    out = torch.empty((T, cfg.hidden), dtype=torch.float32, device=dev)
    # the workspace is allocated outside the capture by a first eager call on
    # this thread; the captured launch happens on a fresh thread
    ref = layer(x).clone()
    torch.cuda.synchronize()
    errors = []

    def capture_and_replay():
        try:
            torch.cuda.set_device(dev)
            s = torch.cuda.Stream(device=dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                layer(x, out)
            g.replay()
            torch.cuda.synchronize()
        except Exception as e:  # noqa: BLE001
            errors.append(repr(e))

    th = threading.Thread(target=capture_and_replay)
    th.start()
    th.join()
    assert errors == []
    assert torch.equal(out, ref)
