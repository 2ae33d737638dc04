"""A routed-MoE layer loaded from a rank file straight into HBM.

The product converter writes one TP4 rank's layer (router, bias, NVFP4 or
EXL3 experts, shared expert) to a .g5n file; the native reader verifies it and
streams every plane with cudaMemcpyAsync from pinned staging into device
tensors.  The placed tensors equal the generated ones byte for byte, and the
layer run on them gives bit-identical output to the layer run on the
generated tensors.  A file with a flipped payload byte is refused after the
stream (its device bytes stay tentative)."""
import numpy as np
import pytest
import torch

from glmaxx_b200 import rank_file as R
from glmaxx_b200 import synth
from glmaxx_b200.moe import MoEConfig, RoutedMoE
from tests.gpu_util import cuda

pytestmark = pytest.mark.gpu
LAYER = 3


def same(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


def write_and_load(tmp_path, w, cfg):
    recs = R.moe_layer_records(w, cfg, LAYER)
    path = tmp_path / f"rank{cfg.rank}.g5n"
    R.RankFileBuilder(cfg.rank, b'{"rank":%d}' % cfg.rank, tensors=recs).write(path, bytes(16))
    with R.NativeRankReader.open(path) as rd:
        loaded, proof = R.load_moe_layers(rd, cfg, [LAYER], device=cuda())
        assert bytes(proof.payload_sha256) == rd.payload_sha256
    torch.cuda.synchronize()
    return loaded[LAYER], proof, path


def test_gpu_nvfp4_layer_from_rank_file(tmp_path):
    cfg = MoEConfig(experts=16, groups=1, topk_groups=1, tp=4, rank=1)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=21, device=dev)
    lw, proof, path = write_and_load(tmp_path, w, cfg)
    planes = sum(t.numel() for t in (w.w13.values, w.w13.scales, w.w2.values, w.w2.scales))
    assert proof.device_bytes == (planes + 4 * 2 * cfg.experts + w.router_weight.numel() * 2 +
                                  cfg.experts * 4 + (w.shared13.numel() + w.shared2.numel()) * 2)
    for a, b in ((lw.router_weight, w.router_weight), (lw.router_bias, w.router_bias),
                 (lw.shared13, w.shared13), (lw.shared2, w.shared2)):
        assert same(a, b)
    for p, q in ((lw.w13, w.w13), (lw.w2, w.w2)):
        for f in ("values", "scales", "global_scale", "global_amax"):
            assert same(getattr(p, f), getattr(q, f)), f
    T = 40
    x = synth.make_input(T, cfg.hidden, seed=21, device=dev)
    ref, got = RoutedMoE(cfg, w, T), RoutedMoE(cfg, lw, T)
    a, b = ref(x), got(x)
    torch.cuda.synchronize()
    assert got.device_status() == [] and torch.equal(a, b)

    bad = bytearray(path.read_bytes())
    d = R.NativeRankReader.open(path).descriptors[5]
    bad[d.payload_offset + 1000] ^= 0x21
    bad_path = tmp_path / "bad.g5n"
    bad_path.write_bytes(bytes(bad))
    with R.NativeRankReader.open(bad_path) as rd:
        with pytest.raises(R.RankFileError) as e:
            R.load_moe_layers(rd, cfg, [LAYER], device=dev)
    assert e.value.kind == "TensorRegion"


def test_gpu_hybrid_layer_from_rank_file(tmp_path):
    """Half the experts EXL3 (source trellis layout, placed as stored), half NVFP4."""
    cfg = MoEConfig(experts=16, groups=1, topk_groups=1, tp=4, rank=2)
    dev = cuda()
    g = torch.Generator().manual_seed(4)
    mask = torch.zeros(cfg.experts, dtype=torch.bool)
    mask[torch.randperm(cfg.experts, generator=g)[:cfg.experts // 2]] = True
    w = synth.make_exl3_rank_weights(cfg, seed=23, device=dev, nvfp4_experts=mask)
    lw, proof, _ = write_and_load(tmp_path, w, cfg)
    assert same(lw.exl3.codec, w.exl3.codec)
    for e in np.flatnonzero(~mask.numpy()):
        for f in ("gate_trellis", "up_trellis", "down_trellis", "gate_suh", "gate_svh", "up_suh",
                  "up_svh", "down_suh", "down_svh"):
            assert same(getattr(lw.exl3, f)[e], getattr(w.exl3, f)[e]), (f, e)
    for p, q in ((lw.w13, w.w13), (lw.w2, w.w2)):
        for f in ("values", "scales", "global_scale"):
            assert same(getattr(p, f), getattr(q, f)), f
    T = 24
    x = synth.make_input(T, cfg.hidden, seed=23, device=dev)
    ref, got = RoutedMoE(cfg, w, T), RoutedMoE(cfg, lw, T)
    a, b = ref(x), got(x)
    torch.cuda.synchronize()
    assert got.device_status() == [] and torch.equal(a, b)
