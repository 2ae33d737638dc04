"""One rank's routed-MoE layer through a rank file, on the host: the product
converter (moe_layer_records) writes it, the native reader places every plane
(load_moe_layers with host destinations), and the placed tensors equal the
originals byte for byte -- router, bias, NVFP4 experts with their global
scales, EXL3 experts (trellis, suh, svh), shared expert -- for an all-NVFP4
and a hybrid NVFP4/EXL3 layer.  Layer 78 (the MTP layer) admits any EXL3
shape that is a multiple of 128, so the geometry stays small."""
import numpy as np
import pytest
import torch

import oracle as O
from oracle import rank_file as OR
from glmaxx_b200 import rank_file as R
from glmaxx_b200.moe import Exl3Experts, MoEConfig, PackedNvfp4, RankWeights

LAYER = 78


def small_weights(cfg: MoEConfig, exl3_mask=None, seed=0) -> RankWeights:
    rng = np.random.default_rng(seed)
    E, H, Ir, Isr = cfg.experts, cfg.hidden, cfg.local_intermediate, cfg.local_shared

    def packed(n, k):
        ps = [O.pack((rng.standard_normal((n, k)) * 0.02).astype(np.float32)) for _ in range(E)]
        return PackedNvfp4(torch.from_numpy(np.stack([p.values.reshape(n, k // 2) for p in ps])),
                           torch.from_numpy(np.stack([p.scales for p in ps])),
                           torch.tensor([p.global_scale for p in ps], dtype=torch.float32),
                           torch.tensor([p.global_amax for p in ps], dtype=torch.float32), n, k)

    bf16 = lambda *s: torch.from_numpy(  # noqa: E731
        O.f32_to_bf16_bits((rng.standard_normal(s) * 0.02).astype(np.float32))).view(torch.bfloat16)
    w = RankWeights(bf16(E, H), torch.from_numpy(rng.standard_normal(E).astype(np.float32)),
                    packed(2 * Ir, H), packed(H, Ir), bf16(2 * Isr, H), bf16(H, Isr))
    if exl3_mask is not None:
        words = lambda k, n: torch.from_numpy(  # noqa: E731
            rng.integers(-32768, 32768, (E, (k // 16) * (n // 16) * 48)).astype(np.int16))
        signs = lambda n: torch.from_numpy(  # noqa: E731
            np.where(rng.random((E, n)) < 0.5, -1.0, 1.0).astype(np.float16))
        w.exl3 = Exl3Experts(words(H, Ir), words(H, Ir), words(Ir, H), signs(H), signs(Ir),
                             signs(H), signs(Ir), signs(Ir), signs(H),
                             torch.from_numpy(exl3_mask.astype(np.uint8)))
        for e in np.flatnonzero(exl3_mask):  # EXL3 experts carry no NVFP4 planes
            for p in (w.w13, w.w2):
                p.values[e].zero_()
                p.scales[e].zero_()
                p.global_scale[e] = 1.0
                p.global_amax[e] = 0.0
    return w


def same(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


@pytest.mark.parametrize("hybrid", [False, True])
def test_layer_round_trip_host(tmp_path, hybrid):
    cfg = MoEConfig(hidden=256, experts=4, intermediate=512, shared_intermediate=512, tp=4,
                    rank=2, groups=1, topk_groups=1)
    mask = np.array([0, 1, 0, 1], bool) if hybrid else None
    w = small_weights(cfg, mask)
    records = R.moe_layer_records(w, cfg, LAYER)
    b = R.RankFileBuilder(cfg.rank, b'{"rank":2,"schema":"layer-test"}', tensors=records)
    conv = bytes(range(16))
    b.write(tmp_path / "layer.g5n", conv)
    data = (tmp_path / "layer.g5n").read_bytes()
    OR.Reader(data).verify()  # the oracle accepts what the product wrote
    with R.NativeRankReader.open(tmp_path / "layer.g5n") as rd:
        assert rd.header_flags == (R.FLAG_NVFP4 | R.FLAG_EXL3 | R.FLAG_HYBRID if hybrid else
                                   R.FLAG_NVFP4 | R.FLAG_DIRECT_KERNEL)
        loaded, proof = R.load_moe_layers(rd, cfg, [LAYER], device="cpu")
    lw = loaded[LAYER]
    assert proof.payload_bytes == rd.file_payload_bytes()
    for a, b_ in ((lw.router_weight, w.router_weight), (lw.router_bias, w.router_bias),
                  (lw.shared13, w.shared13), (lw.shared2, w.shared2)):
        assert same(a, b_)
    for p, q in ((lw.w13, w.w13), (lw.w2, w.w2)):
        for f in ("values", "scales", "global_scale", "global_amax"):
            assert same(getattr(p, f), getattr(q, f)), f
    if hybrid:
        assert same(lw.exl3.codec, w.exl3.codec)
        for f in ("gate_trellis", "up_trellis", "down_trellis", "gate_suh", "gate_svh", "up_suh",
                  "up_svh", "down_suh", "down_svh"):
            for e in np.flatnonzero(mask):
                assert same(getattr(lw.exl3, f)[e], getattr(w.exl3, f)[e]), (f, e)
    else:
        assert lw.exl3 is None


def test_layer_selection_errors(tmp_path):
    cfg = MoEConfig(hidden=256, experts=4, intermediate=512, shared_intermediate=512, tp=4,
                    rank=0, groups=1, topk_groups=1)
    w = small_weights(cfg)
    records = R.moe_layer_records(w, cfg, LAYER)
    R.RankFileBuilder(0, b"{}", tensors=records).write(tmp_path / "l.g5n", bytes(16))
    with R.NativeRankReader.open(tmp_path / "l.g5n") as rd:
        with pytest.raises(ValueError):  # the file has no layer 3
            R.load_moe_layers(rd, cfg, [3], device="cpu")
        bigger = MoEConfig(hidden=256, experts=4, intermediate=1024, shared_intermediate=512,
                           tp=4, rank=0, groups=1, topk_groups=1)
        with pytest.raises(ValueError):  # shapes must match the configuration
            R.load_moe_layers(rd, bigger, [LAYER], device="cpu")


def test_rank_set_loads_concurrently(tmp_path):
    """Four TP rank files, validated as a set and loaded on four threads, place
    every rank's tensors as a sequential load does."""
    cfgs = [MoEConfig(hidden=256, experts=4, intermediate=512, shared_intermediate=512, tp=4,
                      rank=r, groups=1, topk_groups=1) for r in range(4)]
    ws = [small_weights(c, seed=r) for r, c in enumerate(cfgs)]
    builders = [R.RankFileBuilder(r, b'{"rank":%d}' % r,
                                  tensors=R.moe_layer_records(ws[r], cfgs[r], LAYER))
                for r in range(4)]
    conv = R.RankFileBuilder.derive_conversion_uuid(builders)
    for b in builders:
        b.write(tmp_path / f"r{b.rank}.g5n", conv)
    paths = [tmp_path / f"r{r}.g5n" for r in range(4)]
    out, proofs = R.load_rank_set(paths, cfgs, [LAYER], ["cpu"] * 4)
    assert [p.rank for p in proofs] == [0, 1, 2, 3]
    for r in range(4):
        lw, w = out[r][LAYER], ws[r]
        for a, b in ((lw.router_weight, w.router_weight), (lw.shared2, w.shared2),
                     (lw.w13.values, w.w13.values), (lw.w2.scales, w.w2.scales),
                     (lw.w13.global_scale, w.w13.global_scale)):
            assert same(a, b)
    with pytest.raises(R.RankFileError) as e:  # ranks out of order
        R.load_rank_set([paths[1], paths[0], paths[2], paths[3]], cfgs, [LAYER], ["cpu"] * 4)
    assert e.value.kind == "RankSet"


def test_bench_load_inputs_and_reference_arm(tmp_path):
    """The load workload's input file (bench.layer_file_builder: router, bias,
    NVFP4 experts, shared expert of one TP4 layer) verifies natively and in the
    oracle, and the reference arm of `bench.py --workload load` (the oracle
    reader) runs on the CPU and prints its JSON line."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    import bench
    path = tmp_path / "layer.g5n"
    size = bench.write_layer_file(path, 4, 2, seed=5)
    assert size == path.stat().st_size
    with R.NativeRankReader.open(path) as rd:
        assert rd.tensor_count() == 2 * 4 + 5 and rd.rank == 2
        rd.verify()
        cfg = MoEConfig(experts=4, tp=4, rank=2, groups=1, topk_groups=1)
        loaded, _ = R.load_moe_layers(rd, cfg, [bench.LOAD_LAYER], device="cpu")
        assert loaded[bench.LOAD_LAYER].w13.values.shape == (4, 1024, 3072)
    OR.Reader(path.read_bytes()).verify()
    root = Path(bench.__file__).resolve().parent
    r = subprocess.run([sys.executable, str(root / "bench.py"), "--workload", "load", "--impl",
                        "reference", "--steps", "1"], capture_output=True, text=True, timeout=600,
                       cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
