"""The C++ host runtime (include/glmaxx_host.hpp) through its test program
tests/host/host_test.cpp: device-free checks (ABI string, the reference
workspace formulas, row buckets, topology and error rules), and on a GPU one
rank's routed-MoE step through RoutedMoeStep and BucketedMoeGraphs -- routes
bit-exact with the restated router, the layer output within 4 bf16 ulp of the
output scale of the oracle's sequential-fp32 layer, and the bucket graph's rows
bit-identical to eager launches (checked inside the program)."""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from glmaxx_b200 import abi

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "host" / "host_test.cpp"
OUT = ROOT / "tests" / "host" / "_build"


@pytest.fixture(scope="module")
def host_test():
    abi.load()  # builds the library if it is missing
    OUT.mkdir(parents=True, exist_ok=True)
    exe = OUT / "host_test"
    lib_dir = abi.LIB_PATH.parent
    cxx = shutil.which("g++") or "/usr/bin/g++"
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
           str(SRC), f"-L{lib_dir}", "-lglmaxx_sm100", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_host_runtime_device_free_checks(host_test):
    r = subprocess.run([str(host_test), "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout


@pytest.mark.gpu
def test_host_runtime_step_matches_oracle(host_test, tmp_path):
    r = subprocess.run([str(host_test), "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    T, H, E, I, Is, K = 40, 6144, 16, 512, 256, 8
    rd = lambda n, dt: np.fromfile(tmp_path / f"{n}.bin", dtype=dt)  # noqa: E731
    x = rd("x", np.uint16).reshape(T, H)
    router = rd("router", np.uint16).reshape(E, H)
    bias = rd("bias", np.float32)
    ref_e, ref_w = O.router(x, router, bias, 1, 1, K, 2.5)
    got_e = rd("route_experts", np.uint16).reshape(T, K)
    got_w = rd("route_weights", np.float32).reshape(T, K)
    assert np.array_equal(got_e, ref_e)
    assert np.array_equal(got_w.view(np.uint32), ref_w.view(np.uint32))
    routed, shared = O.moe_layer(
        x, ref_e, ref_w, rd("w13v", np.uint8).reshape(E, 2 * I, H // 2),
        rd("w13s", np.uint8), rd("g13", np.float32), rd("w2v", np.uint8).reshape(E, H, I // 2),
        rd("w2s", np.uint8), rd("g2", np.float32), I, rd("sh13", np.uint16).reshape(2 * Is, H),
        rd("sh2", np.uint16).reshape(H, Is))
    ref = routed + shared
    got = rd("out", np.float32).reshape(T, H)
    assert np.isfinite(got).all()
    ulp = 2.0 ** (np.floor(np.log2(np.abs(ref).max())) - 7)
    err = float(np.abs(got - ref).max())
    assert err <= 4 * ulp, (err, ulp)


def test_host_runtime_rank_files(host_test, tmp_path):
    """NativeRankFile over four product-written rank files (the reader test
    fixture of native_reader.rs:1189-1268), device-free."""
    from glmaxx_b200 import rank_file as R
    from tests.test_rank_file import family, to_product
    fam = family("reader")
    builders = [to_product(r, m, s, ident) for r, m, s, ident in fam]
    conv = R.RankFileBuilder.derive_conversion_uuid(builders)
    for b in builders:
        b.write(tmp_path / f"rank{b.rank}.g5n", conv)
    (tmp_path / "truncated.g5n").write_bytes((tmp_path / "rank0.g5n").read_bytes()[:4000])
    r = subprocess.run([str(host_test), "rankfile", str(tmp_path)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("hybrid", [False, True])
def test_host_runtime_layer_from_rank_file(host_test, tmp_path, hybrid):
    """RankLayerWeights::load + RoutedMoeStep on a written layer file (NVFP4, or
    half the experts EXL3) give the same output as the layer run on the
    generated weights, on the same input."""
    import torch

    from glmaxx_b200 import rank_file as R
    from glmaxx_b200 import synth
    from glmaxx_b200.moe import MoEConfig, RoutedMoE
    from tests.gpu_util import assert_layer_close
    cfg = MoEConfig(experts=16, groups=1, topk_groups=1, tp=4, rank=0)
    if hybrid:
        mask = torch.zeros(cfg.experts, dtype=torch.bool)
        mask[::2] = True
        w = synth.make_exl3_rank_weights(cfg, seed=31, device="cuda", nvfp4_experts=mask)
    else:
        w = synth.make_rank_weights(cfg, seed=31, device="cuda")
    path = tmp_path / "layer.g5n"
    R.RankFileBuilder(0, b"{}", tensors=R.moe_layer_records(w, cfg, 3)).write(path, bytes(16))
    r = subprocess.run([str(host_test), "rankgpu", str(path), str(tmp_path)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    T, H = 40, cfg.hidden
    x = torch.from_numpy(np.fromfile(tmp_path / "x.bin", dtype=np.uint16).astype(np.int16)
                         ).view(torch.bfloat16).reshape(T, H).cuda()
    got = np.fromfile(tmp_path / "out.bin", dtype=np.float32).reshape(T, H)
    ref = RoutedMoE(cfg, w, T)(x).cpu().numpy()
    assert ("exl3/hybrid" if hybrid else "nvfp4") in r.stdout
    assert_layer_close(got, ref, "C++ rank-file layer")
