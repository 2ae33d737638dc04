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
