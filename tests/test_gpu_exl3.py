"""EXL3 3-bit trellis path on the GPU against the reference definition.

* The decode-fused projection (glmaxx_exl3_gemv_launch) reproduces the
  reference's warp-staging proof bit for bit: its f16 projection SHA-256 of the
  8 seeded activation rows against the seeded gate-up (K 6144, N 512) and down
  (K 512, N 6144) trellises (fixtures/exl3-warp-staging-proof-v2.json:44-75).
* The full reference-ABI projection (glmaxx_exl3_projection_launch: suh, H128,
  projection, H128, svh) equals Exl3Trellis::matmul_reference_f16
  (crates/glm-format/src/exl3.rs:404-453, restated in oracle/) bit for bit.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from glmaxx_b200 import abi
from exl3_util import f16_bits, warp_activations
from gpu_util import cuda

pytestmark = pytest.mark.gpu


def _dev_u16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(cuda())


def _stream():
    s = torch.cuda.Stream()
    torch.cuda.current_stream().synchronize()
    return s


@pytest.mark.parametrize("index", [0, 1])
def test_exl3_gemv_reproduces_warp_proof(golden, index):
    g = golden["exl3_warp_proof"]["shapes"][index]
    rows, k, n = golden["exl3_warp_proof"]["rows"], g["k"], g["n"]
    tr = O.exl3_xorshift_trellis(g["seed"], O.exl3_trellis_words(k, n, 3))
    x = _dev_u16(f16_bits(warp_activations(rows, k)))
    t = _dev_u16(tr)
    out = torch.empty((rows, n), dtype=torch.int16, device=cuda())
    s = _stream()
    rc = abi.load().glmaxx_exl3_gemv_launch(x.data_ptr(), t.data_ptr(), rows, k, n, 3,
                                            out.data_ptr(), ctypes.c_void_p(s.cuda_stream))
    assert rc == 0
    s.synchronize()
    assert O.u16_hash(out.cpu().numpy().view(np.uint16)) == g["projection_f16_sha256"]


@pytest.mark.parametrize("k,n,rows", [(6144, 512, 5), (512, 6144, 3), (2048, 256, 17)])
def test_exl3_projection_abi_matches_reference(k, n, rows):
    rng = np.random.default_rng(k + n + rows)
    tr = O.exl3_xorshift_trellis(0x5EED0000 + k + n, O.exl3_trellis_words(k, n, 3))
    x = f16_bits(rng.standard_normal((rows, k)).astype(np.float32))
    suh = f16_bits(np.where(rng.random(k) < 0.5, -1.0, 1.0).astype(np.float32) * 0.75)
    svh = f16_bits(np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float32) * 0.0625)
    ref = O.exl3_matmul_reference(tr, k, n, suh, svh, x)
    dx, dt, dsuh, dsvh = _dev_u16(x), _dev_u16(tr), _dev_u16(suh), _dev_u16(svh)
    ws_bytes = abi.load().glmaxx_exl3_projection_workspace_bytes(rows, k, n)
    ws = torch.zeros(ws_bytes // 2 + 8, dtype=torch.int16, device=cuda())
    out = torch.empty((rows, n), dtype=torch.int16, device=cuda())
    err = torch.zeros(1, dtype=torch.int32, device=cuda())
    d = abi.Exl3Descriptor.new(
        abi_version=abi.EXL3_ABI_VERSION, projection=1, rows=rows, logical_k=k, logical_n=n,
        bits=3, input_f16=dx.data_ptr(), trellis_u16=dt.data_ptr(), suh_f16=dsuh.data_ptr(),
        svh_f16=dsvh.data_ptr(), rotated_input_f16=ws.data_ptr(),
        projected_f16=ws.data_ptr() + rows * k * 2, output_f16=out.data_ptr(),
        validation_error_u32=err.data_ptr(), workspace_bytes=ws_bytes)
    s = _stream()
    aerr = ctypes.c_int32(0)
    rc = abi.load().glmaxx_exl3_projection_launch(ctypes.byref(d), ctypes.c_void_p(s.cuda_stream),
                                                  ctypes.byref(aerr))
    assert rc == 0 and aerr.value == 0
    s.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    assert int(err.item()) == 0
    mism = int((got != ref).sum())
    assert mism == 0, f"{mism} of {got.size} outputs differ from matmul_reference_f16"
