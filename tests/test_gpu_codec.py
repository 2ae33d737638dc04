"""The hardware NVFP4 conversions the quantisation kernels use
(cvt.rn.satfinite.e2m1x2 / e4m3x2) give the reference codec's codes
(crates/glm-format/src/float.rs:15-73: nearest, ties to the even code,
saturating) for every fp32 input: an exhaustive on-GPU comparison with the
library's restatement of the codec, through the C ABI."""
import ctypes

import pytest
import torch

from glmaxx_b200 import abi

pytestmark = pytest.mark.gpu


def test_hardware_codec_matches_reference_codec_for_every_float():
    dev = torch.device("cuda:0")
    out = torch.zeros(4, dtype=torch.int64, device=dev)
    L = abi.load()
    abi.check(L.glmaxx_nvfp4_codec_selfcheck_launch(
        ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "codec selfcheck")
    torch.cuda.synchronize()
    bad_e2m1, bad_e4m3, first2, first3 = (int(v) for v in out.cpu())
    assert bad_e2m1 == 0, f"E2M1: {bad_e2m1} mismatches, e.g. bits {first2 - 1:#010x}"
    assert bad_e4m3 == 0, f"E4M3: {bad_e4m3} mismatches, e.g. bits {first3 - 1:#010x}"
