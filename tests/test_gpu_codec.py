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


def test_quotient_codes_match_exact_division_for_every_float():
    """The quantisation kernels' E2M1 code of v / dec (a reciprocal product,
    bracketed by +-2^-20 relative; the exact quotient where an E2M1 midpoint lies
    inside the bracket) equals the code of the exactly rounded quotient for every
    finite fp32 v, over divisors decode(scale) * global as the kernels form them:
    E4M3 scale codes across the range times global scales of several magnitudes,
    plus divisors at and past the fast path's limits."""
    import numpy as np

    import oracle as O
    codes = [1, 7, 8, 0x21, 0x30, 0x38, 0x3b, 0x3d, 0x44, 0x55, 0x66, 0x7e]
    globals_ = np.array([1.0, 3.7193e-3, 1.0 / 2688.0, 0.1234567, 41.25, 7.7e-30], np.float32)
    decs = [np.float32(O.decode_e4m3(c)) * g for c in codes for g in globals_]
    decs += [np.float32(2.0 ** -122), np.float32(2.0 ** 122), np.float32(1e-40),
             np.float32(3e38)]
    d = torch.tensor(np.array(decs, np.float32), device="cuda:0")
    out = torch.zeros(4, dtype=torch.int64, device="cuda:0")
    L = abi.load()
    abi.check(L.glmaxx_nvfp4_quotient_selfcheck_launch(
        ctypes.c_void_p(d.data_ptr()), len(decs), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "quotient selfcheck")
    torch.cuda.synchronize()
    bad, first, fast, checked = (int(v) for v in out.cpu())
    assert checked == len(decs) * ((1 << 32) - (1 << 24))  # every finite bit pattern
    assert bad == 0, (f"{bad} mismatches, e.g. divisor {decs[(first - 1) >> 32]!r}, "
                      f"v bits {(first - 1) & 0xffffffff:#010x}")
    assert fast > checked // 2  # most values are decided on the bracket
