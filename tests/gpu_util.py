"""Shared helpers of the -m gpu parity tests (tolerances stated here)."""
import numpy as np
import torch

# Layer output tolerance: rel-L2 <= 1e-3 against the
# fp32-accumulated CPU oracle, and max-abs <= 4 bf16 ulp of the output scale
# (output scale = max |oracle|; one bf16 ulp of s = 2^(floor(log2 s) - 7)).
REL_L2 = 1e-3
MAX_ABS_ULPS = 4


def bf16_ulp(scale: float) -> float:
    return 2.0 ** (np.floor(np.log2(scale)) - 7)


def rel_l2(got: np.ndarray, ref: np.ndarray) -> float:
    return float(np.linalg.norm((got - ref).ravel()) / max(np.linalg.norm(ref.ravel()), 1e-30))


def assert_layer_close(got: np.ndarray, ref: np.ndarray, what: str = "layer"):
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    r = rel_l2(got, ref)
    scale = float(np.abs(ref).max())
    tol = MAX_ABS_ULPS * bf16_ulp(scale)
    err = float(np.abs(got - ref).max())
    assert r <= REL_L2, f"{what}: rel-L2 {r:.3e} > {REL_L2}"
    assert err <= tol, f"{what}: max-abs {err:.3e} > {MAX_ABS_ULPS} bf16 ulp of {scale:.3e} ({tol:.3e})"
    return r, err


def cuda():
    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    return torch.device("cuda:0")


def to_np_bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
