"""EXL3 fixtures shared by the oracle golden tests and the GPU tests."""
import numpy as np

import oracle as O


def warp_activations(rows: int, k: int) -> np.ndarray:
    """Activations of the reference's warp-staging proof (warp_proof.rs:364-376),
    fp32 values that are exactly fp16-representable."""
    out = np.zeros((rows, k), np.float32)
    for r in range(rows):
        ints = ((r * 1009 + np.arange(k) * 7919 + 17) % 1021).astype(np.int64) - 510
        vals = (ints.astype(np.float32) / np.float32(4096.0))
        out[r] = [O.f16_bits_to_f32(O.f32_to_f16_bits(float(v))) for v in vals]
    return out


def f16_bits(values: np.ndarray) -> np.ndarray:
    flat = [O.f32_to_f16_bits(float(v)) for v in np.asarray(values, np.float32).ravel()]
    return np.array(flat, np.uint16).reshape(np.shape(values))
