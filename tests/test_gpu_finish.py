"""Sparse-layer finish (glmaxx_moe_finish_launch) against the restated
finish_sparse_layer_oracle (crates/glm-reference/src/routed_fc2.rs:214-258):
bit-exact fp32, and bf16 output = round-to-nearest-even of it."""
import numpy as np
import pytest
import torch

import oracle as O
from glmaxx_b200.moe import finish

from gpu_util import cuda

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ranks", [1, 4, 8])
def test_finish_rank_order_bit_exact(ranks):
    rng = np.random.default_rng(ranks)
    n = 4096 * 3
    residual = rng.standard_normal(n).astype(np.float32)
    attention = rng.standard_normal((ranks, n)).astype(np.float32)
    routed = (rng.standard_normal((ranks, n)) * 1e-3).astype(np.float32)
    ref = O.finish_sparse_layer(residual, attention, routed, None)
    dev = cuda()
    parts = [torch.from_numpy(routed[r].copy()).to(dev) for r in range(ranks)]
    res = torch.from_numpy(residual).to(dev)
    att = torch.from_numpy(attention).to(dev)
    out = torch.empty(n, dtype=torch.float32, device=dev)
    outb = torch.empty(n, dtype=torch.bfloat16, device=dev)
    finish(parts, res, attention=att, out_f32=out, out_bf16=outb)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.array_equal(got, ref)
    assert np.array_equal(outb.view(torch.int16).cpu().numpy().view(np.uint16),
                          O.f32_to_bf16_bits(ref))


def test_finish_bf16_residual():
    rng = np.random.default_rng(0)
    n = 1024
    res_bits = O.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32))
    routed = rng.standard_normal((2, n)).astype(np.float32)
    ref = O.finish_sparse_layer(O.bf16_bits_to_f32(res_bits), None, routed, None)
    dev = cuda()
    res = torch.from_numpy(res_bits.view(np.int16)).to(dev).view(torch.bfloat16)
    out = torch.empty(n, dtype=torch.float32, device=dev)
    finish([torch.from_numpy(routed[r].copy()).to(dev) for r in range(2)], res, out_f32=out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref)


def test_finish_rmsnorm_output():
    """Optional next-layer input: bf16(o / sqrt(mean(o^2) + eps)) per row of the
    fp32 finish result o, within one bf16 ulp of a float64 evaluation."""
    rng = np.random.default_rng(5)
    rows, hidden = 6, 6144
    residual = rng.standard_normal(rows * hidden).astype(np.float32)
    routed = (rng.standard_normal((2, rows * hidden)) * 3).astype(np.float32)
    ref_sum = O.finish_sparse_layer(residual, None, routed, None).reshape(rows, hidden)
    o64 = ref_sum.astype(np.float64)
    norm = o64 / np.sqrt((o64 * o64).mean(axis=1, keepdims=True) + 1e-6)
    dev = cuda()
    out = torch.empty(rows * hidden, dtype=torch.float32, device=dev)
    nb = torch.empty(rows * hidden, dtype=torch.bfloat16, device=dev)
    finish([torch.from_numpy(routed[r].copy()).to(dev) for r in range(2)],
           torch.from_numpy(residual).to(dev), out_f32=out, norm_bf16=nb, hidden=hidden)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().reshape(rows, hidden), ref_sum)
    got = nb.float().cpu().numpy().reshape(rows, hidden)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(norm), 1e-30))) - 7)
    assert np.all(np.abs(got - norm) <= ulp)
