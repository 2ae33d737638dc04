"""Token-split routing on the GPU (glmaxx_b200/tp_route.py), ranks emulated on one
device: each rank's slice is routed through glmaxx_router_compact_launch, the
packed slices are concatenated as the all-gather would, and the unpacked routes
must equal, bit for bit, the routes of one router call over all T tokens and the
CPU oracle's routes on a token sample.  Covers the small-T router kernel
(slices under 256 tokens) and the large-T one, at the GLM-5.2 router shape."""
import numpy as np
import pytest
import torch

import oracle as O
from glmaxx_b200 import tp_route
from glmaxx_b200.moe import MoEConfig, RankWeights

from gpu_util import cuda, to_np_bf16_bits

pytestmark = pytest.mark.gpu


def _weights(cfg, seed, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    w = (torch.randn(cfg.experts, cfg.hidden, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    # a skewed bias, so that some experts take many more tokens than others
    b = (torch.randn(cfg.experts, generator=g) * 0.01
         + 0.05 * torch.linspace(1.0, 0.0, cfg.experts) ** 4).to(dev)
    return RankWeights(w, b, None, None)


def _emulated_split(cfg, weights, x, ranks):
    T = x.shape[0]
    dev = x.device
    routers = [tp_route.SplitRouter(cfg, weights, T, r, ranks, dev) for r in range(ranks)]
    for r in routers:
        r.route_slice(x)
    gathered = torch.cat([r.packed for r in routers])
    e = torch.empty((T, cfg.top_k), dtype=torch.int16, device=dev)
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device=dev)
    tp_route.unpack_routes(gathered, ranks, e, w)
    torch.cuda.synchronize()
    for r in routers:
        assert r.device_status() == []
    return e, w


@pytest.mark.parametrize("T,ranks", [(64, 2), (64, 8), (2048, 8), (8192, 8), (8192, 2)])
def test_split_routes_equal_full_router(T, ranks):
    dev = cuda()
    cfg = MoEConfig()
    weights = _weights(cfg, 5 + T + ranks, dev)
    g = torch.Generator(device="cpu").manual_seed(T * 31 + ranks)
    x = torch.randn(T, cfg.hidden, generator=g).to(torch.bfloat16).to(dev)
    e_split, w_split = _emulated_split(cfg, weights, x, ranks)
    e_full, w_full = _emulated_split(cfg, weights, x, 1)   # one router call over all T
    assert torch.equal(e_split, e_full)
    assert torch.equal(w_split.view(torch.int32), w_full.view(torch.int32))
    # the oracle on a token sample spanning every slice
    rng = np.random.default_rng(T + ranks)
    sample = np.unique(np.concatenate([rng.choice(T, min(T, 48), replace=False),
                                       np.arange(ranks) * (T // ranks)]))
    xb = to_np_bf16_bits(x)[sample]
    ref_e, ref_w = O.router(xb, to_np_bf16_bits(weights.router_weight),
                            weights.router_bias.cpu().numpy(), cfg.groups, cfg.topk_groups,
                            cfg.top_k, cfg.route_scale)
    got_e = e_split.cpu().numpy().view(np.uint16)[sample]
    got_w = w_split.cpu().numpy()[sample]
    assert np.array_equal(got_e, ref_e)
    assert np.array_equal(got_w.view(np.uint32), ref_w.view(np.uint32))
