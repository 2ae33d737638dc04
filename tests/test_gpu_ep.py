"""Expert parallelism (glmaxx_b200/ep.py: glmaxx_moe_ep_dispatch_launch, the
owner layer over received rows, glmaxx_moe_ep_return_launch, the
GLMAXX_MOE_EXTERNAL_ROUTED combine) against the TP1 layer on the same tokens.

Every expert row is the TP1 layer's row and the combine is the same kernel, so on
the deterministic decode path every rank's output equals the TP1 layer's output
on that rank's tokens bit for bit.  The ranks are emulated on one GPU (their
buffers local, the same kernels as across GPUs, where the buffers are peer
mappings)."""
import pytest
import torch

from glmaxx_b200 import abi, ep, synth
from glmaxx_b200.moe import MoEConfig, RoutedMoE

from gpu_util import assert_layer_close, cuda

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ranks,tokens", [(2, 24), (4, 24), (4, 300)])
def test_gpu_ep_equals_tp1_layer(ranks, tokens):
    cfg = MoEConfig(experts=64)  # 8 groups / top-4 groups, top-8, shared expert
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=13, device=dev)
    xs = [synth.make_input(tokens, cfg.hidden, seed=100 + r, device=dev) for r in range(ranks)]
    group = ep.make_local_group(cfg, w, ranks, tokens, dev)
    outs = [o.clone() for o in group.step(xs, path=abi.DECODE_PERSISTENT)]
    torch.cuda.synchronize()
    for r in group.ranks:
        assert r.device_status() == []
    # every owner received exactly the assignments routed to its experts
    assert sum(r.rows for r in group.ranks) == ranks * tokens * cfg.top_k
    ref_layer = RoutedMoE(cfg, w, tokens)
    for r, x in enumerate(xs):
        ref = ref_layer(x, path=abi.DECODE_PERSISTENT).clone()
        torch.cuda.synchronize()
        assert torch.equal(outs[r], ref), f"rank {r}"
        # routes are the TP1 router's (replicated router)
        assert torch.equal(group.ranks[r].route_experts[:tokens], ref_layer.route_experts[:tokens])


def test_gpu_ep_prefill_sizes_within_layer_tolerance():
    """Token counts on the prefill path: the TP1 layer adds its slot contributions
    with atomics there, so the two agree to the layer tolerance."""
    cfg = MoEConfig(experts=64)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=14, device=dev)
    ranks, tokens = 2, 512
    xs = [synth.make_input(tokens, cfg.hidden, seed=200 + r, device=dev) for r in range(ranks)]
    group = ep.make_local_group(cfg, w, ranks, tokens, dev)
    outs = [o.clone() for o in group.step(xs)]
    ref_layer = RoutedMoE(cfg, w, tokens)
    for r, x in enumerate(xs):
        ref = ref_layer(x).clone()
        torch.cuda.synchronize()
        assert_layer_close(outs[r].cpu().numpy(), ref.cpu().numpy(), f"ep prefill rank {r}")
