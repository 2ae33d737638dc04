"""Per-row-bucket CUDA graphs (glmaxx_b200.graphs.BucketedMoE): replays padded to
the bucket give the real rows of an unpadded launch -- bit for bit on the
deterministic decode path, to the layer tolerance on the prefill path -- and a
smaller batch after a larger one in the same bucket sees zeroed padding."""
import pytest
import torch

from glmaxx_b200 import synth
from glmaxx_b200.graphs import BucketedMoE
from glmaxx_b200.moe import MoEConfig, RoutedMoE

from gpu_util import assert_layer_close, cuda

pytestmark = pytest.mark.gpu


def test_bucketed_decode_and_prefill_rows():
    cfg = MoEConfig(tp=8, rank=3)
    dev = cuda()
    w = synth.make_rank_weights(cfg, seed=31, device=dev)
    layer = RoutedMoE(cfg, w, 512)
    ref_layer = RoutedMoE(cfg, w, 512)
    b = BucketedMoE(layer, buckets=(4, 64, 128, 512))
    for t in (3, 50, 100, 33):
        x = synth.make_input(t, cfg.hidden, seed=100 + t, device=dev)
        got = b(x).clone()
        ref = ref_layer(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(got, ref), t
    assert sorted(b.graphs) == [4, 64, 128]
    x = synth.make_input(300, cfg.hidden, seed=7, device=dev)
    got = b(x).clone()
    ref = ref_layer(x).clone()
    torch.cuda.synchronize()
    assert_layer_close(got.cpu().numpy(), ref.cpu().numpy(), "bucket 512 (prefill path)")
    assert layer.device_status() == []
