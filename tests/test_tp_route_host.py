"""Host logic of token-split routing (glmaxx_b200/tp_route.py), no GPU: the split
rule, the slice bounds, and the exchange -- each rank packs its slice's routes,
the group all-gathers them over a world-size-2 gloo group and unpacks them into
dense [T, top_k] routes.  The slice router here is the CPU oracle's router, so
the test also checks the property the split rests on: routing a token slice
gives the same routes, bit for bit, as routing all tokens and taking the slice."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from glmaxx_b200 import tp_route
from glmaxx_b200.moe import MoEConfig, RankWeights

T, H, E, K, GROUPS, TOPK_GROUPS = 64, 256, 32, 4, 4, 2


def _inputs():
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((T, H), dtype=np.float32)).astype(np.float32)
    w = (rng.standard_normal((E, H), dtype=np.float32) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(E, dtype=np.float32) * 0.01).astype(np.float32)
    import oracle as O
    return O.f32_to_bf16_bits(x), O.f32_to_bf16_bits(w), bias


def test_split_rule_and_bounds():
    assert not tp_route.split_pays(64, 8)          # decode: 8 tokens per rank
    assert tp_route.split_pays(8192, 8)            # prefill: 1024 per rank
    assert tp_route.split_pays(2048, 8)            # 256 per rank, the threshold
    assert not tp_route.split_pays(2048, 16)
    assert not tp_route.split_pays(8192, 1)
    assert not tp_route.split_pays(8200, 8)        # uneven
    assert not tp_route.split_pays(2056, 8, 8)     # 257 per rank: not a multiple of 8
    assert [tp_route.slice_bounds(8192, 4, r) for r in range(4)] == \
        [(0, 2048), (2048, 4096), (4096, 6144), (6144, 8192)]
    with pytest.raises(ValueError):
        tp_route.slice_bounds(10, 4, 0)


def test_unpack_routes_layout():
    ranks, s, k = 3, 8, 4
    ex = torch.arange(ranks * s * k, dtype=torch.int16).view(ranks * s, k)
    wt = torch.arange(ranks * s * k, dtype=torch.float32).view(ranks * s, k) * 0.5
    blocks = []
    for r in range(ranks):
        blocks.append(torch.cat([ex[r * s:(r + 1) * s].reshape(-1).view(torch.uint8),
                                 wt[r * s:(r + 1) * s].reshape(-1).view(torch.uint8)]))
    gathered = torch.cat(blocks)
    e_out = torch.zeros_like(ex)
    w_out = torch.zeros_like(wt)
    tp_route.unpack_routes(gathered, ranks, e_out, w_out)
    assert torch.equal(e_out, ex) and torch.equal(w_out, wt)


class _OracleSliceRouter(tp_route.SplitRouter):
    """SplitRouter whose slice router is the CPU oracle (the GPU router runs in
    the -m gpu tests); everything after route_slice is the class's own code."""

    def route_slice(self, x):
        import oracle as O
        xb = x.view(torch.int16).numpy().view(np.uint16)[self.lo:self.hi]
        ex, wt = O.router(xb, self._w_bits, self._bias, GROUPS, TOPK_GROUPS, K, 2.5)
        n = self.slice_tokens * K
        self.packed[:2 * n].copy_(torch.from_numpy(ex.astype(np.int16).reshape(-1)).view(torch.uint8))
        self.packed[2 * n:].copy_(torch.from_numpy(wt.reshape(-1).copy()).view(torch.uint8))


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        xb, wb, bias = _inputs()
        cfg = MoEConfig(hidden=H, experts=E, intermediate=256, top_k=K, groups=GROUPS,
                        topk_groups=TOPK_GROUPS, shared_intermediate=0)
        weights = RankWeights(torch.from_numpy(wb.view(np.int16)).view(torch.bfloat16),
                              torch.from_numpy(bias), None, None)
        r = _OracleSliceRouter(cfg, weights, T, rank, world, torch.device("cpu"))
        r._w_bits, r._bias = wb, bias
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
        ex, wt = r(x)
        q.put((rank, ex.numpy().copy(), wt.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_split_routes_all_gather_two_ranks():
    import oracle as O
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + (os.getpid() + 500) % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        rank, ex, wt = q.get(timeout=180)
        got[rank] = (ex, wt)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    xb, wb, bias = _inputs()
    ref_e, ref_w = O.router(xb, wb, bias, GROUPS, TOPK_GROUPS, K, 2.5)
    for rank in range(2):
        ex, wt = got[rank]
        assert np.array_equal(ex.astype(np.uint16), ref_e)
        assert np.array_equal(wt.view(np.uint32), ref_w.view(np.uint32))
