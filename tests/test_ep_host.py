"""Host logic of the expert-parallel step (glmaxx_b200/ep.py), no GPU: the per-owner
row counts from a source's expert offsets, every source's first row in every
owner's receive buffers, the rows each owner receives, and the all-gather of the
count matrix over a world-size-2 gloo group."""
import os

import numpy as np
import torch.multiprocessing as mp

from glmaxx_b200 import ep


def test_owner_counts_and_offsets():
    # 8 experts over 4 owners (2 each); a source with 3, 0, 2, 1, 0, 0, 4, 1 rows per expert
    per_expert = np.array([3, 0, 2, 1, 0, 0, 4, 1])
    offsets = np.concatenate([[0], np.cumsum(per_expert)])
    assert ep.owner_counts(offsets, 4).tolist() == [3, 3, 0, 5]
    counts = np.array([[3, 3, 0, 5], [1, 0, 2, 2], [0, 4, 4, 0], [2, 2, 2, 2]])
    assert ep.dest_row_offsets(counts, 0).tolist() == [0, 0, 0, 0]
    assert ep.dest_row_offsets(counts, 2).tolist() == [4, 3, 2, 7]
    assert ep.dest_row_offsets(counts, 3).tolist() == [4, 7, 6, 7]
    assert [ep.received_rows(counts, d) for d in range(4)] == [6, 9, 8, 9]
    # a source's block ends where the next source's begins, and the last fills the total
    for d in range(4):
        for s in range(3):
            assert ep.dest_row_offsets(counts, s)[d] + counts[s][d] == ep.dest_row_offsets(counts, s + 1)[d]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = ep.exchange_counts(np.array([rank * 10 + d for d in range(world)], np.int64))
        q.put((rank, m.tolist()))
    finally:
        dist.destroy_process_group()


def test_count_matrix_all_gather_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1] == [[0, 1], [10, 11]]
