"""Peer form of the finish (glmaxx_moe_finish_peer_launch): bit-identical to the
local finish (glmaxx_moe_finish_launch, itself bit-exact with the restated
finish_sparse_layer_oracle, crates/glm-reference/src/routed_fc2.rs:214-258) in
both modes, across epochs and CUDA-graph replays; a wait on a rank that never
arrives ends with the peer-timeout status instead of a hang, and the group
recovers after a signal reset.  The two-GPU cases run as child processes and are
skipped on a one-GPU box."""
import ctypes
import os
import socket
import time

import numpy as np
import pytest
import torch

from glmaxx_b200 import abi
from glmaxx_b200.moe import finish

from gpu_util import cuda

pytestmark = pytest.mark.gpu
PEER_TIMEOUT = 1 << 10


def _bits(t):
    return t.contiguous().view(torch.int32 if t.dtype == torch.float32 else torch.int16).cpu()


def _launch(parts, signals, rank, mode, residual=None, out_f32=None, out_bf16=None, norm=None,
            hidden=0, outs=None, status=None):
    """Raw descriptors: parts/signals are lists of device addresses (rank order)."""
    L = abi.load()
    pa = (ctypes.c_uint64 * len(parts))(*parts)
    sa = (ctypes.c_uint64 * len(signals))(*signals)
    keep = [pa, sa]
    d = abi.MoeFinishDescriptor.new(
        abi_version=1, ranks=len(parts), elements=out_ref_elements(parts, out_f32, out_bf16, norm),
        residual_f32=residual.data_ptr() if residual is not None and residual.dtype == torch.float32
        else 0,
        residual_bf16=residual.data_ptr() if residual is not None and
        residual.dtype == torch.bfloat16 else 0,
        partials_f32=ctypes.addressof(pa),
        output_f32=0 if out_f32 is None else out_f32.data_ptr(),
        output_bf16=0 if out_bf16 is None else out_bf16.data_ptr(),
        norm_bf16=0 if norm is None else norm.data_ptr(), hidden=hidden, eps=1e-6)
    p = abi.MoePeerDescriptor.new(abi_version=1, flags=mode, rank=rank,
                                  signals_u32=ctypes.addressof(sa),
                                  status_u32=0 if status is None else status.data_ptr())
    if mode == abi.PEER_TWO_SHOT:
        for field, arr in (outs or {}).items():
            a = (ctypes.c_uint64 * len(arr))(*arr)
            keep.append(a)
            setattr(p, field, ctypes.addressof(a))
    st = L.glmaxx_moe_finish_peer_launch(ctypes.byref(d), ctypes.byref(p),
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    abi.check(st, "finish_peer")


def out_ref_elements(parts, *outs):
    for o in outs:
        if o is not None:
            return o.numel()
    raise ValueError("no output")


@pytest.mark.parametrize("mode", [abi.PEER_ONE_SHOT, abi.PEER_TWO_SHOT])
@pytest.mark.parametrize("residual_kind", [None, "f32", "bf16"])
@pytest.mark.parametrize("rows", [64, 2048])
def test_single_rank_matches_local_finish(mode, residual_kind, rows):
    dev = cuda()
    H = 6144
    g = torch.Generator(device=dev).manual_seed(rows)
    signals = torch.zeros(64, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    part = torch.empty(rows * H, dtype=torch.float32, device=dev)
    residual = None
    if residual_kind:
        residual = torch.randn(rows * H, generator=g, device=dev)
        residual = residual.to(torch.bfloat16) if residual_kind == "bf16" else residual
    outs = [torch.empty(rows * H, dtype=t, device=dev) for t in (torch.float32, torch.bfloat16,
                                                                 torch.bfloat16)]
    refs = [torch.empty_like(o) for o in outs]
    norm_on = residual is not None
    for epoch in range(1, 4):
        part.copy_(torch.randn(rows * H, generator=g, device=dev) * epoch)
        _launch([part.data_ptr()], [signals.data_ptr()], 0, mode, residual=residual,
                out_f32=outs[0], out_bf16=outs[1], norm=outs[2] if norm_on else None,
                hidden=H if norm_on else 0, status=status,
                outs={"outputs_f32": [outs[0].data_ptr()], "outputs_bf16": [outs[1].data_ptr()],
                      **({"norms_bf16": [outs[2].data_ptr()]} if norm_on else {})})
        if residual is None:
            ref0 = part.clone()  # the sum of one partial onto nothing
            assert torch.equal(_bits(outs[0]), _bits(ref0))
            assert torch.equal(_bits(outs[1]), _bits(ref0.to(torch.bfloat16)))
        else:
            finish([part], residual, out_f32=refs[0], out_bf16=refs[1], norm_bf16=refs[2],
                   hidden=H)
            for o, r in zip(outs, refs):
                assert torch.equal(_bits(o), _bits(r))
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert int(signals[2].item()) == epoch  # the epoch word (ranks = 1)
        assert int(signals[3].item()) == 0 and int(signals[4].item()) == 0


def test_peer_finish_replays_in_a_cuda_graph():
    dev = cuda()
    rows, H = 64, 6144
    signals = torch.zeros(64, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    part = torch.zeros(rows * H, dtype=torch.float32, device=dev)
    residual = torch.randn(rows * H, device=dev).to(torch.bfloat16)
    out = torch.empty(rows * H, dtype=torch.float32, device=dev)
    norm = torch.empty(rows * H, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        _launch([part.data_ptr()], [signals.data_ptr()], 0, abi.PEER_ONE_SHOT, residual=residual,
                out_f32=out, norm=norm, hidden=H, status=status)
    torch.cuda.synchronize()
    ref_out, ref_norm = torch.empty_like(out), torch.empty_like(norm)
    for i in range(4):
        part.copy_(torch.randn(rows * H, device=dev))
        graph.replay()
        finish([part], residual, out_f32=ref_out, norm_bf16=ref_norm, hidden=H)
        torch.cuda.synchronize()
        assert torch.equal(_bits(out), _bits(ref_out)) and torch.equal(_bits(norm), _bits(ref_norm))
    assert int(signals[2].item()) == 4 and int(status.item()) == 0


def test_wait_on_absent_rank_times_out_with_status():
    """A flag that nothing sets: rank 1 of a two-rank group never launches (its
    signal buffer and partial are local stand-ins that no kernel writes), so
    both of rank 0's bounded waits run out; the kernel reports it and returns."""
    dev = cuda()
    n = 4096
    sig0 = torch.zeros(64, dtype=torch.int32, device=dev)
    sig1 = torch.zeros(64, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    parts = [torch.ones(n, device=dev), torch.ones(n, device=dev)]
    out = torch.full((n,), -7.0, device=dev)
    torch.cuda.synchronize()
    t0 = time.time()
    _launch([p.data_ptr() for p in parts], [sig0.data_ptr(), sig1.data_ptr()], 0,
            abi.PEER_ONE_SHOT, out_f32=out, status=status)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(status.item()) & PEER_TIMEOUT
    assert 1.0 <= dt < 30.0
    assert torch.all(out == -7.0)  # nothing summed without every rank
    # the context is healthy: a one-rank launch on fresh signals works
    sig = torch.zeros(64, dtype=torch.int32, device=dev)
    status.zero_()
    _launch([parts[0].data_ptr()], [sig.data_ptr()], 0, abi.PEER_ONE_SHOT, out_f32=out,
            status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and torch.all(out == 1.0)


# ------------------------------------------------------------------ two GPUs
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, q):
    import torch.distributed as dist

    from glmaxx_b200.peer import PeerGroup

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    res = {}
    try:
        rows, H = 96, 6144
        n = rows * H
        bufs = {"partial": ((n,), torch.float32), "out": ((n,), torch.float32),
                "next": ((n,), torch.bfloat16), "norm": ((n,), torch.bfloat16)}
        g = PeerGroup(bufs, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        residual = torch.randn(n, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
        residual = residual.to(dev)
        mismatches = []
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            for epoch in range(6):
                gen = torch.Generator().manual_seed(100 * epoch + rank)
                mine = torch.randn(n, generator=gen)
                g.tensor("partial").copy_(mine.to(dev))
                everyone = [None] * world
                dist.all_gather_object(everyone, mine)
                mode = ("one", "two")[epoch % 2]
                norm_on = epoch >= 2
                g.finish("partial", residual=residual, out_f32="out", out_bf16="next",
                         norm_bf16="norm" if norm_on else None, hidden=H if norm_on else 0,
                         mode=mode, status=status)
                parts = [p.to(dev) for p in everyone]
                ro, rb, rn = (torch.empty(n, dtype=t, device=dev)
                              for t in (torch.float32, torch.bfloat16, torch.bfloat16))
                finish(parts, residual, out_f32=ro, out_bf16=rb,
                       norm_bf16=rn if norm_on else None, hidden=H if norm_on else 0)
                stream.synchronize()
                for name, ref in (("out", ro), ("next", rb)) + ((("norm", rn),) if norm_on else ()):
                    if not torch.equal(_bits(g.tensor(name)), _bits(ref)):
                        mismatches.append((epoch, mode, name))
            res["mismatches"] = mismatches
            res["status"] = int(status.item())
            # a rank that never arrives: rank 1 skips one launch; rank 0 times out
            dist.barrier()
            if rank == 0:
                g.finish("partial", out_f32="out", mode="one", status=status)
                stream.synchronize()
            res["timeout_status"] = int(status.item())
            g.reset_signals()
            status.zero_()
            g.tensor("partial").fill_(float(rank + 1))
            stream.synchronize()
            g.finish("partial", out_f32="out", mode="two", status=status)
            stream.synchronize()
            res["recovered"] = bool(torch.all(g.tensor("out") == 3.0).item())
            res["recovered_status"] = int(status.item())
        g.close()
    except Exception as e:  # noqa: BLE001
        res["error"] = repr(e)
    finally:
        q.put((rank, res))
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_gpus_peer_finish_bit_identical_and_recovers():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        res = results[r]
        assert "error" not in res, res
        assert res["mismatches"] == [], res
        assert res["status"] == 0
        assert res["recovered"] and res["recovered_status"] == 0
    assert results[0]["timeout_status"] & PEER_TIMEOUT
    assert results[1]["timeout_status"] == 0
