"""Measurement harness, not library API: reduce-alone timing of the peer finish
against NCCL, one process per GPU.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \\
        --master-addr 127.0.0.1 --master-port 29541 -m glmaxx_b200.peer_bench [--tokens 64,2048]

For each token count T (hidden 6144) every rank maps a PeerGroup of an fp32
partial, an fp32 output and bf16 outputs, and times -- CUDA-graph replays of 20
launches, max over ranks -- the peer finish in one-shot and two-shot form (plain
all-reduce into fp32; and with a bf16 residual, bf16 output and RMSNorm output),
and an NCCL all-reduce of the same fp32 buffer.  Rank 0 prints one JSON line of
microseconds per launch.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from .peer import PeerGroup

HIDDEN = 6144


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", default="64,2048")
    p.add_argument("--launches", type=int, default=20)
    p.add_argument("--replays", type=int, default=20)
    a = p.parse_args()
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    res = {"world": world}
    for T in [int(t) for t in a.tokens.split(",")]:
        n = T * HIDDEN
        g = PeerGroup({"partial": ((n,), torch.float32), "out": ((n,), torch.float32),
                       "nb": ((n,), torch.bfloat16), "norm": ((n,), torch.bfloat16)}, device=dev)
        g.tensor("partial").normal_()
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        resid = torch.randn(n, device=dev).to(torch.bfloat16)
        s = torch.cuda.Stream(device=dev)
        cases = {
            "one": lambda: g.finish("partial", out_f32="out", mode="one", status=status),
            "two": lambda: g.finish("partial", out_f32="out", mode="two", status=status),
            "one_norm": lambda: g.finish("partial", residual=resid, out_bf16="nb", norm_bf16="norm",
                                         hidden=HIDDEN, mode="one", status=status),
            "two_norm": lambda: g.finish("partial", residual=resid, out_bf16="nb", norm_bf16="norm",
                                         hidden=HIDDEN, mode="two", status=status),
            "nccl": lambda: dist.all_reduce(g.tensor("out")),
        }
        for name, fn in cases.items():
            with torch.cuda.stream(s):
                for _ in range(3):
                    fn()
                s.synchronize()
                dist.barrier()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    for _ in range(a.launches):
                        fn()
                graph.replay()
                s.synchronize()
                dist.barrier()
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(s)
                for _ in range(a.replays):
                    graph.replay()
                e1.record(s)
                s.synchronize()
            us = e0.elapsed_time(e1) / (a.launches * a.replays) * 1e3
            t = torch.tensor([us], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[f"T{T}_{name}_us"] = round(float(t.item()), 2)
            del graph
        torch.cuda.synchronize()
        res[f"T{T}_status"] = int(status.item())
        g.close()
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
