#!/usr/bin/env python3
"""Routed-MoE layer benchmark on B200 (BASELINE metric: routed-MoE layer tokens/s).

Workload ("decode"): T=64 tokens, hidden 6144, 256 routed
experts, sigmoid router with correction bias, top-8 over 8 groups / top-4
groups, x2.5; expert intermediate 2048 in NVFP4 (W4A4) sharded over TP = N
ranks; one bf16 shared expert (intermediate 2048, sharded the same way); fp32
partials summed across ranks with an NCCL all-reduce.  A "step" is one full
layer: router, compaction, NVFP4 activation quantisation, grouped FC1+SwiGLU,
FC2 + routing-weighted combine, shared expert, and (N > 1) the all-reduce.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N

Synthetic seeded data of the configured shapes and distributions (no
checkpoint or dataset exists offline).  Weights (5.4 GB at N=1) exceed the
126 MB L2, so every step streams them from HBM; no flush is needed.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, EXPERTS, INTER, TOPK = 6144, 256, 2048, 8
METRIC = "routed-MoE layer tokens/s (decode T=64, 256 experts, top-8, NVFP4 W4A4)"
UNIT = "tokens/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--cpu-sample-tokens", type=int, default=4)
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def routed_bytes_per_expert(local_inter: int) -> dict:
    """Algorithmic HBM bytes of one touched expert per rank (NVFP4 values + E4M3 scales)."""
    fc1 = 2 * local_inter * HIDDEN
    fc2 = HIDDEN * local_inter
    return {"fc1": fc1 // 2 + fc1 // 16, "fc2": fc2 // 2 + fc2 // 16}


def measured_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
               "-lms", "100"]
        if self.uuid:
            cmd += ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [r.split(", ") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        loaded = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def graph_kernel_nodes(graph) -> int | None:
    """Kernel nodes in a captured torch CUDA graph (cudaGraphGetNodes / NodeGetType)."""
    try:
        rt = ctypes.CDLL("libcudart.so.12")
        g = ctypes.c_void_p(graph.raw_cuda_graph())
        n = ctypes.c_size_t(0)
        if rt.cudaGraphGetNodes(g, None, ctypes.byref(n)) != 0:
            return None
        nodes = (ctypes.c_void_p * n.value)()
        if rt.cudaGraphGetNodes(g, nodes, ctypes.byref(n)) != 0:
            return None
        kernels = 0
        for i in range(n.value):
            t = ctypes.c_int(-1)
            rt.cudaGraphNodeGetType(ctypes.c_void_p(nodes[i]), ctypes.byref(t))
            kernels += int(t.value == 0)  # cudaGraphNodeTypeKernel
        return kernels
    except (OSError, AttributeError, TypeError, RuntimeError):
        return None


def cpu_baseline_from_device(layer, x, cfg, n_tokens: int):
    """Oracle port (plain C restatement of crates/glm-reference, sequential fp32,
    weights dequantised inside the call as the reference oracle does) timed on the
    host cores for a bounded token sample of the same workload."""
    import numpy as np

    import oracle as O

    T = x.shape[0]
    sel = list(range(min(n_tokens, T)))
    re, rw = layer.routes(T)
    re = re.cpu().numpy().view(np.uint16)[sel]
    rw = rw.cpu().numpy()[sel]
    used = np.unique(re)
    remap = {int(e): i for i, e in enumerate(used)}
    re_m = np.vectorize(lambda e: remap[int(e)])(re).astype(np.uint16)
    w = layer.w
    idx = torch_index(used)
    xb = x[sel].contiguous().view(torch_int16()).cpu().numpy().view(np.uint16)
    args = (xb, re_m, rw, w.w13.values[idx].cpu().numpy(), w.w13.scales[idx].cpu().numpy(),
            w.w13.global_scale[idx].cpu().numpy(), w.w2.values[idx].cpu().numpy(),
            w.w2.scales[idx].cpu().numpy(), w.w2.global_scale[idx].cpu().numpy(),
            cfg.local_intermediate,
            None if w.shared13 is None else w.shared13.view(torch_int16()).cpu().numpy().view(np.uint16),
            None if w.shared2 is None else w.shared2.view(torch_int16()).cpu().numpy().view(np.uint16))
    O.moe_layer(*args)  # warm (page-in)
    t0 = time.perf_counter()
    O.moe_layer(*args)
    dt = time.perf_counter() - t0
    return {"value": len(sel) / dt, "unit": UNIT, "cores": O.threads(), "kind": "port",
            "sample": f"{len(sel)} of {T} tokens ({len(used)} experts), full layer incl. per-call "
                      f"NVFP4 dequant, {dt:.2f} s"}


def torch_index(used):
    import torch
    return torch.as_tensor(used.astype("int64"))


def torch_int16():
    import torch
    return torch.int16


def run_ours(args):
    import torch
    import torch.distributed as dist

    from glmaxx_b200 import abi, synth
    from glmaxx_b200.moe import MoEConfig, RoutedMoE

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    T = args.tokens
    cfg = MoEConfig(tp=world, rank=rank)
    weights = synth.make_rank_weights(cfg, seed=args.seed, device=dev)
    x = synth.make_input(T, HIDDEN, seed=args.seed, device=dev)
    layer = RoutedMoE(cfg, weights, T)
    out = torch.empty((T, HIDDEN), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def reduce():
        if world > 1:
            dist.all_reduce(out)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            layer(x, out)
            reduce()
        stream.synchronize()
        status = layer.device_status()
        if status:
            raise RuntimeError(f"device status after warm-up: {status}")
        graph = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(graph, stream=stream):
            layer(x, out)
        kernels_per_step = graph_kernel_nodes(graph)
        graph.instantiate()
        for _ in range(3):
            graph.replay()
            reduce()
        stream.synchronize()

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:  # noqa: BLE001
        pass
    clocks = ClockSampler(uuid)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # ---------------------------------------------------------------- timed
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
            reduce()
        e1.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())

    # ------------------------------------------- per-stage kernel timing (roofline)
    L = abi.load()
    nst = len(abi.LAYER_STAGES) + 1
    stage_ms = {s: [] for s in abi.LAYER_STAGES}
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(nst)]
    with torch.cuda.stream(stream):
        for e in evs:
            e.record(stream)  # creates the cudaEvent_t handles
        handles = (ctypes.c_uint64 * nst)(*[e.cuda_event for e in evs])
        abi.check(L.glmaxx_moe_layer_set_stage_events(handles, nst), "stage events")
        for _ in range(min(args.steps, 50)):
            # a short device spin first, so that every launch of the step is queued
            # before the GPU reaches it and the stage events time the GPU alone
            torch.cuda._sleep(2_000_000)
            layer(x, out)
            stream.synchronize()
            for i, s in enumerate(abi.LAYER_STAGES):
                stage_ms[s].append(evs[i].elapsed_time(evs[i + 1]))
        abi.check(L.glmaxx_moe_layer_set_stage_events(None, 0), "stage events off")
    stage_avg = {s: statistics.mean(v) for s, v in stage_ms.items()}

    # ------------------------------------------------------------------ e2e
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((T, HIDDEN), dtype=torch.float32).pin_memory()
    x_dev = x  # the graph reads this buffer
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            x_dev.copy_(x_host, non_blocking=True)
            graph.replay()
            reduce()
            out_host.copy_(out, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())

    # ---------------------------------------------------------- roofline
    re, _ = layer.routes(T)
    touched = int(torch.unique(re.long()).numel())
    per = routed_bytes_per_expert(cfg.local_intermediate)
    A = T * TOPK
    fc1_bytes = touched * per["fc1"] + A * (HIDDEN // 2 + HIDDEN // 16 + 4) + \
        A * cfg.local_intermediate * 2
    fc1_gbs = fc1_bytes / (stage_avg["fc1"] * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()
    shared_bytes = 3 * cfg.local_shared * HIDDEN * 2
    layer_bytes = touched * (per["fc1"] + per["fc2"]) + shared_bytes + EXPERTS * HIDDEN * 2 + \
        T * HIDDEN * (2 + 4)
    traffic = None
    tf = ROOT / "profiles" / "fc1_decode_traffic.json"
    if tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get(f"tp{world}", {}).get("dram_bytes_per_launch")
        except (ValueError, AttributeError):
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_from_device(layer, x, cfg, args.cpu_sample_tokens)
        except Exception as exc:  # noqa: BLE001
            cpu = {"value": None, "unit": UNIT, "error": repr(exc)[:200]}

    if rank == 0:
        line = {
            "metric": METRIC, "value": T / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, N(0,0.01) bias)",
            "config": {"workload": "decode T=64 (BASELINE configs[1])", "tokens": T,
                       "hidden": HIDDEN, "experts": EXPERTS, "top_k": TOPK, "groups": 8,
                       "topk_groups": 4, "intermediate": INTER, "shared_intermediate": INTER,
                       "parallelism": f"tp{world} (expert intermediate sharded, NCCL all-reduce)",
                       "l2": "weights per step >> 126 MB L2 (no flush needed)",
                       "timing": "CUDA-graph replay of the layer + eager NCCL all-reduce, "
                                 "CUDA events on the launch stream, max over ranks"},
            "roofline": {"bound": "hbm", "kernel": "fc1 grouped GEMM (tcgen05 NVFP4, N tile 32)",
                         "achieved": fc1_gbs, "peak": peak, "unit": "GB/s",
                         "frac": fc1_gbs / peak, "peak_kind": peak_kind, "traffic": traffic,
                         "algorithmic_bytes_per_launch": fc1_bytes, "touched_experts": touched,
                         "fc1_ms": stage_avg["fc1"],
                         "layer_weight_bytes": layer_bytes,
                         "layer_achieved_gbs": layer_bytes / (ms * 1e-3) / 1e9,
                         "layer_frac": layer_bytes / (ms * 1e-3) / 1e9 / peak},
            "stage_ms": stage_avg,
            "cpu_baseline": cpu,
            "e2e": {"value": T / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": T * HIDDEN * 2, "d2h_bytes_per_step": T * HIDDEN * 4,
                    "ms_per_step": e2e_ms},
            "gpu_launches": None if kernels_per_step is None else kernels_per_step * args.steps,
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        del graph
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    """Reference arm: the reference's CPU implementation of the path (no Rust
    toolchain exists here, so its C restatement oracle/, which reproduces the
    reference's golden vectors) on this box's host cores, same config/metric."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    import oracle as O

    rng = np.random.default_rng(args.seed)
    T, S = args.tokens, max(1, args.cpu_sample_tokens)
    Ir = INTER // world
    x = O.f32_to_bf16_bits(rng.standard_normal((T, HIDDEN)).astype(np.float32))
    wr = O.f32_to_bf16_bits((rng.standard_normal((EXPERTS, HIDDEN)) * 0.02).astype(np.float32))
    bias = (rng.standard_normal(EXPERTS) * 0.01).astype(np.float32)
    t0 = time.perf_counter()
    experts, weights = O.router(x, wr, bias, 8, 4, TOPK, 2.5)
    router_s = time.perf_counter() - t0
    sel = np.arange(S)
    used = np.unique(experts[sel])
    remap = {int(e): i for i, e in enumerate(used)}
    v13, s13, g13, v2, s2, g2 = [], [], [], [], [], []
    for e in used:
        er = np.random.default_rng(args.seed * 1000 + int(e))
        p13 = O.pack((er.standard_normal((2 * Ir, HIDDEN)) * 0.02).astype(np.float32))
        p2 = O.pack((er.standard_normal((HIDDEN, Ir)) * 0.02).astype(np.float32))
        v13.append(p13.values), s13.append(p13.scales), g13.append(p13.global_scale)
        v2.append(p2.values), s2.append(p2.scales), g2.append(p2.global_scale)
    sh13 = O.f32_to_bf16_bits((rng.standard_normal((2 * Ir, HIDDEN)) * 0.02).astype(np.float32))
    sh2 = O.f32_to_bf16_bits((rng.standard_normal((HIDDEN, Ir)) * 0.02).astype(np.float32))
    re_m = np.vectorize(lambda e: remap[int(e)])(experts[sel]).astype(np.uint16)
    a = (x[sel], re_m, weights[sel], np.stack(v13), np.stack(s13), np.array(g13, np.float32),
         np.stack(v2), np.stack(s2), np.array(g2, np.float32), Ir, sh13, sh2)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        O.moe_layer(*a)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    per_step = statistics.mean(times) + router_s * S / T
    value = S / per_step
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded, same shapes and distributions)",
        "config": {"workload": "decode T=64 (BASELINE configs[1])", "tokens": T,
                   "parallelism": f"tp{world} shard on one host process"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": O.threads(), "kind": "port",
                         "sample": f"{S} tokens of {T} per step ({len(used)} experts), "
                                   "full layer incl. per-call NVFP4 dequant"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
