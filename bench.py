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
UNIT = "tokens/s"
WORKLOADS = {
    "decode": {"tokens": 64, "zipf": False, "bound": "hbm",
               "metric": "routed-MoE layer tokens/s (decode T=64, 256 experts, top-8, NVFP4 W4A4)",
               "name": "decode T=64 (BASELINE configs[1])"},
    "prefill": {"tokens": 8192, "zipf": True, "bound": "tensor",
                "metric": "routed-MoE layer tokens/s (prefill T=8192, Zipf(1.1) routing, 256 "
                          "experts, top-8, NVFP4 W4A4)",
                "name": "prefill T=8192, Zipf(s=1.1) expert counts (BASELINE configs[2])"},
    "exl3": {"tokens": 32, "zipf": False, "bound": "hbm", "codec": "exl3",
             "metric": "routed-MoE layer tokens/s (EXL3 3-bit decode T=32, 256 experts, top-8)",
             "name": "EXL3 trellis decode T=32 (BASELINE configs[3])"},
    "load": {"tokens": 0, "zipf": False, "bound": "host-sha256",
             "metric": "rank-file load GB/s (verify + place one TP4 layer of 256 NVFP4 experts, "
                       "router and shared expert in HBM)",
             "name": "native .g5n reader, one TP4 rank file of one MoE layer"},
    "hybrid": {"tokens": 2048, "zipf": True, "bound": "hbm", "codec": "hybrid", "layers": 4,
               "metric": "4-layer routed-MoE stack tokens/s (2048 tokens, 64 NVFP4 + 192 EXL3 "
                         "experts, Zipf routing, bf16 residual)",
               "name": "hybrid continuous-batch step, 4 stacked layers (BASELINE configs[4])"},
}
HYBRID_NVFP4_EXPERTS = 64
# NVFP4 dense tensor rate / bf16 dense tensor rate on B200 (9 / 2.25 PFLOP/s nominal):
# the NVFP4 roofline is the measured cuBLAS bf16 rate scaled by this ratio.
NVFP4_PER_BF16 = 4.0
NVFP4_NOMINAL_TFLOPS = 9000.0
# The CPU timing plan (BASELINE CPU baseline): configs[1] and configs[3] are timed
# on all their tokens; configs[2] on a seeded 512-token subset (per-token rate).
# Expert weights are dequantised (NVFP4) or decoded (EXL3) once per expert into
# fp32 planes outside the timed region; the timed part is the router and the
# layer arithmetic, OpenMP over assignments with SIMD across output columns.
CPU_PREFILL_SAMPLE_TOKENS = 512
# prepared experts are held for the whole run when they fit in this fraction of
# the host's available memory, else rebuilt (untimed) every step
CPU_HOLD_FRACTION = 0.6
REF_TIME_BUDGET_S = 120.0
# Peer copy over NVLink 5, per direction per GPU: measured live by every
# multi-GPU run with the peer finish (peer_copy_gbs); this earlier measurement on
# the same pool is the denominator only where no live number exists (the NCCL
# reduce mode).
NVLINK_PEER_GBS = 770.0
PEER_PROBE_BYTES = 64 << 20


def peer_copy_gbs(group, dev, stream, reps: int = 10) -> float:
    """Per-direction NVLink copy bandwidth of this box, measured now: every rank
    copies PEER_PROBE_BYTES from its own probe buffer into its right neighbour's
    (cudaMemcpyAsync through the peer mapping; all ranks at once, so every GPU
    sends and receives at the same time), CUDA events around `reps` copies,
    the slowest rank's time."""
    import torch
    import torch.distributed as dist

    from glmaxx_b200.peer import device_view
    half = PEER_PROBE_BYTES
    local = group.tensor("probe")                  # [2 * half] bytes: send half, receive half
    right = (group.rank + 1) % group.ranks
    dst = device_view(group.pointer("probe", right) + half, (half,), torch.uint8, dev)
    src = local[:half]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        dst.copy_(src, non_blocking=True)
        stream.synchronize()
        dist.barrier()
        e0.record(stream)
        for _ in range(reps):
            dst.copy_(src, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return half / (float(t.item()) * 1e-3) / 1e9


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted([*WORKLOADS, "nvfp4-peak"]), default="decode")
    p.add_argument("--tokens", type=int, default=None)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--no-cpu-baseline", action="store_true")
    # N > 1: how the ranks' partials are reduced -- the fused peer-memory finish
    # (one kernel per layer over NVLink) or an NCCL all-reduce plus the finish
    p.add_argument("--reduce", choices=["peer", "nccl"], default="peer")
    p.add_argument("--peer-mode", choices=["auto", "one", "two"], default="auto")
    # N > 1: token-split routing (each rank routes T/N tokens, the routes are
    # all-gathered) where it pays (tp_route.split_pays), always, or never
    p.add_argument("--split-route", choices=["auto", "on", "off"], default="auto")
    # how a prefill-size step combines its routed rows: fp32 atomics into the output
    # (faster: T=8192 layer 3.91 / 2.68 / 1.97 ms at TP1 / TP2 / TP8 shards against
    # 4.56 / 3.23 / 2.33 ms), or the slot plane + expert-order combine
    # (GLMAXX_MOE_DETERMINISTIC, the same bits run after run)
    p.add_argument("--combine", choices=["atomic", "plane"], default="atomic")
    # N > 1, one layer: run the step as this many token chunks, each chunk's peer
    # finish (reduce) on a second stream overlapping the next chunk's layer
    p.add_argument("--chunks", type=int, default=1)
    # --workload load: rank files loaded at once (1, or a TP4 node's 4 on threads)
    p.add_argument("--rank-files", type=int, choices=[1, 4], default=1)
    a = p.parse_args()
    if a.tokens is None:
        a.tokens = WORKLOADS.get(a.workload, {"tokens": 0})["tokens"]
    return a


def routed_bytes_per_expert(local_inter: int) -> dict:
    """Algorithmic HBM bytes of one touched expert per rank (NVFP4 values + E4M3 scales)."""
    fc1 = 2 * local_inter * HIDDEN
    fc2 = HIDDEN * local_inter
    return {"fc1": fc1 // 2 + fc1 // 16, "fc2": fc2 // 2 + fc2 // 16}


def measured_peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, kind) from MEASURED_PEAKS.json, else the fallback."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# tcgen05 NVFP4 MMA-loop cases (N, dual, copy kind, copies per K-block): MMA-only
# rates give the measured NVFP4 peak; the others price the scale-factor copies
# of the grouped GEMMs (dual 128 + 6 atom copies per 4 K-blocks is the decode
# pattern, dual 128 + 1.5 lane-major copies per K-block the prefill pattern).
# copy kind | 4 issues a stage's 4 K-blocks' copies together before its first MMA.
NVFP4_PEAK_CASES = [(256, 0, 0, 0), (128, 0, 0, 0), (128, 1, 0, 0), (128, 1, 1, 3),
                    (128, 1, 2, 1), (128, 1, 2, 2), (256, 0, 1, 3), (256, 0, 2, 1),
                    (256, 0, 2, 2), (128, 0, 2, 1), (128, 0, 1, 2), (128, 1, 6, 1),
                    (256, 0, 6, 1), (256, 0, 6, 2), (256, 0, 5, 3)]


def nvfp4_mma_peak(dev, iters: int = 20000, reps: int = 5):
    """The NVFP4 tensor rate of this GPU measured with the library's own tcgen05
    MMA loop (glmaxx_nvfp4_mma_peak_launch), one CTA per SM, CUDA events around
    each launch (best of `reps`).  Returns (peak TFLOP/s over the MMA-only cases,
    per-case results)."""
    import torch

    from glmaxx_b200 import abi
    L = abi.load()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    cycles = torch.zeros(sms, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = []
    for n, dual, kind, cps in NVFP4_PEAK_CASES:
        def launch():
            abi.check(L.glmaxx_nvfp4_mma_peak_launch(n, dual, kind, cps, iters, sms,
                                                     ctypes.c_void_p(status.data_ptr()),
                                                     ctypes.c_void_p(cycles.data_ptr()),
                                                     ctypes.c_void_p(stream.cuda_stream)),
                      "nvfp4_mma_peak")
        launch()
        best = None
        for _ in range(reps):
            e0.record(stream)
            launch()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        if int(status.item()):
            raise RuntimeError(f"nvfp4 peak loop status {int(status.item())}")
        flops = sms * iters * 4 * (2 if dual else 1) * 2.0 * 128 * n * 64
        kblocks = iters * 4
        out.append({"n": n, "dual": bool(dual), "copy_kind": kind, "copies_per_kblock": cps,
                    "tflops": flops / (best * 1e-3) / 1e12, "ms": best,
                    "cycles_per_kblock": float(cycles.double().median()) / kblocks})
    peak = max(r["tflops"] for r in out if r["copies_per_kblock"] == 0)
    return peak, out


def run_nvfp4_peak(args):
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:  # noqa: BLE001
        pass
    clocks = ClockSampler(uuid)
    nvfp4_mma_peak(dev, iters=2000, reps=1)  # warm-up
    clocks.start()
    peak, cases = nvfp4_mma_peak(dev)
    clock_info = clocks.stop()
    print(json.dumps({"metric": "NVFP4 tcgen05 MMA-loop TFLOP/s (one CTA per SM)", "value": peak,
                      "unit": "TFLOP/s", "nominal_dense": NVFP4_NOMINAL_TFLOPS,
                      "frac_of_nominal": peak / NVFP4_NOMINAL_TFLOPS, "cases": cases,
                      "clocks": clock_info}), flush=True)


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


# FC1 DRAM bytes per launch from ncu (dram__bytes_read.sum + dram__bytes_write.sum)
# of the decode FC1 at 64 experts, T=64, TP1, divided by the touched experts of that
# capture; FC1 traffic grows with the touched experts (weights dominate), so a
# full launch is estimated as this figure x touched experts.
FC1_DECODE_DRAM_BYTES_PER_EXPERT_TP1 = (911.565824e6 + 6.625024e6) / 64


def fc1_traffic_estimate(touched: int, world: int):
    if FC1_DECODE_DRAM_BYTES_PER_EXPERT_TP1 is None:
        return None
    return FC1_DECODE_DRAM_BYTES_PER_EXPERT_TP1 * touched / world


def host_mem_available() -> int:
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


class PreparedExperts:
    """The routed experts of a CPU run, each dequantised (NVFP4) or decoded (EXL3)
    once into fp32 planes outside the timed region.  Held for the whole run when
    they fit in host memory, else rebuilt every step (still untimed)."""

    def __init__(self, make, n_experts: int, bytes_per_expert: int):
        self.make = make
        self.hold = n_experts * bytes_per_expert < CPU_HOLD_FRACTION * host_mem_available()
        self.cache = {}
        self.prep_s = 0.0

    def __call__(self, e: int):
        e = int(e)
        if e in self.cache:
            return self.cache[e]
        t0 = time.perf_counter()
        v = self.make(e)
        self.prep_s += time.perf_counter() - t0
        if self.hold:
            self.cache[e] = v
        return v


def host_u16(t) -> "np.ndarray":
    import numpy as np
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def nvfp4_prepare_fn(w, hidden: int, inter: int):
    """prepare(e): expert e's packed NVFP4 shard copied to the host and dequantised
    once (nvfp4.rs:279-301) into k-major fp32 planes."""
    import oracle as O

    def make(e):
        return O.expert_prepare(w.w13.values[e].cpu().numpy(), w.w13.scales[e].cpu().numpy(),
                                float(w.w13.global_scale[e]), w.w2.values[e].cpu().numpy(),
                                w.w2.scales[e].cpu().numpy(), float(w.w2.global_scale[e]),
                                hidden, inter)
    return make


def exl3_prepare_fn(x3, hidden: int, inter: int):
    """prepare(e): expert e's gate/up/down trellises decoded once (exl3.rs:490-513)
    to fp32, with its fp16 rotation signs."""
    import oracle as O

    def make(e):
        return {"gate": O.exl3_prepare(host_u16(x3.gate_trellis[e]), hidden, inter),
                "up": O.exl3_prepare(host_u16(x3.up_trellis[e]), hidden, inter),
                "down": O.exl3_prepare(host_u16(x3.down_trellis[e]), inter, hidden),
                **{n: host_u16(getattr(x3, n)[e]) for n in
                   ("gate_suh", "gate_svh", "up_suh", "up_svh", "down_suh", "down_svh")}}
    return make


def exl3_layer_cpu(xb, route_experts, route_weights, prep):
    """EXL3 experts of the sample on the CPU: per routed expert (ascending), gate and up
    = matmul_reference_f16 (crates/glm-format/src/exl3.rs:404-453) on the fp16 token
    rows, h = fp16(silu(g) * u), down on h; routing-weighted and summed over the slots
    in ascending expert order.  Returns (routed [S, H], seconds excluding prepare)."""
    import numpy as np

    import oracle as O
    S, K = route_experts.shape
    x16 = (xb.astype(np.uint32) << 16).view(np.float32).astype(np.float16).view(np.uint16)
    busy = 0.0
    contrib = None
    for e in np.unique(route_experts):
        p = prep(int(e))
        t0 = time.perf_counter()
        rows = np.argwhere(route_experts == e)
        xin = x16[rows[:, 0]]
        g = O.exl3_project(p["gate"], p["gate_suh"], p["gate_svh"], xin)
        u = O.exl3_project(p["up"], p["up_suh"], p["up_svh"], xin)
        gf = g.view(np.float16).astype(np.float32)
        uf = u.view(np.float16).astype(np.float32)
        h = (gf / (np.float32(1.0) + np.exp(-gf)) * uf).astype(np.float16).view(np.uint16)
        d = O.exl3_project(p["down"], p["down_suh"], p["down_svh"], h)
        if contrib is None:
            contrib = np.zeros((S, K, d.shape[1]), np.float32)
        contrib[rows[:, 0], rows[:, 1]] = (route_weights[rows[:, 0], rows[:, 1]][:, None] *
                                           d.view(np.float16).astype(np.float32))
        busy += time.perf_counter() - t0
    t0 = time.perf_counter()
    order = np.argsort(route_experts, axis=1, kind="stable")
    out = np.take_along_axis(contrib, order[:, :1, None], 1)[:, 0].copy()
    for j in range(1, K):
        out = out + np.take_along_axis(contrib, order[:, j:j + 1, None], 1)[:, 0]
    busy += time.perf_counter() - t0
    return out, busy


def cpu_sample(T: int, workload: str, seed: int):
    """Token indices the CPU timing covers: every token, except configs[2]'s seeded
    512-token subset."""
    import numpy as np
    if workload == "prefill" and T > CPU_PREFILL_SAMPLE_TOKENS:
        return np.sort(np.random.default_rng(seed).choice(T, CPU_PREFILL_SAMPLE_TOKENS,
                                                          replace=False))
    return np.arange(T)


class CpuLayer:
    """The reference's CPU path of one full layer (oracle/, the C restatement of
    crates/glm-reference: the router restatement, then the NVFP4 or EXL3 experts and
    the bf16 shared expert) on a token sample, on all host cores."""

    def __init__(self, w, cfg, codec, xb):
        import oracle as O
        self.w, self.cfg, self.codec, self.xb = w, cfg, codec, xb
        self.wr = host_u16(w.router_weight)
        self.bias = w.router_bias.cpu().numpy()
        H, Ir = cfg.hidden, cfg.local_intermediate
        per = 3 * H * Ir * 4  # fp32 planes of gate, up and down
        make = exl3_prepare_fn(w.exl3, H, Ir) if codec == "exl3" else nvfp4_prepare_fn(w, H, Ir)
        self.prep = PreparedExperts(make, cfg.experts, per)
        t0 = time.perf_counter()
        self.shared = None if w.shared13 is None else O.shared_prepare(host_u16(w.shared13),
                                                                       host_u16(w.shared2))
        self.prep.prep_s += time.perf_counter() - t0

    def step(self):
        """One timed pass: (seconds excluding expert preparation, touched experts,
        the layer output [S, H] = routed + shared)."""
        import numpy as np

        import oracle as O
        c = self.cfg
        t0 = time.perf_counter()
        ex, wt = O.router(self.xb, self.wr, self.bias, c.groups, c.topk_groups, c.top_k,
                          c.route_scale)
        busy = time.perf_counter() - t0
        shared = None
        if self.codec == "exl3":
            routed, b = exl3_layer_cpu(self.xb, ex.astype(np.int64), wt, self.prep)
            busy += b
            if self.shared is not None:
                t0 = time.perf_counter()
                shared = O.shared_rows(self.xb, np.arange(self.xb.shape[0]), *self.shared)
                busy += time.perf_counter() - t0
        else:
            routed, shared, b = O.moe_layer_prepared(self.xb, ex, wt, self.prep,
                                                     c.local_intermediate, shared=self.shared)
            busy += b
        out = routed if shared is None else routed + shared
        return busy, int(np.unique(ex).size), out


def cpu_baseline(w, cfg, codec, x, workload: str, seed: int):
    """cpu_baseline of our arm: the CPU path timed once on this box's host cores."""
    import oracle as O
    T = x.shape[0]
    sel = cpu_sample(T, workload, seed)
    xb = host_u16(x)[sel]
    cl = CpuLayer(w, cfg, codec, xb)
    busy, touched, _ = cl.step()
    return {"value": len(sel) / busy, "unit": UNIT, "cores": int(O.lib().orc_threads()),
            "kind": "port",
            "sample": f"{len(sel)} of {T} tokens ({touched} experts): router + full layer, "
                      f"{busy:.2f} s; experts dequantised once outside the timing "
                      f"({cl.prep.prep_s:.1f} s)"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    from glmaxx_b200 import abi, synth
    from glmaxx_b200.moe import MoEConfig, RoutedMoE, finish

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        # NCCL's own log lines (e.g. its version banner) go to stderr, so that rank 0's
        # stdout carries only the JSON result line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    T = args.tokens
    wl = WORKLOADS[args.workload]
    cfg = MoEConfig(tp=world, rank=rank)
    zipf = None
    if wl["zipf"]:
        # same beta on every rank: the fit is deterministic in (seed, router, input)
        zipf = synth.fit_zipf_beta(cfg, T, args.seed, dev)
    beta = None if zipf is None else zipf[0]
    codec = wl.get("codec")
    n_layers = wl.get("layers", 1)
    nvfp4_mask = None
    if codec == "hybrid":
        g = torch.Generator().manual_seed(args.seed * 13 + 1)
        nvfp4_mask = torch.zeros(EXPERTS, dtype=torch.bool)
        nvfp4_mask[torch.randperm(EXPERTS, generator=g)[:HYBRID_NVFP4_EXPERTS]] = True
    deterministic = args.combine == "plane"
    layers = []
    for li in range(n_layers):
        seed = args.seed + 7919 * li
        if codec == "exl3":
            w = synth.make_exl3_rank_weights(cfg, seed=seed, device=dev, zipf_beta=beta)
        elif codec == "hybrid":
            w = synth.make_exl3_rank_weights(cfg, seed=seed, device=dev, zipf_beta=beta,
                                             nvfp4_experts=nvfp4_mask)
        else:
            w = synth.make_rank_weights(cfg, seed=seed, device=dev, zipf_beta=beta)
        layers.append(RoutedMoE(cfg, w, T, deterministic=deterministic))
    layer = layers[0]
    weights = layer.w
    x = synth.make_input(T, HIDDEN, seed=args.seed, device=dev)
    use_peer = world > 1 and args.reduce == "peer"
    from glmaxx_b200 import tp_route
    split = world > 1 and (args.split_route == "on" or
                           (args.split_route == "auto" and tp_route.split_pays(T, world)))
    # token-split routing: each layer's routes land in that layer's own route
    # buffers, which its forward() then reads in place (routes given)
    routers = ([tp_route.SplitRouter(cfg, lay.w, T, rank, world, dev, out=lay.routes(T))
                for lay in layers] if split else None)
    group = None
    if use_peer:
        # every rank maps every rank's partial, output and stacked-layer buffers
        from glmaxx_b200.peer import PeerGroup
        bufs = {"partial": ((T, HIDDEN), torch.float32), "out": ((T, HIDDEN), torch.float32),
                "probe": ((2 * PEER_PROBE_BYTES,), torch.uint8)}
        for li in range(1, n_layers):
            bufs[f"rs{li}"] = ((T, HIDDEN), torch.bfloat16)
            bufs[f"xs{li}"] = ((T, HIDDEN), torch.bfloat16)
        group = PeerGroup(bufs, device=dev)
        peer_status = torch.zeros(1, dtype=torch.int32, device=dev)
    # stack: rs[l] is the bf16 residual stream before layer l, xs[l] layer l's MoE
    # input RMSNorm(rs[l]) (unit weight; layer 0 takes the unit-variance input as is)
    if use_peer:
        xs = [x] + [group.tensor(f"xs{li}") for li in range(1, n_layers)]
        rs = [x] + [group.tensor(f"rs{li}") for li in range(1, n_layers)]
        outs = [group.tensor("partial")] * n_layers  # one partial buffer, reused per layer
        out = group.tensor("out")
    else:
        xs = [x] + [torch.empty_like(x) for _ in range(n_layers - 1)]
        rs = [x] + [torch.empty_like(x) for _ in range(n_layers - 1)]
        outs = [torch.empty((T, HIDDEN), dtype=torch.float32, device=dev)
                for _ in range(n_layers)]
        out = outs[-1]
    stream = torch.cuda.Stream(device=dev)

    def reduce(o):
        if world > 1 and not use_peer:
            dist.all_reduce(o)

    def peer_finish(li):
        """The fused reduce + finish of layer li over peer memory: into layer li+1's
        bf16 residual and normalised input, or (last layer) the fp32 output."""
        if li + 1 < n_layers:
            group.finish("partial", residual=rs[li], out_bf16=f"rs{li + 1}",
                         norm_bf16=f"xs{li + 1}", hidden=HIDDEN, mode=args.peer_mode,
                         status=peer_status)
        else:
            group.finish("partial", out_f32="out", mode=args.peer_mode, status=peer_status)

    chunks = args.chunks if (use_peer and n_layers == 1 and args.chunks > 1
                             and T % args.chunks == 0) else 1
    fin_stream = torch.cuda.Stream(device=dev) if chunks > 1 else None
    chunk_done = [torch.cuda.Event() for _ in range(chunks)]
    fin_done = torch.cuda.Event()

    def chunked_layer_and_finish(li):
        """The step as token chunks: chunk c's layer on the launch stream, then its
        rows' peer finish on fin_stream, overlapping chunk c+1's layer; the launch
        stream joins fin_stream at the end.  Every rank issues the same finishes
        in the same order (one signal buffer, used by one finish at a time)."""
        tc = T // chunks
        routes = routers[li](xs[li]) if routers is not None else None
        cur = torch.cuda.current_stream()
        fin_stream.wait_stream(cur)
        for c in range(chunks):
            lo, hi = c * tc, (c + 1) * tc
            r = None if routes is None else (routes[0][lo:hi], routes[1][lo:hi])
            layers[li](xs[li][lo:hi], outs[li][lo:hi], routes=r)
            chunk_done[c].record(cur)
            fin_stream.wait_event(chunk_done[c])
            with torch.cuda.stream(fin_stream):
                group.finish("partial", out_f32="out", mode=args.peer_mode, status=peer_status,
                             rows=(lo, hi), row_elems=HIDDEN)
        fin_done.record(fin_stream)
        cur.wait_event(fin_done)

    def layer_and_finish(li):
        """layer li, and (stack) the finish that forms layer li+1's bf16 input."""
        if chunks > 1:
            chunked_layer_and_finish(li)
            return
        if routers is not None:
            layers[li](xs[li], outs[li], routes=routers[li](xs[li]))
        else:
            layers[li](xs[li], outs[li])
        if use_peer:
            peer_finish(li)

    def finish_into_next(li):
        if li + 1 < n_layers and not use_peer:
            finish([outs[li]], rs[li], out_bf16=rs[li + 1], norm_bf16=xs[li + 1], hidden=HIDDEN)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            for li in range(n_layers):
                layer_and_finish(li)
                reduce(outs[li])
                finish_into_next(li)
        stream.synchronize()
        for lay in layers:
            status = lay.device_status()
            if status:
                raise RuntimeError(f"device status after warm-up: {status}")
        for r in routers or []:
            status = r.device_status()
            if status:
                raise RuntimeError(f"token-slice router status after warm-up: {status}")
        if use_peer and int(peer_status.item()):
            raise RuntimeError(f"peer finish status after warm-up: {int(peer_status.item())}")
        # one graph per layer (its routed step; the finish joins it when no collective
        # sits between a layer and the next)
        graphs = []
        for li in range(n_layers):
            gr = torch.cuda.CUDAGraph(keep_graph=True)
            with torch.cuda.graph(gr, stream=stream):
                layer_and_finish(li)
                if world == 1:
                    finish_into_next(li)
            graphs.append(gr)
        kernels_per_step = 0
        for gr in graphs:
            kn = graph_kernel_nodes(gr)
            kernels_per_step = None if (kn is None or kernels_per_step is None) else \
                kernels_per_step + kn
            gr.instantiate()
        graph = graphs[0]

        def step():
            for li in range(n_layers):
                graphs[li].replay()
                if world > 1 and not use_peer:
                    reduce(outs[li])
                    finish_into_next(li)

        for _ in range(3):
            step()
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
            step()
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
    if use_peer and int(peer_status.item()):
        raise RuntimeError(f"peer finish status: {int(peer_status.item())}")

    # ------------------------------------------- the reduce alone (N > 1)
    reduce_info = None
    if world > 1:
        from glmaxx_b200.peer import two_shot_pays

        def one_reduce():
            if use_peer:
                group.finish("partial", out_f32="out", mode=args.peer_mode, status=peer_status)
            else:
                dist.all_reduce(outs[-1])

        # a CUDA graph of 10 launches, so that host launch cost stays out of the time
        per_graph, n_rep = 10, max(2, min(args.steps, 200) // 10)
        with torch.cuda.stream(stream):
            for _ in range(5):
                one_reduce()
            stream.synchronize()
            rgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(rgraph, stream=stream):
                for _ in range(per_graph):
                    one_reduce()
            rgraph.replay()
            stream.synchronize()
            dist.barrier()
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(n_rep):
                rgraph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        del rgraph
        red_ms = e0.elapsed_time(e1) / (n_rep * per_graph)
        t = torch.tensor([red_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        red_ms = float(t.item())
        S = T * HIDDEN * 4
        mode = args.peer_mode
        if mode == "auto":
            mode = "two" if two_shot_pays(T * HIDDEN, world) else "one"
        busbw = 2 * (world - 1) / world * S / (red_ms * 1e-3) / 1e9
        peer_gbs, peer_live = NVLINK_PEER_GBS, False
        if use_peer:
            try:
                peer_gbs, peer_live = peer_copy_gbs(group, dev, stream), True
            except Exception as exc:  # noqa: BLE001 -- same failure on every rank
                print(f"peer copy probe failed: {exc!r}", file=sys.stderr)
        # bytes each GPU sends (and receives) over NVLink per reduce: one-shot, its
        # partial to each of the N-1 peers; two-shot (and a ring all-reduce), its
        # 1/N slice-reduction inputs to N-1 peers plus its reduced slice to N-1
        # peers, 2(N-1)/N of the partial -- both directions busy at once
        link_bytes = ((world - 1) * S if use_peer and mode == "one"
                      else 2 * (world - 1) * S // world)
        reduce_info = {
            "kind": f"peer {mode}-shot (fused finish kernel)" if use_peer else "NCCL all-reduce",
            "us_per_launch": red_ms * 1e3, "bytes": S,
            "nvlink_bytes_per_rank": link_bytes,
            "busbw_gbs": busbw, "peak_gbs": peer_gbs,
            "peak_kind": ("peer copy measured in this run (every rank into its right "
                          "neighbour at once, 64 MiB, max over ranks)" if peer_live else
                          "earlier peer-copy measurement on this pool"),
            "frac": link_bytes / (red_ms * 1e-3) / 1e9 / peer_gbs,
            "note": "busbw = 2(N-1)/N x bytes / time (the all-reduce convention); frac = the "
                    "bytes each GPU sends per direction (nvlink_bytes_per_rank) / time, "
                    "against the peer copy rate"}
        if use_peer and int(peer_status.item()):
            raise RuntimeError(f"peer finish status: {int(peer_status.item())}")

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
            if routers is not None:
                layer(x, out, routes=routers[0](x))
            else:
                layer(x, out)
            stream.synchronize()
            for i, s in enumerate(abi.LAYER_STAGES):
                stage_ms[s].append(evs[i].elapsed_time(evs[i + 1]))
        abi.check(L.glmaxx_moe_layer_set_stage_events(None, 0), "stage events off")
    stage_avg = {s: statistics.mean(v) for s, v in stage_ms.items()}

    # ------------------------------------------------------------------ e2e
    # Every step uploads its input from pinned host memory and downloads its
    # fp32 output, inside the timed region.  As in a serving loop, the transfers
    # of neighbouring steps overlap the compute: step i+1's input lands in a
    # staging buffer on an upload stream while step i runs, and a device-to-device
    # copy feeds the graph's input buffer; step i's output is snapshotted on the
    # device and downloaded on a download stream while step i+1 runs (the two
    # directions use separate copy engines).  The first upload and the last
    # download are not overlapped.  With N > 1 every rank uploads the input (the
    # TP layout replicates it) and the result -- the same bits on every rank
    # after the reduce -- is read back once, by rank 0.
    reads_result = rank == 0
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((T, HIDDEN), dtype=torch.float32).pin_memory()
    x_dev = x  # the graph reads this buffer
    x_stage = torch.empty_like(x)
    out_stage = torch.empty((T, HIDDEN), dtype=torch.float32, device=dev)
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    x_ready, x_free = torch.cuda.Event(), torch.cuda.Event()
    o_ready, o_free = torch.cuda.Event(), torch.cuda.Event()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        up.wait_event(e0)
        with torch.cuda.stream(up):
            x_stage.copy_(x_host, non_blocking=True)
            x_ready.record(up)
        for i in range(args.steps):
            stream.wait_event(x_ready)
            x_dev.copy_(x_stage, non_blocking=True)
            x_free.record(stream)
            with torch.cuda.stream(up):
                up.wait_event(x_free)
                if i + 1 < args.steps:
                    x_stage.copy_(x_host, non_blocking=True)
                    x_ready.record(up)
            step()
            if reads_result:
                if i > 0:
                    stream.wait_event(o_free)
                out_stage.copy_(out, non_blocking=True)
                o_ready.record(stream)
                with torch.cuda.stream(down):
                    down.wait_event(o_ready)
                    out_host.copy_(out_stage, non_blocking=True)
                    o_free.record(down)
        if reads_result:
            stream.wait_event(o_free)
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
    counts = torch.bincount(re.long().flatten(), minlength=EXPERTS)
    per = routed_bytes_per_expert(cfg.local_intermediate)
    A = T * TOPK
    Ir = cfg.local_intermediate
    hbm_peak, bf16_peak, peak_kind = measured_peaks()
    shared_bytes = 3 * cfg.local_shared * HIDDEN * 2
    layer_bytes = touched * (per["fc1"] + per["fc2"]) + shared_bytes + EXPERTS * HIDDEN * 2 + \
        T * HIDDEN * (2 + 4)
    fc1_ms = stage_avg["fc1"]
    exl3_expert_bytes = 3 * (HIDDEN * Ir * 3 // 8 + (HIDDEN + Ir) * 2)
    if codec == "exl3":
        # the EXL3 chain (rotations, decode-fused gate/up/down projections) runs in
        # the fc1 stage: trellis + suh/svh bytes of every touched expert
        ex_bytes = touched * exl3_expert_bytes
        achieved = ex_bytes / (fc1_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "EXL3 decode-fused projections (gate, up, down)",
                "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "peak_kind": f"{peak_kind} HBM copy",
                "traffic": None, "algorithmic_bytes_per_launch": ex_bytes,
                "alu": {"decoded_weights_per_s": touched * 3 * HIDDEN * Ir / (fc1_ms * 1e-3),
                        "note": "3INST trellis decode is ALU-bound: ~15 thread instructions "
                                "per decoded weight (ncu), one fp32 fma of fp16 factors per "
                                "weight and row (the product is exact, so it equals the "
                                "reference's multiply then add), k ascending"}}
    elif codec == "hybrid":
        layer_ms = ms / n_layers
        nv_touched = int(torch.unique(re.long()[nvfp4_mask.to(re.device)[re.long()]]).numel())
        ex_touched = touched - nv_touched
        hy_bytes = nv_touched * (per["fc1"] + per["fc2"]) + ex_touched * exl3_expert_bytes + \
            shared_bytes
        achieved = hy_bytes / (layer_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "whole layer (NVFP4 + EXL3 experts, shared expert)",
                "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "peak_kind": f"{peak_kind} HBM copy",
                "traffic": None, "algorithmic_bytes_per_layer": hy_bytes,
                "layer_ms": layer_ms, "nvfp4_touched": nv_touched, "exl3_touched": ex_touched,
                "nvfp4_rows": int(nvfp4_mask.to(re.device)[re.long()].sum()),
                "exl3_rows": int((~nvfp4_mask.to(re.device)[re.long()]).sum())}
    elif wl["bound"] == "hbm":
        # FC1 weights of every touched expert, the NVFP4 activation rows (values,
        # scales, global) and the bf16 SwiGLU output rows
        fc1_bytes = touched * per["fc1"] + A * (HIDDEN // 2 + HIDDEN // 16 + 4) + A * Ir * 2
        achieved = fc1_bytes / (fc1_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "fc1 grouped GEMM (tcgen05 NVFP4, N tile 32)",
                "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "peak_kind": f"{peak_kind} HBM copy",
                "traffic": fc1_traffic_estimate(touched, world),
                "algorithmic_bytes_per_launch": fc1_bytes}
    else:
        fc1_flops = 2.0 * A * HIDDEN * (2 * Ir)
        fc2_flops = 2.0 * A * Ir * HIDDEN
        # denominator: this GPU's NVFP4 rate from the library's own tcgen05 MMA loop
        # (outside the timed region); 4 x the measured cuBLAS bf16 burst is kept beside it
        peak, peak_cases = nvfp4_mma_peak(dev)
        achieved = fc1_flops / (fc1_ms * 1e-3) / 1e12
        fc2_tf = fc2_flops / (stage_avg["fc2"] * 1e-3) / 1e12
        roof = {"bound": "tensor", "kernel": "fc1 grouped GEMM (tcgen05 NVFP4, N tile 128)",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_kind": "self-measured tcgen05 NVFP4 MMA loop (best MMA-only case of "
                             "glmaxx_nvfp4_mma_peak_launch, one CTA per SM)",
                "nvfp4_peak_cases": peak_cases,
                "frac_of_4x_bf16": achieved / (NVFP4_PER_BF16 * bf16_peak),
                "frac_of_nominal_9pf": achieved / NVFP4_NOMINAL_TFLOPS,
                "traffic": None, "algorithmic_flops_per_launch": fc1_flops,
                "fc2_tflops": fc2_tf, "fc2_frac": fc2_tf / peak,
                "routed_tflops": (fc1_flops + fc2_flops) / (ms * 1e-3) / 1e12,
                "expert_counts": {"max": int(counts.max()), "min": int(counts.min()),
                                  "zero": int((counts == 0).sum())}}
        if zipf is not None:
            roof["zipf_beta"], roof["zipf_slope"] = zipf
    roof.update({"touched_experts": touched, "fc1_ms": fc1_ms, "layer_weight_bytes": layer_bytes,
                 "layer_achieved_gbs": layer_bytes / (ms * 1e-3) / 1e9,
                 "layer_frac_hbm": layer_bytes / (ms * 1e-3) / 1e9 / hbm_peak})

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            if codec == "hybrid":
                cpu = {"value": None, "unit": UNIT,
                       "note": "see the decode and exl3 workloads' baselines (per codec)"}
            else:
                cpu = cpu_baseline(layer.w, cfg, codec, x, args.workload, args.seed)
        except Exception as exc:  # noqa: BLE001
            cpu = {"value": None, "unit": UNIT, "error": repr(exc)[:200]}

    if reduce_info is not None and n_layers == 1:
        # the part of the step the reduce adds on top of the layer's own stages
        # (stage times: eager launches of the whole step's layer on this rank)
        layer_ms = sum(stage_avg.values())
        reduce_info["layer_stages_ms"] = layer_ms
        reduce_info["exposed_us"] = (ms - layer_ms) * 1e3
        reduce_info["chunks"] = chunks
    if rank == 0:
        line = {
            "metric": wl["metric"], "value": T / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, N(0,0.01) bias"
                    + (", Zipf-skewed bias)" if zipf is not None else ")"),
            "config": {"workload": wl["name"], "tokens": T,
                       "hidden": HIDDEN, "experts": EXPERTS, "top_k": TOPK, "groups": 8,
                       "topk_groups": 4, "intermediate": INTER, "shared_intermediate": INTER,
                       "parallelism": f"tp{world} (expert intermediate sharded, "
                                      + ("fused peer-memory finish over NVLink" if use_peer
                                         else "NCCL all-reduce")
                                      + (", token-split routing + NCCL route all-gather)"
                                         if split else ")"),
                       "routed_combine": ("slot plane + expert-order combine"
                                          if deterministic or T <= 256 or codec is not None
                                          else "fp32 atomics into the output"),
                       "l2": "weights per step >> 126 MB L2 (no flush needed)",
                       "chunks": chunks,
                       "pipeline": (f"{chunks} token chunks; each chunk's peer finish runs on a "
                                    "second stream, overlapping the next chunk's layer"
                                    if chunks > 1 else "none"),
                       "timing": ("CUDA-graph replay of the layer and its peer finish"
                                  if use_peer else "CUDA-graph replay of the layer"
                                  + (" + eager NCCL all-reduce" if world > 1 else ""))
                                 + ", CUDA events on the launch stream, max over ranks"},
            "roofline": roof,
            "stage_ms": stage_avg,
            "reduce": reduce_info,
            "cpu_baseline": cpu,
            "e2e": {"value": T / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": T * HIDDEN * 2, "d2h_bytes_per_step": T * HIDDEN * 4,
                    "ms_per_step": e2e_ms,
                    "transfers": "pinned host buffers; each step's upload and download on "
                                 "copy streams overlap the neighbouring steps' compute"
                                 + ("; every rank uploads the input (h2d bytes are per rank), "
                                    "rank 0 alone reads the result, the same bits on every "
                                    "rank" if world > 1 else "")},
            "gpu_launches": None if kernels_per_step is None else kernels_per_step * args.steps,
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        # every CUDA graph that holds an NCCL call (the split router's all-gather)
        # must be gone before destroy_process_group, or the exit waits for ever
        del graph, gr
        graphs.clear()
        import gc
        gc.collect()
        torch.cuda.synchronize()
        if group is not None:
            outs, out, xs, rs = None, None, None, None
            group.close()
        dist.barrier()
        if routers is not None:
            # the NCCL communicator was used inside captured graphs: end the process
            # once every rank is past the barrier, without waiting on its teardown
            sys.stdout.flush()
            sys.stderr.flush()
            os._exit(0)
        dist.destroy_process_group()


def run_reference(args):
    """Reference arm: the reference's CPU implementation of the path on this box's host
    cores.  No Rust toolchain exists here, so it is the C restatement in oracle/
    (which reproduces the reference's golden vectors) -- the router, the routed
    experts and the shared expert of one full layer, on the same seeded weights and
    inputs as our arm (generated by the same code, on cuda:0 when there is one), per
    the BASELINE CPU plan: configs[1] and [3] on all tokens, configs[2] on a seeded
    512-token subset, each expert dequantised once outside the timed region, OpenMP
    over assignments.  The reference's CPU path has no tensor parallelism, so at any
    N it computes the whole layer (the TP1 weights)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    import oracle as O
    from glmaxx_b200 import synth
    from glmaxx_b200.moe import MoEConfig

    wl = WORKLOADS[args.workload]
    codec = wl.get("codec")
    if codec == "hybrid":
        print(json.dumps({"impl": "reference", "metric": wl["metric"], "unavailable":
                          "the CPU arm times the per-codec workloads (decode, prefill, exl3); the "
                          "hybrid stack has no separate CPU arm"}), flush=True)
        return
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "reference", "metric": wl["metric"], "unavailable":
                          "needs cuda:0 to generate the same seeded weights as our arm (the "
                          "timed part runs on the host cores)"}), flush=True)
        return
    dev = torch.device("cuda", 0)
    T = args.tokens
    cfg = MoEConfig()
    beta = synth.fit_zipf_beta(cfg, T, args.seed, dev)[0] if wl["zipf"] else None
    if codec == "exl3":
        w = synth.make_exl3_rank_weights(cfg, seed=args.seed, device=dev, zipf_beta=beta)
    else:
        w = synth.make_rank_weights(cfg, seed=args.seed, device=dev, zipf_beta=beta)
    x = synth.make_input(T, HIDDEN, seed=args.seed, device=dev)
    sel = cpu_sample(T, args.workload, args.seed)
    cl = CpuLayer(w, cfg, codec, host_u16(x)[sel])

    # warm-up and timed steps stop early once REF_TIME_BUDGET_S is spent, so that the
    # arm ends within a few minutes whatever K and W are; "steps" reports the count run
    warm = min(args.warmup, 1)
    for _ in range(warm):
        cl.step()
    times = []
    t_start = time.perf_counter()
    touched = 0
    while len(times) < args.steps and (not times or
                                       time.perf_counter() - t_start < REF_TIME_BUDGET_S):
        busy, touched, _ = cl.step()
        times.append(busy)
    per_step = statistics.mean(times)
    value = len(sel) / per_step
    cores = int(O.lib().orc_threads())
    what = ("router + EXL3 gate/up/down (trellises decoded once per expert) + bf16 shared "
            "expert" if codec == "exl3" else
            "router + NVFP4 FC1/SwiGLU/FC2 (experts dequantised once) + bf16 shared expert")
    print(json.dumps({
        "impl": "reference", "metric": wl["metric"], "value": value, "unit": UNIT,
        "n_gpus": world, "steps": len(times), "steps_requested": args.steps,
        "warmup": warm, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic, the same seeded weights and inputs as our arm",
        "config": {"workload": wl["name"], "tokens": T,
                   "parallelism": "whole layer on one host process (the reference CPU path "
                                  "has no tensor parallelism)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{len(sel)} of {T} tokens per step ({touched} experts): "
                                   f"{what}; preparation {cl.prep.prep_s:.1f} s untimed, "
                                   f"experts {'held' if cl.prep.hold else 'rebuilt per step'}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


LOAD_LAYER = 3
LOAD_SAMPLE_EXPERTS = 16  # the CPU arms verify a 16-expert layer file (~90 MB)


def write_layer_file(path: Path, experts: int, rank: int, seed: int) -> int:
    """One TP4 rank file of one MoE layer (layer_file_builder); returns its size."""
    return layer_file_builder(experts, rank, seed).write(path, bytes(range(16)))


def layer_file_builder(experts: int, rank: int, seed: int):
    """RankFileBuilder of one TP4 rank file of one MoE layer: router (bf16
    [E, 6144]) and fp32 bias, per expert NVFP4 gate/up [1024, 6144] and down
    [6144, 512] (seeded random codes, E4M3 scales 0x30..0x3f, global scale =
    amax / 2688), bf16 shared expert shard."""
    import numpy as np

    from glmaxx_b200 import rank_file as R
    from glmaxx_b200.moe import MoEConfig

    cfg = MoEConfig(experts=experts, tp=4, rank=rank)
    H, Ir, Isr = cfg.hidden, cfg.local_intermediate, cfg.local_shared
    rng = np.random.default_rng(seed)
    pre = f"model.layers.{LOAD_LAYER}.mlp"
    recs = []

    def add(name, role, expert, axis, flags, payload):
        recs.append(R.TensorRecord(len(recs), name, role, LOAD_LAYER, expert, axis, flags, payload))

    def plain(n, k, dtype="bf16"):
        eb = 4 if dtype == "fp32" else 2
        return R.PlainTensor(dtype, 2 if k else 1, (n, k or 1, 1, 1), (n, k or 1, 1, 1),
                             rng.integers(0, 256, n * (k or 1) * eb, dtype=np.uint8))

    def nvfp4(n, k, e):
        amax = np.float32(1.0 + 0.01 * e)
        return R.Nvfp4Tensor(n, k, n, k, float(amax / np.float32(2688.0)), float(amax),
                             rng.integers(0, 256, n * k // 2, dtype=np.uint8),
                             rng.integers(0x30, 0x40, n * k // 16, dtype=np.uint8))

    add(f"{pre}.gate.weight", R.ROLE_ROUTER_WEIGHT, -1, -1, 1, plain(experts, H))
    add(f"{pre}.gate.e_score_correction_bias", R.ROLE_ROUTER_BIAS, -1, -1, 1,
        plain(experts, 0, "fp32"))
    for e in range(experts):
        add(f"{pre}.experts.{e}.gate_up_proj.weight", R.ROLE_ROUTED_GATE_UP, e, 0, 0b1010,
            nvfp4(2 * Ir, H, e))
        add(f"{pre}.experts.{e}.down_proj.weight", R.ROLE_ROUTED_DOWN, e, 1, 0b1100,
            nvfp4(H, Ir, e))
    for role, n, k, name, axis, flags in ((R.ROLE_SHARED_GATE, Isr, H, "gate_proj", 0, 0b10010),
                                          (R.ROLE_SHARED_UP, Isr, H, "up_proj", 0, 0b10010),
                                          (R.ROLE_SHARED_DOWN, H, Isr, "down_proj", 1, 0b10100)):
        add(f"{pre}.shared_experts.{name}.weight", role, -1, axis, flags, plain(n, k))
    manifest = ('{"rank":%d,"schema":"bench-layer"}' % rank).encode()
    return R.RankFileBuilder(rank, manifest, tensors=recs)


def oracle_load_rate(path: Path) -> tuple[float, float]:
    """The CPU restatement of the reader (oracle/rank_file.py: open + verify,
    one thread) over one file: (GB/s of payload, seconds)."""
    from oracle import rank_file as OR
    data = path.read_bytes()
    t0 = time.perf_counter()
    rd = OR.Reader(data)
    rd.verify()
    dt = time.perf_counter() - t0
    return (rd.pay_region[1] - rd.pay_region[0]) / dt / 1e9, dt


def run_load(args):
    """Rank-file load: the native reader verifies one TP4 rank file of one full
    MoE layer (~1.4 GB) and places every plane in HBM (load_moe_layers).  Wall
    clock around synchronised calls: the path is host-driven (read, SHA-256,
    pinned staging, cudaMemcpyAsync).  The file is page-cache resident."""
    import shutil

    import torch

    from glmaxx_b200 import rank_file as R
    from glmaxx_b200.moe import MoEConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if rank != 0:
        return  # one process measures; a node's ranks load together with --rank-files 4
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    wl = WORKLOADS["load"]
    tmp = Path(tempfile.mkdtemp(prefix="g5n-bench-"))
    try:
        cfg = MoEConfig(tp=4, rank=rank % 4)
        path = tmp / f"glm52-native-v0-rank{cfg.rank}.g5n"
        t0 = time.perf_counter()
        size = write_layer_file(path, EXPERTS, cfg.rank, args.seed + rank)
        write_s = time.perf_counter() - t0
        node = None
        if args.rank_files == 4:
            node = load_node_rate(tmp, dev, args.seed + rank)
        # serial floor: one thread's SHA-256 over the payload; the PCIe copy for context
        buf = torch.empty(512 << 20, dtype=torch.uint8).numpy()
        buf[:] = 7
        sha_gbs = max(buf.nbytes / (lambda t: (R.sha256(buf), time.perf_counter() - t)[1])(
            time.perf_counter()) / 1e9 for _ in range(3))
        pinned = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
        dst = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h2d = []
        for _ in range(3):
            e0.record()
            dst.copy_(pinned, non_blocking=True)
            e1.record()
            e1.synchronize()
            h2d.append(pinned.numel() / (e0.elapsed_time(e1) * 1e-3) / 1e9)
        del pinned, dst
        with R.NativeRankReader.open(path) as rd:
            payload = rd.file_payload_bytes()
            t = time.perf_counter()
            rd.verify()
            verify_gbs = payload / (time.perf_counter() - t) / 1e9
            warm, steps = 3, max(1, min(args.steps, 8))
            for _ in range(warm):
                loaded, _ = R.load_moe_layers(rd, cfg, [LOAD_LAYER], device=dev)
                del loaded
            uuid = None
            try:
                uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
            except Exception:  # noqa: BLE001
                pass
            clocks = ClockSampler(uuid)
            clocks.start()
            wall, native, placed = [], [], 0
            for _ in range(steps):
                torch.cuda.synchronize()
                t = time.perf_counter()
                loaded, proof = R.load_moe_layers(rd, cfg, [LOAD_LAYER], device=dev)
                torch.cuda.synchronize()
                wall.append(time.perf_counter() - t)
                native.append(proof.elapsed_nanoseconds * 1e-9)
                placed = proof.device_bytes
                del loaded
            clock_info = clocks.stop()
        value = payload / statistics.median(native) / 1e9
        e2e = payload / statistics.median(wall) / 1e9
        cpu = None
        if not args.no_cpu_baseline and rank == 0:
            small = tmp / "sample.g5n"
            write_layer_file(small, LOAD_SAMPLE_EXPERTS, cfg.rank, args.seed + 99)
            rate, secs = oracle_load_rate(small)
            cpu = {"value": rate, "unit": "GB/s", "cores": 1, "kind": "port",
                   "sample": f"oracle reader (open + verify) over a {LOAD_SAMPLE_EXPERTS}-expert "
                             f"layer file ({small.stat().st_size / 1e6:.0f} MB, {secs:.1f} s)"}
        if rank == 0:
            print(json.dumps({
                "metric": wl["metric"], "value": value, "unit": "GB/s", "n_gpus": 1,
                "launched_ranks": world,
                "steps": steps, "warmup": warm, "ms_per_step": statistics.median(native) * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
                "data": "synthetic (seeded NVFP4 codes and scales, written by RankFileBuilder)",
                "config": {"workload": wl["name"], "file_bytes": size, "payload_bytes": payload,
                           "tensors": 2 * EXPERTS + 5, "write_s": round(write_s, 2),
                           "page_cache": "resident (file just written)",
                           "rank_set": node,
                           "timing": "wall clock around synchronised calls (host-driven path)"},
                "roofline": {"bound": wl["bound"], "achieved": value, "peak": sha_gbs,
                             "unit": "GB/s", "frac": value / sha_gbs, "traffic": None,
                             "peak_kind": "one host thread's SHA-256 rate measured here (the "
                                          "whole-payload digest is one serial stream)",
                             "h2d_pinned_gbs": statistics.median(h2d),
                             "verify_only_gbs": verify_gbs},
                "cpu_baseline": cpu,
                "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": placed,
                        "d2h_bytes_per_step": 0,
                        "note": "load_moe_layers: allocation, zero fill, verify, placement"},
                "gpu_launches": 0, "clocks": clock_info}), flush=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def load_node_rate(tmp: Path, dev, seed: int) -> dict:
    """Four TP4 rank files of one layer (ranks 0-3, as one node holds them)
    validated as a set and loaded concurrently (load_rank_set, one thread per
    file) into this GPU: aggregate payload GB/s over 3 timed loads."""
    import torch

    from glmaxx_b200 import rank_file as R
    from glmaxx_b200.moe import MoEConfig
    builders = [layer_file_builder(EXPERTS, r, seed + 17 * r) for r in range(4)]
    conv = R.RankFileBuilder.derive_conversion_uuid(builders)  # covers all four files
    paths = [tmp / f"node-rank{r}.g5n" for r in range(4)]
    for b, p in zip(builders, paths):
        b.write(p, conv)
    del builders
    cfgs = [MoEConfig(tp=4, rank=r) for r in range(4)]
    rates, payload = [], 0
    for _ in range(4):
        torch.cuda.synchronize()
        t = time.perf_counter()
        out, proofs = R.load_rank_set(paths, cfgs, [LOAD_LAYER], [dev] * 4)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t
        payload = sum(p.payload_bytes for p in proofs)
        rates.append(payload / dt / 1e9)
        del out
    return {"files": 4, "payload_bytes": payload, "aggregate_gbs": statistics.median(rates[1:]),
            "note": "4 rank files verified and placed concurrently (one thread each)"}


def run_load_reference(args):
    """Reference arm of the load workload: the reader's CPU restatement (the
    reference reader is Rust; no toolchain here) over the sample file."""
    import shutil
    if int(os.environ.get("RANK", "0")) != 0:
        return
    tmp = Path(tempfile.mkdtemp(prefix="g5n-ref-"))
    try:
        path = tmp / "sample.g5n"
        write_layer_file(path, LOAD_SAMPLE_EXPERTS, 0, args.seed + 99)
        rates = [oracle_load_rate(path)[0] for _ in range(max(1, min(args.steps, 3)))]
        v = statistics.median(rates)
        print(json.dumps({
            "impl": "reference", "metric": WORKLOADS["load"]["metric"], "value": v,
            "unit": "GB/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": len(rates),
            "warmup": 0, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8", "data": "synthetic", "config": {"workload": WORKLOADS["load"]["name"]},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": 1, "kind": "port",
                             "sample": f"{LOAD_SAMPLE_EXPERTS}-expert layer file"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def main():
    args = parse()
    if args.workload == "nvfp4-peak":
        run_nvfp4_peak(args)
    elif args.workload == "load":
        run_load_reference(args) if args.impl == "reference" else run_load(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
