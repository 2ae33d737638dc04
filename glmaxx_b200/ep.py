"""Expert-parallel routed-MoE step: the all-to-all alternative to the reference's
tensor-parallel layout (crates/glm-engine/src/manifest.rs:143-165 shards the
expert intermediate; here whole experts are owned by ranks).  This is not a
reference layout, so it adds no arithmetic: every expert row is the TP1 layer's
row, and the step's output equals the TP1 layer's output on the same tokens.

Experts are split in contiguous blocks over N ranks (rank d owns experts
[d*E/N, (d+1)*E/N), with the full intermediate); tokens are split over ranks as
data.  A step on every rank (glmaxx_moe_ep_dispatch_launch and
glmaxx_moe_ep_return_launch, include/glmaxx_kernel.h):

1. route its tokens (glmaxx_router_compact_launch): dense routes, and the
   assignments compacted by expert -- hence grouped by owner;
2. exchange the per-owner row counts (a host all-gather of N x N counts);
3. dispatch every assignment row (bf16 token row, owner-local expert, routing
   weight, source) into its owner's receive buffers;
4. as owner, run the layer over the received rows (routes given, top_k 1, its own
   experts), which gives each row's routing-weighted expert output;
5. return every output row into its source's slot plane [tokens][top_k][hidden];
6. as source, run the layer with GLMAXX_MOE_EXTERNAL_ROUTED: the shared expert and
   the expert-order combine of the plane.

Receive buffers and planes live in a PeerGroup (CUDA IPC) across processes, or in
one process's memory for the single-GPU emulation the tests use.  Exchanges move
rows with plain 16-byte loads and stores.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import abi
from .moe import MoEConfig, PackedNvfp4, RankWeights, RoutedMoE


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def owner_counts(expert_offsets: np.ndarray, ranks: int) -> np.ndarray:
    """Rows a source sends to each owner: the compacted rows of the owner's
    expert block, from the source's expert_offsets [E + 1]."""
    e = len(expert_offsets) - 1
    per = e // ranks
    off = np.asarray(expert_offsets, np.int64)
    return np.array([off[(d + 1) * per] - off[d * per] for d in range(ranks)], np.int64)


def dest_row_offsets(counts: np.ndarray, source: int) -> np.ndarray:
    """First row of `source`'s block in every owner's receive buffers: the rows
    the lower ranks send to that owner (counts[s][d] = rows s sends to d)."""
    return np.asarray(counts, np.int64)[:source].sum(axis=0)


def received_rows(counts: np.ndarray, owner: int) -> int:
    return int(np.asarray(counts, np.int64)[:, owner].sum())


def expert_block(weights: RankWeights, ranks: int, rank: int) -> RankWeights:
    """Rank `rank`'s experts (a contiguous block of E / ranks) of TP1 layer weights,
    with the replicated router and shared expert."""
    e = weights.w13.values.shape[0]
    per = e // ranks
    sl = slice(rank * per, (rank + 1) * per)

    def part(p: PackedNvfp4) -> PackedNvfp4:
        return PackedNvfp4(p.values[sl].contiguous(), p.scales[sl].contiguous(),
                           p.global_scale[sl].contiguous(), p.global_amax[sl].contiguous(),
                           p.n, p.k)
    return RankWeights(weights.router_weight, weights.router_bias, part(weights.w13),
                       part(weights.w2), weights.shared13, weights.shared2)


BUFFERS = ("recv_x", "recv_expert", "recv_weight", "recv_source", "plane")


def buffer_specs(cfg: MoEConfig, max_tokens: int, capacity: int) -> dict:
    """{name: (shape, dtype)} of one rank's exchange buffers."""
    h, k = cfg.hidden, cfg.top_k
    return {"recv_x": ((capacity, h), torch.bfloat16),
            "recv_expert": ((capacity,), torch.int16),
            "recv_weight": ((capacity,), torch.float32),
            "recv_source": ((capacity,), torch.int32),
            "plane": ((max_tokens, k, h), torch.float32)}


class LocalTables:
    """Every rank's exchange buffers in this process's memory (the single-GPU
    emulation of an N-rank group: the same kernels, local pointers)."""

    def __init__(self, specs: dict, ranks: int, device):
        self.ranks = ranks
        self.bufs = [{n: torch.zeros(shape, dtype=dt, device=device)
                      for n, (shape, dt) in specs.items()} for _ in range(ranks)]

    def tensor(self, name: str, rank: int) -> torch.Tensor:
        return self.bufs[rank][name]

    def pointers(self, name: str) -> list[int]:
        return [b[name].data_ptr() for b in self.bufs]


class PeerTables:
    """Every rank's exchange buffers mapped through a PeerGroup (one process per
    GPU); this rank's tensors are views of its own block."""

    def __init__(self, group):
        self.group = group
        self.ranks = group.ranks

    def tensor(self, name: str, rank: int) -> torch.Tensor:
        assert rank == self.group.rank
        return self.group.tensor(name)

    def pointers(self, name: str) -> list[int]:
        return self.group.pointers(name)


class EpRank:
    """One rank of an expert-parallel group: routes and combines its own tokens,
    owns the expert block [rank*E/N, (rank+1)*E/N)."""

    def __init__(self, cfg: MoEConfig, weights: RankWeights, ranks: int, rank: int,
                 max_tokens: int, capacity: int, tables, device):
        if cfg.tp != 1 or cfg.experts % ranks:
            raise ValueError("expert parallelism needs the TP1 geometry and E % ranks == 0")
        self.cfg, self.ranks, self.rank = cfg, ranks, rank
        self.max_tokens, self.capacity, self.tables, self.device = max_tokens, capacity, tables, device
        per = cfg.experts // ranks
        self.L = abi.load()
        block = expert_block(weights, ranks, rank)
        self.owner = RoutedMoE(MoEConfig(hidden=cfg.hidden, experts=per,
                                         intermediate=cfg.intermediate, top_k=1, groups=1,
                                         topk_groups=1, shared_intermediate=0),
                               RankWeights(None, None, block.w13, block.w2), capacity, device)
        self.source = RoutedMoE(cfg, RankWeights(weights.router_weight, weights.router_bias,
                                                 None, None, weights.shared13, weights.shared2),
                                max_tokens, device)
        t, k, e = max_tokens, cfg.top_k, cfg.experts
        self.route_experts = torch.empty((t, k), dtype=torch.int16, device=device)
        self.route_weights = torch.empty((t, k), dtype=torch.float32, device=device)
        self.comp_tokens = torch.empty(t * k, dtype=torch.int32, device=device)
        self.comp_experts = torch.empty(t * k, dtype=torch.int16, device=device)
        self.comp_slots = torch.empty(t * k, dtype=torch.uint8, device=device)
        self.comp_weights = torch.empty(t * k, dtype=torch.float32, device=device)
        self.offsets = torch.empty(e + 1, dtype=torch.int32, device=device)
        self.status = torch.zeros(4, dtype=torch.int32, device=device)
        self.rows_out = torch.empty((capacity, cfg.hidden), dtype=torch.float32, device=device)
        self._router_ws = {}
        self.tokens = 0

    # ------------------------------------------------------------------ phases
    def route(self, x: torch.Tensor) -> None:
        """Phase 1: router + compaction of this rank's tokens."""
        c = self.cfg
        t = x.shape[0]
        assert 0 < t <= self.max_tokens and x.is_contiguous()
        self.tokens, self.x = t, x
        need = int(self.L.glmaxx_router_workspace_bytes(t, c.hidden, c.experts, c.top_k))
        ws = self._router_ws.get(t)
        if ws is None:
            ws = self._router_ws[t] = torch.empty(need, dtype=torch.uint8, device=self.device)
        w = self.source.w
        d = abi.RouterDescriptor.new(
            abi_version=abi.ROUTER_ABI_VERSION, tokens=t, hidden=c.hidden, experts=c.experts,
            top_k=c.top_k, groups=c.groups, topk_groups=c.topk_groups,
            route_scale=c.route_scale, input_bf16=x.data_ptr(),
            router_weight_bf16=w.router_weight.data_ptr(), router_bias_f32=w.router_bias.data_ptr(),
            route_experts_u16=self.route_experts.data_ptr(),
            route_weights_f32=self.route_weights.data_ptr(),
            compacted_tokens_u32=self.comp_tokens.data_ptr(),
            compacted_experts_u16=self.comp_experts.data_ptr(),
            compacted_slots_u8=self.comp_slots.data_ptr(),
            compacted_weights_f32=self.comp_weights.data_ptr(),
            expert_offsets_u32=self.offsets.data_ptr(), validation_error_u32=self.status.data_ptr(),
            workspace=ws.data_ptr(), workspace_bytes=ws.numel())
        err = ctypes.c_int32(0)
        abi.check(self.L.glmaxx_router_compact_launch(ctypes.byref(d), ctypes.c_void_p(_stream()),
                                                      ctypes.byref(err)), "router_compact")

    def counts(self) -> np.ndarray:
        """Phase 2 input: rows this rank sends to every owner (synchronises)."""
        return owner_counts(self.offsets.cpu().numpy(), self.ranks)

    def _descriptor(self, **kw) -> abi.MoeEpDescriptor:
        c = self.cfg
        d = abi.MoeEpDescriptor.new(abi_version=abi.MOE_EP_ABI_VERSION, ranks=self.ranks,
                                    rank=self.rank, hidden=c.hidden, experts=c.experts,
                                    top_k=c.top_k, validation_error_u32=self.status.data_ptr(),
                                    **kw)
        for name, field in (("recv_x", "recv_x_bf16"), ("recv_expert", "recv_expert_u16"),
                            ("recv_weight", "recv_weight_f32"), ("recv_source", "recv_source_u32")):
            getattr(d, field)[:self.ranks] = self.tables.pointers(name)
        d.recv_capacity[:self.ranks] = [self.capacity] * self.ranks
        return d

    def dispatch(self, counts: np.ndarray) -> None:
        """Phase 3: this rank's assignment rows into their owners' receive buffers."""
        for dst in range(self.ranks):
            if received_rows(counts, dst) > self.capacity:
                raise abi.KernelError(f"owner {dst} would receive more than {self.capacity} rows",
                                      abi.ERR_DESCRIPTOR)
        d = self._descriptor(
            tokens=self.tokens, input_bf16=self.x.data_ptr(),
            compacted_tokens_u32=self.comp_tokens.data_ptr(),
            compacted_experts_u16=self.comp_experts.data_ptr(),
            compacted_slots_u8=self.comp_slots.data_ptr(),
            compacted_weights_f32=self.comp_weights.data_ptr(),
            expert_offsets_u32=self.offsets.data_ptr())
        d.dest_row_offset[:self.ranks] = [int(v) for v in dest_row_offsets(counts, self.rank)]
        abi.check(self.L.glmaxx_moe_ep_dispatch_launch(ctypes.byref(d), ctypes.c_void_p(_stream())),
                  "moe_ep_dispatch")

    def own(self, counts: np.ndarray, path: int = abi.DECODE_PERSISTENT) -> int:
        """Phase 4: the layer over the rows this rank received (its experts)."""
        rows = received_rows(counts, self.rank)
        if rows:
            tb = self.tables
            x = tb.tensor("recv_x", self.rank)[:rows]
            experts = tb.tensor("recv_expert", self.rank)[:rows].view(rows, 1)
            weights = tb.tensor("recv_weight", self.rank)[:rows].view(rows, 1)
            self.owner(x, self.rows_out[:rows], routes=(experts, weights), path=path)
        self.rows = rows
        return rows

    def give_back(self, plane_tokens: list[int]) -> None:
        """Phase 5: every received row's output into its source's slot plane."""
        if not self.rows:
            return
        d = self._descriptor(rows=self.rows, rows_out_f32=self.rows_out.data_ptr())
        d.planes_f32[:self.ranks] = self.tables.pointers("plane")
        d.plane_tokens[:self.ranks] = plane_tokens
        abi.check(self.L.glmaxx_moe_ep_return_launch(ctypes.byref(d), ctypes.c_void_p(_stream())),
                  "moe_ep_return")

    def combine(self, out: torch.Tensor | None = None, path: int = 0) -> torch.Tensor:
        """Phase 6: shared expert + expert-order combine of this rank's slot plane."""
        plane = self.tables.tensor("plane", self.rank)
        return self.source(self.x, out,
                           routes=(self.route_experts[:self.tokens],
                                   self.route_weights[:self.tokens]),
                           path=path, external_plane=plane)

    def device_status(self) -> list[str]:
        words = [int(self.status[0].item())]
        words += [int(self.owner.status[0].item()), int(self.source.status[0].item())]
        out = []
        for w in words:
            out += abi.decode_status(w)
        return out


@dataclass
class LocalEpGroup:
    """An N-rank expert-parallel group emulated in one process on one GPU (every
    rank's buffers local, phases run rank after rank on one stream)."""
    ranks: list

    def step(self, xs: list[torch.Tensor], path: int = 0) -> list[torch.Tensor]:
        for r, x in zip(self.ranks, xs):
            r.route(x)
        counts = np.stack([r.counts() for r in self.ranks])
        for r in self.ranks:
            r.dispatch(counts)
        for r in self.ranks:
            r.own(counts)
        plane_tokens = [r.tokens for r in self.ranks]
        for r in self.ranks:
            r.give_back(plane_tokens)
        return [r.combine(path=path) for r in self.ranks]


def make_local_group(cfg: MoEConfig, weights: RankWeights, ranks: int, max_tokens: int,
                     device) -> LocalEpGroup:
    """N emulated ranks over one set of TP1 layer weights; each owner's receive
    capacity holds every assignment of every rank."""
    capacity = ranks * max_tokens * cfg.top_k
    tables = LocalTables(buffer_specs(cfg, max_tokens, capacity), ranks, device)
    return LocalEpGroup([EpRank(cfg, weights, ranks, r, max_tokens, capacity, tables, device)
                         for r in range(ranks)])


def exchange_counts(local: np.ndarray, group=None) -> np.ndarray:
    """The N x N row-count matrix (row s: rows rank s sends to every owner) from
    every rank's own counts, over a torch.distributed group (host all-gather)."""
    import torch.distributed as dist
    n = dist.get_world_size(group)
    t = torch.as_tensor(np.asarray(local, np.int64))
    parts = [torch.zeros_like(t) for _ in range(n)]
    dist.all_gather(parts, t, group=group)
    return torch.stack(parts).numpy()


class DistEpGroup:
    """One process per GPU: this rank's EpRank, its exchange buffers mapped on
    every rank through a PeerGroup, the counts all-gathered over the process
    group, and a device synchronisation plus host barrier between the phases
    that read other ranks' writes (dispatch -> owner, return -> combine)."""

    def __init__(self, cfg: MoEConfig, weights: RankWeights, max_tokens: int, device,
                 group=None, count_group=None):
        import torch.distributed as dist

        from .peer import PeerGroup
        ranks = dist.get_world_size(group)
        rank = dist.get_rank(group)
        capacity = ranks * max_tokens * cfg.top_k
        self.group, self.count_group = group, count_group
        self.peer = PeerGroup(buffer_specs(cfg, max_tokens, capacity), group=group, device=device)
        self.rank = EpRank(cfg, weights, ranks, rank, max_tokens, capacity,
                           PeerTables(self.peer), device)

    def _sync(self):
        import torch.distributed as dist
        torch.cuda.synchronize(self.rank.device)
        dist.barrier(group=self.group)

    def step(self, x: torch.Tensor, path: int = 0) -> torch.Tensor:
        r = self.rank
        r.route(x)
        counts = exchange_counts(r.counts(), self.count_group)
        tokens = exchange_counts(np.array([x.shape[0]], np.int64), self.count_group)[:, 0]
        r.dispatch(counts)
        self._sync()
        r.own(counts)
        r.give_back([int(t) for t in tokens])
        self._sync()
        return r.combine(path=path)

    def close(self):
        self.peer.close()
