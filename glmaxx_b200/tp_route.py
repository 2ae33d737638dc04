"""Token-split routing for a tensor-parallel group.

In the reference's tensor-parallel layout (crates/glm-engine/src/manifest.rs:
143-165) every rank holds the whole router and routes every token of the step
(the router itself is specified at manifest.rs:166-194), so at prefill sizes the
router's T x E x H multiply-adds are repeated on every rank.  A token's route
depends on that token's row alone, so here rank r routes only its slice of the
step, tokens [r*T/N, (r+1)*T/N) (glmaxx_router_compact_launch on that slice),
and the group all-gathers the dense routes (experts u16 and weights f32, 6 bytes
per (token, slot)) before the layer runs with GLMAXX_MOE_ROUTES_GIVEN.  Every
rank then holds the same routes, bit for bit, as if it had routed all T tokens
itself: the router kernels compute each token's logits in one fixed order
whatever the token count, and selection is per token.

The exchange is one all-gather of a packed byte buffer per layer step
(T x top_k x 6 bytes in total: 384 KiB at T = 8192, top-8).  It pays where the
router's work is large against the collective's latency: from `min_slice`
tokens per rank on (the tiled router kernel's range); a decode step of 64
tokens routes on every rank as before.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import abi
from .moe import MoEConfig, RankWeights

# Tokens per rank from which the split pays (the large-T router kernel's range).
MIN_SLICE = 256


def split_pays(tokens: int, ranks: int, min_slice: int = MIN_SLICE) -> bool:
    """Whether a step of `tokens` over `ranks` routes token slices: more than one
    rank, an even split into slices of a multiple of 8 tokens (so each slice's
    weights start 16-byte aligned in its packed block), and at least `min_slice`
    tokens per rank."""
    return (ranks > 1 and tokens % ranks == 0 and (tokens // ranks) % 8 == 0
            and tokens // ranks >= min_slice)


def slice_bounds(tokens: int, ranks: int, rank: int) -> tuple[int, int]:
    """Token range [lo, hi) that `rank` routes."""
    if tokens % ranks:
        raise ValueError(f"{tokens} tokens do not split evenly over {ranks} ranks")
    s = tokens // ranks
    return rank * s, (rank + 1) * s


def unpack_routes(gathered: torch.Tensor, ranks: int, experts: torch.Tensor,
                  weights: torch.Tensor) -> None:
    """Scatter the all-gathered byte buffer [ranks][slice*top_k*6] -- rank r's
    block holds its slice's experts (int16), then their weights (f32) -- into
    dense routes experts [T, top_k] int16 and weights [T, top_k] f32."""
    n2 = experts.numel() * 2 // ranks
    blocks = gathered.view(ranks, gathered.numel() // ranks)
    experts.view(torch.uint8).view(ranks, n2).copy_(blocks[:, :n2])
    weights.view(torch.uint8).view(ranks, 2 * n2).copy_(blocks[:, n2:])


class SplitRouter:
    """Routes this rank's token slice and all-gathers the group's routes.

    `weights` needs the router weight and bias (the same on every rank).
    Calling it with the step's full input [T, H] returns (experts [T, K] int16,
    weights [T, K] f32) on every rank, ready for RoutedMoE.forward(routes=...);
    with out=layer.routes(max_tokens) they are the layer's own route buffers and
    forward() reads them without a copy.
    The launches go to the current stream, so a step can be captured in a CUDA
    graph (the all-gather is an NCCL collective on the process group)."""

    def __init__(self, cfg: MoEConfig, weights: RankWeights, tokens: int, rank: int,
                 ranks: int, device: torch.device, group=None,
                 out: tuple[torch.Tensor, torch.Tensor] | None = None):
        self.cfg, self.w, self.tokens = cfg, weights, tokens
        self.rank, self.ranks, self.group, self.device = rank, ranks, group, device
        self.lo, self.hi = slice_bounds(tokens, ranks, rank)
        s, k, e = self.hi - self.lo, cfg.top_k, cfg.experts
        if s % 8:
            raise ValueError("token slices must be a multiple of 8 tokens")
        self.slice_tokens = s
        self.L = abi.load()
        # this rank's packed routes: experts (2 bytes) then weights (4 bytes) per slot
        self.packed = torch.empty(6 * s * k, dtype=torch.uint8, device=device)
        self.gathered = torch.empty(ranks * 6 * s * k, dtype=torch.uint8, device=device)
        self.comp_tokens = torch.empty(s * k, dtype=torch.int32, device=device)
        self.comp_experts = torch.empty(s * k, dtype=torch.int16, device=device)
        self.comp_slots = torch.empty(s * k, dtype=torch.uint8, device=device)
        self.comp_weights = torch.empty(s * k, dtype=torch.float32, device=device)
        self.offsets = torch.empty(e + 1, dtype=torch.int32, device=device)
        self.status = torch.zeros(4, dtype=torch.int32, device=device)
        need = int(self.L.glmaxx_router_workspace_bytes(s, cfg.hidden, e, k))
        self.ws = torch.empty(need, dtype=torch.uint8, device=device)
        # the gathered routes land here: by default new buffers, or (out) the
        # layer's own route buffers, which RoutedMoE.forward then reads in place
        if out is None:
            out = (torch.empty((tokens, k), dtype=torch.int16, device=device),
                   torch.empty((tokens, k), dtype=torch.float32, device=device))
        self.experts, self.weights = out[0][:tokens], out[1][:tokens]

    def route_slice(self, x: torch.Tensor) -> None:
        """glmaxx_router_compact_launch over tokens [lo, hi) of x, its dense routes
        written into this rank's packed buffer."""
        c = self.cfg
        assert x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape == (self.tokens, c.hidden)
        n = self.slice_tokens * c.top_k
        d = abi.RouterDescriptor.new(
            abi_version=abi.ROUTER_ABI_VERSION, tokens=self.slice_tokens, hidden=c.hidden,
            experts=c.experts, top_k=c.top_k, groups=c.groups, topk_groups=c.topk_groups,
            route_scale=c.route_scale, input_bf16=x[self.lo:self.hi].data_ptr(),
            router_weight_bf16=self.w.router_weight.data_ptr(),
            router_bias_f32=self.w.router_bias.data_ptr(),
            route_experts_u16=self.packed.data_ptr(),
            route_weights_f32=self.packed.data_ptr() + 2 * n,
            compacted_tokens_u32=self.comp_tokens.data_ptr(),
            compacted_experts_u16=self.comp_experts.data_ptr(),
            compacted_slots_u8=self.comp_slots.data_ptr(),
            compacted_weights_f32=self.comp_weights.data_ptr(),
            expert_offsets_u32=self.offsets.data_ptr(), validation_error_u32=self.status.data_ptr(),
            workspace=self.ws.data_ptr(), workspace_bytes=self.ws.numel())
        err = ctypes.c_int32(0)
        abi.check(self.L.glmaxx_router_compact_launch(
            ctypes.byref(d), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
            ctypes.byref(err)), "router_compact (token slice)")

    def __call__(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        self.route_slice(x)
        dist.all_gather_into_tensor(self.gathered, self.packed, group=self.group)
        unpack_routes(self.gathered, self.ranks, self.experts, self.weights)
        return self.experts, self.weights

    def device_status(self) -> list[str]:
        return abi.decode_status(int(self.status[0].item()))
