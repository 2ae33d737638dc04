"""Host-side routed-MoE layer on the C ABI (the "glm-cuda backend" of this repo).

Mirrors the reference operator surface for the routed-expert step
(crates/glm-reference/src/routed_fc2.rs:93-109 operation order; weights in the
packed rank layout of crates/glm-reference/src/manifest.rs:143-165): a
``RoutedMoE`` owns one rank's NVFP4 expert shards, the bf16 shared-expert shard,
the replicated router and a device workspace, and runs the whole step with one
``glmaxx_moe_layer_launch`` call on the current CUDA stream.  torch supplies
device memory and streams only; all arithmetic is in libglmaxx_sm100.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import abi


def _ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


@dataclass
class MoEConfig:
    """Geometry of one rank's routed-MoE layer (GLM-5.2: hidden 6144, 256
    experts, top-8 over 8 groups / top-4 groups, intermediate 2048, x2.5)."""
    hidden: int = 6144
    experts: int = 256
    intermediate: int = 2048          # full expert intermediate (all ranks)
    top_k: int = 8
    groups: int = 8
    topk_groups: int = 4
    route_scale: float = 2.5
    shared_intermediate: int = 2048   # full shared-expert intermediate (0 = none)
    tp: int = 1
    rank: int = 0

    @property
    def local_intermediate(self) -> int:
        return self.intermediate // self.tp

    @property
    def local_shared(self) -> int:
        return self.shared_intermediate // self.tp


@dataclass
class PackedNvfp4:
    """Batch of NVFP4 tensors in the reference layout (nvfp4.rs:165-301):
    values [batch, n, k/2] u8 (even element low nibble), scales [batch, n*k/16]
    u8 in the 128x4 atom layout, global [batch] f32."""
    values: torch.Tensor
    scales: torch.Tensor
    global_scale: torch.Tensor
    global_amax: torch.Tensor
    n: int
    k: int


def pack_nvfp4(src: torch.Tensor) -> PackedNvfp4:
    """PackedNvfp4::pack (1-D codec) of [batch, n, k] f32/bf16 on the GPU
    (n % 128 == 0, k % 64 == 0), bit-exact with the reference codec."""
    if src.dim() == 2:
        src = src.unsqueeze(0)
    assert src.is_cuda and src.is_contiguous() and src.dtype in (torch.float32, torch.bfloat16)
    b, n, k = src.shape
    dev = src.device
    values = torch.empty((b, n, k // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((b, n * k // 16), dtype=torch.uint8, device=dev)
    gscale = torch.empty(b, dtype=torch.float32, device=dev)
    gamax = torch.empty(b, dtype=torch.float32, device=dev)
    scratch = torch.empty(max(b, 4), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    abi.check(abi.load().glmaxx_nvfp4_pack_launch(
        src.data_ptr(), int(src.dtype == torch.bfloat16), b, n, k, values.data_ptr(),
        scales.data_ptr(), gscale.data_ptr(), gamax.data_ptr(), scratch.data_ptr(),
        status.data_ptr(), ctypes.c_void_p(_stream())), "nvfp4_pack")
    word = int(status.item())
    if word:
        raise abi.KernelError(f"nvfp4_pack device status {abi.decode_status(word)}", word)
    return PackedNvfp4(values, scales, gscale, gamax, n, k)


@dataclass
class Exl3Experts:
    """One rank's EXL3 3-bit expert shards (glmaxx_moe_exl3_experts): trellises
    in the reference tile layout (exl3.rs) as int16 words, expert-major; fp16
    suh (input) / svh (output) scales; codec [E] uint8 (1 = EXL3, 0 = the
    NVFP4 weights) or None for an all-EXL3 layer."""
    gate_trellis: torch.Tensor   # [E, (H/16)*(I_r/16)*48] int16  (K = H, N = I_r)
    up_trellis: torch.Tensor     # [E, (H/16)*(I_r/16)*48] int16
    down_trellis: torch.Tensor   # [E, (I_r/16)*(H/16)*48] int16  (K = I_r, N = H)
    gate_suh: torch.Tensor       # [E, H] f16
    gate_svh: torch.Tensor       # [E, I_r] f16
    up_suh: torch.Tensor         # [E, H] f16
    up_svh: torch.Tensor         # [E, I_r] f16
    down_suh: torch.Tensor       # [E, I_r] f16
    down_svh: torch.Tensor       # [E, H] f16
    codec: torch.Tensor | None = None


@dataclass
class RankWeights:
    """One rank's layer weights (device tensors)."""
    router_weight: torch.Tensor          # [E, H] bf16 (replicated)
    router_bias: torch.Tensor            # [E] f32 (replicated)
    w13: PackedNvfp4 | None              # [E] x [2*I_r, H]: rank gate rows then up rows
    w2: PackedNvfp4 | None               # [E] x [H, I_r]
    shared13: torch.Tensor | None = None  # [2*Is_r, H] bf16
    shared2: torch.Tensor | None = None   # [H, Is_r] bf16
    exl3: Exl3Experts | None = None       # EXL3 experts (all, or those codec selects)


class RoutedMoE:
    """One rank's routed-MoE step (router, compaction, NVFP4 FC1+SwiGLU, FC2 +
    weighted combine, shared expert) for up to ``max_tokens`` tokens."""

    def __init__(self, cfg: MoEConfig, weights: RankWeights, max_tokens: int,
                 device: torch.device | None = None, deterministic: bool = False):
        """deterministic: GLMAXX_MOE_DETERMINISTIC -- prefill-size steps combine the
        routed rows through the slot plane in expert order (bit-reproducible)
        instead of fp32 atomics."""
        self.cfg = cfg
        self.deterministic = deterministic
        self.w = weights
        self.device = device or weights.router_weight.device
        self.lib = abi.load()
        self.max_tokens = max_tokens
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._ws = {}
        self.route_experts = torch.empty((max_tokens, cfg.top_k), dtype=torch.int16,
                                         device=self.device)
        self.route_weights = torch.empty((max_tokens, cfg.top_k), dtype=torch.float32,
                                         device=self.device)

    def _descriptor(self, tokens: int, x: torch.Tensor, out: torch.Tensor,
                    routes_given: bool, path: int,
                    external_plane: torch.Tensor | None = None) -> abi.MoeLayerDescriptor:
        c, w = self.cfg, self.w
        flags = (abi.MOE_ROUTES_GIVEN if routes_given else 0)
        if external_plane is not None:
            flags |= abi.MOE_EXTERNAL_ROUTED
        if self.deterministic:
            flags |= abi.MOE_DETERMINISTIC
        if c.shared_intermediate and w.shared13 is not None:
            flags |= abi.MOE_SHARED_EXPERT
        xd = None
        if w.exl3 is not None:
            flags |= abi.MOE_EXL3_EXPERTS
            x3 = w.exl3
            xd = abi.MoeExl3Experts.new(
                abi_version=abi.MOE_EXL3_ABI_VERSION, bits=3, codec_u8=_ptr(x3.codec),
                gate_trellis_u16=_ptr(x3.gate_trellis), up_trellis_u16=_ptr(x3.up_trellis),
                down_trellis_u16=_ptr(x3.down_trellis), gate_suh_f16=_ptr(x3.gate_suh),
                gate_svh_f16=_ptr(x3.gate_svh), up_suh_f16=_ptr(x3.up_suh),
                up_svh_f16=_ptr(x3.up_svh), down_suh_f16=_ptr(x3.down_suh),
                down_svh_f16=_ptr(x3.down_svh))
        w13 = w.w13
        w2 = w.w2
        d = abi.MoeLayerDescriptor.new(
            abi_version=abi.MOE_LAYER_ABI_VERSION, flags=flags, path=path, tokens=tokens,
            hidden=c.hidden, experts=c.experts, local_intermediate=c.local_intermediate,
            top_k=c.top_k, groups=c.groups, topk_groups=c.topk_groups,
            route_scale=c.route_scale,
            shared_intermediate=c.local_shared if flags & abi.MOE_SHARED_EXPERT else 0,
            input_bf16=x.data_ptr(), router_weight_bf16=_ptr(w.router_weight),
            router_bias_f32=_ptr(w.router_bias),
            w13_values=_ptr(w13.values if w13 else None),
            w13_scales=_ptr(w13.scales if w13 else None),
            w13_global_f32=_ptr(w13.global_scale if w13 else None),
            w2_values=_ptr(w2.values if w2 else None), w2_scales=_ptr(w2.scales if w2 else None),
            w2_global_f32=_ptr(w2.global_scale if w2 else None), shared13_bf16=_ptr(w.shared13),
            shared2_bf16=_ptr(w.shared2), route_experts_u16=self.route_experts.data_ptr(),
            route_weights_f32=self.route_weights.data_ptr(), output_f32=out.data_ptr(),
            validation_error_u32=self.status.data_ptr(), sequence=1,
            exl3_experts=ctypes.addressof(xd) if xd is not None else 0,
            routed_plane_f32=_ptr(external_plane))
        d._exl3 = xd  # the library reads it through exl3_experts at launch
        need = int(self.lib.glmaxx_moe_layer_workspace_bytes(ctypes.byref(d)))
        key = (tokens, flags, path)
        ws = self._ws.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        d.workspace = ws.data_ptr()
        d.workspace_bytes = ws.numel()
        self._last, self._last_key = d, key
        return d

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None,
                routes: tuple[torch.Tensor, torch.Tensor] | None = None,
                path: int = 0, external_plane: torch.Tensor | None = None) -> torch.Tensor:
        """x: [T, H] bf16 -> fp32 rank partial [T, H] (routed + shared).
        routes: optional (experts [T, K] int16, weights [T, K] f32) to bypass the router.
        external_plane: [T, K, H] fp32 routed contributions computed elsewhere (expert
        parallelism): only the shared expert and the expert-order combine run."""
        if external_plane is not None:
            assert routes is not None, "the external plane needs the routes (combine order)"
            assert external_plane.dtype == torch.float32 and external_plane.is_contiguous()
        assert x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape[1] == self.cfg.hidden
        t = x.shape[0]
        assert t <= self.max_tokens
        if out is None:
            out = torch.empty((t, self.cfg.hidden), dtype=torch.float32, device=self.device)
        if routes is not None:
            # routes already in this layer's own buffers (a SplitRouter's output) are read in place
            if routes[0].data_ptr() != self.route_experts.data_ptr():
                self.route_experts[:t].copy_(routes[0])
            if routes[1].data_ptr() != self.route_weights.data_ptr():
                self.route_weights[:t].copy_(routes[1])
        d = self._descriptor(t, x, out, routes is not None, path, external_plane)
        err = ctypes.c_int32(0)
        abi.check(self.lib.glmaxx_moe_layer_launch(ctypes.byref(d), ctypes.c_void_p(_stream()),
                                                   ctypes.byref(err)), "moe_layer_launch")
        return out

    __call__ = forward

    def plane(self, name: str) -> torch.Tensor:
        """Device view of an intermediate workspace plane of the last forward()
        (glmaxx_moe_layer_plane), as raw bytes."""
        d = self._last
        addr, nbytes = ctypes.c_uint64(0), ctypes.c_uint64(0)
        abi.check(self.lib.glmaxx_moe_layer_plane(ctypes.byref(d), abi.PLANES[name],
                                                  ctypes.byref(addr), ctypes.byref(nbytes)),
                  f"plane {name}")
        ws = self._ws[self._last_key]
        off = addr.value - ws.data_ptr()
        return ws[off:off + nbytes.value]

    def device_status(self) -> list[str]:
        """Decode the device validation word of the last step (synchronises)."""
        return abi.decode_status(int(self.status[0].item()))

    def routes(self, tokens: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.route_experts[:tokens], self.route_weights[:tokens]


def finish(partials: list[torch.Tensor], residual: torch.Tensor,
           attention: torch.Tensor | None = None, out_f32: torch.Tensor | None = None,
           out_bf16: torch.Tensor | None = None, norm_bf16: torch.Tensor | None = None,
           hidden: int = 0, eps: float = 1e-6) -> None:
    """Sparse-layer finish (glmaxx_moe_finish_launch, finish_sparse_layer_oracle
    order): residual (fp32 or bf16) + attention[r] for each rank + partials[r] for
    each rank, in rank order, into out_f32 and/or out_bf16, and optionally the
    row-wise RMSNorm (rows of `hidden`) of the result into norm_bf16, on the
    current stream."""
    n = residual.numel()
    ptrs = (ctypes.c_uint64 * len(partials))(*[p.data_ptr() for p in partials])
    d = abi.MoeFinishDescriptor.new(
        abi_version=abi.MOE_FINISH_ABI_VERSION, ranks=len(partials), elements=n,
        residual_f32=residual.data_ptr() if residual.dtype == torch.float32 else 0,
        residual_bf16=residual.data_ptr() if residual.dtype == torch.bfloat16 else 0,
        attention_f32=_ptr(attention), partials_f32=ctypes.addressof(ptrs),
        output_f32=_ptr(out_f32), output_bf16=_ptr(out_bf16), norm_bf16=_ptr(norm_bf16),
        hidden=hidden, eps=eps)
    abi.check(abi.load().glmaxx_moe_finish_launch(ctypes.byref(d), ctypes.c_void_p(_stream())),
              "moe_finish_launch")
