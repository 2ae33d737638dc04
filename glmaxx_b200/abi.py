"""ctypes binding of libglmaxx_sm100.so (include/glmaxx_kernel.h).

This is the Python counterpart of the reference's Rust FFI block
(crates/glm-cuda/src/ffi.rs:21-151) and descriptor mirror
(crates/glm-cuda/src/abi.rs:95-191): plain structs, device addresses as
uint64, int32 status returns.  Importing this module loads the CUDA library;
there is no fallback -- a missing or unbuildable library raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libglmaxx_sm100.so"

FC1_ABI_VERSION = 1
FC2_ABI_VERSION = 1
EXL3_ABI_VERSION = 1
MOE_EXL3_ABI_VERSION = 1
MOE_FINISH_ABI_VERSION = 1
MOE_PEER_ABI_VERSION = 1
MOE_EP_ABI_VERSION = 1
PEER_ONE_SHOT, PEER_TWO_SHOT = 1, 2
ROUTER_ABI_VERSION = 3
MOE_LAYER_ABI_VERSION = 3
DECODE_PERSISTENT = 1
PREFILL_GROUPED = 2
ERR_NULL, ERR_DESCRIPTOR, ERR_WRONG_ARCH = -1, -2, -120
EXL3_GATE, EXL3_UP, EXL3_DOWN = 1, 2, 3
PLANES = {"fc1_output_bf16": 0, "row_token_u32": 1, "row_slot_u32": 2, "row_weight_f32": 3,
          "expert_offsets_u32": 4, "shared_f32": 5, "routed_f32": 6}
LAYER_STAGES = ["router", "compact", "quant", "fc1", "fc2_quant", "shared", "fc2", "combine"]
ROUTER_STATIC_SCRATCH_BYTES = 4 << 20
MOE_ROUTES_GIVEN = 1 << 0
MOE_SHARED_EXPERT = 1 << 1
MOE_EXL3_EXPERTS = 1 << 2
MOE_EXTERNAL_ROUTED = 1 << 3
MOE_DETERMINISTIC = 1 << 4

STATUS_BITS = {
    1 << 0: "route-token-out-of-range",
    1 << 1: "route-slot-out-of-range",
    1 << 2: "duplicate-token-slot",
    1 << 3: "expert-out-of-range",
    1 << 4: "route-weight-not-finite",
    1 << 5: "non-finite-input",
    1 << 6: "capacity-exceeded",
    1 << 8: "wait-timeout",
    1 << 9: "tmem-timeout",
    1 << 10: "peer-timeout",
}

u32, u64, f32 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float


class _Desc(ctypes.Structure):
    """Descriptor base.  Use ``Cls.new(**fields)``: the C side declares the
    structs alignas(16), so instances are placed at 16-byte aligned addresses."""

    @classmethod
    def new(cls, **kw):
        size = ctypes.sizeof(cls)
        buf = (ctypes.c_uint8 * (size + 16))()
        addr = (ctypes.addressof(buf) + 15) & ~15
        obj = cls.from_address(addr)
        obj._keepalive = buf
        ctypes.memset(addr, 0, size)
        obj.struct_bytes = size
        for k, v in kw.items():
            setattr(obj, k, v)
        return obj


class Fc1Descriptor(_Desc):
    """glmaxx_fc1_descriptor (glmaxx_kernel.h:22-57), 224 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "flags", "path", "rows",
                                   "assignments", "hidden", "local_gate_up",
                                   "local_intermediate", "experts", "top_k", "reserved0")] + \
        [(n, u64) for n in ("input_bf16", "expert_value_base", "expert_scale_base",
                            "expert_global_scales", "route_experts_u16", "route_tokens_u32",
                            "route_slots_u8", "route_weights_f32", "expert_offsets_u32",
                            "compacted_input_bf16", "activation_values", "activation_scales",
                            "activation_global_scales", "gate_up_accum_f32", "output_bf16",
                            "workspace_bytes", "sequence")] + [("reserved", u64 * 4),
                                                                ("_tail", ctypes.c_uint8 * 8)]


class Fc2Descriptor(_Desc):
    """glmaxx_fc2_descriptor (glmaxx_kernel.h:59-95), 224 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "flags", "path", "rows",
                                   "assignments", "hidden", "local_intermediate", "experts",
                                   "top_k", "reserved0", "reserved1")] + \
        [(n, u64) for n in ("input_bf16", "expert_value_base", "expert_scale_base",
                            "expert_global_scales", "route_experts_u16", "route_tokens_u32",
                            "route_slots_u8", "route_weights_f32", "expert_offsets_u32",
                            "activation_values", "activation_scales",
                            "activation_global_scales", "assignment_down_f32",
                            "token_output_f32", "slot_assignment_u32", "validation_error_u32",
                            "workspace_bytes", "sequence")] + [("reserved", u64 * 4)]


class Exl3Descriptor(_Desc):
    """glmaxx_exl3_descriptor (glmaxx_kernel.h:97-121), 144 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "flags", "projection", "rows",
                                   "logical_k", "logical_n", "bits")] + \
        [(n, u64) for n in ("input_f16", "trellis_u16", "suh_f16", "svh_f16",
                            "rotated_input_f16", "projected_f16", "output_f16",
                            "validation_error_u32", "workspace_bytes", "sequence")] + \
        [("reserved", u64 * 4)]


class RouterDescriptor(_Desc):
    """glmaxx_router_descriptor (new), 192 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "flags", "tokens", "hidden",
                                   "experts", "top_k", "groups", "topk_groups")] + \
        [("route_scale", f32), ("reserved0", u32 * 2)] + \
        [(n, u64) for n in ("input_bf16", "router_weight_bf16", "router_bias_f32",
                            "route_experts_u16", "route_weights_f32", "compacted_tokens_u32",
                            "compacted_experts_u16", "compacted_slots_u8",
                            "compacted_weights_f32", "expert_offsets_u32",
                            "validation_error_u32", "workspace", "workspace_bytes",
                            "sequence")] + [("reserved", u64 * 4)]


class MoeLayerDescriptor(_Desc):
    """glmaxx_moe_layer_descriptor (new), 240 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "flags", "path", "tokens",
                                   "hidden", "experts", "local_intermediate", "top_k", "groups",
                                   "topk_groups")] + \
        [("route_scale", f32), ("shared_intermediate", u32), ("reserved0", u32 * 3)] + \
        [(n, u64) for n in ("input_bf16", "router_weight_bf16", "router_bias_f32", "w13_values",
                            "w13_scales", "w13_global_f32", "w2_values", "w2_scales",
                            "w2_global_f32", "shared13_bf16", "shared2_bf16",
                            "route_experts_u16", "route_weights_f32", "output_f32",
                            "validation_error_u32", "workspace", "workspace_bytes",
                            "sequence", "exl3_experts", "routed_plane_f32")] + \
        [("reserved", u64 * 2)]


class MoeFinishDescriptor(_Desc):
    """glmaxx_moe_finish_descriptor (new), 112 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "flags", "ranks")] + \
        [(n, u64) for n in ("elements", "residual_f32", "residual_bf16", "attention_f32",
                            "partials_f32", "output_f32", "output_bf16", "norm_bf16")] + \
        [("hidden", u32), ("eps", f32), ("reserved", u64 * 3)]


class MoePeerDescriptor(_Desc):
    """glmaxx_moe_peer_descriptor (new), 80 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "flags", "rank")] + \
        [(n, u64) for n in ("signals_u32", "outputs_f32", "outputs_bf16", "norms_bf16",
                            "status_u32")] + [("reserved", u64 * 3)]


class MoeExl3Experts(_Desc):
    """glmaxx_moe_exl3_experts (new), 128 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "bits", "reserved0")] + \
        [(n, u64) for n in ("codec_u8", "gate_trellis_u16", "up_trellis_u16", "down_trellis_u16",
                            "gate_suh_f16", "gate_svh_f16", "up_suh_f16", "up_svh_f16",
                            "down_suh_f16", "down_svh_f16")] + [("reserved", u64 * 4)]


class MoeEpDescriptor(_Desc):
    """glmaxx_moe_ep_descriptor (new, expert parallelism), 560 bytes."""
    _fields_ = [(n, u32) for n in ("abi_version", "struct_bytes", "ranks", "rank", "tokens",
                                   "hidden", "experts", "top_k", "rows")] + \
        [("reserved0", u32 * 3)] + \
        [(n, u64) for n in ("input_bf16", "compacted_tokens_u32", "compacted_experts_u16",
                            "compacted_slots_u8", "compacted_weights_f32",
                            "expert_offsets_u32")] + \
        [(n, u64 * 8) for n in ("recv_x_bf16", "recv_expert_u16", "recv_weight_f32",
                                "recv_source_u32")] + \
        [("recv_capacity", u32 * 8), ("dest_row_offset", u32 * 8), ("rows_out_f32", u64),
         ("planes_f32", u64 * 8), ("plane_tokens", u32 * 8), ("validation_error_u32", u64),
         ("reserved", u64 * 4)]


EXPECTED_SIZES = {Fc1Descriptor: 224, Fc2Descriptor: 224, Exl3Descriptor: 144,
                  RouterDescriptor: 192, MoeLayerDescriptor: 240, MoeExl3Experts: 128,
                  MoeFinishDescriptor: 112, MoePeerDescriptor: 80, MoeEpDescriptor: 560}

_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)
_U64P = ctypes.POINTER(u64)
_U16P = ctypes.POINTER(ctypes.c_uint16)

# name -> (restype, argtypes); every symbol include/glmaxx_kernel.h declares.
SIGNATURES = {
    "glmaxx_nvfp4_routed_fc1_launch": (ctypes.c_int32, [_P, _P, _I32P]),
    "glmaxx_nvfp4_routed_fc1_graph_instantiate": (ctypes.c_int32, [_P, _P, _U64P]),
    "glmaxx_nvfp4_quantize_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_grouped_quantize_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_core_swiglu_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_dense_control_launch": (ctypes.c_int32, [_P, u32, _P, _I32P]),
    "glmaxx_nvfp4_grouped_control_launch": (ctypes.c_int32, [_P, _U16P, u32, _P, _I32P]),
    "glmaxx_nvfp4_grouped_core_swiglu_launch": (ctypes.c_int32, [_P, _U16P, u32, _P, _I32P]),
    "glmaxx_nvfp4_grouped_prepare_launch": (ctypes.c_int32, [_P, _U16P, u32, _P]),
    "glmaxx_nvfp4_grouped_prepared_control_launch": (ctypes.c_int32, [_P, u32, _P, _I32P]),
    "glmaxx_nvfp4_grouped_prepared_core_swiglu_launch": (ctypes.c_int32, [_P, u32, _P, _I32P]),
    "glmaxx_nvfp4_routed_fc2_launch": (ctypes.c_int32, [_P, _P, _I32P]),
    "glmaxx_nvfp4_fc2_quantize_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_fc2_grouped_quantize_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_fc2_core_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_fc2_reduce_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_fc2_dense_control_launch": (ctypes.c_int32, [_P, u32, _P, _I32P]),
    "glmaxx_nvfp4_fc2_grouped_control_launch": (ctypes.c_int32, [_P, _U16P, u32, _P, _I32P]),
    "glmaxx_exl3_projection_launch": (ctypes.c_int32, [_P, _P, _I32P]),
    "glmaxx_moe_finish_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_moe_finish_peer_launch": (ctypes.c_int32, [_P, _P, _P]),
    "glmaxx_moe_peer_signal_bytes": (u64, [u32]),
    "glmaxx_ipc_handle": (ctypes.c_int32, [u64, ctypes.POINTER(ctypes.c_uint8)]),
    "glmaxx_ipc_open": (ctypes.c_int32, [ctypes.POINTER(ctypes.c_uint8), _U64P]),
    "glmaxx_ipc_close": (ctypes.c_int32, [u64]),
    "glmaxx_exl3_gemv_launch": (ctypes.c_int32, [u64, u64, u32, u32, u32, u32, u64, _P]),
    "glmaxx_graph_exec_launch": (ctypes.c_int32, [u64, u64]),
    "glmaxx_graph_exec_destroy": (ctypes.c_int32, [u64]),
    "glmaxx_stream_begin_capture": (ctypes.c_int32, [u64]),
    "glmaxx_stream_end_capture": (ctypes.c_int32, [u64, _U64P]),
    "glmaxx_event_create": (ctypes.c_int32, [_U64P]),
    "glmaxx_event_record": (ctypes.c_int32, [u64, u64]),
    "glmaxx_event_synchronize": (ctypes.c_int32, [u64]),
    "glmaxx_event_elapsed_ms": (ctypes.c_int32, [u64, u64, ctypes.POINTER(f32)]),
    "glmaxx_event_destroy": (ctypes.c_int32, [u64]),
    "glmaxx_profiler_start": (ctypes.c_int32, []),
    "glmaxx_profiler_stop": (ctypes.c_int32, []),
    "glmaxx_nvtx_range_push": (ctypes.c_int32, [ctypes.c_char_p]),
    "glmaxx_nvtx_range_pop": (ctypes.c_int32, []),
    "glmaxx_nvfp4_routed_fc1_workspace_bytes": (u64, [u32]),
    "glmaxx_nvfp4_grouped_workspace_bytes": (u64, [u32]),
    "glmaxx_nvfp4_routed_fc2_workspace_bytes": (u64, [u32, u32]),
    "glmaxx_nvfp4_grouped_fc2_workspace_bytes": (u64, [u32, u32]),
    "glmaxx_exl3_projection_workspace_bytes": (u64, [u32, u32, u32]),
    "glmaxx_kernel_abi": (ctypes.c_char_p, []),
    "glmaxx_exl3_kernel_abi": (ctypes.c_char_p, []),
    "glmaxx_device_count": (ctypes.c_int32, [_I32P]),
    "glmaxx_device_bind": (ctypes.c_int32, [ctypes.c_int32, _I32P, _I32P, _U64P,
                                             ctypes.POINTER(ctypes.c_uint8)]),
    "glmaxx_device_memory_info": (ctypes.c_int32, [_U64P, _U64P]),
    "glmaxx_device_alloc": (ctypes.c_int32, [u64, _U64P]),
    "glmaxx_device_free": (ctypes.c_int32, [u64]),
    "glmaxx_pinned_alloc": (ctypes.c_int32, [u64, _U64P]),
    "glmaxx_pinned_free": (ctypes.c_int32, [u64]),
    "glmaxx_stream_create": (ctypes.c_int32, [_U64P]),
    "glmaxx_stream_destroy": (ctypes.c_int32, [u64]),
    "glmaxx_stream_query": (ctypes.c_int32, [u64, _I32P]),
    "glmaxx_stream_synchronize": (ctypes.c_int32, [u64]),
    "glmaxx_memcpy_h2d": (ctypes.c_int32, [u64, _P, u64, u64]),
    "glmaxx_memcpy_d2d": (ctypes.c_int32, [u64, u64, u64, u64]),
    "glmaxx_memcpy_d2h": (ctypes.c_int32, [_P, u64, u64, u64]),
    "glmaxx_memset_zero": (ctypes.c_int32, [u64, u64, u64]),
    "glmaxx_nvfp4_routed_fc1_workspace_bytes_v3": (u64, [u32] * 6),
    "glmaxx_nvfp4_routed_fc2_workspace_bytes_v3": (u64, [u32] * 6),
    "glmaxx_router_workspace_bytes": (u64, [u32] * 4),
    "glmaxx_moe_layer_workspace_bytes": (u64, [_P]),
    "glmaxx_router_compact_launch": (ctypes.c_int32, [_P, _P, _I32P]),
    "glmaxx_router_compact_launch_static": (ctypes.c_int32, [_P, _P, _I32P]),
    "glmaxx_moe_layer_launch": (ctypes.c_int32, [_P, _P, _I32P]),
    "glmaxx_moe_layer_set_stage_events": (ctypes.c_int32, [_U64P, u32]),
    "glmaxx_moe_layer_plane": (ctypes.c_int32, [_P, u32, _U64P, _U64P]),
    "glmaxx_peer_enable": (ctypes.c_int32, [ctypes.c_int32]),
    "glmaxx_moe_ep_dispatch_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_moe_ep_return_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_codec_selfcheck_launch": (ctypes.c_int32, [_P, _P]),
    "glmaxx_nvfp4_quotient_selfcheck_launch": (ctypes.c_int32, [_P, ctypes.c_uint32, _P, _P]),
    "glmaxx_nvfp4_mma_peak_launch": (ctypes.c_int32, [u32, u32, u32, u32, u32, u32, _P, _P, _P]),
    "glmaxx_nvfp4_pack_launch": (ctypes.c_int32, [u64, ctypes.c_int32, u32, u32, u32, u64, u64,
                                                  u64, u64, u64, u64, _P]),
}

_lib = None


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load the CUDA library, building it in-tree first if it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            if not build_if_missing:
                raise RuntimeError(f"{LIB_PATH} is missing; run python -m glmaxx_b200.build")
            from . import build as _build
            _build.build()
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class KernelError(RuntimeError):
    """A launch returned a non-zero status (crates/glm-cuda/src/abi.rs:686-698)."""

    def __init__(self, what: str, status: int):
        kinds = {-1: "null argument", -2: "invalid descriptor or workspace",
                 -120: "device is not compute capability 10.x"}
        super().__init__(f"{what}: status {status} ({kinds.get(status, 'cudaError')})")
        self.status = status


def check(status: int, what: str) -> None:
    if status != 0:
        raise KernelError(what, status)


def decode_status(word: int) -> list[str]:
    return [name for bit, name in STATUS_BITS.items() if word & bit]


def abi_string() -> str:
    return load().glmaxx_kernel_abi().decode()
