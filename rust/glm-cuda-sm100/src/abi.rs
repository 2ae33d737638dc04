//! C structs and constants of `include/glmaxx_kernel.h` (the v3 routed-MoE ABI of
//! libglmaxx_sm100), field for field.  The three reference descriptors
//! (`Fc1Descriptor`, `Fc2Descriptor`, `Exl3Descriptor`) keep the layout of the
//! reference's `crates/glm-cuda/src/abi.rs:95-191` and are not repeated here; the
//! structs below are the entry points the reference does not have.

/// ABI string of this library (`glmaxx_kernel_abi()`).
pub const KERNEL_ABI: &str = "glmaxx.sm100.nvfp4.routed_moe.v3";

pub const ROUTER_ABI_VERSION: u32 = 3;
pub const MOE_LAYER_ABI_VERSION: u32 = 3;
pub const MOE_EXL3_ABI_VERSION: u32 = 1;
pub const MOE_FINISH_ABI_VERSION: u32 = 1;
pub const MOE_PEER_ABI_VERSION: u32 = 1;
pub const MOE_EP_ABI_VERSION: u32 = 1;

/// `path` of [`MoeLayerDescriptor`]: 0 picks by token count.
pub const PATH_AUTO: u32 = 0;
pub const PATH_DECODE_PERSISTENT: u32 = 1;
pub const PATH_PREFILL_GROUPED: u32 = 2;

/// `flags` of [`MoeLayerDescriptor`].
pub const MOE_ROUTES_GIVEN: u32 = 1 << 0;
pub const MOE_SHARED_EXPERT: u32 = 1 << 1;
pub const MOE_EXL3_EXPERTS: u32 = 1 << 2;
pub const MOE_EXTERNAL_ROUTED: u32 = 1 << 3;
/// Routed contributions through the per-slot plane and the expert-order combine
/// at every token count (bit-reproducible prefill).
pub const MOE_DETERMINISTIC: u32 = 1 << 4;

/// `flags` of [`MoePeerDescriptor`].
pub const MOE_PEER_ONE_SHOT: u32 = 1;
pub const MOE_PEER_TWO_SHOT: u32 = 2;

/// Return codes (0 = success; positive values are `cudaError_t`).
pub const ERR_NULL: i32 = -1;
pub const ERR_DESCRIPTOR: i32 = -2;
pub const ERR_WRONG_ARCH: i32 = -120;

/// Device status bits (`validation_error_u32`); bits 0-4 keep the reference's
/// meaning (`kernels/sm120/nvfp4_routed_fc2.cu:33-39`).
pub const STATUS_ROUTE_TOKEN_OUT_OF_RANGE: u32 = 1 << 0;
pub const STATUS_ROUTE_SLOT_OUT_OF_RANGE: u32 = 1 << 1;
pub const STATUS_DUPLICATE_TOKEN_SLOT: u32 = 1 << 2;
pub const STATUS_EXPERT_OUT_OF_RANGE: u32 = 1 << 3;
pub const STATUS_ROUTE_WEIGHT_NOT_FINITE: u32 = 1 << 4;
pub const STATUS_NON_FINITE_INPUT: u32 = 1 << 5;
pub const STATUS_CAPACITY_EXCEEDED: u32 = 1 << 6;
pub const STATUS_WAIT_TIMEOUT: u32 = 1 << 8;
pub const STATUS_TMEM_TIMEOUT: u32 = 1 << 9;
pub const STATUS_PEER_TIMEOUT: u32 = 1 << 10;

/// Largest scratch need (`glmaxx_router_workspace_bytes`) the allocation-free
/// router accepts: 256 experts at top-8 fit up to 507 tokens.
pub const ROUTER_STATIC_SCRATCH_BYTES: u64 = 4 << 20;

/// `glmaxx_router_descriptor` (192 bytes): router + stable compaction.
#[repr(C, align(16))]
#[derive(Clone, Copy, Debug, Default)]
pub struct RouterDescriptor {
    pub abi_version: u32,
    pub struct_bytes: u32,
    pub flags: u32,
    pub tokens: u32,
    pub hidden: u32,
    pub experts: u32,
    pub top_k: u32,
    pub groups: u32,
    pub topk_groups: u32,
    pub route_scale: f32,
    pub reserved0: [u32; 2],
    pub input_bf16: u64,
    pub router_weight_bf16: u64,
    pub router_bias_f32: u64,
    pub route_experts_u16: u64,
    pub route_weights_f32: u64,
    pub compacted_tokens_u32: u64,
    pub compacted_experts_u16: u64,
    pub compacted_slots_u8: u64,
    pub compacted_weights_f32: u64,
    pub expert_offsets_u32: u64,
    pub validation_error_u32: u64,
    pub workspace: u64,
    pub workspace_bytes: u64,
    pub sequence: u64,
    pub reserved: [u64; 4],
}

/// `glmaxx_moe_exl3_experts` (128 bytes): a layer's EXL3 3-bit experts,
/// expert-major device arrays; `codec_u8` (device, `[experts]`, 0 = NVFP4,
/// 1 = EXL3) or 0 for an all-EXL3 layer.
#[repr(C, align(16))]
#[derive(Clone, Copy, Debug, Default)]
pub struct MoeExl3Experts {
    pub abi_version: u32,
    pub struct_bytes: u32,
    pub bits: u32,
    pub reserved0: u32,
    pub codec_u8: u64,
    pub gate_trellis_u16: u64,
    pub up_trellis_u16: u64,
    pub down_trellis_u16: u64,
    pub gate_suh_f16: u64,
    pub gate_svh_f16: u64,
    pub up_suh_f16: u64,
    pub up_svh_f16: u64,
    pub down_suh_f16: u64,
    pub down_svh_f16: u64,
    pub reserved: [u64; 4],
}

/// `glmaxx_moe_layer_descriptor` (240 bytes): one rank's routed-MoE step.
/// `exl3_experts` is the host address of a [`MoeExl3Experts`] (flag
/// [`MOE_EXL3_EXPERTS`]), read at launch.
#[repr(C, align(16))]
#[derive(Clone, Copy, Debug, Default)]
pub struct MoeLayerDescriptor {
    pub abi_version: u32,
    pub struct_bytes: u32,
    pub flags: u32,
    pub path: u32,
    pub tokens: u32,
    pub hidden: u32,
    pub experts: u32,
    pub local_intermediate: u32,
    pub top_k: u32,
    pub groups: u32,
    pub topk_groups: u32,
    pub route_scale: f32,
    pub shared_intermediate: u32,
    pub reserved0: [u32; 3],
    pub input_bf16: u64,
    pub router_weight_bf16: u64,
    pub router_bias_f32: u64,
    pub w13_values: u64,
    pub w13_scales: u64,
    pub w13_global_f32: u64,
    pub w2_values: u64,
    pub w2_scales: u64,
    pub w2_global_f32: u64,
    pub shared13_bf16: u64,
    pub shared2_bf16: u64,
    pub route_experts_u16: u64,
    pub route_weights_f32: u64,
    pub output_f32: u64,
    pub validation_error_u32: u64,
    pub workspace: u64,
    pub workspace_bytes: u64,
    pub sequence: u64,
    pub exl3_experts: u64,
    /// Flag [`MOE_EXTERNAL_ROUTED`]: the `[tokens][top_k][hidden]` fp32 slot plane
    /// the experts' owner ranks wrote (expert parallelism), else 0.
    pub routed_plane_f32: u64,
    pub reserved: [u64; 2],
}

/// `glmaxx_moe_finish_descriptor` (112 bytes): residual + attention + every
/// rank's partial in rank order (`finish_sparse_layer_oracle`,
/// `crates/glm-reference/src/routed_fc2.rs:214-258`).  `partials_f32` is the host
/// address of an array of `ranks` device pointers.
#[repr(C, align(16))]
#[derive(Clone, Copy, Debug, Default)]
pub struct MoeFinishDescriptor {
    pub abi_version: u32,
    pub struct_bytes: u32,
    pub flags: u32,
    pub ranks: u32,
    pub elements: u64,
    pub residual_f32: u64,
    pub residual_bf16: u64,
    pub attention_f32: u64,
    pub partials_f32: u64,
    pub output_f32: u64,
    pub output_bf16: u64,
    pub norm_bf16: u64,
    pub hidden: u32,
    pub eps: f32,
    pub reserved: [u64; 3],
}

/// `glmaxx_moe_peer_descriptor` (80 bytes): this rank's part of the peer-memory
/// finish; `signals_u32`, `outputs_*` and `norms_bf16` are host addresses of
/// arrays of `ranks` device addresses.
#[repr(C, align(16))]
#[derive(Clone, Copy, Debug, Default)]
pub struct MoePeerDescriptor {
    pub abi_version: u32,
    pub struct_bytes: u32,
    pub flags: u32,
    pub rank: u32,
    pub signals_u32: u64,
    pub outputs_f32: u64,
    pub outputs_bf16: u64,
    pub norms_bf16: u64,
    pub status_u32: u64,
    pub reserved: [u64; 3],
}

/// `glmaxx_moe_ep_descriptor` (560 bytes): the expert-parallel dispatch and
/// return.  The arrays of 8 hold every rank's buffers in rank order.
#[repr(C, align(16))]
#[derive(Clone, Copy, Debug, Default)]
pub struct MoeEpDescriptor {
    pub abi_version: u32,
    pub struct_bytes: u32,
    pub ranks: u32,
    pub rank: u32,
    pub tokens: u32,
    pub hidden: u32,
    pub experts: u32,
    pub top_k: u32,
    pub rows: u32,
    pub reserved0: [u32; 3],
    pub input_bf16: u64,
    pub compacted_tokens_u32: u64,
    pub compacted_experts_u16: u64,
    pub compacted_slots_u8: u64,
    pub compacted_weights_f32: u64,
    pub expert_offsets_u32: u64,
    pub recv_x_bf16: [u64; 8],
    pub recv_expert_u16: [u64; 8],
    pub recv_weight_f32: [u64; 8],
    pub recv_source_u32: [u64; 8],
    pub recv_capacity: [u32; 8],
    pub dest_row_offset: [u32; 8],
    pub rows_out_f32: u64,
    pub planes_f32: [u64; 8],
    pub plane_tokens: [u32; 8],
    pub validation_error_u32: u64,
    pub reserved: [u64; 4],
}

// Frozen layouts (the C header static_asserts the same sizes).
const _: () = assert!(core::mem::size_of::<RouterDescriptor>() == 192);
const _: () = assert!(core::mem::size_of::<MoeExl3Experts>() == 128);
const _: () = assert!(core::mem::size_of::<MoeLayerDescriptor>() == 240);
const _: () = assert!(core::mem::size_of::<MoeFinishDescriptor>() == 112);
const _: () = assert!(core::mem::size_of::<MoePeerDescriptor>() == 80);
const _: () = assert!(core::mem::size_of::<MoeEpDescriptor>() == 560);
const _: () = assert!(core::mem::align_of::<MoeLayerDescriptor>() == 16);

impl RouterDescriptor {
    #[must_use]
    pub fn new() -> Self {
        Self {
            abi_version: ROUTER_ABI_VERSION,
            struct_bytes: core::mem::size_of::<Self>() as u32,
            ..Self::default()
        }
    }
}

impl MoeLayerDescriptor {
    #[must_use]
    pub fn new() -> Self {
        Self {
            abi_version: MOE_LAYER_ABI_VERSION,
            struct_bytes: core::mem::size_of::<Self>() as u32,
            ..Self::default()
        }
    }
}

impl MoeExl3Experts {
    #[must_use]
    pub fn new() -> Self {
        Self {
            abi_version: MOE_EXL3_ABI_VERSION,
            struct_bytes: core::mem::size_of::<Self>() as u32,
            bits: 3,
            ..Self::default()
        }
    }
}

impl MoeFinishDescriptor {
    #[must_use]
    pub fn new() -> Self {
        Self {
            abi_version: MOE_FINISH_ABI_VERSION,
            struct_bytes: core::mem::size_of::<Self>() as u32,
            eps: 1e-6,
            ..Self::default()
        }
    }
}

impl MoeEpDescriptor {
    #[must_use]
    pub fn new() -> Self {
        Self {
            abi_version: MOE_EP_ABI_VERSION,
            struct_bytes: core::mem::size_of::<Self>() as u32,
            ..Self::default()
        }
    }
}

impl MoePeerDescriptor {
    #[must_use]
    pub fn new() -> Self {
        Self {
            abi_version: MOE_PEER_ABI_VERSION,
            struct_bytes: core::mem::size_of::<Self>() as u32,
            ..Self::default()
        }
    }
}

/// Error kinds of the reference's `KernelError` (`crates/glm-cuda/src/abi.rs:686-698`),
/// mapped from this library's return codes and device status words.
#[derive(Clone, Copy, Debug, Eq, PartialEq)]
pub enum KernelError {
    Abi,
    Null,
    Descriptor,
    Arch,
    Driver(i32),
    DeviceValidation(u32),
    Topology,
}

impl core::fmt::Display for KernelError {
    fn fmt(&self, f: &mut core::fmt::Formatter<'_>) -> core::fmt::Result {
        write!(f, "{self:?}")
    }
}

impl std::error::Error for KernelError {}

/// Maps a launch's return value to `Ok` or the matching [`KernelError`].
pub fn check(status: i32) -> Result<(), KernelError> {
    match status {
        0 => Ok(()),
        ERR_NULL => Err(KernelError::Null),
        ERR_DESCRIPTOR => Err(KernelError::Descriptor),
        ERR_WRONG_ARCH => Err(KernelError::Arch),
        other => Err(KernelError::Driver(other)),
    }
}
