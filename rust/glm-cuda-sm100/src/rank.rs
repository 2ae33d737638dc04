//! One rank's thread-owned B200 context and its routed-MoE step.
//!
//! Mirrors the reference's `NativeRankContext` (`crates/glm-cuda/src/ffi.rs:185-298`):
//! created on the persistent rank thread, every method checks that it is still
//! called from that thread.  `bind` accepts compute capability 10.x and a
//! tensor-parallel group of 1, 2, 4 or 8 visible devices (the reference requires
//! exactly four SM120 devices).

use core::ffi::c_void;
use std::thread::ThreadId;

use crate::abi::{self, check, KernelError, MoeExl3Experts, MoeLayerDescriptor};
use crate::ffi;

/// Device memory owned by one rank (freed on drop, on the owner thread).
pub struct DeviceBuffer {
    pub ptr: u64,
    pub bytes: u64,
}

impl DeviceBuffer {
    pub fn alloc(bytes: u64) -> Result<Self, KernelError> {
        let mut ptr = 0_u64;
        // SAFETY: `ptr` is a valid out-parameter; the library returns a device
        // address on the current (rank-bound) device.
        check(unsafe { ffi::glmaxx_device_alloc(bytes.max(16), &mut ptr) })?;
        Ok(Self { ptr, bytes })
    }

    pub fn zeroed(bytes: u64, stream: u64) -> Result<Self, KernelError> {
        let b = Self::alloc(bytes)?;
        // SAFETY: the buffer was just allocated with at least `bytes` bytes.
        check(unsafe { ffi::glmaxx_memset_zero(b.ptr, bytes, stream) })?;
        Ok(b)
    }
}

impl Drop for DeviceBuffer {
    fn drop(&mut self) {
        // SAFETY: `ptr` came from glmaxx_device_alloc and is freed once.
        let _ = unsafe { ffi::glmaxx_device_free(self.ptr) };
    }
}

/// A rank's device, bound on its owner thread, with one execution stream.
pub struct RankContext {
    pub rank: u32,
    pub ranks: u32,
    pub compute_capability: i32,
    pub multiprocessors: i32,
    pub total_memory_bytes: u64,
    pub device_uuid: [u8; 16],
    stream: u64,
    owner: ThreadId,
}

impl RankContext {
    /// Binds device `rank` of a `ranks`-wide group to the calling thread.
    pub fn bind(rank: u32, ranks: u32) -> Result<Self, KernelError> {
        if !matches!(ranks, 1 | 2 | 4 | 8) || rank >= ranks {
            return Err(KernelError::Topology);
        }
        let mut visible = 0_i32;
        // SAFETY: valid out-parameter.
        check(unsafe { ffi::glmaxx_device_count(&mut visible) })?;
        if visible < ranks as i32 {
            return Err(KernelError::Topology);
        }
        let (mut cc, mut sms, mut total) = (0_i32, 0_i32, 0_u64);
        let mut uuid = [0_u8; 16];
        // SAFETY: every out-parameter is valid; `rank` < visible devices.
        check(unsafe {
            ffi::glmaxx_device_bind(rank as i32, &mut cc, &mut sms, &mut total, uuid.as_mut_ptr())
        })?;
        if cc / 10 != 10 || sms <= 0 || total == 0 {
            return Err(KernelError::Arch);
        }
        let mut stream = 0_u64;
        // SAFETY: valid out-parameter on the bound device.
        check(unsafe { ffi::glmaxx_stream_create(&mut stream) })?;
        Ok(Self {
            rank,
            ranks,
            compute_capability: cc,
            multiprocessors: sms,
            total_memory_bytes: total,
            device_uuid: uuid,
            stream,
            owner: std::thread::current().id(),
        })
    }

    pub fn stream(&self) -> Result<u64, KernelError> {
        self.require_owner()?;
        Ok(self.stream)
    }

    pub fn synchronize(&self) -> Result<(), KernelError> {
        self.require_owner()?;
        // SAFETY: the stream belongs to this context.
        check(unsafe { ffi::glmaxx_stream_synchronize(self.stream) })
    }

    fn require_owner(&self) -> Result<(), KernelError> {
        if std::thread::current().id() == self.owner {
            Ok(())
        } else {
            Err(KernelError::Topology)
        }
    }
}

impl Drop for RankContext {
    fn drop(&mut self) {
        // SAFETY: the stream was created by bind and is destroyed once.
        let _ = unsafe { ffi::glmaxx_stream_destroy(self.stream) };
    }
}

/// Device addresses of one rank's layer weights, in the reference's packed rank
/// layout (`crates/glm-reference/src/manifest.rs:143-165`): NVFP4 gate/up
/// `[experts][2*I_r][H/2]` + scales + globals, down `[experts][H][I_r/2]`, the
/// replicated router, and the bf16 shared-expert shard.
#[derive(Clone, Copy, Debug, Default)]
pub struct RankLayerWeights {
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
    /// EXL3 or hybrid experts (`MoeExl3Experts`), else `None`.
    pub exl3: Option<MoeExl3Experts>,
}

/// Geometry of a rank-local layer (GLM-5.2: hidden 6144, 256 experts, top-8 of
/// 8 groups / top-4 groups, x2.5, intermediate 2048 / ranks).
#[derive(Clone, Copy, Debug)]
pub struct LayerGeometry {
    pub hidden: u32,
    pub experts: u32,
    pub local_intermediate: u32,
    pub shared_intermediate: u32,
    pub top_k: u32,
    pub groups: u32,
    pub topk_groups: u32,
    pub route_scale: f32,
}

impl LayerGeometry {
    #[must_use]
    pub const fn glm52(ranks: u32) -> Self {
        Self {
            hidden: 6144,
            experts: 256,
            local_intermediate: 2048 / ranks,
            shared_intermediate: 2048 / ranks,
            top_k: 8,
            groups: 8,
            topk_groups: 4,
            route_scale: 2.5,
        }
    }
}

/// One rank's routed-MoE step (`glmaxx_moe_layer_launch`): router, compaction,
/// NVFP4 FC1 + SwiGLU, FC2 + routing-weighted combine and the shared expert into
/// an fp32 partial.  Workspace and route buffers are sized once for `max_tokens`.
pub struct RoutedMoeStep {
    pub geometry: LayerGeometry,
    pub weights: RankLayerWeights,
    pub max_tokens: u32,
    route_experts: DeviceBuffer,
    route_weights: DeviceBuffer,
    status: DeviceBuffer,
    workspace: DeviceBuffer,
    exl3: Option<Box<MoeExl3Experts>>,
}

impl RoutedMoeStep {
    pub fn new(
        ctx: &RankContext,
        geometry: LayerGeometry,
        weights: RankLayerWeights,
        max_tokens: u32,
    ) -> Result<Self, KernelError> {
        let stream = ctx.stream()?;
        let k = u64::from(geometry.top_k);
        let mut step = Self {
            geometry,
            weights,
            max_tokens,
            route_experts: DeviceBuffer::alloc(u64::from(max_tokens) * k * 2)?,
            route_weights: DeviceBuffer::alloc(u64::from(max_tokens) * k * 4)?,
            status: DeviceBuffer::zeroed(16, stream)?,
            workspace: DeviceBuffer::alloc(16)?,
            exl3: weights.exl3.map(Box::new),
        };
        // the prefill path (most tokens) needs the largest workspace
        let need = step.workspace_bytes(max_tokens, abi::PATH_PREFILL_GROUPED)?.max(
            step.workspace_bytes(max_tokens.min(256), abi::PATH_DECODE_PERSISTENT)?,
        );
        step.workspace = DeviceBuffer::alloc(need)?;
        Ok(step)
    }

    fn descriptor(&self, tokens: u32, input_bf16: u64, output_f32: u64, path: u32) -> MoeLayerDescriptor {
        let g = self.geometry;
        let w = self.weights;
        let mut flags = 0;
        if g.shared_intermediate != 0 && w.shared13_bf16 != 0 {
            flags |= abi::MOE_SHARED_EXPERT;
        }
        let mut d = MoeLayerDescriptor::new();
        if let Some(x) = &self.exl3 {
            flags |= abi::MOE_EXL3_EXPERTS;
            d.exl3_experts = core::ptr::from_ref::<MoeExl3Experts>(x) as u64;
        }
        d.flags = flags;
        d.path = path;
        d.tokens = tokens;
        d.hidden = g.hidden;
        d.experts = g.experts;
        d.local_intermediate = g.local_intermediate;
        d.top_k = g.top_k;
        d.groups = g.groups;
        d.topk_groups = g.topk_groups;
        d.route_scale = g.route_scale;
        d.shared_intermediate = if flags & abi::MOE_SHARED_EXPERT != 0 { g.shared_intermediate } else { 0 };
        d.input_bf16 = input_bf16;
        d.router_weight_bf16 = w.router_weight_bf16;
        d.router_bias_f32 = w.router_bias_f32;
        d.w13_values = w.w13_values;
        d.w13_scales = w.w13_scales;
        d.w13_global_f32 = w.w13_global_f32;
        d.w2_values = w.w2_values;
        d.w2_scales = w.w2_scales;
        d.w2_global_f32 = w.w2_global_f32;
        d.shared13_bf16 = w.shared13_bf16;
        d.shared2_bf16 = w.shared2_bf16;
        d.route_experts_u16 = self.route_experts.ptr;
        d.route_weights_f32 = self.route_weights.ptr;
        d.output_f32 = output_f32;
        d.validation_error_u32 = self.status.ptr;
        d.workspace = self.workspace.ptr;
        d.workspace_bytes = self.workspace.bytes;
        d.sequence = 1;
        d
    }

    fn workspace_bytes(&self, tokens: u32, path: u32) -> Result<u64, KernelError> {
        let d = self.descriptor(tokens, 0, 0, path);
        // SAFETY: `d` is a fully initialised descriptor (pointers unused here).
        let need = unsafe { ffi::glmaxx_moe_layer_workspace_bytes(&d) };
        if need == 0 {
            return Err(KernelError::Descriptor);
        }
        Ok(need)
    }

    /// Enqueues the step for `tokens` bf16 rows at `input_bf16`; writes the fp32
    /// partial `[tokens][hidden]` to `output_f32` on the rank's stream.
    pub fn launch(&self, ctx: &RankContext, tokens: u32, input_bf16: u64, output_f32: u64) -> Result<(), KernelError> {
        if tokens == 0 || tokens > self.max_tokens {
            return Err(KernelError::Descriptor);
        }
        let d = self.descriptor(tokens, input_bf16, output_f32, abi::PATH_AUTO);
        let mut async_err = 0_i32;
        // SAFETY: the descriptor's buffers are owned by this step or the caller and
        // stay alive until the stream has run the launch.
        check(unsafe {
            ffi::glmaxx_moe_layer_launch(&d, ctx.stream()? as *mut c_void, &mut async_err)
        })
    }

    /// Reads the device status word of the last step (synchronises the stream).
    pub fn device_status(&self, ctx: &RankContext) -> Result<u32, KernelError> {
        let mut word = 0_u32;
        let stream = ctx.stream()?;
        // SAFETY: 4 bytes from the status buffer into `word`.
        check(unsafe {
            ffi::glmaxx_memcpy_d2h(core::ptr::from_mut(&mut word).cast(), self.status.ptr, 4, stream)
        })?;
        ctx.synchronize()?;
        if word == 0 { Ok(0) } else { Err(KernelError::DeviceValidation(word)) }
    }
}
