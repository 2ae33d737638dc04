//! The `extern "C"` block of libglmaxx_sm100 (`include/glmaxx_kernel.h`).
//!
//! The first group is the reference's block (`crates/glm-cuda/src/ffi.rs:21-151`)
//! with the same names and signatures, so the reference's safe wrappers keep
//! working against this library; the second group is the v3 routed-MoE surface.
//! Descriptor pointers of the reference structs are passed as `*const c_void`
//! here, so this module does not depend on the reference's `abi.rs`.

use core::ffi::{c_char, c_void};

use crate::abi::{
    MoeEpDescriptor, MoeFinishDescriptor, MoeLayerDescriptor, MoePeerDescriptor, RouterDescriptor,
};

#[link(name = "glmaxx_sm100")]
unsafe extern "C" {
    // ---- reference entry points (glmaxx_kernel.h:123-250) ----
    pub fn glmaxx_nvfp4_routed_fc1_launch(
        descriptor: *const c_void,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_nvfp4_routed_fc1_graph_instantiate(
        descriptor: *const c_void,
        stream: *mut c_void,
        graph_exec: *mut u64,
    ) -> i32;
    pub fn glmaxx_nvfp4_quantize_launch(descriptor: *const c_void, stream: *mut c_void) -> i32;
    pub fn glmaxx_nvfp4_grouped_quantize_launch(descriptor: *const c_void, stream: *mut c_void) -> i32;
    pub fn glmaxx_nvfp4_core_swiglu_launch(descriptor: *const c_void, stream: *mut c_void) -> i32;
    pub fn glmaxx_nvfp4_dense_control_launch(
        descriptor: *const c_void,
        expert: u32,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_nvfp4_grouped_control_launch(
        descriptor: *const c_void,
        active_experts: *const u16,
        active_expert_count: u32,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_nvfp4_grouped_core_swiglu_launch(
        descriptor: *const c_void,
        active_experts: *const u16,
        active_expert_count: u32,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_nvfp4_grouped_prepare_launch(
        descriptor: *const c_void,
        active_experts: *const u16,
        active_expert_count: u32,
        stream: *mut c_void,
    ) -> i32;
    pub fn glmaxx_nvfp4_grouped_prepared_control_launch(
        descriptor: *const c_void,
        active_expert_count: u32,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_nvfp4_grouped_prepared_core_swiglu_launch(
        descriptor: *const c_void,
        active_expert_count: u32,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_nvfp4_routed_fc2_launch(
        descriptor: *const c_void,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_nvfp4_fc2_quantize_launch(descriptor: *const c_void, stream: *mut c_void) -> i32;
    pub fn glmaxx_nvfp4_fc2_grouped_quantize_launch(
        descriptor: *const c_void,
        stream: *mut c_void,
    ) -> i32;
    pub fn glmaxx_nvfp4_fc2_core_launch(descriptor: *const c_void, stream: *mut c_void) -> i32;
    pub fn glmaxx_nvfp4_fc2_reduce_launch(descriptor: *const c_void, stream: *mut c_void) -> i32;
    pub fn glmaxx_nvfp4_fc2_dense_control_launch(
        descriptor: *const c_void,
        expert: u32,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_nvfp4_fc2_grouped_control_launch(
        descriptor: *const c_void,
        active_experts: *const u16,
        active_expert_count: u32,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_exl3_projection_launch(
        descriptor: *const c_void,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_graph_exec_launch(graph_exec: u64, stream: u64) -> i32;
    pub fn glmaxx_graph_exec_destroy(graph_exec: u64) -> i32;
    pub fn glmaxx_event_create(event: *mut u64) -> i32;
    pub fn glmaxx_event_record(event: u64, stream: u64) -> i32;
    pub fn glmaxx_event_synchronize(event: u64) -> i32;
    pub fn glmaxx_event_elapsed_ms(start: u64, end: u64, milliseconds: *mut f32) -> i32;
    pub fn glmaxx_event_destroy(event: u64) -> i32;
    pub fn glmaxx_profiler_start() -> i32;
    pub fn glmaxx_profiler_stop() -> i32;
    pub fn glmaxx_nvtx_range_push(message: *const c_char) -> i32;
    pub fn glmaxx_nvtx_range_pop() -> i32;
    pub fn glmaxx_nvfp4_routed_fc1_workspace_bytes(assignments: u32) -> u64;
    pub fn glmaxx_nvfp4_grouped_workspace_bytes(assignments: u32) -> u64;
    pub fn glmaxx_nvfp4_routed_fc2_workspace_bytes(rows: u32, assignments: u32) -> u64;
    pub fn glmaxx_nvfp4_grouped_fc2_workspace_bytes(rows: u32, assignments: u32) -> u64;
    pub fn glmaxx_exl3_projection_workspace_bytes(rows: u32, logical_k: u32, logical_n: u32) -> u64;
    pub fn glmaxx_kernel_abi() -> *const c_char;
    pub fn glmaxx_exl3_kernel_abi() -> *const c_char;
    pub fn glmaxx_device_count(count: *mut i32) -> i32;
    pub fn glmaxx_device_bind(
        device_index: i32,
        compute_capability: *mut i32,
        multiprocessor_count: *mut i32,
        total_memory_bytes: *mut u64,
        device_uuid: *mut u8,
    ) -> i32;
    pub fn glmaxx_device_memory_info(free_memory_bytes: *mut u64, total_memory_bytes: *mut u64) -> i32;
    pub fn glmaxx_device_alloc(bytes: u64, pointer: *mut u64) -> i32;
    pub fn glmaxx_device_free(pointer: u64) -> i32;
    pub fn glmaxx_pinned_alloc(bytes: u64, pointer: *mut u64) -> i32;
    pub fn glmaxx_pinned_free(pointer: u64) -> i32;
    pub fn glmaxx_stream_create(stream: *mut u64) -> i32;
    pub fn glmaxx_stream_destroy(stream: u64) -> i32;
    pub fn glmaxx_stream_query(stream: u64, complete: *mut i32) -> i32;
    pub fn glmaxx_stream_synchronize(stream: u64) -> i32;
    pub fn glmaxx_memcpy_h2d(destination: u64, source: *const c_void, bytes: u64, stream: u64) -> i32;
    pub fn glmaxx_memcpy_d2d(destination: u64, source: u64, bytes: u64, stream: u64) -> i32;
    pub fn glmaxx_memcpy_d2h(destination: *mut c_void, source: u64, bytes: u64, stream: u64) -> i32;
    pub fn glmaxx_memset_zero(destination: u64, bytes: u64, stream: u64) -> i32;

    // ---- v3 routed-MoE surface (new) ----
    pub fn glmaxx_stream_begin_capture(stream: u64) -> i32;
    pub fn glmaxx_stream_end_capture(stream: u64, graph_exec: *mut u64) -> i32;
    pub fn glmaxx_nvfp4_routed_fc1_workspace_bytes_v3(
        rows: u32,
        assignments: u32,
        hidden: u32,
        local_intermediate: u32,
        experts: u32,
        top_k: u32,
    ) -> u64;
    pub fn glmaxx_nvfp4_routed_fc2_workspace_bytes_v3(
        rows: u32,
        assignments: u32,
        hidden: u32,
        local_intermediate: u32,
        experts: u32,
        top_k: u32,
    ) -> u64;
    pub fn glmaxx_router_workspace_bytes(tokens: u32, hidden: u32, experts: u32, top_k: u32) -> u64;
    pub fn glmaxx_moe_layer_workspace_bytes(descriptor: *const MoeLayerDescriptor) -> u64;
    pub fn glmaxx_exl3_gemv_launch(
        input_f16: u64,
        trellis_u16: u64,
        rows: u32,
        logical_k: u32,
        logical_n: u32,
        bits: u32,
        output_f16: u64,
        stream: *mut c_void,
    ) -> i32;
    pub fn glmaxx_router_compact_launch(
        descriptor: *const RouterDescriptor,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_router_compact_launch_static(
        descriptor: *const RouterDescriptor,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_moe_layer_launch(
        descriptor: *const MoeLayerDescriptor,
        stream: *mut c_void,
        asynchronous_error: *mut i32,
    ) -> i32;
    pub fn glmaxx_moe_finish_launch(descriptor: *const MoeFinishDescriptor, stream: *mut c_void) -> i32;
    pub fn glmaxx_moe_peer_signal_bytes(ranks: u32) -> u64;
    pub fn glmaxx_moe_finish_peer_launch(
        descriptor: *const MoeFinishDescriptor,
        peer: *const MoePeerDescriptor,
        stream: *mut c_void,
    ) -> i32;
    pub fn glmaxx_ipc_handle(pointer: u64, handle: *mut u8) -> i32;
    pub fn glmaxx_ipc_open(handle: *const u8, pointer: *mut u64) -> i32;
    pub fn glmaxx_ipc_close(pointer: u64) -> i32;
    pub fn glmaxx_peer_enable(peer_device: i32) -> i32;
    pub fn glmaxx_moe_layer_set_stage_events(events: *mut u64, count: u32) -> i32;
    pub fn glmaxx_moe_layer_plane(
        descriptor: *const MoeLayerDescriptor,
        which: u32,
        address: *mut u64,
        bytes: *mut u64,
    ) -> i32;
    pub fn glmaxx_nvfp4_pack_launch(
        src: u64,
        src_is_bf16: i32,
        batch: u32,
        n: u32,
        k: u32,
        values: u64,
        scales: u64,
        global_scale_f32: u64,
        global_amax_f32: u64,
        scratch: u64,
        validation_error_u32: u64,
        stream: *mut c_void,
    ) -> i32;
    pub fn glmaxx_moe_ep_dispatch_launch(descriptor: *const MoeEpDescriptor, stream: *mut c_void) -> i32;
    pub fn glmaxx_moe_ep_return_launch(descriptor: *const MoeEpDescriptor, stream: *mut c_void) -> i32;
    pub fn glmaxx_nvfp4_codec_selfcheck_launch(result_u64x4: *mut u64, stream: *mut c_void) -> i32;
    pub fn glmaxx_nvfp4_quotient_selfcheck_launch(
        decs: *const f32,
        n_decs: u32,
        result_u64x4: *mut u64,
        stream: *mut c_void,
    ) -> i32;
    pub fn glmaxx_nvfp4_mma_peak_launch(
        n: u32,
        dual: u32,
        copy_kind: u32,
        copies_per_kblock: u32,
        iters: u32,
        ctas: u32,
        status_u32: *mut u32,
        cycles_u64: *mut u64,
        stream: *mut c_void,
    ) -> i32;
}
