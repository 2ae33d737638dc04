/*
 * glmaxx routed-MoE kernel library for NVIDIA B200 (sm_100a): C ABI.
 *
 * Drop-in replacement for the reference's kernel library
 * (yatesdr/glmaxx kernels/include/glmaxx_kernel.h, bound from Rust in
 * crates/glm-cuda/src/ffi.rs:21-151), shipped as libglmaxx_sm100.so.
 *
 *  - Descriptor structs keep the reference layouts byte for byte
 *    (glmaxx_kernel.h:22-121; 224/224/144 bytes, 16-byte aligned, POSIX
 *    ownership: the caller owns every buffer, pointers are device addresses
 *    as uint64_t, launches are asynchronous on the caller's stream).
 *  - Geometry fields (hidden, local_intermediate, experts, top_k) are honoured
 *    instead of being pinned to the TP4 constants, so TP = 1/2/4/8 shards and
 *    the 16-expert reduced layer run through the same entry points.
 *  - Status convention (reference nvfp4_routed_fc1.cu:542-566): 0 success,
 *    -1 null argument, -2 invalid descriptor or short workspace, -120 device is
 *    not the supported architecture (here: compute capability 10.x), a positive
 *    cudaError_t otherwise.  Device-detected problems are reported as bit flags
 *    in the caller's validation word (bits 0..4 as the reference's FC2 word,
 *    nvfp4_routed_fc2.cu:33-39; see GLMAXX_STATUS_* below).
 *
 * New in this library (ABI string "glmaxx.sm100.nvfp4.routed_moe.v3"):
 *  - glmaxx_router_compact_launch: the protected router (manifest.rs:188-194)
 *    and the stable (expert, token, slot) compaction (routed_fc1.rs:20-58) on
 *    the device.
 *  - glmaxx_moe_layer_launch: the full rank-local routed-MoE step (router,
 *    compaction, NVFP4 quantisation, grouped FC1+SwiGLU, FC2 + weighted
 *    combine, bf16 shared expert) producing the fp32 partial that the TP
 *    all-reduce sums (manifest.rs:223-229).
 *  - glmaxx_nvfp4_pack_launch: PackedNvfp4::pack (nvfp4.rs:170-273) on the GPU.
 */
#ifndef GLMAXX_KERNEL_H_
#define GLMAXX_KERNEL_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__cplusplus)
extern "C" {
#endif

enum {
  GLMAXX_FC1_ABI_VERSION = 1,
  GLMAXX_FC2_ABI_VERSION = 1,
  GLMAXX_EXL3_ABI_VERSION = 1,
  GLMAXX_ROUTER_ABI_VERSION = 3,
  GLMAXX_MOE_LAYER_ABI_VERSION = 3,
  GLMAXX_MOE_EXL3_ABI_VERSION = 1,
  GLMAXX_MOE_FINISH_ABI_VERSION = 1,
  GLMAXX_MOE_PEER_ABI_VERSION = 1,
  GLMAXX_MOE_EP_ABI_VERSION = 1,
  GLMAXX_FC1_DECODE_PERSISTENT = 1,
  GLMAXX_FC1_PREFILL_GROUPED = 2,
  GLMAXX_EXL3_GATE = 1,
  GLMAXX_EXL3_UP = 2,
  GLMAXX_EXL3_DOWN = 3,
};

/* Status codes returned by the launch functions. */
enum {
  GLMAXX_OK = 0,
  GLMAXX_ERR_NULL = -1,
  GLMAXX_ERR_DESCRIPTOR = -2,
  GLMAXX_ERR_WRONG_ARCH = -120,
};

/* Bits of the device validation word. */
enum {
  GLMAXX_STATUS_ROUTE_TOKEN_OUT_OF_RANGE = 1u << 0,
  GLMAXX_STATUS_ROUTE_SLOT_OUT_OF_RANGE = 1u << 1,
  GLMAXX_STATUS_DUPLICATE_TOKEN_SLOT = 1u << 2,
  GLMAXX_STATUS_EXPERT_OUT_OF_RANGE = 1u << 3,
  GLMAXX_STATUS_ROUTE_WEIGHT_NOT_FINITE = 1u << 4,
  GLMAXX_STATUS_NON_FINITE_INPUT = 1u << 5,
  GLMAXX_STATUS_CAPACITY_EXCEEDED = 1u << 6,
  GLMAXX_STATUS_WAIT_TIMEOUT = 1u << 8,
  GLMAXX_STATUS_TMEM_TIMEOUT = 1u << 9,
  GLMAXX_STATUS_PEER_TIMEOUT = 1u << 10,
};

/* Flags of glmaxx_moe_layer_descriptor.flags. */
enum {
  GLMAXX_MOE_ROUTES_GIVEN = 1u << 0,   /* route_experts/route_weights are inputs */
  GLMAXX_MOE_SHARED_EXPERT = 1u << 1,  /* add the bf16 shared expert            */
  GLMAXX_MOE_EXL3_EXPERTS = 1u << 2,   /* exl3_experts describes EXL3 experts   */
  /* the routed contributions are already in routed_plane_f32 [tokens][top_k][hidden]
   * (expert parallelism: written there by the experts' owner ranks); the step runs
   * the shared expert and the deterministic expert-order combine only.  Needs
   * GLMAXX_MOE_ROUTES_GIVEN (route_experts_u16 orders the combine). */
  GLMAXX_MOE_EXTERNAL_ROUTED = 1u << 3,
  /* routed contributions go through the per-slot plane and the expert-order
   * combine at every token count (decode and EXL3 layers always do), so the
   * step's output is the same bits run after run; without it, prefill-size
   * steps (more than 256 tokens) add each routed row into the output with fp32
   * atomics, whose order varies.  The plane takes tokens x top_k x hidden x 4
   * bytes of workspace (glmaxx_moe_layer_workspace_bytes counts it). */
  GLMAXX_MOE_DETERMINISTIC = 1u << 4,
};

/* glmaxx_kernel.h:22-57 (unchanged layout). */
#if defined(__cplusplus)
struct alignas(16) glmaxx_fc1_descriptor {
#else
struct glmaxx_fc1_descriptor {
#endif
  uint32_t abi_version;
  uint32_t struct_bytes;
  uint32_t flags;
  uint32_t path;
  uint32_t rows;
  uint32_t assignments;
  uint32_t hidden;
  uint32_t local_gate_up;
  uint32_t local_intermediate;
  uint32_t experts;
  uint32_t top_k;
  uint32_t reserved0;
  uint64_t input_bf16;
  uint64_t expert_value_base;
  uint64_t expert_scale_base;
  uint64_t expert_global_scales;
  uint64_t route_experts_u16;
  uint64_t route_tokens_u32;
  uint64_t route_slots_u8;
  uint64_t route_weights_f32;
  uint64_t expert_offsets_u32;
  uint64_t compacted_input_bf16;
  uint64_t activation_values;
  uint64_t activation_scales;
  uint64_t activation_global_scales;
  uint64_t gate_up_accum_f32;
  uint64_t output_bf16;
  uint64_t workspace_bytes;
  uint64_t sequence;
  uint64_t reserved[4];
};

/* glmaxx_kernel.h:59-95 (unchanged layout). */
#if defined(__cplusplus)
struct alignas(16) glmaxx_fc2_descriptor {
#else
struct glmaxx_fc2_descriptor {
#endif
  uint32_t abi_version;
  uint32_t struct_bytes;
  uint32_t flags;
  uint32_t path;
  uint32_t rows;
  uint32_t assignments;
  uint32_t hidden;
  uint32_t local_intermediate;
  uint32_t experts;
  uint32_t top_k;
  uint32_t reserved0;
  uint32_t reserved1;
  uint64_t input_bf16;
  uint64_t expert_value_base;
  uint64_t expert_scale_base;
  uint64_t expert_global_scales;
  uint64_t route_experts_u16;
  uint64_t route_tokens_u32;
  uint64_t route_slots_u8;
  uint64_t route_weights_f32;
  uint64_t expert_offsets_u32;
  uint64_t activation_values;
  uint64_t activation_scales;
  uint64_t activation_global_scales;
  uint64_t assignment_down_f32;
  uint64_t token_output_f32;
  uint64_t slot_assignment_u32;
  uint64_t validation_error_u32;
  uint64_t workspace_bytes;
  uint64_t sequence;
  uint64_t reserved[4];
};

/* glmaxx_kernel.h:97-121 (unchanged layout). */
#if defined(__cplusplus)
struct alignas(16) glmaxx_exl3_descriptor {
#else
struct glmaxx_exl3_descriptor {
#endif
  uint32_t abi_version;
  uint32_t struct_bytes;
  uint32_t flags;
  uint32_t projection;
  uint32_t rows;
  uint32_t logical_k;
  uint32_t logical_n;
  uint32_t bits;
  uint64_t input_f16;
  uint64_t trellis_u16;
  uint64_t suh_f16;
  uint64_t svh_f16;
  uint64_t rotated_input_f16;
  uint64_t projected_f16;
  uint64_t output_f16;
  uint64_t validation_error_u32;
  uint64_t workspace_bytes;
  uint64_t sequence;
  uint64_t reserved[4];
};

/*
 * Router + compaction (new).  Replaces the host-side route preparation of the
 * reference (crates/glm-cuda/src/ffi.rs:1692-1750 validate_case, which builds
 * expert_offsets on the CPU) and the unbuilt router of manifest.rs:188-194.
 * Outputs: dense routes [tokens][top_k] (slot order = descending choice
 * score) and the compacted arrays in (expert, token, slot) order with
 * expert_offsets[experts + 1], exactly the inputs of the FC1/FC2 descriptors.
 */
#if defined(__cplusplus)
struct alignas(16) glmaxx_router_descriptor {
#else
struct glmaxx_router_descriptor {
#endif
  uint32_t abi_version;
  uint32_t struct_bytes;
  uint32_t flags;
  uint32_t tokens;
  uint32_t hidden;
  uint32_t experts;
  uint32_t top_k;
  uint32_t groups;
  uint32_t topk_groups;
  float route_scale;
  uint32_t reserved0[2];
  uint64_t input_bf16;          /* [tokens][hidden]                      */
  uint64_t router_weight_bf16;  /* [experts][hidden]                     */
  uint64_t router_bias_f32;     /* [experts] e_score_correction_bias      */
  uint64_t route_experts_u16;   /* out [tokens][top_k]                    */
  uint64_t route_weights_f32;   /* out [tokens][top_k]                    */
  uint64_t compacted_tokens_u32;   /* out [tokens*top_k]                  */
  uint64_t compacted_experts_u16;  /* out [tokens*top_k]                  */
  uint64_t compacted_slots_u8;     /* out [tokens*top_k]                  */
  uint64_t compacted_weights_f32;  /* out [tokens*top_k]                  */
  uint64_t expert_offsets_u32;  /* out [experts + 1]                      */
  uint64_t validation_error_u32;
  uint64_t workspace;
  uint64_t workspace_bytes;
  uint64_t sequence;
  uint64_t reserved[4];
};

/*
 * EXL3 routed experts of a layer (new; the reference's per-expert hybrid codec,
 * crates/glm-engine/src/weight.rs:37-50,116-215).  Each expert's gate, up and
 * down projections are 3-bit trellises in the reference layout (exl3.rs, 16x16
 * tiles of 48 halves, K x N logical: gate/up hidden x local_intermediate, down
 * local_intermediate x hidden), with fp16 input signs/scales suh [K] and output
 * scales svh [N]; arrays are expert-major ([experts][...]).  codec_u8 (device,
 * [experts]) selects per expert: 0 = the descriptor's NVFP4 weights, 1 = EXL3;
 * codec_u8 = 0 (null) makes every expert EXL3.  Per assignment row the layer
 * computes y = proj(x) exactly as Exl3Trellis::matmul_reference_f16 (exl3.rs:
 * 404-453) for gate and up (x = fp16 of the bf16 token row), h = fp16(silu(g)
 * * u), down = proj(h), and adds the routing-weighted fp32 value in the
 * deterministic expert order of the decode combine.
 */
#if defined(__cplusplus)
struct alignas(16) glmaxx_moe_exl3_experts {
#else
struct glmaxx_moe_exl3_experts {
#endif
  uint32_t abi_version; /* GLMAXX_MOE_EXL3_ABI_VERSION */
  uint32_t struct_bytes;
  uint32_t bits; /* 3 */
  uint32_t reserved0;
  uint64_t codec_u8;
  uint64_t gate_trellis_u16;
  uint64_t up_trellis_u16;
  uint64_t down_trellis_u16;
  uint64_t gate_suh_f16;
  uint64_t gate_svh_f16;
  uint64_t up_suh_f16;
  uint64_t up_svh_f16;
  uint64_t down_suh_f16;
  uint64_t down_svh_f16;
  uint64_t reserved[4];
};

/*
 * Full rank-local routed-MoE step (new).  Weights are in the reference's
 * packed rank layout: per expert, gate/up NVFP4 [2*local_intermediate][hidden]
 * (rank-local gate rows, then up rows: nvfp4-physical-abi.md:18-28) and down
 * NVFP4 [hidden][local_intermediate]; values row-major, two codes per byte
 * (even element in the low nibble), scales in the 128x4 atom layout of
 * nvfp4.rs:493-521, one fp32 global scale per tensor.  Experts are contiguous:
 * expert e's gate/up values start at w13_values + e * 2*I*H/2, and so on.
 * Shared expert (optional): bf16 gate/up [2*shared_intermediate][hidden] and
 * down [hidden][shared_intermediate] rank shards (checkpoint.rs:1408-1436).
 * Output: fp32 partial [tokens][hidden] = routed + shared (routed_fc2.rs:
 * 250-256), the operand of the TP all-reduce.
 */
#if defined(__cplusplus)
struct alignas(16) glmaxx_moe_layer_descriptor {
#else
struct glmaxx_moe_layer_descriptor {
#endif
  uint32_t abi_version;
  uint32_t struct_bytes;
  uint32_t flags;
  uint32_t path; /* 0 = auto, GLMAXX_FC1_DECODE_PERSISTENT, GLMAXX_FC1_PREFILL_GROUPED */
  uint32_t tokens;
  uint32_t hidden;
  uint32_t experts;
  uint32_t local_intermediate;
  uint32_t top_k;
  uint32_t groups;
  uint32_t topk_groups;
  float route_scale;
  uint32_t shared_intermediate;
  uint32_t reserved0[3];
  uint64_t input_bf16;
  uint64_t router_weight_bf16;
  uint64_t router_bias_f32;
  uint64_t w13_values;
  uint64_t w13_scales;
  uint64_t w13_global_f32;
  uint64_t w2_values;
  uint64_t w2_scales;
  uint64_t w2_global_f32;
  uint64_t shared13_bf16;
  uint64_t shared2_bf16;
  uint64_t route_experts_u16;
  uint64_t route_weights_f32;
  uint64_t output_f32;
  uint64_t validation_error_u32;
  uint64_t workspace;
  uint64_t workspace_bytes;
  uint64_t sequence;
  /* host address of a glmaxx_moe_exl3_experts (flag GLMAXX_MOE_EXL3_EXPERTS), else 0 */
  uint64_t exl3_experts;
  /* flag GLMAXX_MOE_EXTERNAL_ROUTED: [tokens][top_k][hidden] fp32 slot plane, else 0 */
  uint64_t routed_plane_f32;
  uint64_t reserved[2];
};

/*
 * Sparse-layer finish (new; finish_sparse_layer_oracle, crates/glm-reference/src/
 * routed_fc2.rs:214-258): output[i] = residual[i], then += attention[r][i] for
 * r = 0..ranks-1, then += partial_r[i] (each rank's routed + shared partial, the
 * output of glmaxx_moe_layer_launch) for r = 0..ranks-1, in fp32 and in that
 * order, so the result is the same bit for bit whatever launch does it.
 * partials_f32 is the host address of an array of `ranks` device pointers
 * (rank order; other GPUs' buffers when peer access is enabled).  The residual
 * is fp32 or bf16 (exactly one given); outputs fp32 and/or bf16 (round to
 * nearest even).  ranks 1..8.  The row-wise RMSNorm output (not in the reference,
 * which stops at the residual) feeds the next layer of a stacked benchmark.
 */
#if defined(__cplusplus)
struct alignas(16) glmaxx_moe_finish_descriptor {
#else
struct glmaxx_moe_finish_descriptor {
#endif
  uint32_t abi_version; /* GLMAXX_MOE_FINISH_ABI_VERSION */
  uint32_t struct_bytes;
  uint32_t flags;
  uint32_t ranks;
  uint64_t elements;
  uint64_t residual_f32;
  uint64_t residual_bf16;
  uint64_t attention_f32;
  uint64_t partials_f32;
  uint64_t output_f32;
  uint64_t output_bf16;
  /* optional: the next layer's MoE input, bf16(o / sqrt(mean(o^2) + eps)) over each
   * row of `hidden` elements of the fp32 result o (RMSNorm with unit weight) */
  uint64_t norm_bf16;
  uint32_t hidden;
  float eps;
  uint64_t reserved[3];
};

/*
 * Peer form of the finish (new; replaces the NCCL all-reduce of the partials,
 * crates/glm-engine/src/manifest.rs:228, and the finish after it): every rank of a
 * tensor-parallel group calls glmaxx_moe_finish_peer_launch at the same point of
 * its stream with the same finish descriptor except for its own outputs;
 * partials_f32 then holds every rank's partial buffer as mapped on this GPU (CUDA
 * IPC).  The residual may be absent (a plain all-reduce).  A flag barrier over
 * the ranks' signal buffers orders the launch after every rank's partial and keeps
 * each partial unchanged until every rank has read it.  The result is the same
 * bit for bit as glmaxx_moe_finish_launch on the same partials, on every rank.
 *  GLMAXX_MOE_PEER_ONE_SHOT: every rank reads all partials and writes its own
 *    outputs (the outputs_* arrays are 0).
 *  GLMAXX_MOE_PEER_TWO_SHOT: rank r reduces the r-th slice (of rows with the
 *    RMSNorm output) and writes it into every rank's outputs; outputs_f32,
 *    outputs_bf16, norms_bf16 are host arrays of `ranks` device addresses (rank
 *    order, entry `rank` equal to the descriptor's own output), 0 exactly when the
 *    descriptor's output is 0.
 * signals_u32: host array of `ranks` device addresses, every rank's signal buffer
 * (glmaxx_moe_peer_signal_bytes(ranks) bytes each, zeroed once before the first
 * launch, 16-byte aligned).  A wait on another rank gives up after 1 s and sets
 * GLMAXX_STATUS_PEER_TIMEOUT in status_u32 (optional device word); the signal
 * buffers must then be zeroed on every rank, after a host barrier, before the next
 * launch.  norm_bf16 and output_bf16 are 8-byte aligned, hidden % 4 == 0 with the
 * RMSNorm.
 */
enum {
  GLMAXX_MOE_PEER_ONE_SHOT = 1,
  GLMAXX_MOE_PEER_TWO_SHOT = 2,
};
#if defined(__cplusplus)
struct alignas(16) glmaxx_moe_peer_descriptor {
#else
struct glmaxx_moe_peer_descriptor {
#endif
  uint32_t abi_version; /* GLMAXX_MOE_PEER_ABI_VERSION */
  uint32_t struct_bytes;
  uint32_t flags;       /* GLMAXX_MOE_PEER_ONE_SHOT or GLMAXX_MOE_PEER_TWO_SHOT */
  uint32_t rank;
  uint64_t signals_u32;
  uint64_t outputs_f32;
  uint64_t outputs_bf16;
  uint64_t norms_bf16;
  uint64_t status_u32;
  uint64_t reserved[3];
};

/*
 * Expert-parallel exchange (new; the all-to-all alternative to the reference's
 * tensor-parallel layout, crates/glm-engine/src/manifest.rs:143-165 -- not a
 * reference layout).  Experts are split in contiguous blocks over `ranks`
 * owners (owner of e = e / (experts / ranks)); tokens are split over ranks as
 * data.  Per step, on every rank: glmaxx_router_compact_launch on its tokens;
 * glmaxx_moe_ep_dispatch_launch sends each compacted row to its expert's owner
 * (bf16 token row, owner-local expert, routing weight, source); the owner runs
 * glmaxx_moe_layer_launch over its received rows (GLMAXX_MOE_ROUTES_GIVEN,
 * top_k 1, its experts' weights); glmaxx_moe_ep_return_launch copies each output
 * row into the source rank's slot plane [tokens][top_k][hidden]; the source runs
 * glmaxx_moe_layer_launch with GLMAXX_MOE_EXTERNAL_ROUTED (shared expert +
 * expert-order combine).  The arrays of 8 hold every rank's buffers as mapped on
 * this GPU, in rank order (entries >= ranks are 0).  dest_row_offset[d] is the
 * first row of this rank's block in owner d's buffers: the sum of the row counts
 * ranks before this one send to d (their expert_offsets, exchanged by the host).
 * Rows move with plain 16-byte loads and stores, peer memory included.  A row
 * past an owner's capacity sets GLMAXX_STATUS_CAPACITY_EXCEEDED and is dropped.
 */
#if defined(__cplusplus)
struct alignas(16) glmaxx_moe_ep_descriptor {
#else
struct glmaxx_moe_ep_descriptor {
#endif
  uint32_t abi_version; /* GLMAXX_MOE_EP_ABI_VERSION */
  uint32_t struct_bytes;
  uint32_t ranks;       /* 1..8 */
  uint32_t rank;
  uint32_t tokens;      /* dispatch: this rank's tokens */
  uint32_t hidden;
  uint32_t experts;     /* all experts (a multiple of ranks) */
  uint32_t top_k;
  uint32_t rows;        /* return: rows this rank received */
  uint32_t reserved0[3];
  uint64_t input_bf16;            /* dispatch: [tokens][hidden]                   */
  uint64_t compacted_tokens_u32;  /* dispatch: glmaxx_router_compact_launch outputs */
  uint64_t compacted_experts_u16;
  uint64_t compacted_slots_u8;
  uint64_t compacted_weights_f32;
  uint64_t expert_offsets_u32;
  uint64_t recv_x_bf16[8];        /* every rank's receive buffers                 */
  uint64_t recv_expert_u16[8];
  uint64_t recv_weight_f32[8];
  uint64_t recv_source_u32[8];
  uint32_t recv_capacity[8];      /* rows each rank's receive buffers hold        */
  uint32_t dest_row_offset[8];
  uint64_t rows_out_f32;          /* return: [rows][hidden], this rank's owner output */
  uint64_t planes_f32[8];         /* every rank's slot plane [tokens_r][top_k][hidden] */
  uint32_t plane_tokens[8];
  uint64_t validation_error_u32;
  uint64_t reserved[4];
};

/* ---- reference entry points (glmaxx_kernel.h:123-250) ---- */
int32_t glmaxx_nvfp4_routed_fc1_launch(const struct glmaxx_fc1_descriptor* descriptor,
                                       void* cuda_stream, int32_t* asynchronous_error);
int32_t glmaxx_nvfp4_routed_fc1_graph_instantiate(const struct glmaxx_fc1_descriptor* descriptor,
                                                  void* cuda_stream, uint64_t* graph_exec);
int32_t glmaxx_nvfp4_quantize_launch(const struct glmaxx_fc1_descriptor* descriptor,
                                     void* cuda_stream);
int32_t glmaxx_nvfp4_grouped_quantize_launch(const struct glmaxx_fc1_descriptor* descriptor,
                                             void* cuda_stream);
int32_t glmaxx_nvfp4_core_swiglu_launch(const struct glmaxx_fc1_descriptor* descriptor,
                                        void* cuda_stream);
int32_t glmaxx_nvfp4_dense_control_launch(const struct glmaxx_fc1_descriptor* descriptor,
                                          uint32_t expert, void* cuda_stream,
                                          int32_t* asynchronous_error);
int32_t glmaxx_nvfp4_grouped_control_launch(const struct glmaxx_fc1_descriptor* descriptor,
                                            const uint16_t* active_experts,
                                            uint32_t active_expert_count, void* cuda_stream,
                                            int32_t* asynchronous_error);
int32_t glmaxx_nvfp4_grouped_core_swiglu_launch(const struct glmaxx_fc1_descriptor* descriptor,
                                                const uint16_t* active_experts,
                                                uint32_t active_expert_count, void* cuda_stream,
                                                int32_t* asynchronous_error);
int32_t glmaxx_nvfp4_grouped_prepare_launch(const struct glmaxx_fc1_descriptor* descriptor,
                                            const uint16_t* active_experts,
                                            uint32_t active_expert_count, void* cuda_stream);
int32_t glmaxx_nvfp4_grouped_prepared_control_launch(
    const struct glmaxx_fc1_descriptor* descriptor, uint32_t active_expert_count,
    void* cuda_stream, int32_t* asynchronous_error);
int32_t glmaxx_nvfp4_grouped_prepared_core_swiglu_launch(
    const struct glmaxx_fc1_descriptor* descriptor, uint32_t active_expert_count,
    void* cuda_stream, int32_t* asynchronous_error);
int32_t glmaxx_nvfp4_routed_fc2_launch(const struct glmaxx_fc2_descriptor* descriptor,
                                       void* cuda_stream, int32_t* asynchronous_error);
int32_t glmaxx_nvfp4_fc2_quantize_launch(const struct glmaxx_fc2_descriptor* descriptor,
                                         void* cuda_stream);
int32_t glmaxx_nvfp4_fc2_grouped_quantize_launch(const struct glmaxx_fc2_descriptor* descriptor,
                                                 void* cuda_stream);
int32_t glmaxx_nvfp4_fc2_core_launch(const struct glmaxx_fc2_descriptor* descriptor,
                                     void* cuda_stream);
int32_t glmaxx_nvfp4_fc2_reduce_launch(const struct glmaxx_fc2_descriptor* descriptor,
                                       void* cuda_stream);
int32_t glmaxx_nvfp4_fc2_dense_control_launch(const struct glmaxx_fc2_descriptor* descriptor,
                                              uint32_t expert, void* cuda_stream,
                                              int32_t* asynchronous_error);
int32_t glmaxx_nvfp4_fc2_grouped_control_launch(const struct glmaxx_fc2_descriptor* descriptor,
                                                const uint16_t* active_experts,
                                                uint32_t active_expert_count, void* cuda_stream,
                                                int32_t* asynchronous_error);
int32_t glmaxx_exl3_projection_launch(const struct glmaxx_exl3_descriptor* descriptor,
                                      void* cuda_stream, int32_t* asynchronous_error);
int32_t glmaxx_graph_exec_launch(uint64_t graph_exec, uint64_t stream);
int32_t glmaxx_graph_exec_destroy(uint64_t graph_exec);
/* Stream capture (new): begin capturing `stream` (thread-local capture mode); end
 * it and instantiate the captured work into an executable graph for
 * glmaxx_graph_exec_launch / glmaxx_graph_exec_destroy. */
int32_t glmaxx_stream_begin_capture(uint64_t stream);
int32_t glmaxx_stream_end_capture(uint64_t stream, uint64_t* graph_exec);
int32_t glmaxx_event_create(uint64_t* event);
int32_t glmaxx_event_record(uint64_t event, uint64_t stream);
int32_t glmaxx_event_synchronize(uint64_t event);
int32_t glmaxx_event_elapsed_ms(uint64_t start, uint64_t end, float* milliseconds);
int32_t glmaxx_event_destroy(uint64_t event);
int32_t glmaxx_profiler_start(void);
int32_t glmaxx_profiler_stop(void);
int32_t glmaxx_nvtx_range_push(const char* message);
int32_t glmaxx_nvtx_range_pop(void);

/* Workspace sizes for the reference GLM-5.2 TP4 geometry (hidden 6144, local
 * intermediate 512, 256 experts), as the reference defines them
 * (nvfp4_routed_fc1.cu:346-368, nvfp4_routed_fc2.cu:512-544). */
uint64_t glmaxx_nvfp4_routed_fc1_workspace_bytes(uint32_t assignments);
uint64_t glmaxx_nvfp4_grouped_workspace_bytes(uint32_t assignments);
uint64_t glmaxx_nvfp4_routed_fc2_workspace_bytes(uint32_t rows, uint32_t assignments);
uint64_t glmaxx_nvfp4_grouped_fc2_workspace_bytes(uint32_t rows, uint32_t assignments);
uint64_t glmaxx_exl3_projection_workspace_bytes(uint32_t rows, uint32_t logical_k,
                                                uint32_t logical_n);
const char* glmaxx_kernel_abi(void);
const char* glmaxx_exl3_kernel_abi(void);

/* Runtime helpers (glmaxx_kernel.h:221-250, same signatures). */
int32_t glmaxx_device_count(int32_t* count);
int32_t glmaxx_device_bind(int32_t device_index, int32_t* compute_capability,
                           int32_t* multiprocessor_count, uint64_t* total_memory_bytes,
                           uint8_t device_uuid[16]);
int32_t glmaxx_device_memory_info(uint64_t* free_memory_bytes, uint64_t* total_memory_bytes);
int32_t glmaxx_device_alloc(uint64_t bytes, uint64_t* pointer);
int32_t glmaxx_device_free(uint64_t pointer);
int32_t glmaxx_pinned_alloc(uint64_t bytes, uint64_t* pointer);
int32_t glmaxx_pinned_free(uint64_t pointer);
int32_t glmaxx_stream_create(uint64_t* stream);
int32_t glmaxx_stream_destroy(uint64_t stream);
int32_t glmaxx_stream_query(uint64_t stream, int32_t* complete);
int32_t glmaxx_stream_synchronize(uint64_t stream);
int32_t glmaxx_memcpy_h2d(uint64_t destination, const void* source, uint64_t bytes,
                          uint64_t stream);
int32_t glmaxx_memcpy_d2d(uint64_t destination, uint64_t source, uint64_t bytes, uint64_t stream);
int32_t glmaxx_memcpy_d2h(void* destination, uint64_t source, uint64_t bytes, uint64_t stream);
int32_t glmaxx_memset_zero(uint64_t destination, uint64_t bytes, uint64_t stream);

/* ---- new entry points ---- */

/* Geometry-aware workspace sizes (replace the fixed-geometry formulas above
 * for TP != 4 and for the 16-expert reduced layer). */
uint64_t glmaxx_nvfp4_routed_fc1_workspace_bytes_v3(uint32_t rows, uint32_t assignments,
                                                    uint32_t hidden, uint32_t local_intermediate,
                                                    uint32_t experts, uint32_t top_k);
uint64_t glmaxx_nvfp4_routed_fc2_workspace_bytes_v3(uint32_t rows, uint32_t assignments,
                                                    uint32_t hidden, uint32_t local_intermediate,
                                                    uint32_t experts, uint32_t top_k);
uint64_t glmaxx_router_workspace_bytes(uint32_t tokens, uint32_t hidden, uint32_t experts,
                                       uint32_t top_k);
uint64_t glmaxx_moe_layer_workspace_bytes(const struct glmaxx_moe_layer_descriptor* descriptor);

/* EXL3 decode-fused projection alone (the core of glmaxx_exl3_projection_launch
 * without the suh/H128 input and H128/svh output rotations): output[r][n] =
 * f16(sum_k input[r][k] * W[k][n]) over the 3-bit trellis W (exl3.rs layout,
 * K x N logical), fp32 multiply-then-add in ascending k exactly as
 * Exl3Trellis::matmul_reference_f16 (crates/glm-format/src/exl3.rs:404-453)
 * and the reference's warp-staging proof (warp_proof.rs:378-381).  k % 16 == 0,
 * n % 32 == 0, bits == 3.  Returns 0, GLMAXX_ERR_NULL, GLMAXX_ERR_DESCRIPTOR, an
 * arch error, or a cudaError_t. */
int32_t glmaxx_exl3_gemv_launch(uint64_t input_f16, uint64_t trellis_u16, uint32_t rows,
                                uint32_t logical_k, uint32_t logical_n, uint32_t bits,
                                uint64_t output_f16, void* cuda_stream);

int32_t glmaxx_router_compact_launch(const struct glmaxx_router_descriptor* descriptor,
                                     void* cuda_stream, int32_t* asynchronous_error);

/* Allocation-free variant of glmaxx_router_compact_launch (no counterpart in the
 * reference library).  For callers that cannot provide or allocate scratch
 * memory -- an engine whose HBM is planned up front with no per-call
 * workspace, or code that must not call cudaMalloc (it can synchronise the
 * device) -- the router's scratch lives in a device array of
 * GLMAXX_ROUTER_STATIC_SCRATCH_BYTES inside this library, held by every GPU
 * that loads it until exit.  The descriptor's workspace fields are ignored;
 * inputs and outputs are the caller's.  Shapes needing more scratch than the
 * array (glmaxx_router_workspace_bytes > 4 MiB; with 256 experts and top-8
 * that is T > 507) return GLMAXX_ERR_DESCRIPTOR.  The first call on a device
 * looks up the array's address (cached for the process; cudaDeviceReset is not
 * supported) and should be made before any stream capture.  All calls share
 * the array: calls whose GPU work overlaps race and must be serialised by the
 * caller. */
#define GLMAXX_ROUTER_STATIC_SCRATCH_BYTES (4ull << 20)
int32_t glmaxx_router_compact_launch_static(const struct glmaxx_router_descriptor* descriptor,
                                            void* cuda_stream, int32_t* asynchronous_error);
int32_t glmaxx_moe_layer_launch(const struct glmaxx_moe_layer_descriptor* descriptor,
                                void* cuda_stream, int32_t* asynchronous_error);
int32_t glmaxx_moe_finish_launch(const struct glmaxx_moe_finish_descriptor* descriptor,
                                 void* cuda_stream);
uint64_t glmaxx_moe_peer_signal_bytes(uint32_t ranks);
int32_t glmaxx_moe_finish_peer_launch(const struct glmaxx_moe_finish_descriptor* descriptor,
                                      const struct glmaxx_moe_peer_descriptor* peer,
                                      void* cuda_stream);

/* CUDA IPC of a glmaxx_device_alloc allocation between the processes of one host
 * (new; the peer form of the finish maps every rank's buffers with these).
 * glmaxx_ipc_handle writes the 64-byte handle of the allocation starting at
 * `pointer`; glmaxx_ipc_open maps another process's handle on the current device
 * (peer access enabled lazily); glmaxx_ipc_close unmaps it. */
int32_t glmaxx_ipc_handle(uint64_t pointer, uint8_t handle[64]);
int32_t glmaxx_ipc_open(const uint8_t handle[64], uint64_t* pointer);
int32_t glmaxx_ipc_close(uint64_t pointer);
/* One process driving several GPUs (a thread per rank): lets the current device
 * read and write peer_device's memory directly (cudaDeviceEnablePeerAccess; a
 * repeat call succeeds).  Returns GLMAXX_ERR_DESCRIPTOR for the current device or
 * an index out of range, cudaErrorPeerAccessUnsupported without a peer path. */
int32_t glmaxx_peer_enable(int32_t peer_device);

/* Profiling (the CUDA-event timing of the reference, crates/glm-cuda/src/
 * ffi.rs:3057-3079, per stage): while set, layer launches on the calling
 * thread record events[s] (cudaEvent_t handles) before stage s of
 * GLMAXX_LAYER_STAGE_* and events[GLMAXX_LAYER_STAGES] after the last, on the
 * launch stream.  count must be >= GLMAXX_LAYER_STAGES + 1; events = NULL clears. */
enum {
  GLMAXX_LAYER_STAGE_ROUTER = 0,
  GLMAXX_LAYER_STAGE_COMPACT = 1,
  GLMAXX_LAYER_STAGE_QUANT = 2,
  GLMAXX_LAYER_STAGE_FC1 = 3,
  GLMAXX_LAYER_STAGE_FC2_QUANT = 4,
  GLMAXX_LAYER_STAGE_SHARED = 5,
  GLMAXX_LAYER_STAGE_FC2 = 6,
  GLMAXX_LAYER_STAGE_COMBINE = 7,
  GLMAXX_LAYER_STAGES = 8,
};
int32_t glmaxx_moe_layer_set_stage_events(uint64_t* events, uint32_t count);

/* Workspace introspection: device address and size of an intermediate plane
 * of the last glmaxx_moe_layer_launch with this descriptor (valid after the
 * launch completes).  Rows are in compacted (expert, token, slot) order, the
 * order of crates/glm-reference/src/routed_fc1.rs:20-58. */
enum {
  GLMAXX_PLANE_FC1_OUTPUT_BF16 = 0,    /* [assignments][local_intermediate] SwiGLU output */
  GLMAXX_PLANE_ROW_TOKEN_U32 = 1,      /* [assignments] token of each compacted row       */
  GLMAXX_PLANE_ROW_SLOT_U32 = 2,       /* [assignments] route slot                        */
  GLMAXX_PLANE_ROW_WEIGHT_F32 = 3,     /* [assignments] routing weight                    */
  GLMAXX_PLANE_EXPERT_OFFSETS_U32 = 4, /* [experts + 1] exclusive compacted offsets       */
  GLMAXX_PLANE_SHARED_F32 = 5,         /* [tokens][hidden] shared expert (decode path)     */
  GLMAXX_PLANE_ROUTED_F32 = 6,         /* [tokens][top_k][hidden] routing-weighted expert
                                          outputs per slot (decode path, EXL3 experts)   */
};
int32_t glmaxx_moe_layer_plane(const struct glmaxx_moe_layer_descriptor* descriptor,
                               uint32_t which, uint64_t* address, uint64_t* bytes);

/* PackedNvfp4::pack (1-D codec) of `batch` row-major [n][k] tensors (f32 when
 * src_is_bf16 == 0, else bf16), n % 128 == 0, k % 64 == 0.  Tensor b writes
 * values + b*n*k/2, scales + b*n*k/16, global_scale[b], global_amax[b]
 * (global_amax may be 0).  scratch: >= 4*batch bytes of device memory. */
int32_t glmaxx_nvfp4_pack_launch(uint64_t src, int32_t src_is_bf16, uint32_t batch, uint32_t n,
                                 uint32_t k, uint64_t values, uint64_t scales,
                                 uint64_t global_scale_f32, uint64_t global_amax_f32,
                                 uint64_t scratch, uint64_t validation_error_u32,
                                 void* cuda_stream);

/* Measurement entry point (no reference counterpart: the reference publishes no
 * NVFP4 tensor peak).  `ctas` CTAs (one per SM) each issue `iters` x 4 (x2 when
 * dual) back-to-back tcgen05 block-scaled NVFP4 MMAs, M = 128, N = n (128 or
 * 256; dual needs 128), K = 64, on operands resident in shared memory and scales
 * resident in TMEM, with copies_per_kblock tcgen05.cp scale copies before each
 * K-block's MMAs (copy_kind 1: 32x128b.warpx4, 512 bytes; 2: 128x256b, 4 KB;
 * 0: none; copy_kind | 4: a 4-K-block stage's copies all issued before its first
 * MMA).  FLOPs per launch = ctas * iters * 4 * (dual ? 2 : 1) * 2*128*n*64.
 * iters <= 200000.  cycles_u64 (optional, [ctas]) receives each CTA's %clock64
 * span of its MMA loop; status_u32 receives GLMAXX_STATUS bits. */
int32_t glmaxx_nvfp4_mma_peak_launch(uint32_t n, uint32_t dual, uint32_t copy_kind,
                                     uint32_t copies_per_kblock, uint32_t iters, uint32_t ctas,
                                     uint32_t* status_u32, unsigned long long* cycles_u64,
                                     void* cuda_stream);

int32_t glmaxx_moe_ep_dispatch_launch(const struct glmaxx_moe_ep_descriptor* descriptor,
                                      void* cuda_stream);
int32_t glmaxx_moe_ep_return_launch(const struct glmaxx_moe_ep_descriptor* descriptor,
                                    void* cuda_stream);

/* Self-check (no reference counterpart): runs every fp32 bit pattern through the
 * hardware E2M1 / E4M3 conversions the quantisation kernels use and through this
 * library's restatement of the reference codec (float.rs:15-73), on the GPU.
 * result_u64x4 (device): [0] E2M1 mismatches over all finite values, [1] E4M3
 * mismatches over all positive finite values, [2]/[3] bits + 1 of one
 * mismatching input (0 = none). */
int32_t glmaxx_nvfp4_codec_selfcheck_launch(unsigned long long* result_u64x4, void* cuda_stream);

/* Self-check (no reference counterpart): every finite fp32 value v against each
 * divisor decs[0..n_decs) (device, n_decs <= 4096): the E2M1 code the
 * quantisation kernels give v / dec (a reciprocal product bracketed within
 * 2^-20, the exact quotient where an E2M1 midpoint is that close) against the
 * code of the exactly rounded quotient fl(v / dec), the reference's
 * (nvfp4.rs:567-608).  result_u64x4 (device): [0] mismatches, [1] (divisor
 * index << 32 | v bits) + 1 of one mismatch (0 = none), [2] values decided on
 * the bracket alone, [3] values checked. */
int32_t glmaxx_nvfp4_quotient_selfcheck_launch(const float* decs, uint32_t n_decs,
                                               unsigned long long* result_u64x4,
                                               void* cuda_stream);

#if defined(__cplusplus)
}

static_assert(sizeof(glmaxx_fc1_descriptor) == 224, "Rust/C descriptor size mismatch");
static_assert(alignof(glmaxx_fc1_descriptor) == 16, "Rust/C descriptor alignment mismatch");
static_assert(sizeof(glmaxx_fc2_descriptor) == 224, "Rust/C FC2 descriptor size mismatch");
static_assert(alignof(glmaxx_fc2_descriptor) == 16, "Rust/C FC2 descriptor alignment mismatch");
static_assert(sizeof(glmaxx_exl3_descriptor) == 144, "Rust/C EXL3 descriptor size mismatch");
static_assert(alignof(glmaxx_exl3_descriptor) == 16, "Rust/C EXL3 descriptor alignment mismatch");
static_assert(sizeof(glmaxx_router_descriptor) == 192, "router descriptor size");
static_assert(sizeof(glmaxx_moe_layer_descriptor) == 240, "layer descriptor size");
static_assert(sizeof(glmaxx_moe_exl3_experts) == 128, "EXL3 experts descriptor size");
static_assert(sizeof(glmaxx_moe_finish_descriptor) == 112, "finish descriptor size");
static_assert(sizeof(glmaxx_moe_peer_descriptor) == 80, "peer descriptor size");
static_assert(sizeof(glmaxx_moe_ep_descriptor) == 560, "expert-parallel descriptor size");
#endif

#endif /* GLMAXX_KERNEL_H_ */
