// Internal host-side interface between the C ABI (abi.cu), the routed-MoE
// step orchestration (layer.cu) and the kernels (moe_kernels.cu, gemm.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "gemm.cuh"

namespace glmaxx {

struct QuantScatterArgs {
  const uint16_t* x;              // [T][H] bf16
  const uint16_t* route_experts;  // [T][K]
  const float* route_weights;     // [T][K]
  const uint32_t* bitmap;         // [E][W]
  const uint32_t* wprefix;        // [E][W]
  const uint32_t* poffs;          // [E+1]
  const uint32_t* offsets;        // [E+1]
  uint8_t* xq;                    // [A][H/2], compacted rows
  uint8_t* xsf;                   // atoms, padded row space
  uint32_t* row_token;            // [A] compacted row -> token
  uint32_t* row_slot;             // [A] -> slot
  float* row_weight;              // [A] -> routing weight
  float* row_gscale;              // [A] -> NVFP4 global scale of the row
  uint32_t* row_prow;             // [A] -> padded (scale-factor) row
  uint32_t* route_row;            // [T*K] -> compacted row
  uint32_t* status;
  uint32_t T, H, E, top_k, sf_row_cap, nt;
};

// Compacted-order route arrays of the reference FC1/FC2 ABI, written from the
// device-side compaction (router_compact).
struct CompactWriteArgs {
  const uint16_t* route_experts;  // [T*K]
  const float* route_weights;     // [T*K]
  const uint32_t* bitmap;
  const uint32_t* wprefix;
  const uint32_t* offsets;
  uint32_t* comp_token;
  uint16_t* comp_expert;
  uint8_t* comp_slot;
  float* comp_weight;
  uint32_t T, E, top_k;
};

// From reference-ABI compacted routes (expert, token, slot per assignment,
// expert_offsets[E+1]): padded offsets, per-row padded row, n tiles.
struct CompatPrepareArgs {
  const uint16_t* route_experts;  // [A] compacted order
  const uint32_t* offsets;        // [E+1]
  uint32_t* poffs;                // [E+1]
  uint32_t* row_prow;             // [A]
  NTile* tiles;
  uint32_t* tile_count;
  uint32_t A, E, nt, sf_row_cap, max_tiles;
  uint32_t* status;
  uint32_t expert_mask[8];        // experts that receive tiles (bit e of word e/32)
};

// Reference-ABI quantiser: NVFP4 rows of src[src_row(r)] for compacted rows r
// (FC1: src = input_bf16, src_row = route_tokens; FC2: src = h, src_row = r).
struct QuantRowsArgs {
  const uint16_t* src;       // [*][K] bf16
  const uint32_t* src_row;   // [A] or null (identity)
  const uint32_t* row_prow;  // [A] padded scale-factor row
  uint8_t* values;           // [A][K/2]
  uint8_t* scales;           // atoms
  float* gscale;             // [A]
  uint32_t* status;
  uint32_t A, K, src_rows, sf_row_cap;
};

// Reference FC2 slot table and slot-ordered reduce
// (kernels/sm120/nvfp4_routed_fc2.cu:187-230, 318-348).
struct SlotArgs {
  const uint16_t* route_experts;  // [A] compacted
  const uint32_t* route_tokens;
  const uint8_t* route_slots;
  const float* route_weights;
  uint32_t* slot_assignment;      // [rows][top_k]
  const float* assignment_down;   // [A][H]
  float* token_output;            // [rows][H]
  uint32_t* status;
  uint32_t A, rows, H, E, top_k;
};

struct Fc2QuantArgs {
  const uint16_t* h;         // [A][I] bf16, compacted rows
  const uint32_t* row_prow;  // [A] compacted row -> padded (scale-factor) row
  uint8_t* hq;               // [A][I/2]
  uint8_t* hsf;              // atoms, padded row space
  float* gscale;             // [A]
  uint32_t* status;
  const uint32_t* count_ptr; // device count of rows (offsets[E]) or null
  uint32_t count, I, sf_row_cap;
  // optional: rows of experts with skip_codec[e] == 1 (EXL3) are not quantised
  const uint32_t* offsets;   // [E + 1] compacted row offsets
  const uint8_t* skip_codec; // [E]
  uint32_t E;
};

struct FinishArgs {
  const float* residual_f32;
  const uint16_t* residual_bf16;
  const float* attention_f32;  // [ranks][elements] or null
  const float* partials[8];    // rank order
  float* output_f32;
  uint16_t* output_bf16;
  uint16_t* norm_bf16;         // optional row-wise RMSNorm output
  uint64_t elements;           // multiple of 4
  uint32_t ranks;
  uint32_t hidden;             // row length (norm_bf16)
  float eps;
};
cudaError_t launch_finish(const FinishArgs& a, cudaStream_t stream);
// Peer form of the finish: every rank's signal buffer and, for two-shot, every
// rank's outputs (rank order).
struct FinishPeer {
  uint32_t* signals[8];
  float* outputs_f32[8];
  uint16_t* outputs_bf16[8];
  uint16_t* norms_bf16[8];
  uint32_t* status;
  uint32_t rank;
  bool two_shot;
};
cudaError_t launch_finish_peer(const FinishArgs& a, const FinishPeer& p, cudaStream_t stream);

cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* w, float* partial, uint32_t T,
                                 uint32_t H, uint32_t E, uint32_t* bitmap, uint32_t bitmap_words,
                                 cudaStream_t stream);
cudaError_t launch_router_select(const float* partial, const float* bias, uint32_t T, uint32_t E,
                                 uint32_t groups, uint32_t topk_groups, uint32_t top_k,
                                 float route_scale, uint16_t* experts, float* weights,
                                 uint32_t* bitmap, uint32_t bitmap_stride, uint32_t* status,
                                 cudaStream_t stream);
cudaError_t launch_routes_to_bitmap(const uint16_t* experts, const float* weights, uint32_t T,
                                    uint32_t E, uint32_t top_k, uint32_t* bitmap,
                                    uint32_t bitmap_words, uint32_t* status, cudaStream_t stream);
cudaError_t launch_compact(const uint32_t* bitmap, uint32_t T, uint32_t E, uint32_t nt,
                           uint32_t sf_row_cap, uint32_t max_tiles, uint32_t* wprefix,
                           uint32_t* counts, uint32_t* offsets, uint32_t* poffs, NTile* tiles,
                           uint32_t* tile_count, uint32_t* status, cudaStream_t stream,
                           const uint8_t* no_tiles = nullptr);
cudaError_t launch_quant_scatter(const QuantScatterArgs& a, cudaStream_t stream);
cudaError_t launch_compact_write(const CompactWriteArgs& a, cudaStream_t stream);
cudaError_t launch_compat_prepare(const CompatPrepareArgs& a, cudaStream_t stream);
cudaError_t launch_fc2_quant(const Fc2QuantArgs& a, cudaStream_t stream);
cudaError_t launch_quant_rows(const QuantRowsArgs& a, cudaStream_t stream);
cudaError_t launch_slot_table(const SlotArgs& a, cudaStream_t stream);
cudaError_t launch_slot_reduce(const SlotArgs& a, cudaStream_t stream);
cudaError_t launch_combine(const float* plane, const uint16_t* experts, const float* shared,
                           uint32_t shared_splits, float* shared_out, float* out, uint32_t T,
                           uint32_t H, uint32_t top_k, cudaStream_t stream);
// Bulk L2 prefetch of [a, a + a_bytes) and [b, b + b_bytes) (16-byte aligned).
cudaError_t launch_l2_prefetch(const void* a, uint64_t a_bytes, const void* b, uint64_t b_bytes,
                               cudaStream_t stream);
cudaError_t launch_swiglu_finish(const float* parts, uint32_t splits, uint32_t T, uint32_t I,
                                 uint16_t* h, cudaStream_t stream);
cudaError_t launch_pack(const void* src, int src_bf16, uint32_t batch, uint32_t N, uint32_t K,
                        uint8_t* values, uint8_t* scales, float* global_scale, float* global_amax,
                        uint32_t* amax_scratch, uint32_t* status, cudaStream_t stream);

// ------------------------------------------------------------------ GEMMs
// A operand: [experts][a_rows][a_row_bytes] bytes (weights); B operand:
// [b_rows][b_row_bytes] bytes (activations).  Row bytes = K/2 (NVFP4) or 2K (BF16).
struct GemmLaunch {
  const void* a;
  uint32_t a_experts, a_rows, a_row_bytes;
  const void* b;
  uint32_t b_rows, b_row_bytes;
  GemmArgs args;
};

enum GemmVariant : int {
  kFc1DecodeFp4 = 0,    // NVFP4, gate+up, N tile 32, SwiGLU
  kFc2DecodeFp4 = 1,    // NVFP4, N tile 32, routed plane
  kFc1PrefillFp4 = 2,   // NVFP4, gate+up, N tile 128, SwiGLU
  kFc2PrefillFp4 = 3,   // NVFP4, N tile 128, routed atomics
  kShared1Bf16N64 = 4,  // BF16, gate+up, N tile 64, SwiGLU
  kShared2Bf16N64 = 5,  // BF16, N tile 64, store f32
  kShared1Bf16N128 = 6,
  kShared2Bf16N128 = 7,
  kFc2DecodeFp4Store = 8,  // NVFP4, N tile 32, store f32 (reference FC2 assignment plane)
  kFc2PrefillFp4Store = 9, // NVFP4, N tile 128, store f32
  kShared1Bf16N64Split = 10,  // BF16, gate+up, N tile 64, split-K partials
  kShared2Bf16N64Split = 11,  // BF16, N tile 64, split-K partials
  kFc2DecodeFp4Pair = 12,     // NVFP4, two adjacent M tiles per item, N tile 32, routed plane
  kFc2PrefillFp4PairAtomic = 13, // NVFP4, two adjacent M tiles per item, N tile 128, routed atomics
  kFc2PrefillFp4PairPlane = 14,  // as 13, writing the routed plane (deterministic combine)
};

// Number of K slices (and chunks per slice) that spread `tiles` output tiles of
// k_chunks chunks over about `sms` CTAs, every slice non-empty.
void choose_k_splits(uint32_t tiles, uint32_t k_chunks, int sms, uint32_t max_splits,
                     uint32_t* splits, uint32_t* kc_per);

int gemm_tile_rows(GemmVariant v);
cudaError_t launch_gemm(GemmVariant v, const GemmLaunch& g, int num_sms, cudaStream_t stream);

}  // namespace glmaxx
