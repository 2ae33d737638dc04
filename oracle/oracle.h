/*
 * CPU oracle for the routed-MoE hot path: TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, in plain C, the reference arithmetic of yatesdr/glmaxx
 * for the routed-expert MoE step (NVFP4 codec, route compaction, FC1/FC2
 * oracles, rank-order finish, EXL3 trellis decode) plus this project's own
 * router definition (the reference specifies the router in one sentence only).
 * Each function names the reference file:line it follows.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the
 * product library never links or calls it.
 *
 * Build: oracle/Makefile (gcc -O3 -ffp-contract=off, no fast-math) so that
 * every floating-point operation rounds exactly once, like Rust's f32 ops.
 */
#ifndef GLMAXX_ORACLE_H_
#define GLMAXX_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_OK = 0, ORC_ERR_NONFINITE = -1, ORC_ERR_SHAPE = -2, ORC_ERR_ROUTE = -3,
       ORC_ERR_INDEX = -4, ORC_ERR_ALLOC = -5 };
enum { ORC_CODEC_1D = 1, ORC_CODEC_2D = 2 };

typedef struct {
  uint32_t token;
  uint16_t expert;
  uint8_t slot;
  uint8_t pad;
  float weight;
} orc_route;

typedef struct {
  uint32_t token;
  uint16_t expert;
  uint8_t slot;
  uint8_t pad;
} orc_compacted_route;

/* crates/glm-format/src/float.rs */
float orc_decode_e2m1(uint8_t code);
int orc_encode_e2m1(float value, uint8_t* code);
float orc_decode_e4m3(uint8_t code);
int orc_encode_e4m3(float value, uint8_t* code);

/* crates/glm-format/src/crc32c.rs, nvfp4.rs */
uint32_t orc_crc32c(const uint8_t* bytes, uint64_t length);
int64_t orc_scale_offset(uint64_t n, uint64_t group, uint64_t padded_n, uint64_t padded_k);
int orc_nvfp4_pack(const float* input, uint64_t logical_n, uint64_t logical_k, int codec,
                   uint8_t* values, uint8_t* scales, float* global_scale, float* global_amax);
int orc_nvfp4_dequantize(const uint8_t* values, const uint8_t* scales, float global_scale,
                         uint64_t logical_n, uint64_t logical_k, float* output);
void orc_nvfp4_metadata_encode(int codec, uint32_t logical_n, uint32_t logical_k,
                               uint32_t padded_n, uint32_t padded_k, float global_scale,
                               float global_amax, uint32_t value_bytes, uint32_t scale_bytes,
                               uint8_t out[128]);

/* crates/glm-reference/src/routed_fc1.rs */
float orc_bf16_round(float value);
int orc_compact_routes(const orc_route* routes, uint64_t count, uint64_t token_count,
                       orc_compacted_route* output);
int orc_routed_fc1(const float* activations, uint64_t rows, uint64_t k, const uint8_t* w_values,
                   const uint8_t* w_scales, float w_global, uint64_t n, float* output);
int orc_routed_fc1_fixed_tree_at(const float* activation, uint64_t k, const uint8_t* w_values,
                                 const uint8_t* w_scales, float w_global, uint64_t n,
                                 uint64_t column, float* output);

/* crates/glm-reference/src/routed_fc2.rs */
int orc_routed_fc2(const float* activated, const orc_route* routes, uint64_t route_count,
                   uint64_t token_count, uint64_t local_intermediate, uint64_t hidden,
                   const uint16_t* weight_experts, const uint8_t* const* down_values,
                   const uint8_t* const* down_scales, const float* down_globals,
                   uint64_t weight_count, float* output);
int orc_finish_sparse_layer(const float* input_residual, const float* attention,
                            const float* routed, const float* shared, uint32_t ranks,
                            uint64_t elements, float* output);

/* crates/glm-reference/src/matrix.rs, crates/glm-cli/src/main.rs */
int orc_generate_routes(int routing_case, uint64_t token_count, orc_route* routes,
                        uint64_t* count);
int orc_generate_numerical_fixture(int numerical_case, uint64_t rows, uint64_t n, uint64_t k,
                                   float* activations, float* weights);
void orc_actual_shape_values(uint64_t n, uint64_t k, float* output);

/* Router restatement (crates/glm-reference/src/manifest.rs:188-194). */
float orc_router_exp(float x);
float orc_router_sigmoid(float x);
void orc_router_logits(const uint16_t* x_bf16, uint64_t tokens, uint64_t hidden,
                       const uint16_t* w_bf16, uint64_t experts, float* logits, int threads);
int orc_router_select(const float* logits, uint64_t tokens, uint64_t experts, const float* bias,
                      uint32_t groups, uint32_t topk_groups, uint32_t topk, float route_scale,
                      uint16_t* experts_out, float* weights_out);

/* Full rank-local routed-MoE layer (routes given), per the reference op order. */
int orc_moe_layer(uint32_t tokens, uint32_t hidden, uint32_t experts, uint32_t local_inter,
                  uint32_t topk, const uint16_t* x_bf16, const uint16_t* route_experts,
                  const float* route_weights, const uint8_t* w13_values,
                  const uint8_t* w13_scales, const float* w13_global, const uint8_t* w2_values,
                  const uint8_t* w2_scales, const float* w2_global,
                  const uint16_t* shared13_bf16, const uint16_t* shared2_bf16,
                  uint32_t shared_inter, const uint32_t* token_subset, uint32_t subset_count,
                  float* routed_out, float* shared_out, int threads);

/* Prepared-expert form of orc_moe_layer (same bits): an expert's weights
 * dequantised once into k-major fp32 planes (w13t [H][2I], w2t [I][H]; shared
 * s13t [H][2Is], s2t [Is][H]), then its assignments in parallel with SIMD
 * across output columns.  Calling orc_moe_expert_rows per expert in ascending
 * order reproduces the compacted accumulation order of orc_moe_layer. */
int orc_expert_prepare(const uint8_t* w13_values, const uint8_t* w13_scales, float w13_global,
                       const uint8_t* w2_values, const uint8_t* w2_scales, float w2_global,
                       uint32_t hidden, uint32_t local_inter, float* w13t, float* w2t);
int orc_shared_prepare(const uint16_t* shared13_bf16, const uint16_t* shared2_bf16,
                       uint32_t hidden, uint32_t shared_inter, float* s13t, float* s2t);
int orc_moe_expert_h(uint32_t hidden, uint32_t local_inter, const uint16_t* x_bf16,
                     const uint32_t* tokens, uint32_t rows, const float* w13t, float* h,
                     int threads);
int orc_moe_expert_rows(uint32_t hidden, uint32_t local_inter, const uint16_t* x_bf16,
                        const uint32_t* tokens, const float* weights, const uint32_t* out_rows,
                        uint32_t rows, const float* w13t, const float* w2t, float* out,
                        int threads);
int orc_shared_rows(uint32_t hidden, uint32_t shared_inter, const uint16_t* x_bf16,
                    const uint32_t* tokens, uint32_t rows, const float* s13t, const float* s2t,
                    float* shared_out, int threads);
int orc_threads(void);

/* crates/glm-format/src/exl3.rs */
uint16_t orc_f32_to_f16_bits(float value);
float orc_f16_bits_to_f32(uint16_t bits);
void orc_exl3_xorshift_trellis(uint64_t seed, uint64_t words, uint16_t* trellis);
uint16_t orc_exl3_decode_native_at(const uint16_t* trellis, uint64_t logical_n, uint32_t bits,
                                   uint64_t row, uint64_t column);
void orc_exl3_reconstruct_native(const uint16_t* trellis, uint64_t k, uint64_t n, uint32_t bits,
                                 uint16_t* output);
int orc_exl3_prepare(const uint16_t* trellis, uint64_t k, uint64_t n, uint32_t bits,
                     float* nativef);
int orc_exl3_project(const float* nativef, uint64_t k, uint64_t n, const uint16_t* suh,
                     const uint16_t* svh, const uint16_t* activations, uint64_t rows,
                     uint16_t* output, int threads);
int orc_exl3_matmul_reference(const uint16_t* trellis, uint64_t k, uint64_t n, uint32_t bits,
                              const uint16_t* suh, const uint16_t* svh,
                              const uint16_t* activations, uint64_t rows, uint16_t* output,
                              int threads);

#ifdef __cplusplus
}
#endif
#endif
