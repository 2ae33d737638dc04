// Device properties cache and the architecture gate shared by the entry points.
#pragma once

#include <cstdint>

struct glmaxx_moe_layer_descriptor;
struct glmaxx_router_descriptor;

namespace glmaxx {

struct DeviceInfo {
  int device;
  int sms;
  int major;
  int minor;
};

// Fills `info` for the current device.  Returns 0, GLMAXX_ERR_WRONG_ARCH when
// the device is not compute capability 10.x (B200 / sm_100a), or a cudaError_t.
int32_t current_device_info(DeviceInfo* info);

enum LayerStage : uint32_t {
  kStageRouter = 0,
  kStageCompact = 1,
  kStageQuant = 2,
  kStageFc1 = 3,
  kStageFc2Quant = 4,
  kStageShared = 5,
  kStageFc2 = 6,
  kStageCombine = 7,
  kLayerStages = 8,
};
int32_t set_stage_events(uint64_t* events, uint32_t count);

uint64_t layer_workspace_bytes(const glmaxx_moe_layer_descriptor& d);
int32_t layer_plane(const glmaxx_moe_layer_descriptor* desc, uint32_t which, uint64_t* address,
                    uint64_t* bytes);
int32_t moe_layer_launch(const glmaxx_moe_layer_descriptor* desc, void* stream, int32_t* async_err);
uint64_t router_workspace_bytes(uint32_t tokens, uint32_t experts, uint32_t top_k);
int32_t router_compact_launch(const glmaxx_router_descriptor* desc, void* stream,
                              int32_t* async_err);

// EXL3 decode-fused projection (exl3.cu): P = f16(x . W) in the reference's
// order; single matrix over `rows` rows, or groups of rows (one trellis each).
cudaError_t launch_exl3_gemv_single(const uint16_t* x, const uint16_t* trellis, uint32_t rows,
                                    uint32_t K, uint32_t N, uint16_t* out, cudaStream_t stream);
// EXL3 routed experts of the layer (exl3.cu): rows in compacted order, every
// EXL3 expert's rows through gate/up projections, SwiGLU and down projection,
// the routing-weighted result into plane[token][slot][hidden].
struct Exl3ExpertsLaunch {
  uint32_t A, H, I, E, top_k;
  const uint16_t* x_bf16;      // layer input [T][H]
  const uint32_t* offsets;     // [E + 1] compacted row offsets
  const uint8_t* codec;        // [E] or null
  const uint32_t* row_token;
  const uint32_t* row_slot;
  const float* row_weight;
  const uint16_t *gate_trellis, *up_trellis, *down_trellis;
  const uint16_t *gate_suh, *gate_svh, *up_suh, *up_svh, *down_suh, *down_svh;
  float* plane;                // [T][top_k][H]
  void* workspace;             // exl3_experts_workspace_bytes
  uint32_t* status;            // device status word
  int num_sms;
};
uint64_t exl3_experts_workspace_bytes(uint32_t A, uint32_t H, uint32_t I, uint32_t E);
struct NTile;  // grouped-GEMM tile descriptor (gemm.cuh)
// Tensor-core EXL3 projection (exl3_gemm.cu) of the experts with many rows.
cudaError_t launch_exl3_tc_tiles(const uint32_t* offsets, uint32_t E, const uint8_t* codec,
                                 uint32_t min_rows, NTile* tiles, uint32_t* tile_count,
                                 cudaStream_t stream);
cudaError_t launch_exl3_tc(const uint16_t* x, uint32_t x_rows, uint32_t K, const uint16_t* trellis,
                           uint64_t trellis_stride, const NTile* tiles, const uint32_t* tile_count,
                           uint32_t Nproj, uint16_t* out, uint32_t* status, int num_sms,
                           cudaStream_t stream);
cudaError_t launch_exl3_experts(const Exl3ExpertsLaunch& launch, cudaStream_t stream);

}  // namespace glmaxx
