// extern "C" entry points of libglmaxx_sm100.so (include/glmaxx_kernel.h).
//
// The reference FC1/FC2 launches (kernels/sm120/nvfp4_routed_fc1.cu:542-600,
// nvfp4_routed_fc2.cu:546-620) are implemented on the caller's planes with
// the same meaning: FC1 turns compacted routes + bf16 input into the bf16
// SwiGLU output [assignments][local_intermediate] in compacted order; FC2
// turns that into the unweighted per-assignment projection
// [assignments][hidden] and the slot-ordered weighted token output
// [rows][hidden].  The work runs on the tcgen05 grouped GEMMs; scratch for
// tile lists lives in planes the reference itself declares as workspace
// (FC1: compacted_input_bf16 past its 257-entry SFA plan; FC2: token_output_f32,
// which is only written by the final reduce).
#include <cuda_profiler_api.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cstring>

#include "../../include/glmaxx_kernel.h"
#include "moe.h"
#include "runtime.h"

namespace glmaxx {

int32_t current_device_info(DeviceInfo* info) {
  static thread_local int cached_device = -1;
  static thread_local DeviceInfo cached{};
  int dev = -1;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return int32_t(st);
  if (dev != cached_device) {
    cudaDeviceProp p{};
    st = cudaGetDeviceProperties(&p, dev);
    if (st != cudaSuccess) return int32_t(st);
    cached.device = dev;
    cached.sms = p.multiProcessorCount;
    cached.major = p.major;
    cached.minor = p.minor;
    cached_device = dev;
  }
  *info = cached;
  return info->major == 10 ? 0 : GLMAXX_ERR_WRONG_ARCH;
}

namespace {

constexpr uint32_t kRefHidden = 6144, kRefInter = 512, kRefExperts = 256, kRefTopK = 8;

uint64_t round128(uint64_t v) { return (v + 127) / 128 * 128; }
uint64_t up256(uint64_t v) { return (v + 255) / 256 * 256; }

// Grouped (expert-local 128-padded) scale rows, crates/glm-cuda/src/abi.rs:77-91.
uint64_t grouped_sf_rows(uint64_t assignments, uint64_t experts) {
  return assignments + 127 * (assignments < experts ? assignments : experts);
}

bool geometry_ok(uint32_t hidden, uint32_t inter, uint32_t experts, uint32_t top_k) {
  return hidden >= 256 && hidden % 256 == 0 && hidden <= 16384 && inter >= 256 &&
         (inter & (inter - 1)) == 0 && inter <= 2048 && experts >= 1 && experts <= 256 &&
         top_k >= 1 && top_k <= 8;
}

bool valid_fc1(const glmaxx_fc1_descriptor& d) {
  if (d.abi_version != GLMAXX_FC1_ABI_VERSION || d.struct_bytes != sizeof(d) || d.flags != 0 ||
      d.reserved0 != 0)
    return false;
  for (uint64_t r : d.reserved)
    if (r) return false;
  if (!geometry_ok(d.hidden, d.local_intermediate, d.experts, d.top_k) ||
      d.local_gate_up != 2 * d.local_intermediate)
    return false;
  if (d.rows == 0 || d.assignments == 0 || d.assignments > 65536 ||
      uint64_t(d.assignments) > uint64_t(d.rows) * d.top_k)
    return false;
  if (d.path != GLMAXX_FC1_DECODE_PERSISTENT && d.path != GLMAXX_FC1_PREFILL_GROUPED) return false;
  if (d.path == GLMAXX_FC1_DECODE_PERSISTENT && d.rows > 128) return false;
  return d.input_bf16 && d.expert_value_base && d.expert_scale_base && d.expert_global_scales &&
         d.route_experts_u16 && d.route_tokens_u32 && d.route_slots_u8 && d.route_weights_f32 &&
         d.expert_offsets_u32 && d.compacted_input_bf16 && d.activation_values &&
         d.activation_scales && d.activation_global_scales && d.gate_up_accum_f32 &&
         d.output_bf16 && d.expert_value_base % 256 == 0 && d.expert_scale_base % 256 == 0 &&
         d.activation_values % 256 == 0 && d.activation_scales % 16 == 0 &&
         d.compacted_input_bf16 % 16 == 0 && d.input_bf16 % 16 == 0;
}

bool valid_fc2(const glmaxx_fc2_descriptor& d) {
  if (d.abi_version != GLMAXX_FC2_ABI_VERSION || d.struct_bytes != sizeof(d) || d.flags != 0 ||
      d.reserved0 != 0 || d.reserved1 != 0)
    return false;
  for (uint64_t r : d.reserved)
    if (r) return false;
  if (!geometry_ok(d.hidden, d.local_intermediate, d.experts, d.top_k)) return false;
  if (d.rows == 0 || d.assignments == 0 || d.assignments > 65536 ||
      uint64_t(d.assignments) > uint64_t(d.rows) * d.top_k)
    return false;
  if (d.path != GLMAXX_FC1_DECODE_PERSISTENT && d.path != GLMAXX_FC1_PREFILL_GROUPED) return false;
  return d.input_bf16 && d.expert_value_base && d.expert_scale_base && d.expert_global_scales &&
         d.route_experts_u16 && d.route_tokens_u32 && d.route_slots_u8 && d.route_weights_f32 &&
         d.expert_offsets_u32 && d.activation_values && d.activation_scales &&
         d.activation_global_scales && d.assignment_down_f32 && d.token_output_f32 &&
         d.slot_assignment_u32 && d.validation_error_u32 && d.expert_value_base % 256 == 0 &&
         d.expert_scale_base % 256 == 0 && d.activation_values % 256 == 0 &&
         d.activation_scales % 16 == 0 && d.token_output_f32 % 256 == 0 && d.input_bf16 % 16 == 0;
}

// Scratch carved from a caller plane: padded offsets, row -> padded row, tiles.
struct CompatScratch {
  uint32_t* poffs;
  uint32_t* row_prow;
  NTile* tiles;
  uint32_t* tile_count;
  uint32_t max_tiles;
  uint64_t bytes;
  void carve(uint64_t base, uint32_t A, uint32_t E, uint32_t nt) {
    const uint32_t active = A < E ? A : E;
    max_tiles = (A + nt - 1) / nt + active;
    uint64_t c = up256(base);
    poffs = reinterpret_cast<uint32_t*>(c);
    c = up256(c + uint64_t(E + 1) * 4);
    row_prow = reinterpret_cast<uint32_t*>(c);
    c = up256(c + uint64_t(A) * 4);
    tiles = reinterpret_cast<NTile*>(c);
    c = up256(c + uint64_t(max_tiles) * sizeof(NTile));
    tile_count = reinterpret_cast<uint32_t*>(c);
    c = up256(c + 16);
    bytes = c - base;
  }
};

// FC1 scratch starts past the reference's 257 x u64 grouped-SFA plan that the
// caller stores at the head of compacted_input_bf16 (crates/glm-cuda/src/ffi.rs:2224-2229).
constexpr uint64_t kFc1ScratchOffset = 4096;

struct Fc1Plan {
  CompatScratch s;
  uint32_t nt;
  GemmVariant variant;
  uint64_t sf_rows;
  bool build(const glmaxx_fc1_descriptor& d) {
    // 128-row tiles keep the scale plane within the reference's grouped SFA
    // capacity (A + 127 * min(A, E) rows) for any per-expert count.
    nt = 128;
    variant = kFc1PrefillFp4;
    sf_rows = round128(grouped_sf_rows(d.assignments, d.experts));
    s.carve(d.compacted_input_bf16 + kFc1ScratchOffset, d.assignments, d.experts, nt);
    const uint64_t plane = uint64_t(d.assignments) * d.hidden * 2;
    return kFc1ScratchOffset + s.bytes + 256 <= plane;
  }
};

int32_t fc1_prepare(const glmaxx_fc1_descriptor& d, Fc1Plan& p, const uint32_t mask[8],
                    cudaStream_t stream) {
  CompatPrepareArgs a{};
  a.route_experts = reinterpret_cast<const uint16_t*>(d.route_experts_u16);
  a.offsets = reinterpret_cast<const uint32_t*>(d.expert_offsets_u32);
  a.poffs = p.s.poffs;
  a.row_prow = p.s.row_prow;
  a.tiles = p.s.tiles;
  a.tile_count = p.s.tile_count;
  a.A = d.assignments;
  a.E = d.experts;
  a.nt = p.nt;
  a.sf_row_cap = static_cast<uint32_t>(p.sf_rows);
  a.max_tiles = p.s.max_tiles;
  a.status = nullptr;
  std::memcpy(a.expert_mask, mask, sizeof(a.expert_mask));
  return int32_t(launch_compat_prepare(a, stream));
}

int32_t fc1_quantize(const glmaxx_fc1_descriptor& d, Fc1Plan& p, cudaStream_t stream) {
  QuantRowsArgs q{};
  q.src = reinterpret_cast<const uint16_t*>(d.input_bf16);
  q.src_row = reinterpret_cast<const uint32_t*>(d.route_tokens_u32);
  q.row_prow = p.s.row_prow;
  q.values = reinterpret_cast<uint8_t*>(d.activation_values);
  q.scales = reinterpret_cast<uint8_t*>(d.activation_scales);
  q.gscale = reinterpret_cast<float*>(d.activation_global_scales);
  q.A = d.assignments;
  q.K = d.hidden;
  q.src_rows = d.rows;
  q.sf_row_cap = static_cast<uint32_t>(p.sf_rows);
  return int32_t(launch_quant_rows(q, stream));
}

int32_t fc1_core(const glmaxx_fc1_descriptor& d, Fc1Plan& p, int sms, cudaStream_t stream) {
  GemmLaunch g{};
  g.a = reinterpret_cast<const void*>(d.expert_value_base);
  g.a_experts = d.experts;
  g.a_rows = 2 * d.local_intermediate;
  g.a_row_bytes = d.hidden / 2;
  g.b = reinterpret_cast<const void*>(d.activation_values);
  g.b_rows = d.assignments;
  g.b_row_bytes = d.hidden / 2;
  GemmArgs& a = g.args;
  a.tiles = p.s.tiles;
  a.tile_count = p.s.tile_count;
  a.m_tiles = d.local_intermediate / 128;
  a.k_chunks = d.hidden / 256;
  a.up_row_offset = d.local_intermediate;
  a.kblocks = d.hidden / 64;
  a.ldo = d.local_intermediate;
  a.top_k = d.top_k;
  a.sfa = reinterpret_cast<const uint8_t*>(d.expert_scale_base);
  a.sfa_expert_bytes = 2ull * d.local_intermediate * d.hidden / 16;
  a.sfb = reinterpret_cast<const uint8_t*>(d.activation_scales);
  a.a_global = reinterpret_cast<const float*>(d.expert_global_scales);
  a.b_global = reinterpret_cast<const float*>(d.activation_global_scales);
  a.out = reinterpret_cast<void*>(d.output_bf16);
  return int32_t(launch_gemm(p.variant, g, sms, stream));
}

uint64_t fc1_required_bytes(const glmaxx_fc1_descriptor& d) {
  // Reference grouped workspace formula generalised to the descriptor geometry.
  const uint64_t A = d.assignments, H = d.hidden;
  return A * (H * 2 + 4 + uint64_t(d.local_gate_up) * 4) + round128(A) * H / 2 +
         grouped_sf_rows(A, d.experts) * H / 16 + uint64_t(d.experts + 1) * 4;
}

uint64_t fc2_required_bytes(const glmaxx_fc2_descriptor& d) {
  const uint64_t A = d.assignments, R = d.rows, H = d.hidden, I = d.local_intermediate;
  return round128(A) * I / 2 + grouped_sf_rows(A, d.experts) * I / 16 + A * 4 + A * H * 4 +
         A * H * 2 + R * H * 4 + R * d.top_k * 4 + 4;
}

int32_t check_mask(const uint16_t* active, uint32_t count, const glmaxx_fc1_descriptor* d,
                   uint32_t mask[8]) {
  std::memset(mask, 0, 32);
  if (active == nullptr || count == 0 || count > 256 || count > d->assignments) return -1;
  for (uint32_t i = 0; i < count; ++i) {
    if (active[i] >= d->experts || (i && active[i - 1] >= active[i])) return -2;
    mask[active[i] / 32] |= 1u << (active[i] % 32);
  }
  return 0;
}

int32_t fc1_common(const glmaxx_fc1_descriptor* descriptor, void* cuda_stream, bool quantize,
                   bool prepare, bool core, const uint32_t* mask_in) {
  if (descriptor == nullptr || cuda_stream == nullptr) return GLMAXX_ERR_NULL;
  const glmaxx_fc1_descriptor& d = *descriptor;
  if (!valid_fc1(d) || d.workspace_bytes < fc1_required_bytes(d)) return GLMAXX_ERR_DESCRIPTOR;
  Fc1Plan p;
  if (!p.build(d)) return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
  uint32_t all[8];
  std::memset(all, 0xff, sizeof(all));
  int32_t st = 0;
  if (prepare) st = fc1_prepare(d, p, mask_in ? mask_in : all, stream);
  if (st == 0 && quantize) st = fc1_quantize(d, p, stream);
  if (st == 0 && core) st = fc1_core(d, p, info.sms, stream);
  return st;
}

}  // namespace
}  // namespace glmaxx

using namespace glmaxx;

extern "C" {

const char* glmaxx_kernel_abi(void) { return "glmaxx.sm100.nvfp4.routed_moe.v3"; }
const char* glmaxx_exl3_kernel_abi(void) { return "glmaxx.sm100.exl3.source_projection.v1"; }

// ------------------------------------------------------------ workspace sizes
// Reference formulas for the GLM-5.2 TP4 geometry (nvfp4_routed_fc1.cu:346-368,
// nvfp4_routed_fc2.cu:512-544); the Rust caller checks them for equality.
uint64_t glmaxx_nvfp4_routed_fc1_workspace_bytes(uint32_t assignments) {
  const uint64_t padded = round128(assignments);
  return uint64_t(assignments) * (kRefHidden * 2 + 4 + 2 * kRefInter * 4) + padded * kRefHidden / 2 +
         padded * kRefHidden / 16 + uint64_t(kRefExperts + 1) * 4;
}

uint64_t glmaxx_nvfp4_grouped_workspace_bytes(uint32_t assignments) {
  if (assignments == 0 || assignments > 65535) return 0;
  return glmaxx_nvfp4_routed_fc1_workspace_bytes(assignments) -
         round128(assignments) * kRefHidden / 16 +
         grouped_sf_rows(assignments, kRefExperts) * kRefHidden / 16;
}

uint64_t glmaxx_nvfp4_routed_fc2_workspace_bytes(uint32_t rows, uint32_t assignments) {
  if (rows == 0 || assignments == 0 || assignments > uint64_t(rows) * kRefTopK) return 0;
  const uint64_t padded = round128(assignments);
  return padded * kRefInter / 2 + padded * kRefInter / 16 + uint64_t(assignments) * 4 +
         uint64_t(assignments) * kRefHidden * 4 + uint64_t(assignments) * kRefHidden * 2 +
         uint64_t(rows) * kRefHidden * 4 + uint64_t(rows) * kRefTopK * 4 + 4;
}

uint64_t glmaxx_nvfp4_grouped_fc2_workspace_bytes(uint32_t rows, uint32_t assignments) {
  if (rows == 0 || assignments == 0 || assignments > 65535 ||
      assignments > uint64_t(rows) * kRefTopK)
    return 0;
  return glmaxx_nvfp4_routed_fc2_workspace_bytes(rows, assignments) -
         round128(assignments) * kRefInter / 16 +
         grouped_sf_rows(assignments, kRefExperts) * kRefInter / 16;
}

// exl3_projection_control.cu:216-225: rotated input + projected planes (fp16).
// Geometry generalised from the TP4 shapes to any K, N that are multiples of 128.
uint64_t glmaxx_exl3_projection_workspace_bytes(uint32_t rows, uint32_t logical_k,
                                                uint32_t logical_n) {
  if (rows == 0 || rows > 3072 || logical_k == 0 || logical_n == 0 || logical_k % 128 ||
      logical_n % 128)
    return 0;
  return uint64_t(rows) * (uint64_t(logical_k) + logical_n) * 2;
}

uint64_t glmaxx_nvfp4_routed_fc1_workspace_bytes_v3(uint32_t rows, uint32_t assignments,
                                                    uint32_t hidden, uint32_t local_intermediate,
                                                    uint32_t experts, uint32_t top_k) {
  glmaxx_fc1_descriptor d{};
  d.rows = rows;
  d.assignments = assignments;
  d.hidden = hidden;
  d.local_intermediate = local_intermediate;
  d.local_gate_up = 2 * local_intermediate;
  d.experts = experts;
  d.top_k = top_k;
  return fc1_required_bytes(d);
}

uint64_t glmaxx_nvfp4_routed_fc2_workspace_bytes_v3(uint32_t rows, uint32_t assignments,
                                                    uint32_t hidden, uint32_t local_intermediate,
                                                    uint32_t experts, uint32_t top_k) {
  glmaxx_fc2_descriptor d{};
  d.rows = rows;
  d.assignments = assignments;
  d.hidden = hidden;
  d.local_intermediate = local_intermediate;
  d.experts = experts;
  d.top_k = top_k;
  return fc2_required_bytes(d);
}

uint64_t glmaxx_router_workspace_bytes(uint32_t tokens, uint32_t hidden, uint32_t experts,
                                       uint32_t top_k) {
  (void)hidden;
  return router_workspace_bytes(tokens, experts, top_k);
}

uint64_t glmaxx_moe_layer_workspace_bytes(const glmaxx_moe_layer_descriptor* descriptor) {
  if (descriptor == nullptr) return 0;
  return layer_workspace_bytes(*descriptor);
}

// ------------------------------------------------------------------ launches
int32_t glmaxx_router_compact_launch(const glmaxx_router_descriptor* descriptor, void* cuda_stream,
                                     int32_t* asynchronous_error) {
  return router_compact_launch(descriptor, cuda_stream, asynchronous_error);
}

int32_t glmaxx_moe_layer_launch(const glmaxx_moe_layer_descriptor* descriptor, void* cuda_stream,
                                int32_t* asynchronous_error) {
  return moe_layer_launch(descriptor, cuda_stream, asynchronous_error);
}

int32_t glmaxx_moe_layer_set_stage_events(uint64_t* events, uint32_t count) {
  return set_stage_events(events, count);
}

int32_t glmaxx_moe_layer_plane(const glmaxx_moe_layer_descriptor* descriptor, uint32_t which,
                               uint64_t* address, uint64_t* bytes) {
  return layer_plane(descriptor, which, address, bytes);
}

int32_t glmaxx_nvfp4_routed_fc1_launch(const glmaxx_fc1_descriptor* descriptor, void* cuda_stream,
                                       int32_t* asynchronous_error) {
  if (asynchronous_error == nullptr) return GLMAXX_ERR_NULL;
  *asynchronous_error = 0;
  return fc1_common(descriptor, cuda_stream, true, true, true, nullptr);
}

int32_t glmaxx_nvfp4_routed_fc1_graph_instantiate(const glmaxx_fc1_descriptor* descriptor,
                                                  void* cuda_stream, uint64_t* graph_exec) {
  if (descriptor == nullptr || cuda_stream == nullptr || graph_exec == nullptr)
    return GLMAXX_ERR_NULL;
  *graph_exec = 0;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
  cudaError_t st = cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal);
  if (st != cudaSuccess) return int32_t(st);
  const int32_t launch = fc1_common(descriptor, cuda_stream, true, true, true, nullptr);
  cudaGraph_t graph = nullptr;
  st = cudaStreamEndCapture(stream, &graph);
  if (launch != 0) {
    if (graph) cudaGraphDestroy(graph);
    return launch;
  }
  if (st != cudaSuccess) return int32_t(st);
  cudaGraphExec_t exec = nullptr;
  st = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (st != cudaSuccess) return int32_t(st);
  *graph_exec = reinterpret_cast<uint64_t>(exec);
  return 0;
}

// Quantisation writes the expert-local (grouped) scale layout in both forms:
// the tcgen05 grouped GEMM consumes only that layout.
int32_t glmaxx_nvfp4_quantize_launch(const glmaxx_fc1_descriptor* descriptor, void* cuda_stream) {
  return fc1_common(descriptor, cuda_stream, true, true, false, nullptr);
}

int32_t glmaxx_nvfp4_grouped_quantize_launch(const glmaxx_fc1_descriptor* descriptor,
                                             void* cuda_stream) {
  return fc1_common(descriptor, cuda_stream, true, true, false, nullptr);
}

int32_t glmaxx_nvfp4_core_swiglu_launch(const glmaxx_fc1_descriptor* descriptor,
                                        void* cuda_stream) {
  return fc1_common(descriptor, cuda_stream, false, true, true, nullptr);
}

int32_t glmaxx_nvfp4_dense_control_launch(const glmaxx_fc1_descriptor* descriptor,
                                          uint32_t expert, void* cuda_stream,
                                          int32_t* asynchronous_error) {
  if (descriptor == nullptr || asynchronous_error == nullptr) return GLMAXX_ERR_NULL;
  if (expert >= descriptor->experts) return GLMAXX_ERR_DESCRIPTOR;
  *asynchronous_error = 0;
  uint32_t mask[8] = {0};
  mask[expert / 32] = 1u << (expert % 32);
  return fc1_common(descriptor, cuda_stream, true, true, true, mask);
}

int32_t glmaxx_nvfp4_grouped_control_launch(const glmaxx_fc1_descriptor* descriptor,
                                            const uint16_t* active_experts,
                                            uint32_t active_expert_count, void* cuda_stream,
                                            int32_t* asynchronous_error) {
  if (descriptor == nullptr || asynchronous_error == nullptr || cuda_stream == nullptr)
    return GLMAXX_ERR_NULL;
  uint32_t mask[8];
  const int32_t m = check_mask(active_experts, active_expert_count, descriptor, mask);
  if (m != 0) return m;
  *asynchronous_error = 0;
  return fc1_common(descriptor, cuda_stream, true, true, true, mask);
}

int32_t glmaxx_nvfp4_grouped_core_swiglu_launch(const glmaxx_fc1_descriptor* descriptor,
                                                const uint16_t* active_experts,
                                                uint32_t active_expert_count, void* cuda_stream,
                                                int32_t* asynchronous_error) {
  if (descriptor == nullptr || asynchronous_error == nullptr || cuda_stream == nullptr)
    return GLMAXX_ERR_NULL;
  uint32_t mask[8];
  const int32_t m = check_mask(active_experts, active_expert_count, descriptor, mask);
  if (m != 0) return m;
  *asynchronous_error = 0;
  return fc1_common(descriptor, cuda_stream, false, true, true, mask);
}

int32_t glmaxx_nvfp4_grouped_prepare_launch(const glmaxx_fc1_descriptor* descriptor,
                                            const uint16_t* active_experts,
                                            uint32_t active_expert_count, void* cuda_stream) {
  if (descriptor == nullptr || cuda_stream == nullptr) return GLMAXX_ERR_NULL;
  uint32_t mask[8];
  const int32_t m = check_mask(active_experts, active_expert_count, descriptor, mask);
  if (m != 0) return m;
  return fc1_common(descriptor, cuda_stream, false, true, false, mask);
}

int32_t glmaxx_nvfp4_grouped_prepared_control_launch(const glmaxx_fc1_descriptor* descriptor,
                                                     uint32_t active_expert_count,
                                                     void* cuda_stream,
                                                     int32_t* asynchronous_error) {
  if (descriptor == nullptr || asynchronous_error == nullptr || cuda_stream == nullptr ||
      active_expert_count == 0 || active_expert_count > 256)
    return GLMAXX_ERR_NULL;
  *asynchronous_error = 0;
  return fc1_common(descriptor, cuda_stream, true, false, true, nullptr);
}

int32_t glmaxx_nvfp4_grouped_prepared_core_swiglu_launch(
    const glmaxx_fc1_descriptor* descriptor, uint32_t active_expert_count, void* cuda_stream,
    int32_t* asynchronous_error) {
  if (descriptor == nullptr || asynchronous_error == nullptr || cuda_stream == nullptr ||
      active_expert_count == 0 || active_expert_count > 256)
    return GLMAXX_ERR_NULL;
  *asynchronous_error = 0;
  return fc1_common(descriptor, cuda_stream, false, false, true, nullptr);
}

}  // extern "C"

// ------------------------------------------------------------------------ FC2
namespace glmaxx {
namespace {

struct Fc2Plan {
  CompatScratch s;
  uint32_t nt;
  uint64_t sf_rows;
  bool build(const glmaxx_fc2_descriptor& d) {
    nt = 128;
    sf_rows = round128(grouped_sf_rows(d.assignments, d.experts));
    s.carve(d.token_output_f32, d.assignments, d.experts, nt);
    return s.bytes + 256 <= uint64_t(d.rows) * d.hidden * 4;
  }
};

enum Fc2Stage : int { kFc2Prepare = 1, kFc2Quantize = 2, kFc2Core = 4, kFc2Reduce = 8 };

int32_t fc2_run(const glmaxx_fc2_descriptor* descriptor, void* cuda_stream, int stages,
                const uint32_t* mask_in) {
  if (descriptor == nullptr || cuda_stream == nullptr) return GLMAXX_ERR_NULL;
  const glmaxx_fc2_descriptor& d = *descriptor;
  if (!valid_fc2(d) || d.workspace_bytes < fc2_required_bytes(d)) return GLMAXX_ERR_DESCRIPTOR;
  Fc2Plan p;
  if (!p.build(d)) return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
  uint32_t* status = reinterpret_cast<uint32_t*>(d.validation_error_u32);
  SlotArgs sl{};
  sl.route_experts = reinterpret_cast<const uint16_t*>(d.route_experts_u16);
  sl.route_tokens = reinterpret_cast<const uint32_t*>(d.route_tokens_u32);
  sl.route_slots = reinterpret_cast<const uint8_t*>(d.route_slots_u8);
  sl.route_weights = reinterpret_cast<const float*>(d.route_weights_f32);
  sl.slot_assignment = reinterpret_cast<uint32_t*>(d.slot_assignment_u32);
  sl.assignment_down = reinterpret_cast<const float*>(d.assignment_down_f32);
  sl.token_output = reinterpret_cast<float*>(d.token_output_f32);
  sl.status = status;
  sl.A = d.assignments;
  sl.rows = d.rows;
  sl.H = d.hidden;
  sl.E = d.experts;
  sl.top_k = d.top_k;
  cudaError_t st = cudaSuccess;
  if (stages & kFc2Prepare) {
    st = cudaMemsetAsync(status, 0, 4, stream);
    if (st == cudaSuccess) st = launch_slot_table(sl, stream);
    if (st == cudaSuccess) {
      uint32_t all[8];
      std::memset(all, 0xff, sizeof(all));
      CompatPrepareArgs a{};
      a.route_experts = sl.route_experts;
      a.offsets = reinterpret_cast<const uint32_t*>(d.expert_offsets_u32);
      a.poffs = p.s.poffs;
      a.row_prow = p.s.row_prow;
      a.tiles = p.s.tiles;
      a.tile_count = p.s.tile_count;
      a.A = d.assignments;
      a.E = d.experts;
      a.nt = p.nt;
      a.sf_row_cap = static_cast<uint32_t>(p.sf_rows);
      a.max_tiles = p.s.max_tiles;
      a.status = status;
      std::memcpy(a.expert_mask, mask_in ? mask_in : all, sizeof(a.expert_mask));
      st = launch_compat_prepare(a, stream);
    }
  }
  if (st == cudaSuccess && (stages & kFc2Quantize)) {
    QuantRowsArgs q{};
    q.src = reinterpret_cast<const uint16_t*>(d.input_bf16);
    q.src_row = nullptr;
    q.row_prow = p.s.row_prow;
    q.values = reinterpret_cast<uint8_t*>(d.activation_values);
    q.scales = reinterpret_cast<uint8_t*>(d.activation_scales);
    q.gscale = reinterpret_cast<float*>(d.activation_global_scales);
    q.status = status;
    q.A = d.assignments;
    q.K = d.local_intermediate;
    q.src_rows = d.assignments;
    q.sf_row_cap = static_cast<uint32_t>(p.sf_rows);
    st = launch_quant_rows(q, stream);
  }
  if (st == cudaSuccess && (stages & kFc2Core)) {
    GemmLaunch g{};
    g.a = reinterpret_cast<const void*>(d.expert_value_base);
    g.a_experts = d.experts;
    g.a_rows = d.hidden;
    g.a_row_bytes = d.local_intermediate / 2;
    g.b = reinterpret_cast<const void*>(d.activation_values);
    g.b_rows = d.assignments;
    g.b_row_bytes = d.local_intermediate / 2;
    GemmArgs& a = g.args;
    a.tiles = p.s.tiles;
    a.tile_count = p.s.tile_count;
    a.m_tiles = d.hidden / 128;
    a.k_chunks = d.local_intermediate / 256;
    a.kblocks = d.local_intermediate / 64;
    a.ldo = d.hidden;
    a.top_k = d.top_k;
    a.sfa = reinterpret_cast<const uint8_t*>(d.expert_scale_base);
    a.sfa_expert_bytes = uint64_t(d.hidden) * d.local_intermediate / 16;
    a.sfb = reinterpret_cast<const uint8_t*>(d.activation_scales);
    a.a_global = reinterpret_cast<const float*>(d.expert_global_scales);
    a.b_global = reinterpret_cast<const float*>(d.activation_global_scales);
    a.out = reinterpret_cast<void*>(d.assignment_down_f32);
    a.status = status;
    st = launch_gemm(p.nt == 32 ? kFc2DecodeFp4Store : kFc2PrefillFp4Store, g, info.sms, stream);
  }
  if (st == cudaSuccess && (stages & kFc2Reduce)) st = launch_slot_reduce(sl, stream);
  return int32_t(st);
}

}  // namespace
}  // namespace glmaxx

extern "C" {

int32_t glmaxx_nvfp4_routed_fc2_launch(const glmaxx_fc2_descriptor* descriptor, void* cuda_stream,
                                       int32_t* asynchronous_error) {
  if (asynchronous_error == nullptr) return GLMAXX_ERR_NULL;
  *asynchronous_error = 0;
  return fc2_run(descriptor, cuda_stream, kFc2Prepare | kFc2Quantize | kFc2Core | kFc2Reduce,
                 nullptr);
}

int32_t glmaxx_nvfp4_fc2_quantize_launch(const glmaxx_fc2_descriptor* descriptor,
                                         void* cuda_stream) {
  return fc2_run(descriptor, cuda_stream, kFc2Prepare | kFc2Quantize, nullptr);
}

int32_t glmaxx_nvfp4_fc2_grouped_quantize_launch(const glmaxx_fc2_descriptor* descriptor,
                                                 void* cuda_stream) {
  return fc2_run(descriptor, cuda_stream, kFc2Prepare | kFc2Quantize, nullptr);
}

int32_t glmaxx_nvfp4_fc2_core_launch(const glmaxx_fc2_descriptor* descriptor, void* cuda_stream) {
  return fc2_run(descriptor, cuda_stream, kFc2Prepare | kFc2Core, nullptr);
}

int32_t glmaxx_nvfp4_fc2_reduce_launch(const glmaxx_fc2_descriptor* descriptor,
                                       void* cuda_stream) {
  return fc2_run(descriptor, cuda_stream, kFc2Reduce, nullptr);
}

int32_t glmaxx_nvfp4_fc2_dense_control_launch(const glmaxx_fc2_descriptor* descriptor,
                                              uint32_t expert, void* cuda_stream,
                                              int32_t* asynchronous_error) {
  if (descriptor == nullptr || asynchronous_error == nullptr) return GLMAXX_ERR_NULL;
  if (expert >= descriptor->experts) return GLMAXX_ERR_DESCRIPTOR;
  *asynchronous_error = 0;
  uint32_t mask[8] = {0};
  mask[expert / 32] = 1u << (expert % 32);
  return fc2_run(descriptor, cuda_stream, kFc2Prepare | kFc2Quantize | kFc2Core | kFc2Reduce,
                 mask);
}

int32_t glmaxx_nvfp4_fc2_grouped_control_launch(const glmaxx_fc2_descriptor* descriptor,
                                                const uint16_t* active_experts,
                                                uint32_t active_expert_count, void* cuda_stream,
                                                int32_t* asynchronous_error) {
  if (descriptor == nullptr || asynchronous_error == nullptr || active_experts == nullptr ||
      active_expert_count == 0 || active_expert_count > 256 ||
      active_expert_count > descriptor->assignments)
    return GLMAXX_ERR_NULL;
  uint32_t mask[8] = {0};
  for (uint32_t i = 0; i < active_expert_count; ++i) {
    if (active_experts[i] >= descriptor->experts || (i && active_experts[i - 1] >= active_experts[i]))
      return GLMAXX_ERR_DESCRIPTOR;
    mask[active_experts[i] / 32] |= 1u << (active_experts[i] % 32);
  }
  *asynchronous_error = 0;
  return fc2_run(descriptor, cuda_stream, kFc2Prepare | kFc2Quantize | kFc2Core | kFc2Reduce,
                 mask);
}

int32_t glmaxx_nvfp4_pack_launch(uint64_t src, int32_t src_is_bf16, uint32_t batch, uint32_t n,
                                 uint32_t k, uint64_t values, uint64_t scales,
                                 uint64_t global_scale_f32, uint64_t global_amax_f32,
                                 uint64_t scratch, uint64_t validation_error_u32,
                                 void* cuda_stream) {
  if (!src || !values || !scales || !global_scale_f32 || !scratch || !validation_error_u32)
    return GLMAXX_ERR_NULL;
  if (batch == 0 || n == 0 || k == 0 || n % 128 || k % 64 || values % 16 || scales % 4 ||
      (src_is_bf16 ? src % 2 : src % 4))
    return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
  return int32_t(launch_pack(reinterpret_cast<const void*>(src), src_is_bf16, batch, n, k,
                             reinterpret_cast<uint8_t*>(values), reinterpret_cast<uint8_t*>(scales),
                             reinterpret_cast<float*>(global_scale_f32),
                             reinterpret_cast<float*>(global_amax_f32),
                             reinterpret_cast<uint32_t*>(scratch),
                             reinterpret_cast<uint32_t*>(validation_error_u32), stream));
}

// ------------------------------------------------------------ runtime helpers
int32_t glmaxx_graph_exec_launch(uint64_t graph_exec, uint64_t stream) {
  if (graph_exec == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaGraphLaunch(reinterpret_cast<cudaGraphExec_t>(graph_exec),
                                 reinterpret_cast<cudaStream_t>(stream)));
}
int32_t glmaxx_graph_exec_destroy(uint64_t graph_exec) {
  if (graph_exec == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaGraphExecDestroy(reinterpret_cast<cudaGraphExec_t>(graph_exec)));
}
int32_t glmaxx_stream_begin_capture(uint64_t stream) {
  if (stream == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaStreamBeginCapture(reinterpret_cast<cudaStream_t>(stream),
                                        cudaStreamCaptureModeThreadLocal));
}
int32_t glmaxx_stream_end_capture(uint64_t stream, uint64_t* graph_exec) {
  if (stream == 0 || graph_exec == nullptr) return GLMAXX_ERR_NULL;
  cudaGraph_t graph = nullptr;
  cudaError_t st = cudaStreamEndCapture(reinterpret_cast<cudaStream_t>(stream), &graph);
  if (st != cudaSuccess) return int32_t(st);
  cudaGraphExec_t exec = nullptr;
  st = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (st == cudaSuccess) *graph_exec = reinterpret_cast<uint64_t>(exec);
  return int32_t(st);
}
int32_t glmaxx_event_create(uint64_t* event) {
  if (event == nullptr) return GLMAXX_ERR_NULL;
  cudaEvent_t e = nullptr;
  const cudaError_t st = cudaEventCreate(&e);
  if (st == cudaSuccess) *event = reinterpret_cast<uint64_t>(e);
  return int32_t(st);
}
int32_t glmaxx_event_record(uint64_t event, uint64_t stream) {
  if (event == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event),
                                 reinterpret_cast<cudaStream_t>(stream)));
}
int32_t glmaxx_event_synchronize(uint64_t event) {
  if (event == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaEventSynchronize(reinterpret_cast<cudaEvent_t>(event)));
}
int32_t glmaxx_event_elapsed_ms(uint64_t start, uint64_t end, float* milliseconds) {
  if (start == 0 || end == 0 || milliseconds == nullptr) return GLMAXX_ERR_NULL;
  return int32_t(cudaEventElapsedTime(milliseconds, reinterpret_cast<cudaEvent_t>(start),
                                      reinterpret_cast<cudaEvent_t>(end)));
}
int32_t glmaxx_event_destroy(uint64_t event) {
  if (event == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaEventDestroy(reinterpret_cast<cudaEvent_t>(event)));
}
int32_t glmaxx_profiler_start(void) { return int32_t(cudaProfilerStart()); }
int32_t glmaxx_profiler_stop(void) { return int32_t(cudaProfilerStop()); }
int32_t glmaxx_nvtx_range_push(const char* message) {
  if (message == nullptr) return GLMAXX_ERR_NULL;
  return nvtxRangePushA(message) < 0 ? -3 : 0;
}
int32_t glmaxx_nvtx_range_pop(void) { return nvtxRangePop() < 0 ? -3 : 0; }

int32_t glmaxx_device_count(int32_t* count) {
  if (count == nullptr) return GLMAXX_ERR_NULL;
  int n = 0;
  const cudaError_t st = cudaGetDeviceCount(&n);
  if (st == cudaSuccess) *count = n;
  return int32_t(st);
}

int32_t glmaxx_device_bind(int32_t device_index, int32_t* compute_capability,
                           int32_t* multiprocessor_count, uint64_t* total_memory_bytes,
                           uint8_t device_uuid[16]) {
  if (device_index < 0 || !compute_capability || !multiprocessor_count || !total_memory_bytes ||
      !device_uuid)
    return GLMAXX_ERR_NULL;
  cudaError_t st = cudaSetDevice(device_index);
  cudaDeviceProp p{};
  if (st == cudaSuccess) st = cudaGetDeviceProperties(&p, device_index);
  if (st == cudaSuccess) {
    *compute_capability = p.major * 10 + p.minor;
    *multiprocessor_count = p.multiProcessorCount;
    *total_memory_bytes = static_cast<uint64_t>(p.totalGlobalMem);
    for (int i = 0; i < 16; ++i) device_uuid[i] = static_cast<uint8_t>(p.uuid.bytes[i]);
  }
  return int32_t(st);
}

int32_t glmaxx_device_memory_info(uint64_t* free_memory_bytes, uint64_t* total_memory_bytes) {
  if (!free_memory_bytes || !total_memory_bytes) return GLMAXX_ERR_NULL;
  size_t f = 0, t = 0;
  const cudaError_t st = cudaMemGetInfo(&f, &t);
  if (st == cudaSuccess) {
    *free_memory_bytes = f;
    *total_memory_bytes = t;
  }
  return int32_t(st);
}

int32_t glmaxx_device_alloc(uint64_t bytes, uint64_t* pointer) {
  if (bytes == 0 || pointer == nullptr) return GLMAXX_ERR_NULL;
  void* p = nullptr;
  const cudaError_t st = cudaMalloc(&p, bytes);
  if (st == cudaSuccess) *pointer = reinterpret_cast<uint64_t>(p);
  return int32_t(st);
}
int32_t glmaxx_device_free(uint64_t pointer) {
  if (pointer == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaFree(reinterpret_cast<void*>(pointer)));
}
int32_t glmaxx_ipc_handle(uint64_t pointer, uint8_t handle[64]) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handle size");
  if (pointer == 0 || handle == nullptr) return GLMAXX_ERR_NULL;
  cudaIpcMemHandle_t h;
  const cudaError_t st = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(pointer));
  if (st == cudaSuccess) std::memcpy(handle, &h, sizeof(h));
  return int32_t(st);
}
int32_t glmaxx_ipc_open(const uint8_t handle[64], uint64_t* pointer) {
  if (handle == nullptr || pointer == nullptr) return GLMAXX_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t st = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (st == cudaSuccess) *pointer = reinterpret_cast<uint64_t>(p);
  return int32_t(st);
}
int32_t glmaxx_ipc_close(uint64_t pointer) {
  if (pointer == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaIpcCloseMemHandle(reinterpret_cast<void*>(pointer)));
}
int32_t glmaxx_peer_enable(int32_t peer_device) {
  int dev = -1, count = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st == cudaSuccess) st = cudaGetDeviceCount(&count);
  if (st != cudaSuccess) return int32_t(st);
  if (peer_device < 0 || peer_device >= count || peer_device == dev) return GLMAXX_ERR_DESCRIPTOR;
  int can = 0;
  st = cudaDeviceCanAccessPeer(&can, dev, peer_device);
  if (st != cudaSuccess) return int32_t(st);
  if (!can) return int32_t(cudaErrorPeerAccessUnsupported);
  st = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (st == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();  // clear the error state the repeated enable left behind
    st = cudaSuccess;
  }
  return int32_t(st);
}
int32_t glmaxx_pinned_alloc(uint64_t bytes, uint64_t* pointer) {
  if (bytes == 0 || pointer == nullptr) return GLMAXX_ERR_NULL;
  void* p = nullptr;
  const cudaError_t st = cudaHostAlloc(&p, bytes, cudaHostAllocDefault);
  if (st == cudaSuccess) *pointer = reinterpret_cast<uint64_t>(p);
  return int32_t(st);
}
int32_t glmaxx_pinned_free(uint64_t pointer) {
  if (pointer == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaFreeHost(reinterpret_cast<void*>(pointer)));
}
int32_t glmaxx_stream_create(uint64_t* stream) {
  if (stream == nullptr) return GLMAXX_ERR_NULL;
  cudaStream_t s = nullptr;
  const cudaError_t st = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (st == cudaSuccess) *stream = reinterpret_cast<uint64_t>(s);
  return int32_t(st);
}
int32_t glmaxx_stream_destroy(uint64_t stream) {
  return int32_t(cudaStreamDestroy(reinterpret_cast<cudaStream_t>(stream)));
}
int32_t glmaxx_stream_query(uint64_t stream, int32_t* complete) {
  if (stream == 0 || complete == nullptr) return GLMAXX_ERR_NULL;
  const cudaError_t st = cudaStreamQuery(reinterpret_cast<cudaStream_t>(stream));
  *complete = st == cudaSuccess ? 1 : 0;
  return (st == cudaSuccess || st == cudaErrorNotReady) ? 0 : int32_t(st);
}
int32_t glmaxx_stream_synchronize(uint64_t stream) {
  return int32_t(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
}
int32_t glmaxx_memcpy_h2d(uint64_t destination, const void* source, uint64_t bytes,
                          uint64_t stream) {
  return int32_t(cudaMemcpyAsync(reinterpret_cast<void*>(destination), source, bytes,
                                 cudaMemcpyHostToDevice, reinterpret_cast<cudaStream_t>(stream)));
}
int32_t glmaxx_memcpy_d2d(uint64_t destination, uint64_t source, uint64_t bytes, uint64_t stream) {
  return int32_t(cudaMemcpyAsync(reinterpret_cast<void*>(destination),
                                 reinterpret_cast<const void*>(source), bytes,
                                 cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream)));
}
int32_t glmaxx_memcpy_d2h(void* destination, uint64_t source, uint64_t bytes, uint64_t stream) {
  return int32_t(cudaMemcpyAsync(destination, reinterpret_cast<const void*>(source), bytes,
                                 cudaMemcpyDeviceToHost, reinterpret_cast<cudaStream_t>(stream)));
}
int32_t glmaxx_memset_zero(uint64_t destination, uint64_t bytes, uint64_t stream) {
  if (destination == 0 || bytes == 0 || stream == 0) return GLMAXX_ERR_NULL;
  return int32_t(cudaMemsetAsync(reinterpret_cast<void*>(destination), 0, bytes,
                                 reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"
