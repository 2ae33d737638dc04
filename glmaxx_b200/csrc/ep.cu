// Expert-parallel exchange of the routed-MoE step: the all-to-all alternative
// to the reference's tensor-parallel layout (not a reference layout; every
// expert row is still computed exactly as the TP1 layer computes it).
//
// Experts are partitioned in contiguous blocks over `ranks` owners (the owner of
// expert e is e / (experts / ranks)), and tokens over ranks as data.  Each rank
// routes its own tokens (glmaxx_router_compact_launch), so its compacted
// assignments are already grouped by owner: owner d's rows are the compacted
// rows [offsets[d*E/N], offsets[(d+1)*E/N]).
//  - dispatch: the rows for owner d go to d's receive buffers at row
//    dest_row_offset[d] + (compacted row - first row of d): the bf16 token row,
//    the owner-local expert (u16), the routing weight (f32) and the source
//    (rank << 24 | token << 4 | slot, u32).
//  - the owner runs glmaxx_moe_layer_launch over its received rows with
//    GLMAXX_MOE_ROUTES_GIVEN, top_k = 1 and its own experts' weights: each row's
//    routing-weighted expert output w * FC2(FC1(x)) in fp32.
//  - return: the owner copies each output row into its source rank's slot plane
//    [tokens][top_k][hidden] at (token, slot).
//  - the source then runs glmaxx_moe_layer_launch with GLMAXX_MOE_EXTERNAL_ROUTED:
//    the shared expert and the expert-order combine of the plane.
// Receive buffers and planes may be other GPUs' memory (peer access or CUDA
// IPC): the kernels move rows with plain 16-byte loads and stores -- no TMA and no
// multicast touches another GPU's memory.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/glmaxx_kernel.h"
#include "device.cuh"
#include "runtime.h"

namespace glmaxx {
namespace {

constexpr uint32_t kEpMaxRanks = 8;
constexpr uint32_t kEpThreads = 256;

struct EpArgs {
  const uint16_t* x;
  const uint32_t* comp_token;
  const uint16_t* comp_expert;
  const uint8_t* comp_slot;
  const float* comp_weight;
  const uint32_t* offsets;
  uint16_t* recv_x[kEpMaxRanks];
  uint16_t* recv_expert[kEpMaxRanks];
  float* recv_weight[kEpMaxRanks];
  uint32_t* recv_source[kEpMaxRanks];
  uint32_t recv_capacity[kEpMaxRanks];
  uint32_t dest_row[kEpMaxRanks];
  const float* rows_out;
  float* planes[kEpMaxRanks];
  uint32_t plane_tokens[kEpMaxRanks];
  uint32_t* status;
  uint32_t ranks, rank, hidden, experts, top_k, rows;
};

// One CTA per compacted row (grid-stride): the row goes to its expert's owner.
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(EpArgs a) {
  const uint32_t assignments = a.offsets[a.experts];
  const uint32_t per = a.experts / a.ranks;
  for (uint32_t row = blockIdx.x; row < assignments; row += gridDim.x) {
    const uint32_t e = a.comp_expert[row];
    const uint32_t d = e / per;
    if (d >= a.ranks) {
      if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusExpertOutOfRange);
      continue;
    }
    const uint32_t dst = a.dest_row[d] + (row - a.offsets[d * per]);
    if (dst >= a.recv_capacity[d]) {
      if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusCapacityExceeded);
      continue;
    }
    const uint32_t t = a.comp_token[row];
    const uint4* src = reinterpret_cast<const uint4*>(a.x + uint64_t(t) * a.hidden);
    uint4* out = reinterpret_cast<uint4*>(a.recv_x[d] + uint64_t(dst) * a.hidden);
    for (uint32_t i = threadIdx.x; i < a.hidden / 8; i += kEpThreads) out[i] = src[i];
    if (threadIdx.x == 0) {
      a.recv_expert[d][dst] = static_cast<uint16_t>(e - d * per);
      a.recv_weight[d][dst] = a.comp_weight[row];
      a.recv_source[d][dst] = (a.rank << 24) | (t << 4) | a.comp_slot[row];
    }
  }
}

// One CTA per received row (grid-stride): its output row goes to the source
// rank's slot plane.
__global__ void __launch_bounds__(kEpThreads) ep_return_kernel(EpArgs a) {
  const uint32_t* src_of = a.recv_source[a.rank];
  for (uint32_t j = blockIdx.x; j < a.rows; j += gridDim.x) {
    const uint32_t src = src_of[j];
    const uint32_t s = src >> 24, t = (src >> 4) & 0xfffffu, slot = src & 15u;
    if (s >= a.ranks || t >= a.plane_tokens[s] || slot >= a.top_k) {
      if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusRouteTokenOutOfRange);
      continue;
    }
    const float4* in = reinterpret_cast<const float4*>(a.rows_out + uint64_t(j) * a.hidden);
    float4* out = reinterpret_cast<float4*>(a.planes[s] + (uint64_t(t) * a.top_k + slot) * a.hidden);
    for (uint32_t i = threadIdx.x; i < a.hidden / 4; i += kEpThreads) out[i] = in[i];
  }
}

bool aligned16(uint64_t p) { return p != 0 && p % 16 == 0; }

int32_t ep_common(const glmaxx_moe_ep_descriptor* d, EpArgs* a) {
  if (d == nullptr) return GLMAXX_ERR_NULL;
  if (d->abi_version != GLMAXX_MOE_EP_ABI_VERSION || d->struct_bytes != sizeof(*d))
    return GLMAXX_ERR_DESCRIPTOR;
  for (uint32_t v : d->reserved0)
    if (v) return GLMAXX_ERR_DESCRIPTOR;
  for (uint64_t v : d->reserved)
    if (v) return GLMAXX_ERR_DESCRIPTOR;
  if (d->ranks == 0 || d->ranks > kEpMaxRanks || d->rank >= d->ranks) return GLMAXX_ERR_DESCRIPTOR;
  if (d->experts == 0 || d->experts > 256 || d->experts % d->ranks) return GLMAXX_ERR_DESCRIPTOR;
  if (d->hidden == 0 || d->hidden % 8 || d->top_k == 0 || d->top_k > 8)
    return GLMAXX_ERR_DESCRIPTOR;
  *a = EpArgs{};
  a->ranks = d->ranks;
  a->rank = d->rank;
  a->hidden = d->hidden;
  a->experts = d->experts;
  a->top_k = d->top_k;
  a->rows = d->rows;
  a->status = reinterpret_cast<uint32_t*>(d->validation_error_u32);
  for (uint32_t r = 0; r < d->ranks; ++r) {
    a->recv_x[r] = reinterpret_cast<uint16_t*>(d->recv_x_bf16[r]);
    a->recv_expert[r] = reinterpret_cast<uint16_t*>(d->recv_expert_u16[r]);
    a->recv_weight[r] = reinterpret_cast<float*>(d->recv_weight_f32[r]);
    a->recv_source[r] = reinterpret_cast<uint32_t*>(d->recv_source_u32[r]);
    a->recv_capacity[r] = d->recv_capacity[r];
    a->dest_row[r] = d->dest_row_offset[r];
    a->planes[r] = reinterpret_cast<float*>(d->planes_f32[r]);
    a->plane_tokens[r] = d->plane_tokens[r];
  }
  DeviceInfo info;
  return current_device_info(&info);
}

}  // namespace
}  // namespace glmaxx

extern "C" int32_t glmaxx_moe_ep_dispatch_launch(const glmaxx_moe_ep_descriptor* d,
                                                 void* cuda_stream) {
  using namespace glmaxx;
  EpArgs a;
  const int32_t st = ep_common(d, &a);
  if (st != 0) return st;
  if (d->tokens == 0 || d->tokens > (1u << 20) || !aligned16(d->input_bf16) ||
      d->compacted_tokens_u32 == 0 || d->compacted_experts_u16 == 0 ||
      d->compacted_slots_u8 == 0 || d->compacted_weights_f32 == 0 || d->expert_offsets_u32 == 0)
    return GLMAXX_ERR_DESCRIPTOR;
  for (uint32_t r = 0; r < d->ranks; ++r)
    if (!aligned16(d->recv_x_bf16[r]) || d->recv_expert_u16[r] == 0 ||
        d->recv_weight_f32[r] == 0 || d->recv_source_u32[r] == 0)
      return GLMAXX_ERR_DESCRIPTOR;
  a.x = reinterpret_cast<const uint16_t*>(d->input_bf16);
  a.comp_token = reinterpret_cast<const uint32_t*>(d->compacted_tokens_u32);
  a.comp_expert = reinterpret_cast<const uint16_t*>(d->compacted_experts_u16);
  a.comp_slot = reinterpret_cast<const uint8_t*>(d->compacted_slots_u8);
  a.comp_weight = reinterpret_cast<const float*>(d->compacted_weights_f32);
  a.offsets = reinterpret_cast<const uint32_t*>(d->expert_offsets_u32);
  const uint32_t rows = d->tokens * d->top_k;
  const uint32_t grid = rows < 4096 ? rows : 4096;
  ep_dispatch_kernel<<<grid, kEpThreads, 0, static_cast<cudaStream_t>(cuda_stream)>>>(a);
  return int32_t(cudaPeekAtLastError());
}

extern "C" int32_t glmaxx_moe_ep_return_launch(const glmaxx_moe_ep_descriptor* d,
                                               void* cuda_stream) {
  using namespace glmaxx;
  EpArgs a;
  const int32_t st = ep_common(d, &a);
  if (st != 0) return st;
  if (d->rows == 0) return 0;
  if (!aligned16(d->rows_out_f32) || d->recv_source_u32[d->rank] == 0 ||
      d->rows > d->recv_capacity[d->rank])
    return GLMAXX_ERR_DESCRIPTOR;
  for (uint32_t r = 0; r < d->ranks; ++r)
    if (d->plane_tokens[r] != 0 && !aligned16(d->planes_f32[r])) return GLMAXX_ERR_DESCRIPTOR;
  a.rows_out = reinterpret_cast<const float*>(d->rows_out_f32);
  const uint32_t grid = d->rows < 4096 ? d->rows : 4096;
  ep_return_kernel<<<grid, kEpThreads, 0, static_cast<cudaStream_t>(cuda_stream)>>>(a);
  return int32_t(cudaPeekAtLastError());
}
