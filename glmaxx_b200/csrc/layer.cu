// Rank-local routed-MoE step and device router/compaction: descriptor
// validation, workspace carving and the launch sequence.  The operation order
// is the reference's frozen sparse-layer order (crates/glm-reference/src/
// routed_fc2.rs:93-109): ProtectedRouter -> StableRouteCompaction -> RoutedFc1
// -> Swiglu -> RoutedFc2WeightedScatter -> SharedExpert, producing the partial
// that MoeTpReduce sums across ranks.
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/glmaxx_kernel.h"
#include "moe.h"
#include "runtime.h"

namespace glmaxx {

namespace {

constexpr uint64_t kAlign = 256;
uint64_t up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

struct Carve {
  uint64_t cursor = 0;
  uint64_t take(uint64_t bytes) {
    const uint64_t off = cursor;
    cursor = up(cursor + (bytes ? bytes : 1), kAlign);
    return off;
  }
};

// Planes shared by the router/compaction and the full layer.
struct RoutePlan {
  uint32_t T, E, K, W, A;
  uint64_t partial, bitmap, wprefix, counts, offsets, poffs, status;
  void carve(Carve& c, uint32_t tokens, uint32_t experts, uint32_t top_k) {
    T = tokens;
    E = experts;
    K = top_k;
    W = (T + 31) / 32;
    A = T * K;
    partial = c.take(8ull * T * E * 4);
    bitmap = c.take(uint64_t(E) * W * 4);
    wprefix = c.take(uint64_t(E) * W * 4);
    counts = c.take(uint64_t(E) * 4);
    offsets = c.take(uint64_t(E + 1) * 4);
    poffs = c.take(uint64_t(E + 1) * 4);
    status = c.take(16);
  }
};

// SMs the decode shared expert (split-K over this many work items) takes while
// it overlaps the router, compaction and quantisation on the other SMs.  Measured
// decode step (T=64, TP1): 0.895 ms at 148, 0.893 at 96, 0.891 at 64, 0.888 at 40.
constexpr uint32_t kSharedDecodeSms = 40;
// Gate/up weight bytes of the first experts prefetched into L2 at decode.
// Graph-replayed step of one TP8 shard (T=64): 0.1989 ms without, 0.1850 at
// 32 MB, 0.1844 at 64 MB, 0.1980 at 96 MB; TP1: 0.855 without, 0.847 at 32 MB.
constexpr uint64_t kFc1PrefetchBytes = 32ull << 20;

struct LayerPlan {
  RoutePlan r;
  uint32_t H, I, Is, nt, sf_rows, max_tiles;
  uint32_t s1_splits, s1_kc, s2_splits, s2_kc;  // shared-expert split-K (decode)
  bool decode, shared;
  // exl3: some experts are EXL3; nvfp4: some experts are NVFP4 (the NVFP4 stages
  // run); plane_mode: routed results go through the per-slot plane and the
  // deterministic expert-order combine (decode, and any layer with EXL3 experts)
  bool exl3, nvfp4, plane_mode;
  // external: the routed plane is the caller's (expert parallelism); only the
  // shared expert and the combine run
  bool external;
  uint64_t exl3_ws;
  uint64_t tiles, tile_count, route_row, row_token, row_slot, row_weight, gx, gh, row_prow;
  uint64_t xq, xsf, hbuf, hq, hsf, plane, hs, sbuf, sparts1, sparts2, total;

  void build(const glmaxx_moe_layer_descriptor& d) {
    Carve c;
    r.carve(c, d.tokens, d.experts, d.top_k);
    H = d.hidden;
    I = d.local_intermediate;
    shared = (d.flags & GLMAXX_MOE_SHARED_EXPERT) != 0;
    Is = shared ? d.shared_intermediate : 0;
    decode = d.path == GLMAXX_FC1_DECODE_PERSISTENT || (d.path == 0 && d.tokens <= 256);
    exl3 = (d.flags & GLMAXX_MOE_EXL3_EXPERTS) != 0;
    const glmaxx_moe_exl3_experts* xe =
        exl3 ? reinterpret_cast<const glmaxx_moe_exl3_experts*>(d.exl3_experts) : nullptr;
    external = (d.flags & GLMAXX_MOE_EXTERNAL_ROUTED) != 0;
    nvfp4 = !external && (!exl3 || (xe != nullptr && xe->codec_u8 != 0));
    plane_mode = decode || exl3 || external || (d.flags & GLMAXX_MOE_DETERMINISTIC) != 0;
    nt = decode ? 32 : 128;
    const uint32_t A = r.A;
    const uint32_t active = A < r.E ? A : r.E;
    max_tiles = (A + nt - 1) / nt + active;
    sf_rows = max_tiles * 128;  // each n tile owns a 128-row scale atom
    const uint64_t rA = external ? 0 : A;  // the routed stages' planes (none when external)
    tiles = c.take(external ? 0 : uint64_t(max_tiles) * sizeof(NTile));
    tile_count = c.take(16);
    route_row = c.take(rA * 4);
    row_token = c.take(rA * 4);
    row_slot = c.take(rA * 4);
    row_weight = c.take(rA * 4);
    gx = c.take(rA * 4);
    gh = c.take(rA * 4);
    row_prow = c.take(rA * 4);
    xq = c.take(rA * H / 2);
    xsf = c.take(external ? 0 : uint64_t(sf_rows) * H / 16);
    hbuf = c.take(rA * I * 2);
    hq = c.take(rA * I / 2);
    hsf = c.take(external ? 0 : uint64_t(sf_rows) * I / 16);
    plane = (plane_mode && !external) ? c.take(uint64_t(A) * H * 4) : c.take(0);
    hs = shared ? c.take(uint64_t(r.T) * Is * 2) : c.take(0);
    sbuf = (shared && plane_mode) ? c.take(uint64_t(r.T) * H * 4) : c.take(0);
    exl3_ws = exl3 ? c.take(exl3_experts_workspace_bytes(A, H, I, r.E)) : c.take(0);
    // Decode runs the shared expert as split-K GEMMs so that its few output
    // tiles still cover every SM (sized for up to 148 SMs).
    s1_splits = s1_kc = s2_splits = s2_kc = 1;
    if (shared && decode) {
      const uint32_t nt_tiles = (r.T + 63) / 64;
      choose_k_splits(nt_tiles * (Is / 128), 2 * H / 128, kSharedDecodeSms, 16, &s1_splits,
                      &s1_kc);
      choose_k_splits(nt_tiles * (H / 128), 2 * Is / 128, kSharedDecodeSms, 16, &s2_splits,
                      &s2_kc);
    }
    sparts1 = (shared && decode) ? c.take(uint64_t(s1_splits) * r.T * 2 * Is * 4) : c.take(0);
    sparts2 = (shared && decode) ? c.take(uint64_t(s2_splits) * r.T * H * 4) : c.take(0);
    total = c.cursor + kAlign;  // slack so the caller's base need only be 16-byte aligned
  }
};

bool aligned(uint64_t p, uint64_t a) { return p != 0 && p % a == 0; }

bool valid_layer(const glmaxx_moe_layer_descriptor& d) {
  if (d.abi_version != GLMAXX_MOE_LAYER_ABI_VERSION || d.struct_bytes != sizeof(d)) return false;
  for (uint32_t v : d.reserved0)
    if (v) return false;
  for (uint64_t v : d.reserved)
    if (v) return false;
  if (d.flags & ~uint32_t(GLMAXX_MOE_ROUTES_GIVEN | GLMAXX_MOE_SHARED_EXPERT |
                          GLMAXX_MOE_EXL3_EXPERTS | GLMAXX_MOE_EXTERNAL_ROUTED |
                          GLMAXX_MOE_DETERMINISTIC))
    return false;
  if (d.flags & GLMAXX_MOE_EXTERNAL_ROUTED) {
    if (!(d.flags & GLMAXX_MOE_ROUTES_GIVEN) || (d.flags & GLMAXX_MOE_EXL3_EXPERTS) ||
        !aligned(d.routed_plane_f32, 16))
      return false;
  } else if (d.routed_plane_f32) {
    return false;
  }
  bool nvfp4_weights = true;
  if (d.flags & GLMAXX_MOE_EXL3_EXPERTS) {
    if (d.exl3_experts == 0) return false;
    const auto& xe = *reinterpret_cast<const glmaxx_moe_exl3_experts*>(d.exl3_experts);
    if (xe.abi_version != GLMAXX_MOE_EXL3_ABI_VERSION || xe.struct_bytes != sizeof(xe) ||
        xe.bits != 3 || xe.reserved0)
      return false;
    for (uint64_t v : xe.reserved)
      if (v) return false;
    if (!aligned(xe.gate_trellis_u16, 16) || !aligned(xe.up_trellis_u16, 16) ||
        !aligned(xe.down_trellis_u16, 16) || !aligned(xe.gate_suh_f16, 2) ||
        !aligned(xe.gate_svh_f16, 2) || !aligned(xe.up_suh_f16, 2) || !aligned(xe.up_svh_f16, 2) ||
        !aligned(xe.down_suh_f16, 2) || !aligned(xe.down_svh_f16, 2))
      return false;
    if (d.hidden % 128 || d.local_intermediate % 128) return false;
    nvfp4_weights = xe.codec_u8 != 0;
  } else if (d.exl3_experts) {
    return false;
  }
  if (d.path > GLMAXX_FC1_PREFILL_GROUPED) return false;
  if (d.tokens == 0 || d.tokens > 65536) return false;
  if (d.hidden == 0 || d.hidden % 256 != 0 || d.hidden > 16384) return false;  // <= 256 k-blocks
  if (d.experts == 0 || d.experts > 256) return false;
  if (d.top_k == 0 || d.top_k > 8 || d.top_k > d.experts) return false;
  if (uint64_t(d.tokens) * d.top_k > (1u << 20)) return false;
  // power of two in [256, 2048]: FC2 quantisation reduces a row over I/64 lanes
  if (d.local_intermediate < 256 || d.local_intermediate > 2048 ||
      (d.local_intermediate & (d.local_intermediate - 1)))
    return false;
  if (!(d.flags & GLMAXX_MOE_ROUTES_GIVEN)) {
    if (d.groups == 0 || d.groups > 32 || d.experts % d.groups) return false;
    if (d.topk_groups == 0 || d.topk_groups > d.groups) return false;
    if (d.top_k > (d.experts / d.groups) * d.topk_groups) return false;
    if (!(d.route_scale == d.route_scale)) return false;
    if (!aligned(d.router_weight_bf16, 16) || !aligned(d.router_bias_f32, 4)) return false;
  }
  if (d.flags & GLMAXX_MOE_SHARED_EXPERT) {
    if (d.shared_intermediate == 0 || d.shared_intermediate % 128 || d.shared_intermediate > 8192)
      return false;
    if (!aligned(d.shared13_bf16, 256) || !aligned(d.shared2_bf16, 256)) return false;
  }
  if (d.flags & GLMAXX_MOE_EXTERNAL_ROUTED) nvfp4_weights = false;  // no routed GEMMs run
  if (nvfp4_weights &&
      !(aligned(d.w13_values, 256) && aligned(d.w13_scales, 16) && aligned(d.w13_global_f32, 4) &&
        aligned(d.w2_values, 256) && aligned(d.w2_scales, 16) && aligned(d.w2_global_f32, 4)))
    return false;
  return aligned(d.input_bf16, 256) && aligned(d.route_experts_u16, 4) &&
         aligned(d.route_weights_f32, 4) && aligned(d.output_f32, 16) && aligned(d.workspace, 16);
}

template <typename T>
T* at(uint64_t base, uint64_t off) {
  return reinterpret_cast<T*>(base + off);
}

// Optional per-stage CUDA events (profiling): when set, the next layer
// launches on this thread record event[s] before stage s and event[kStages]
// after the last stage, on the launch stream.
thread_local uint64_t* g_stage_events = nullptr;
thread_local uint32_t g_stage_event_count = 0;

}  // namespace

int32_t set_stage_events(uint64_t* events, uint32_t count) {
  if (events != nullptr && count < kLayerStages + 1) return GLMAXX_ERR_DESCRIPTOR;
  g_stage_events = events;
  g_stage_event_count = events ? count : 0;
  return 0;
}

namespace {
// The shared expert depends only on x, so it runs on a second stream forked
// from the launch stream after the status word is cleared, and joins before the
// kernel that consumes it (the combine, or FC2 when FC2 adds onto its output).
// It then overlaps the latency-bound router, compaction and quantisation at
// decode.  One side stream and event pair per thread and device; CUDA-graph
// capture turns the fork and join into graph edges.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
thread_local SideStream g_side[64];

// *out stays null (the shared expert then runs in order on the launch stream)
// when the side stream does not exist yet and the launch stream is capturing:
// creating streams and events is left to an uncaptured launch.
cudaError_t side_stream(cudaStream_t launch, SideStream** out) {
  *out = nullptr;
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  SideStream& s = g_side[dev];
  if (s.stream == nullptr) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if ((st = cudaStreamIsCapturing(launch, &cap)) != cudaSuccess) return st;
    if (cap != cudaStreamCaptureStatusNone) return cudaSuccess;
    if ((st = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking)) != cudaSuccess) return st;
    if ((st = cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming)) != cudaSuccess) return st;
    if ((st = cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming)) != cudaSuccess) return st;
  }
  *out = &s;
  return cudaSuccess;
}

cudaError_t mark(uint32_t stage, cudaStream_t stream) {
  if (g_stage_events == nullptr || stage >= g_stage_event_count) return cudaSuccess;
  return cudaEventRecord(reinterpret_cast<cudaEvent_t>(g_stage_events[stage]), stream);
}
}  // namespace

uint64_t layer_workspace_bytes(const glmaxx_moe_layer_descriptor& d) {
  LayerPlan p;
  p.build(d);
  return p.total;
}

int32_t layer_plane(const glmaxx_moe_layer_descriptor* desc, uint32_t which, uint64_t* address,
                    uint64_t* bytes) {
  if (desc == nullptr || address == nullptr || bytes == nullptr) return GLMAXX_ERR_NULL;
  if (!valid_layer(*desc)) return GLMAXX_ERR_DESCRIPTOR;
  LayerPlan p;
  p.build(*desc);
  const uint64_t ws = up(desc->workspace, kAlign);
  const uint64_t A = p.r.A;
  switch (which) {
    case GLMAXX_PLANE_FC1_OUTPUT_BF16:
      *address = ws + p.hbuf, *bytes = A * p.I * 2;
      break;
    case GLMAXX_PLANE_ROW_TOKEN_U32:
      *address = ws + p.row_token, *bytes = A * 4;
      break;
    case GLMAXX_PLANE_ROW_SLOT_U32:
      *address = ws + p.row_slot, *bytes = A * 4;
      break;
    case GLMAXX_PLANE_ROW_WEIGHT_F32:
      *address = ws + p.row_weight, *bytes = A * 4;
      break;
    case GLMAXX_PLANE_EXPERT_OFFSETS_U32:
      *address = ws + p.r.offsets, *bytes = uint64_t(p.r.E + 1) * 4;
      break;
    case GLMAXX_PLANE_SHARED_F32:
      if (!p.shared || !p.plane_mode) return GLMAXX_ERR_DESCRIPTOR;
      *address = ws + p.sbuf, *bytes = uint64_t(p.r.T) * p.H * 4;
      break;
    case GLMAXX_PLANE_ROUTED_F32:
      if (!p.plane_mode) return GLMAXX_ERR_DESCRIPTOR;
      *address = ws + p.plane, *bytes = A * p.H * 4;
      break;
    default:
      return GLMAXX_ERR_DESCRIPTOR;
  }
  return 0;
}

int32_t moe_layer_launch(const glmaxx_moe_layer_descriptor* desc, void* cuda_stream,
                         int32_t* async_err) {
  if (desc == nullptr || async_err == nullptr) return GLMAXX_ERR_NULL;
  *async_err = 0;
  const glmaxx_moe_layer_descriptor& d = *desc;
  if (!valid_layer(d)) return GLMAXX_ERR_DESCRIPTOR;
  LayerPlan p;
  p.build(d);
  if (d.workspace_bytes < p.total) return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
  const uint64_t ws = up(d.workspace, kAlign);
  const RoutePlan& r = p.r;
  uint32_t* status = d.validation_error_u32 ? reinterpret_cast<uint32_t*>(d.validation_error_u32)
                                            : at<uint32_t>(ws, r.status);
  uint16_t* experts = reinterpret_cast<uint16_t*>(d.route_experts_u16);
  float* weights = reinterpret_cast<float*>(d.route_weights_f32);
  const uint16_t* x = reinterpret_cast<const uint16_t*>(d.input_bf16);
  float* out = reinterpret_cast<float*>(d.output_f32);
  const uint32_t bitmap_words = r.E * r.W;
#define CHECK(expr)                          \
  do {                                       \
    cudaError_t _st = (expr);                \
    if (_st != cudaSuccess) return int32_t(_st); \
  } while (0)
  CHECK(mark(kStageRouter, stream));
  CHECK(cudaMemsetAsync(status, 0, 4, stream));
  SideStream* side = nullptr;
  cudaStream_t sstream = stream;  // the shared expert's stream
  if (p.shared) {
    CHECK(side_stream(stream, &side));
    if (side) {
      sstream = side->stream;
      CHECK(cudaEventRecord(side->fork, stream));
      CHECK(cudaStreamWaitEvent(sstream, side->fork, 0));
      // Decode: HBM idles through the latency-bound router chain, and FC1 then
      // streams the experts' gate/up weights in ascending expert order; the
      // first experts' weights are prefetched into L2 meanwhile.
      if (p.decode && p.nvfp4 && !p.exl3) {
        const uint64_t vals = uint64_t(2) * p.I * p.H / 2, scales = uint64_t(2) * p.I * p.H / 16;
        uint64_t n = kFc1PrefetchBytes / (vals + scales);
        if (n > r.E) n = r.E;
        if (n > 0)
          CHECK(launch_l2_prefetch(reinterpret_cast<const void*>(d.w13_values), n * vals,
                                   reinterpret_cast<const void*>(d.w13_scales), n * scales,
                                   sstream));
      }
    }
  }
  // shared expert (bf16) on the side stream, and the output initialisation it
  // provides outside plane mode
  if (p.shared) {
    GemmLaunch g1{};
    g1.a = reinterpret_cast<const void*>(d.shared13_bf16);
    g1.a_experts = 1;
    g1.a_rows = 2 * p.Is;
    g1.a_row_bytes = 2 * p.H;
    g1.b = x;
    g1.b_rows = r.T;
    g1.b_row_bytes = 2 * p.H;
    g1.args.implicit_rows = r.T;
    g1.args.m_tiles = p.Is / 128;
    g1.args.k_chunks = 2 * p.H / 128;
    g1.args.up_row_offset = p.Is;
    g1.args.status = status;
    GemmLaunch g2{};
    g2.a = reinterpret_cast<const void*>(d.shared2_bf16);
    g2.a_experts = 1;
    g2.a_rows = p.H;
    g2.a_row_bytes = 2 * p.Is;
    g2.b = at<void>(ws, p.hs);
    g2.b_rows = r.T;
    g2.b_row_bytes = 2 * p.Is;
    g2.args.implicit_rows = r.T;
    g2.args.m_tiles = p.H / 128;
    g2.args.k_chunks = 2 * p.Is / 128;
    g2.args.ldo = p.H;
    g2.args.status = status;
    if (p.decode) {
      // split-K partial planes, reduced in slice order by the finish / combine kernels
      g1.args.k_splits = p.s1_splits;
      g1.args.kc_per_split = p.s1_kc;
      g1.args.ldo = 2 * p.Is;
      g1.args.ldo_up = p.Is;
      g1.args.split_stride = uint64_t(r.T) * 2 * p.Is;
      g1.args.out = at<void>(ws, p.sparts1);
      const int shared_sms = info.sms < int(kSharedDecodeSms) ? info.sms : int(kSharedDecodeSms);
      CHECK(launch_gemm(kShared1Bf16N64Split, g1, shared_sms, sstream));
      CHECK(launch_swiglu_finish(at<float>(ws, p.sparts1), p.s1_splits, r.T, p.Is,
                                 at<uint16_t>(ws, p.hs), sstream));
      g2.args.k_splits = p.s2_splits;
      g2.args.kc_per_split = p.s2_kc;
      g2.args.split_stride = uint64_t(r.T) * p.H;
      g2.args.out = at<void>(ws, p.sparts2);
      CHECK(launch_gemm(kShared2Bf16N64Split, g2, shared_sms, sstream));
    } else {
      g1.args.ldo = p.Is;
      g1.args.out = at<void>(ws, p.hs);
      CHECK(launch_gemm(kShared1Bf16N128, g1, info.sms, sstream));
      // plane mode: the combine adds the shared expert from sbuf
      g2.args.out = p.plane_mode ? at<void>(ws, p.sbuf) : static_cast<void*>(out);
      CHECK(launch_gemm(kShared2Bf16N128, g2, info.sms, sstream));
    }
    if (side) CHECK(cudaEventRecord(side->join, sstream));
  }

  if (p.external) {
    // Expert parallelism: the routed slot plane was written by the experts'
    // owner ranks; what is left is the deterministic combine with the shared
    // expert, the same kernel (and so the same bits) as the local plane path.
    for (uint32_t stage = kStageCompact; stage <= kStageFc2; ++stage) CHECK(mark(stage, stream));
    CHECK(mark(kStageCombine, stream));
    if (side) CHECK(cudaStreamWaitEvent(stream, side->join, 0));
    const float* shared_in = !p.shared ? nullptr
                             : (p.decode ? at<float>(ws, p.sparts2) : at<float>(ws, p.sbuf));
    CHECK(launch_combine(reinterpret_cast<const float*>(d.routed_plane_f32), experts, shared_in,
                         p.decode ? p.s2_splits : 1,
                         (p.shared && p.decode) ? at<float>(ws, p.sbuf) : nullptr, out, r.T, p.H,
                         r.K, stream));
    CHECK(mark(kLayerStages, stream));
    return 0;
  }

  // 1. router (or caller routes) -> dense routes + token-in-expert bitmap
  if (d.flags & GLMAXX_MOE_ROUTES_GIVEN) {
    CHECK(launch_routes_to_bitmap(experts, weights, r.T, r.E, r.K, at<uint32_t>(ws, r.bitmap),
                                  bitmap_words, status, stream));
  } else {
    CHECK(launch_router_logits(x, reinterpret_cast<const uint16_t*>(d.router_weight_bf16),
                               at<float>(ws, r.partial), r.T, p.H, r.E, at<uint32_t>(ws, r.bitmap),
                               bitmap_words, stream));
    CHECK(launch_router_select(at<float>(ws, r.partial),
                               reinterpret_cast<const float*>(d.router_bias_f32), r.T, r.E,
                               d.groups, d.topk_groups, r.K, d.route_scale, experts, weights,
                               at<uint32_t>(ws, r.bitmap), r.W, status, stream));
  }
  // 2. stable compaction
  CHECK(mark(kStageCompact, stream));
  NTile* tiles = at<NTile>(ws, p.tiles);
  uint32_t* tile_count = at<uint32_t>(ws, p.tile_count);
  const glmaxx_moe_exl3_experts* xe =
      p.exl3 ? reinterpret_cast<const glmaxx_moe_exl3_experts*>(d.exl3_experts) : nullptr;
  const uint8_t* codec = xe ? reinterpret_cast<const uint8_t*>(xe->codec_u8) : nullptr;
  CHECK(launch_compact(at<uint32_t>(ws, r.bitmap), r.T, r.E, p.nt, p.sf_rows, p.max_tiles,
                       at<uint32_t>(ws, r.wprefix), at<uint32_t>(ws, r.counts),
                       at<uint32_t>(ws, r.offsets), at<uint32_t>(ws, r.poffs), tiles, tile_count,
                       status, stream, codec));
  // 3. NVFP4 quantisation of x into the assignment rows
  CHECK(mark(kStageQuant, stream));
  QuantScatterArgs q{};
  q.x = x;
  q.route_experts = experts;
  q.route_weights = weights;
  q.bitmap = at<uint32_t>(ws, r.bitmap);
  q.wprefix = at<uint32_t>(ws, r.wprefix);
  q.poffs = at<uint32_t>(ws, r.poffs);
  q.offsets = at<uint32_t>(ws, r.offsets);
  q.xq = at<uint8_t>(ws, p.xq);
  q.xsf = at<uint8_t>(ws, p.xsf);
  q.row_token = at<uint32_t>(ws, p.row_token);
  q.row_slot = at<uint32_t>(ws, p.row_slot);
  q.row_weight = at<float>(ws, p.row_weight);
  q.row_gscale = at<float>(ws, p.gx);
  q.row_prow = at<uint32_t>(ws, p.row_prow);
  q.route_row = at<uint32_t>(ws, p.route_row);
  q.status = status;
  q.T = r.T;
  q.H = p.H;
  q.E = r.E;
  q.top_k = r.K;
  q.sf_row_cap = p.sf_rows;
  q.nt = p.nt;
  CHECK(launch_quant_scatter(q, stream));
  // 4. grouped FC1 (gate+up) with fused SwiGLU -> h [A][I] bf16 (NVFP4 experts);
  //    EXL3 experts: gate/up/down projections straight into the routed plane
  CHECK(mark(kStageFc1, stream));
  if (p.exl3) {
    Exl3ExpertsLaunch L{};
    L.A = r.A;
    L.H = p.H;
    L.I = p.I;
    L.E = r.E;
    L.top_k = r.K;
    L.x_bf16 = x;
    L.offsets = at<uint32_t>(ws, r.offsets);
    L.codec = codec;
    L.row_token = q.row_token;
    L.row_slot = q.row_slot;
    L.row_weight = q.row_weight;
    L.gate_trellis = reinterpret_cast<const uint16_t*>(xe->gate_trellis_u16);
    L.up_trellis = reinterpret_cast<const uint16_t*>(xe->up_trellis_u16);
    L.down_trellis = reinterpret_cast<const uint16_t*>(xe->down_trellis_u16);
    L.gate_suh = reinterpret_cast<const uint16_t*>(xe->gate_suh_f16);
    L.gate_svh = reinterpret_cast<const uint16_t*>(xe->gate_svh_f16);
    L.up_suh = reinterpret_cast<const uint16_t*>(xe->up_suh_f16);
    L.up_svh = reinterpret_cast<const uint16_t*>(xe->up_svh_f16);
    L.down_suh = reinterpret_cast<const uint16_t*>(xe->down_suh_f16);
    L.down_svh = reinterpret_cast<const uint16_t*>(xe->down_svh_f16);
    L.plane = at<float>(ws, p.plane);
    L.workspace = at<void>(ws, p.exl3_ws);
    L.status = status;
    L.num_sms = info.sms;
    CHECK(launch_exl3_experts(L, stream));
  }
  if (p.nvfp4) {
    GemmLaunch g{};
    g.a = reinterpret_cast<const void*>(d.w13_values);
    g.a_experts = r.E;
    g.a_rows = 2 * p.I;
    g.a_row_bytes = p.H / 2;
    g.b = q.xq;
    g.b_rows = r.A;
    g.b_row_bytes = p.H / 2;
    GemmArgs& a = g.args;
    a.tiles = tiles;
    a.tile_count = tile_count;
    a.m_tiles = p.I / 128;
    a.k_chunks = p.H / 256;
    a.up_row_offset = p.I;
    a.kblocks = p.H / 64;
    a.ldo = p.I;
    a.top_k = r.K;
    a.sfa = reinterpret_cast<const uint8_t*>(d.w13_scales);
    a.sfa_expert_bytes = 2ull * p.I * p.H / 16;
    a.sfb = q.xsf;
    a.a_global = reinterpret_cast<const float*>(d.w13_global_f32);
    a.b_global = q.row_gscale;
    a.out = at<void>(ws, p.hbuf);
    a.status = status;
    CHECK(launch_gemm(p.decode ? kFc1DecodeFp4 : kFc1PrefillFp4, g, info.sms, stream));
  }
  // 5. NVFP4 quantisation of h
  CHECK(mark(kStageFc2Quant, stream));
  Fc2QuantArgs f{};
  f.h = at<uint16_t>(ws, p.hbuf);
  f.row_prow = q.row_prow;
  f.hq = at<uint8_t>(ws, p.hq);
  f.hsf = at<uint8_t>(ws, p.hsf);
  f.gscale = at<float>(ws, p.gh);
  f.status = status;
  f.count_ptr = at<uint32_t>(ws, r.offsets) + r.E;
  f.count = r.A;
  f.I = p.I;
  f.sf_row_cap = p.sf_rows;
  f.offsets = at<uint32_t>(ws, r.offsets);
  f.skip_codec = codec;
  f.E = r.E;
  if (p.nvfp4) CHECK(launch_fc2_quant(f, stream));
  // 6. the shared expert ran on the side stream (launched before the router)
  CHECK(mark(kStageShared, stream));
  if (!p.shared && !p.plane_mode) {
    CHECK(cudaMemsetAsync(out, 0, uint64_t(r.T) * p.H * 4, stream));
  }
  if (side && !p.plane_mode) CHECK(cudaStreamWaitEvent(stream, side->join, 0));
  // 7. grouped FC2 with the routing-weighted combine
  CHECK(mark(kStageFc2, stream));
  if (p.nvfp4) {
    GemmLaunch g{};
    g.a = reinterpret_cast<const void*>(d.w2_values);
    g.a_experts = r.E;
    g.a_rows = p.H;
    g.a_row_bytes = p.I / 2;
    g.b = f.hq;
    g.b_rows = r.A;
    g.b_row_bytes = p.I / 2;
    GemmArgs& a = g.args;
    a.tiles = tiles;
    a.tile_count = tile_count;
    // Decode and plane mode: two adjacent 128-row M tiles per item share one B
    // tile (twice the weight bytes per pipeline stage, half the B-tile and
    // scale-copy work per FLOP).  Prefill with the atomic combine: one M tile per
    // item, whose two accumulator buffers let the MMA run through the atomic
    // epilogue (FC2 1.34 -> 1.21 ms at T=8192) -- except on narrow shards
    // (local intermediate <= 256, one K stage per item), where the shared B tile
    // wins again (T=8192 TP8-shard layer 1.80 -> 1.73 ms; at TP1 and a TP2 shard
    // the pair measured slower, 3.89 -> 3.95 and 2.50 -> 2.63 ms).
    const bool single = !p.decode && !p.plane_mode && p.I > 256;
    a.m_tiles = single ? p.H / 128 : p.H / 256;
    a.m_stride = single ? 128 : 256;
    a.up_row_offset = single ? 0 : 128;
    a.k_chunks = p.I / 256;
    a.kblocks = p.I / 64;
    a.ldo = p.H;
    a.top_k = r.K;
    a.sfa = reinterpret_cast<const uint8_t*>(d.w2_scales);
    a.sfa_expert_bytes = uint64_t(p.H) * p.I / 16;
    a.sfb = f.hsf;
    a.a_global = reinterpret_cast<const float*>(d.w2_global_f32);
    a.b_global = f.gscale;
    a.out = p.plane_mode ? at<void>(ws, p.plane) : static_cast<void*>(out);
    a.row_token = q.row_token;
    a.row_slot = q.row_slot;
    a.row_weight = q.row_weight;
    a.status = status;
    CHECK(launch_gemm(p.decode       ? kFc2DecodeFp4Pair
                      : p.plane_mode ? kFc2PrefillFp4PairPlane
                      : single       ? kFc2PrefillFp4
                                     : kFc2PrefillFp4PairAtomic,
                      g, info.sms, stream));
  }
  // 8. deterministic combine (plane mode): ascending-expert sum + shared
  CHECK(mark(kStageCombine, stream));
  if (side && p.plane_mode) CHECK(cudaStreamWaitEvent(stream, side->join, 0));
  if (p.plane_mode) {
    const float* shared_in = !p.shared ? nullptr
                             : (p.decode ? at<float>(ws, p.sparts2) : at<float>(ws, p.sbuf));
    CHECK(launch_combine(at<float>(ws, p.plane), experts, shared_in, p.decode ? p.s2_splits : 1,
                         (p.shared && p.decode) ? at<float>(ws, p.sbuf) : nullptr, out, r.T, p.H,
                         r.K, stream));
  }
  CHECK(mark(kLayerStages, stream));
#undef CHECK
  return 0;
}

// -------------------------------------------------------------- router only
namespace {
bool valid_router(const glmaxx_router_descriptor& d) {
  if (d.abi_version != GLMAXX_ROUTER_ABI_VERSION || d.struct_bytes != sizeof(d) || d.flags)
    return false;
  for (uint32_t v : d.reserved0)
    if (v) return false;
  for (uint64_t v : d.reserved)
    if (v) return false;
  if (d.tokens == 0 || d.tokens > 65536 || d.hidden == 0 || d.hidden % 256 || d.hidden > 16384)
    return false;
  if (d.experts == 0 || d.experts > 256 || d.top_k == 0 || d.top_k > 8) return false;
  if (d.groups == 0 || d.groups > 32 || d.experts % d.groups) return false;
  if (d.topk_groups == 0 || d.topk_groups > d.groups) return false;
  if (d.top_k > (d.experts / d.groups) * d.topk_groups) return false;
  return aligned(d.input_bf16, 16) && aligned(d.router_weight_bf16, 16) &&
         aligned(d.router_bias_f32, 4) && aligned(d.route_experts_u16, 2) &&
         aligned(d.route_weights_f32, 4) && aligned(d.compacted_tokens_u32, 4) &&
         aligned(d.compacted_experts_u16, 2) && d.compacted_slots_u8 != 0 &&
         aligned(d.compacted_weights_f32, 4) && aligned(d.expert_offsets_u32, 4) &&
         aligned(d.workspace, 16);
}
}  // namespace

uint64_t router_workspace_bytes(uint32_t tokens, uint32_t experts, uint32_t top_k) {
  Carve c;
  RoutePlan r;
  r.carve(c, tokens, experts, top_k);
  return c.cursor + kAlign;
}

int32_t router_compact_launch(const glmaxx_router_descriptor* desc, void* cuda_stream,
                              int32_t* async_err) {
  if (desc == nullptr || async_err == nullptr) return GLMAXX_ERR_NULL;
  *async_err = 0;
  const glmaxx_router_descriptor& d = *desc;
  if (!valid_router(d)) return GLMAXX_ERR_DESCRIPTOR;
  if (d.workspace_bytes < router_workspace_bytes(d.tokens, d.experts, d.top_k))
    return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
  Carve c;
  RoutePlan r;
  r.carve(c, d.tokens, d.experts, d.top_k);
  const uint64_t ws = up(d.workspace, kAlign);
  uint32_t* status = d.validation_error_u32 ? reinterpret_cast<uint32_t*>(d.validation_error_u32)
                                            : at<uint32_t>(ws, r.status);
  uint16_t* experts = reinterpret_cast<uint16_t*>(d.route_experts_u16);
  float* weights = reinterpret_cast<float*>(d.route_weights_f32);
  cudaError_t st = cudaMemsetAsync(status, 0, 4, stream);
  if (st == cudaSuccess)
    st = launch_router_logits(reinterpret_cast<const uint16_t*>(d.input_bf16),
                              reinterpret_cast<const uint16_t*>(d.router_weight_bf16),
                              at<float>(ws, r.partial), r.T, d.hidden, r.E,
                              at<uint32_t>(ws, r.bitmap), r.E * r.W, stream);
  if (st == cudaSuccess)
    st = launch_router_select(at<float>(ws, r.partial),
                              reinterpret_cast<const float*>(d.router_bias_f32), r.T, r.E,
                              d.groups, d.topk_groups, r.K, d.route_scale, experts, weights,
                              at<uint32_t>(ws, r.bitmap), r.W, status, stream);
  // Offsets only: the n-tile list is not needed here (nt = 128, no tiles written).
  if (st == cudaSuccess)
    st = launch_compact(at<uint32_t>(ws, r.bitmap), r.T, r.E, 128, 0xffffffffu, 0xffffffffu,
                        at<uint32_t>(ws, r.wprefix), at<uint32_t>(ws, r.counts),
                        reinterpret_cast<uint32_t*>(d.expert_offsets_u32),
                        at<uint32_t>(ws, r.poffs), nullptr, at<uint32_t>(ws, r.status) + 1,
                        status, stream);
  if (st == cudaSuccess) {
    CompactWriteArgs a{};
    a.route_experts = experts;
    a.route_weights = weights;
    a.bitmap = at<uint32_t>(ws, r.bitmap);
    a.wprefix = at<uint32_t>(ws, r.wprefix);
    a.offsets = reinterpret_cast<const uint32_t*>(d.expert_offsets_u32);
    a.comp_token = reinterpret_cast<uint32_t*>(d.compacted_tokens_u32);
    a.comp_expert = reinterpret_cast<uint16_t*>(d.compacted_experts_u16);
    a.comp_slot = reinterpret_cast<uint8_t*>(d.compacted_slots_u8);
    a.comp_weight = reinterpret_cast<float*>(d.compacted_weights_f32);
    a.T = r.T;
    a.E = r.E;
    a.top_k = r.K;
    st = launch_compact_write(a, stream);
  }
  return int32_t(st);
}

}  // namespace glmaxx
