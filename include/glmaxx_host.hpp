// C++ host runtime of the routed-MoE path over the C ABI of libglmaxx_sm100.so
// (glmaxx_kernel.h).  It is the counterpart, in C++17, of the reference's Rust
// binding layer crates/glm-cuda/src/ffi.rs and abi.rs: an owner-thread rank
// context (NativeRankContext::bind, ffi.rs:185-298), move-only device buffer,
// stream, event and graph handles (ffi.rs:649-790), the KernelError kinds
// (abi.rs:686-698), the ABI validation entry (validate_native_moe_abi,
// ffi.rs:3227-3245), and the operator this library adds for the whole rank-local
// step: RoutedMoeStep, its per-row-bucket graphs (the engine's GraphKey
// verifier_row_bucket, crates/glm-engine/src/graph.rs:13-80, with the buckets of
// crates/glm-cli/src/profile.rs:10-11), and PeerFinish, the fused tensor-parallel
// reduce over CUDA IPC mappings.  NativeRankFile and RankLayerWeights read
// .g5n rank files (glmaxx_rank_file.h; the reference's NativeRankReader,
// crates/glm-format/src/native_reader.rs) straight into a step's weights.
//
// Header-only: it calls only the extern "C" functions of glmaxx_kernel.h, so a
// C++ engine links libglmaxx_sm100.so and includes this file.  Every failure
// raises KernelError; no call falls back to another implementation.
#pragma once

#include <algorithm>
#include <array>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "glmaxx_kernel.h"
#include "glmaxx_rank_file.h"

namespace glmaxx {
namespace host {

// ------------------------------------------------------------------ errors
enum class ErrorKind {
  Abi,
  Path,
  Shape,
  Null,
  Alignment,
  Overflow,
  Workspace,
  Driver,
  Async,
  DeviceValidation,
  Topology,
};

inline const char* error_kind_name(ErrorKind k) {
  switch (k) {
    case ErrorKind::Abi: return "Abi";
    case ErrorKind::Path: return "Path";
    case ErrorKind::Shape: return "Shape";
    case ErrorKind::Null: return "Null";
    case ErrorKind::Alignment: return "Alignment";
    case ErrorKind::Overflow: return "Overflow";
    case ErrorKind::Workspace: return "Workspace";
    case ErrorKind::Driver: return "Driver";
    case ErrorKind::Async: return "Async";
    case ErrorKind::DeviceValidation: return "DeviceValidation";
    case ErrorKind::Topology: return "Topology";
  }
  return "?";
}

class KernelError : public std::runtime_error {
 public:
  KernelError(ErrorKind kind, int64_t code = 0, uint64_t required = 0, uint64_t provided = 0)
      : std::runtime_error(std::string(error_kind_name(kind)) + "(" + std::to_string(code) + ")"),
        kind_(kind), code_(code), required_(required), provided_(provided) {}
  ErrorKind kind() const { return kind_; }
  int64_t code() const { return code_; }           // status, async error or device word
  uint64_t required() const { return required_; }  // Workspace
  uint64_t provided() const { return provided_; }

 private:
  ErrorKind kind_;
  int64_t code_;
  uint64_t required_, provided_;
};

// A non-zero status of an extern "C" call is a Driver error carrying it
// (ffi.rs:3170-3176).
inline void check(int32_t status) {
  if (status != 0) throw KernelError(ErrorKind::Driver, status);
}

inline uint64_t checked_add(uint64_t a, uint64_t b) {
  if (a > UINT64_MAX - b) throw KernelError(ErrorKind::Overflow);
  return a + b;
}

// ------------------------------------------------------------------ handles
class NativeStream {
 public:
  static NativeStream create() {
    uint64_t s = 0;
    check(glmaxx_stream_create(&s));
    return NativeStream(s);
  }
  NativeStream() = default;
  NativeStream(NativeStream&& o) noexcept : s_(std::exchange(o.s_, 0)) {}
  NativeStream& operator=(NativeStream&& o) noexcept {
    std::swap(s_, o.s_);
    return *this;
  }
  NativeStream(const NativeStream&) = delete;
  NativeStream& operator=(const NativeStream&) = delete;
  ~NativeStream() {
    if (s_) glmaxx_stream_destroy(s_);
  }
  uint64_t get() const { return s_; }
  void synchronize() const { check(glmaxx_stream_synchronize(s_)); }

 private:
  explicit NativeStream(uint64_t s) : s_(s) {}
  uint64_t s_ = 0;
};

class NativeEvent {
 public:
  static NativeEvent create() {
    uint64_t e = 0;
    check(glmaxx_event_create(&e));
    if (e == 0) throw KernelError(ErrorKind::Driver, -1);
    return NativeEvent(e);
  }
  NativeEvent(NativeEvent&& o) noexcept : e_(std::exchange(o.e_, 0)) {}
  NativeEvent& operator=(NativeEvent&& o) noexcept {
    std::swap(e_, o.e_);
    return *this;
  }
  NativeEvent(const NativeEvent&) = delete;
  NativeEvent& operator=(const NativeEvent&) = delete;
  ~NativeEvent() {
    if (e_) glmaxx_event_destroy(e_);
  }
  void record(uint64_t stream) const { check(glmaxx_event_record(e_, stream)); }
  void synchronize() const { check(glmaxx_event_synchronize(e_)); }
  float elapsed_ms(const NativeEvent& end) const {
    float ms = 0.0f;
    check(glmaxx_event_elapsed_ms(e_, end.e_, &ms));
    return ms;
  }

 private:
  explicit NativeEvent(uint64_t e) : e_(e) {}
  uint64_t e_ = 0;
};

// An executable graph of the work captured on a stream between begin() and
// end() (glmaxx_stream_begin_capture / glmaxx_stream_end_capture).
class NativeGraph {
 public:
  static void begin(uint64_t stream) { check(glmaxx_stream_begin_capture(stream)); }
  static NativeGraph end(uint64_t stream) {
    uint64_t exec = 0;
    check(glmaxx_stream_end_capture(stream, &exec));
    return NativeGraph(exec);
  }
  NativeGraph() = default;
  NativeGraph(NativeGraph&& o) noexcept : g_(std::exchange(o.g_, 0)) {}
  NativeGraph& operator=(NativeGraph&& o) noexcept {
    std::swap(g_, o.g_);
    return *this;
  }
  NativeGraph(const NativeGraph&) = delete;
  NativeGraph& operator=(const NativeGraph&) = delete;
  ~NativeGraph() {
    if (g_) glmaxx_graph_exec_destroy(g_);
  }
  void launch(uint64_t stream) const { check(glmaxx_graph_exec_launch(g_, stream)); }
  bool valid() const { return g_ != 0; }

 private:
  explicit NativeGraph(uint64_t g) : g_(g) {}
  uint64_t g_ = 0;
};

// Device allocation with range-checked copies (ffi.rs:649-724).
class NativeBuffer {
 public:
  static NativeBuffer allocate(uint64_t bytes) {
    if (bytes == 0) throw KernelError(ErrorKind::Shape);
    uint64_t p = 0;
    check(glmaxx_device_alloc(bytes, &p));
    return NativeBuffer(p, bytes);
  }
  static NativeBuffer upload(const void* host, uint64_t bytes, uint64_t stream) {
    NativeBuffer b = allocate(bytes);
    b.upload_at(host, bytes, 0, stream);
    return b;
  }
  NativeBuffer() = default;
  NativeBuffer(NativeBuffer&& o) noexcept
      : p_(std::exchange(o.p_, 0)), bytes_(std::exchange(o.bytes_, 0)) {}
  NativeBuffer& operator=(NativeBuffer&& o) noexcept {
    std::swap(p_, o.p_);
    std::swap(bytes_, o.bytes_);
    return *this;
  }
  NativeBuffer(const NativeBuffer&) = delete;
  NativeBuffer& operator=(const NativeBuffer&) = delete;
  ~NativeBuffer() {
    if (p_) glmaxx_device_free(p_);
  }
  uint64_t ptr() const { return p_; }
  uint64_t bytes() const { return bytes_; }
  void upload_at(const void* host, uint64_t bytes, uint64_t offset, uint64_t stream) const {
    if (checked_add(offset, bytes) > bytes_) throw KernelError(ErrorKind::Shape);
    check(glmaxx_memcpy_h2d(p_ + offset, host, bytes, stream));
  }
  void download_at(void* host, uint64_t bytes, uint64_t offset, uint64_t stream) const {
    if (checked_add(offset, bytes) > bytes_) throw KernelError(ErrorKind::Shape);
    check(glmaxx_memcpy_d2h(host, p_ + offset, bytes, stream));
  }
  void copy_within(uint64_t src_offset, uint64_t dst_offset, uint64_t bytes, uint64_t stream) const {
    if (checked_add(src_offset, bytes) > bytes_ || checked_add(dst_offset, bytes) > bytes_)
      throw KernelError(ErrorKind::Shape);
    check(glmaxx_memcpy_d2d(p_ + dst_offset, p_ + src_offset, bytes, stream));
  }
  void zero(uint64_t stream) const { check(glmaxx_memset_zero(p_, bytes_, stream)); }

 private:
  NativeBuffer(uint64_t p, uint64_t b) : p_(p), bytes_(b) {}
  uint64_t p_ = 0, bytes_ = 0;
};

// ------------------------------------------------------------------ rank context
struct NativeDeviceIdentity {
  uint32_t visible_devices = 0;
  uint32_t device_index = 0;
  uint32_t compute_capability = 0;
  uint32_t multiprocessor_count = 0;
  uint64_t total_memory_bytes = 0;
  std::array<uint8_t, 16> device_uuid{};
};

// One rank's device and non-blocking stream, bound on and owned by the calling
// thread; every method checks that it runs on that thread (ffi.rs:185-298).
// ranks: the tensor-parallel degree (1, 2, 4 or 8; the reference fixes 4); the
// rank's device is device `rank`, of compute capability 10.x.
class NativeRankContext {
 public:
  static NativeRankContext bind(uint32_t rank, uint32_t ranks) {
    if (!(ranks == 1 || ranks == 2 || ranks == 4 || ranks == 8) || rank >= ranks)
      throw KernelError(ErrorKind::Topology);
    int32_t visible = 0;
    check(glmaxx_device_count(&visible));
    if (visible < int32_t(ranks)) throw KernelError(ErrorKind::Topology);
    int32_t cc = 0, sms = 0;
    uint64_t total = 0;
    NativeDeviceIdentity id;
    check(glmaxx_device_bind(int32_t(rank), &cc, &sms, &total, id.device_uuid.data()));
    if (cc / 10 != 10 || sms <= 0 || total == 0) throw KernelError(ErrorKind::Topology);
    id.visible_devices = uint32_t(visible);
    id.device_index = rank;
    id.compute_capability = uint32_t(cc);
    id.multiprocessor_count = uint32_t(sms);
    id.total_memory_bytes = total;
    return NativeRankContext(id, NativeStream::create());
  }
  NativeRankContext(NativeRankContext&&) = default;
  NativeRankContext& operator=(NativeRankContext&&) = default;
  const NativeDeviceIdentity& identity() const { return id_; }
  uint64_t stream() const {
    require_owner();
    return stream_.get();
  }
  void synchronize() const {
    require_owner();
    stream_.synchronize();
  }
  uint64_t free_memory_bytes() const {
    require_owner();
    uint64_t free_b = 0, total_b = 0;
    check(glmaxx_device_memory_info(&free_b, &total_b));
    if (free_b == 0 || total_b != id_.total_memory_bytes || free_b > total_b)
      throw KernelError(ErrorKind::Topology);
    return free_b;
  }
  void require_owner() const {
    if (std::this_thread::get_id() != owner_) throw KernelError(ErrorKind::Topology);
  }

 private:
  NativeRankContext(NativeDeviceIdentity id, NativeStream s)
      : id_(id), stream_(std::move(s)), owner_(std::this_thread::get_id()) {}
  NativeDeviceIdentity id_;
  NativeStream stream_;
  std::thread::id owner_;
};

// The reference workspace formulas for the fixed TP4 geometry
// (crates/glm-cuda/src/abi.rs:454-559), which the library's workspace queries
// must reproduce.
inline uint64_t reference_fc1_workspace_bytes(uint64_t a) {
  const uint64_t p = (a + 127) / 128 * 128;
  return a * 6144 * 2 + p * 3072 + p * 384 + a * 4 + a * 1024 * 4 + 257 * 4;
}
inline uint64_t reference_fc2_workspace_bytes(uint64_t rows, uint64_t a) {
  const uint64_t p = (a + 127) / 128 * 128;
  return p * 256 + p * 32 + a * 4 + a * 6144 * 4 + a * 6144 * 2 + rows * 6144 * 4 +
         rows * 8 * 4 + 4;
}

// Checks, without a device, that the loaded library is this ABI and that its
// routed FC1/FC2 workspace sizes for (rows, assignments) are the reference's
// (ffi.rs:3227-3235).
inline void validate_native_moe_abi(uint32_t rows, uint32_t assignments) {
  const char* abi = glmaxx_kernel_abi();
  if (abi == nullptr || std::string(abi) != "glmaxx.sm100.nvfp4.routed_moe.v3")
    throw KernelError(ErrorKind::Abi);
  if (rows == 0 || assignments == 0 || uint64_t(assignments) > uint64_t(rows) * 8)
    throw KernelError(ErrorKind::Shape);
  const uint64_t fc1 = glmaxx_nvfp4_routed_fc1_workspace_bytes(assignments);
  const uint64_t fc2 = glmaxx_nvfp4_routed_fc2_workspace_bytes(rows, assignments);
  if (fc1 != reference_fc1_workspace_bytes(assignments))
    throw KernelError(ErrorKind::Workspace, 1, reference_fc1_workspace_bytes(assignments), fc1);
  if (fc2 != reference_fc2_workspace_bytes(rows, assignments))
    throw KernelError(ErrorKind::Workspace, 2, reference_fc2_workspace_bytes(rows, assignments),
                      fc2);
}

// ------------------------------------------------------------------ the step
// Geometry of one rank's routed-MoE layer (tensor-parallel shard).
struct MoeGeometry {
  uint32_t max_tokens = 0;
  uint32_t hidden = 6144;
  uint32_t experts = 256;
  uint32_t local_intermediate = 2048;  // 2048 / tp
  uint32_t top_k = 8;
  uint32_t groups = 8;
  uint32_t topk_groups = 4;
  float route_scale = 2.5f;
  uint32_t shared_intermediate = 2048;  // 0: no shared expert
};

// Device addresses of one rank's weights, in the layouts glmaxx_kernel.h
// documents for glmaxx_moe_layer_descriptor.  exl3 (optional) is a host struct
// that must outlive the step.
struct MoeWeights {
  uint64_t router_weight_bf16 = 0, router_bias_f32 = 0;
  uint64_t w13_values = 0, w13_scales = 0, w13_global_f32 = 0;
  uint64_t w2_values = 0, w2_scales = 0, w2_global_f32 = 0;
  uint64_t shared13_bf16 = 0, shared2_bf16 = 0;
  const glmaxx_moe_exl3_experts* exl3 = nullptr;
};

// One rank's routed-MoE step (glmaxx_moe_layer_launch): owns the route arrays,
// the validation word and the workspace, sized for max_tokens on both paths.
// The step runs on the caller's stream; launches on one step object must not
// overlap on the device.
class RoutedMoeStep {
 public:
  RoutedMoeStep(const NativeRankContext& ctx, const MoeGeometry& g, const MoeWeights& w)
      : geom_(g), w_(w) {
    ctx.require_owner();
    if (g.max_tokens == 0 || g.top_k == 0) throw KernelError(ErrorKind::Shape);
    route_experts_ = NativeBuffer::allocate(uint64_t(g.max_tokens) * g.top_k * 2);
    route_weights_ = NativeBuffer::allocate(uint64_t(g.max_tokens) * g.top_k * 4);
    status_ = NativeBuffer::allocate(16);
    uint64_t need = 0;
    for (uint32_t path : {0u, uint32_t(GLMAXX_FC1_PREFILL_GROUPED)}) {
      glmaxx_moe_layer_descriptor d = descriptor(g.max_tokens, 0, 0, path, 0, 0);
      const uint64_t b = glmaxx_moe_layer_workspace_bytes(&d);
      if (b == 0) throw KernelError(ErrorKind::Shape);
      need = std::max(need, b);
    }
    workspace_ = NativeBuffer::allocate(need);
  }

  const MoeGeometry& geometry() const { return geom_; }
  uint64_t workspace_bytes() const { return workspace_.bytes(); }
  uint64_t route_experts_u16() const { return route_experts_.ptr(); }
  uint64_t route_weights_f32() const { return route_weights_.ptr(); }

  // out[tokens][hidden] fp32 = routed + shared partial of x[tokens][hidden] bf16.
  // path: 0 auto (decode up to 256 tokens), GLMAXX_FC1_DECODE_PERSISTENT or
  // GLMAXX_FC1_PREFILL_GROUPED.
  void launch(uint64_t input_bf16, uint64_t output_f32, uint32_t tokens, uint64_t stream,
              uint32_t path = 0) {
    if (tokens == 0 || tokens > geom_.max_tokens) throw KernelError(ErrorKind::Shape);
    if (input_bf16 == 0 || output_f32 == 0) throw KernelError(ErrorKind::Null);
    glmaxx_moe_layer_descriptor d =
        descriptor(tokens, input_bf16, output_f32, path, workspace_.ptr(), workspace_.bytes());
    int32_t async_error = 0;
    const int32_t st =
        glmaxx_moe_layer_launch(&d, reinterpret_cast<void*>(static_cast<uintptr_t>(stream)),
                                &async_error);
    if (st == GLMAXX_ERR_NULL) throw KernelError(ErrorKind::Null, st);
    if (st == GLMAXX_ERR_DESCRIPTOR) throw KernelError(ErrorKind::Shape, st);
    if (st == GLMAXX_ERR_WRONG_ARCH) throw KernelError(ErrorKind::Abi, st);
    check(st);
    if (async_error != 0) throw KernelError(ErrorKind::Async, async_error);
  }

  // The device validation word of the last launch (waits for `stream`); a
  // non-zero word raises DeviceValidation with it.
  void check_device_status(uint64_t stream) const {
    uint32_t word = 0;
    status_.download_at(&word, 4, 0, stream);
    check(glmaxx_stream_synchronize(stream));
    if (word != 0) throw KernelError(ErrorKind::DeviceValidation, word);
  }

 private:
  glmaxx_moe_layer_descriptor descriptor(uint32_t tokens, uint64_t x, uint64_t out, uint32_t path,
                                         uint64_t ws, uint64_t ws_bytes) const {
    glmaxx_moe_layer_descriptor d;
    std::memset(&d, 0, sizeof(d));
    d.abi_version = GLMAXX_MOE_LAYER_ABI_VERSION;
    d.struct_bytes = sizeof(d);
    d.flags = (geom_.shared_intermediate ? uint32_t(GLMAXX_MOE_SHARED_EXPERT) : 0u) |
              (w_.exl3 ? uint32_t(GLMAXX_MOE_EXL3_EXPERTS) : 0u);
    d.path = path;
    d.tokens = tokens;
    d.hidden = geom_.hidden;
    d.experts = geom_.experts;
    d.local_intermediate = geom_.local_intermediate;
    d.top_k = geom_.top_k;
    d.groups = geom_.groups;
    d.topk_groups = geom_.topk_groups;
    d.route_scale = geom_.route_scale;
    d.shared_intermediate = geom_.shared_intermediate;
    d.input_bf16 = x;
    d.router_weight_bf16 = w_.router_weight_bf16;
    d.router_bias_f32 = w_.router_bias_f32;
    d.w13_values = w_.w13_values;
    d.w13_scales = w_.w13_scales;
    d.w13_global_f32 = w_.w13_global_f32;
    d.w2_values = w_.w2_values;
    d.w2_scales = w_.w2_scales;
    d.w2_global_f32 = w_.w2_global_f32;
    d.shared13_bf16 = w_.shared13_bf16;
    d.shared2_bf16 = w_.shared2_bf16;
    d.route_experts_u16 = route_experts_.ptr();
    d.route_weights_f32 = route_weights_.ptr();
    d.output_f32 = out;
    d.validation_error_u32 = status_.ptr();
    d.workspace = ws;
    d.workspace_bytes = ws_bytes;
    d.sequence = 1;
    d.exl3_experts = reinterpret_cast<uint64_t>(w_.exl3);
    return d;
  }

  MoeGeometry geom_;
  MoeWeights w_;
  NativeBuffer route_experts_, route_weights_, status_, workspace_;
};

// ------------------------------------------------------------------ row buckets
constexpr std::array<uint32_t, 8> kDecodeRows = {1, 2, 4, 8, 16, 32, 64, 128};
constexpr std::array<uint32_t, 5> kPrefillRows = {256, 512, 1024, 2048, 3072};

// The smallest bucket holding `rows` rows (sorted buckets); Shape past the last.
inline uint32_t bucket_for(uint32_t rows, const std::vector<uint32_t>& buckets) {
  if (rows == 0) throw KernelError(ErrorKind::Shape);
  for (uint32_t b : buckets)
    if (b >= rows) return b;
  throw KernelError(ErrorKind::Shape);
}

inline std::vector<uint32_t> reference_buckets() {
  std::vector<uint32_t> b(kDecodeRows.begin(), kDecodeRows.end());
  b.insert(b.end(), kPrefillRows.begin(), kPrefillRows.end());
  return b;
}

// One executable graph of a RoutedMoeStep per row bucket over persistent,
// bucket-sized input and output buffers.  run() copies T rows in, zeroes the
// rows up to the bucket that an earlier call left behind, and replays the
// bucket's graph; real rows equal an unpadded launch (bit for bit on the decode
// path: every stage is per row and the split-K layout depends on ceil(T/64)).
class BucketedMoeGraphs {
 public:
  BucketedMoeGraphs(RoutedMoeStep& step, std::vector<uint32_t> buckets)
      : step_(step), buckets_(std::move(buckets)) {
    std::sort(buckets_.begin(), buckets_.end());
    if (buckets_.empty() || buckets_.back() > step.geometry().max_tokens)
      throw KernelError(ErrorKind::Shape);
    const uint64_t rows = buckets_.back(), h = step.geometry().hidden;
    x_ = NativeBuffer::allocate(rows * h * 2);
    out_ = NativeBuffer::allocate(rows * h * 4);
  }

  uint64_t output_f32() const { return out_.ptr(); }
  size_t captured() const { return graphs_.size(); }

  // x_bf16: device rows [rows][hidden]; returns the device address of the fp32
  // output rows (valid until the next run).
  uint64_t run(uint64_t x_bf16, uint32_t rows, uint64_t stream) {
    const uint32_t b = bucket_for(rows, buckets_);
    const uint64_t h = step_.geometry().hidden;
    if (dirty_ == 0) x_.zero(stream);
    check(glmaxx_memcpy_d2d(x_.ptr(), x_bf16, uint64_t(rows) * h * 2, stream));
    if (dirty_ > rows)
      check(glmaxx_memset_zero(x_.ptr() + uint64_t(rows) * h * 2, uint64_t(dirty_ - rows) * h * 2,
                               stream));
    dirty_ = rows;
    auto it = graphs_.find(b);
    if (it == graphs_.end()) {
      // an uncaptured launch first sizes nothing new (the step's workspace is
      // fixed) but creates the library's side stream outside the capture
      step_.launch(x_.ptr(), out_.ptr(), b, stream);
      NativeGraph::begin(stream);
      try {
        step_.launch(x_.ptr(), out_.ptr(), b, stream);
      } catch (...) {
        uint64_t discard = 0;
        glmaxx_stream_end_capture(stream, &discard);
        if (discard) glmaxx_graph_exec_destroy(discard);
        throw;
      }
      it = graphs_.emplace(b, NativeGraph::end(stream)).first;
    }
    it->second.launch(stream);
    return out_.ptr();
  }

 private:
  RoutedMoeStep& step_;
  std::vector<uint32_t> buckets_;
  NativeBuffer x_, out_;
  std::map<uint32_t, NativeGraph> graphs_;
  uint32_t dirty_ = 0;
};

// ------------------------------------------------------------------ peer finish
// The fused tensor-parallel reduce of the ranks' partials over CUDA IPC
// (glmaxx_moe_finish_peer_launch).  Each rank allocates one block holding a
// 256-byte signal buffer and the named slots at the same offsets on every rank;
// the engine's control channel carries local_handle() to the other ranks, and
// open() maps theirs.  Collective: every rank calls finish() at the same point
// of its stream.
class PeerFinish {
 public:
  // slot_bytes: the byte size of each named buffer, in order (e.g. partial,
  // output); every slot is 256-byte aligned.
  PeerFinish(const NativeRankContext& ctx, uint32_t rank, uint32_t ranks,
             std::vector<uint64_t> slot_bytes)
      : rank_(rank), ranks_(ranks) {
    ctx.require_owner();
    if (ranks == 0 || ranks > 8 || rank >= ranks) throw KernelError(ErrorKind::Topology);
    offsets_.push_back(256);
    uint64_t off = 256;
    for (uint64_t b : slot_bytes) {
      if (b == 0) throw KernelError(ErrorKind::Shape);
      off = checked_add(off, (b + 255) / 256 * 256);
      offsets_.push_back(off);
    }
    block_ = NativeBuffer::allocate(off);
    block_.zero(ctx.stream());
    ctx.synchronize();
    bases_.assign(ranks, 0);
    bases_[rank] = block_.ptr();
  }
  PeerFinish(const PeerFinish&) = delete;
  PeerFinish& operator=(const PeerFinish&) = delete;
  ~PeerFinish() {
    for (uint32_t r = 0; r < ranks_; ++r)
      if (r != rank_ && bases_[r]) glmaxx_ipc_close(bases_[r]);
  }

  std::array<uint8_t, 64> local_handle() const {
    std::array<uint8_t, 64> h{};
    check(glmaxx_ipc_handle(block_.ptr(), h.data()));
    return h;
  }
  // handles[r]: rank r's local_handle() (this rank's entry is ignored).
  void open(const std::vector<std::array<uint8_t, 64>>& handles) {
    if (handles.size() != ranks_) throw KernelError(ErrorKind::Shape);
    for (uint32_t r = 0; r < ranks_; ++r) {
      if (r == rank_ || bases_[r]) continue;
      uint64_t p = 0;
      check(glmaxx_ipc_open(handles[r].data(), &p));
      bases_[r] = p;
    }
  }
  // Device address of slot `slot` on rank `r` as mapped here.
  uint64_t slot(uint32_t slot, uint32_t r) const {
    if (slot + 1 >= offsets_.size() || r >= ranks_ || bases_[r] == 0)
      throw KernelError(ErrorKind::Shape);
    return bases_[r] + offsets_[slot];
  }
  uint64_t local(uint32_t s) const { return slot(s, rank_); }

  // out (slot out_slot, fp32) = residual (optional, bf16 or fp32 device
  // address) + sum over ranks of slot partial_slot, in rank order, on every rank.
  // two_shot: each rank reduces a slice and writes it into every rank's output.
  void finish(uint32_t partial_slot, uint32_t out_slot, uint64_t elements, uint64_t stream,
              bool two_shot, uint64_t residual_f32 = 0, uint64_t residual_bf16 = 0,
              uint64_t status_u32 = 0) const {
    std::vector<uint64_t> parts(ranks_), sigs(ranks_), outs(ranks_);
    for (uint32_t r = 0; r < ranks_; ++r) {
      parts[r] = slot(partial_slot, r);
      sigs[r] = bases_[r];
      outs[r] = slot(out_slot, r);
    }
    glmaxx_moe_finish_descriptor d;
    std::memset(&d, 0, sizeof(d));
    d.abi_version = GLMAXX_MOE_FINISH_ABI_VERSION;
    d.struct_bytes = sizeof(d);
    d.ranks = ranks_;
    d.elements = elements;
    d.residual_f32 = residual_f32;
    d.residual_bf16 = residual_bf16;
    d.partials_f32 = reinterpret_cast<uint64_t>(parts.data());
    d.output_f32 = outs[rank_];
    glmaxx_moe_peer_descriptor p;
    std::memset(&p, 0, sizeof(p));
    p.abi_version = GLMAXX_MOE_PEER_ABI_VERSION;
    p.struct_bytes = sizeof(p);
    p.flags = two_shot ? GLMAXX_MOE_PEER_TWO_SHOT : GLMAXX_MOE_PEER_ONE_SHOT;
    p.rank = rank_;
    p.signals_u32 = reinterpret_cast<uint64_t>(sigs.data());
    p.outputs_f32 = two_shot ? reinterpret_cast<uint64_t>(outs.data()) : 0;
    p.status_u32 = status_u32;
    check(glmaxx_moe_finish_peer_launch(&d, &p,
                                        reinterpret_cast<void*>(static_cast<uintptr_t>(stream))));
  }

 private:
  uint32_t rank_, ranks_;
  std::vector<uint64_t> offsets_;  // [0] signal buffer end / first slot, then slot ends
  NativeBuffer block_;
  std::vector<uint64_t> bases_;
};

// ------------------------------------------------------------------ rank files
// A reader error: code is a GLMAXX_RANK_ERR_* value (or a cudaError_t), kind()
// the reference variant it mirrors (RankFileError, Nvfp4Error, Exl3Error or the
// reader's I/O / UnsafeFile / Changed / Sink arms, native_reader.rs:664-671).
class RankFileError : public std::runtime_error {
 public:
  explicit RankFileError(int32_t code)
      : std::runtime_error(std::string("RankFile(") + glmaxx_rank_file_error_name(code) + ")"),
        code_(code) {}
  int32_t code() const { return code_; }
  const char* kind() const { return glmaxx_rank_file_error_name(code_); }

 private:
  int32_t code_;
};

inline void check_rank(int32_t status) {
  if (status != 0) throw RankFileError(status);
}

// One opened, validated rank file (NativeRankReader::open, native_reader.rs:
// 119-335); move-only.  verify / load read the payload once (verify_and_stream).
class NativeRankFile {
 public:
  static NativeRankFile open(const std::string& path) {
    glmaxx_rank_file* h = nullptr;
    check_rank(glmaxx_rank_file_open(path.c_str(), &h));
    NativeRankFile f(h);
    check_rank(glmaxx_rank_file_info_get(h, &f.info_));
    f.tensors_.resize(f.info_.tensor_count);
    for (uint32_t i = 0; i < f.info_.tensor_count; ++i)
      check_rank(glmaxx_rank_file_tensor(h, i, &f.tensors_[i]));
    return f;
  }
  NativeRankFile(NativeRankFile&& o) noexcept
      : h_(std::exchange(o.h_, nullptr)), info_(o.info_), tensors_(std::move(o.tensors_)) {}
  NativeRankFile& operator=(NativeRankFile&& o) noexcept {
    std::swap(h_, o.h_);
    std::swap(info_, o.info_);
    std::swap(tensors_, o.tensors_);
    return *this;
  }
  NativeRankFile(const NativeRankFile&) = delete;
  NativeRankFile& operator=(const NativeRankFile&) = delete;
  ~NativeRankFile() {
    if (h_) glmaxx_rank_file_close(h_);
  }

  const glmaxx_rank_file* handle() const { return h_; }
  const glmaxx_rank_file_info& info() const { return info_; }
  size_t tensor_count() const { return tensors_.size(); }
  const glmaxx_rank_tensor_info& tensor(size_t i) const {
    if (i >= tensors_.size()) throw RankFileError(GLMAXX_RANK_ERR_TENSOR_ID);
    return tensors_[i];
  }
  std::string tensor_name(size_t i) const {
    const glmaxx_rank_tensor_info& t = tensor(i);
    return std::string(t.name, t.name_bytes);
  }
  // The manifest bytes, digest-checked at open (JSON, not interpreted here).
  std::string manifest() const {
    const uint8_t* p = nullptr;
    uint64_t n = 0;
    check_rank(glmaxx_rank_file_manifest(h_, &p, &n));
    return std::string(reinterpret_cast<const char*>(p), n);
  }
  std::vector<uint8_t> codec_metadata(size_t i) const {
    const uint8_t* p = nullptr;
    uint64_t n = 0;
    check_rank(glmaxx_rank_file_codec_metadata(h_, uint32_t(i), &p, &n));
    return std::vector<uint8_t>(p, p + n);
  }
  // Tensors of one role, layer and expert (-1: not expert-specific); EXL3
  // projection 1/2/3 or 0 for any.  Selection is by role id, never by name
  // (format-v0.md section 18).
  std::vector<size_t> find(uint16_t role, int16_t layer, int16_t expert,
                           uint8_t projection = 0) const {
    std::vector<size_t> out;
    for (size_t i = 0; i < tensors_.size(); ++i) {
      const glmaxx_rank_tensor_info& t = tensors_[i];
      if (t.role_id == role && t.layer_id == layer && t.expert_id == expert &&
          (projection == 0 || t.exl3_projection == projection))
        out.push_back(i);
    }
    return out;
  }
  glmaxx_rank_payload_proof verify() const { return load({}, 0, 0); }
  glmaxx_rank_payload_proof load(const std::vector<glmaxx_rank_placement>& placements,
                                 uint64_t stream, uint32_t flags = 0) const {
    glmaxx_rank_payload_proof proof;
    check_rank(glmaxx_rank_file_verify_and_stream(
        h_, placements.empty() ? nullptr : placements.data(), uint32_t(placements.size()), flags,
        reinterpret_cast<void*>(static_cast<uintptr_t>(stream)), &proof));
    return proof;
  }
  // validate_rank_set (native_reader.rs:543-588): ranks 0..3 in order.
  static void validate_set(const std::array<const NativeRankFile*, 4>& files) {
    const glmaxx_rank_file* h[4];
    for (int r = 0; r < 4; ++r) h[r] = files[r] ? files[r]->h_ : nullptr;
    check_rank(glmaxx_rank_file_validate_set(h));
  }

 private:
  explicit NativeRankFile(glmaxx_rank_file* h) : h_(h) { std::memset(&info_, 0, sizeof(info_)); }
  glmaxx_rank_file* h_ = nullptr;
  glmaxx_rank_file_info info_;
  std::vector<glmaxx_rank_tensor_info> tensors_;
};

// One MoE layer of a rank file placed in new device buffers, laid out as
// MoeWeights documents: router [E, H] bf16 (role 0x0301), bias [E] fp32
// (0x0302), per expert either NVFP4 gate/up [2*I_r, H] (0x0501) and down
// [H, I_r] (0x0502) with their global scales, or EXL3 gate, up (0x0501,
// K = H, N = I_r) and down (0x0502, K = I_r, N = H) trellises with suh / svh;
// shared gate/up/down bf16 (0x0601-0x0603).  A hybrid layer gets a codec
// vector (1 = EXL3) and zero NVFP4 planes with global scale 1 for its EXL3
// experts; an all-EXL3 layer has no NVFP4 slabs.  Shapes must equal the
// geometry (logical and padded); one verified pass over the file.
class RankLayerWeights {
 public:
  static constexpr uint16_t kRouterWeight = 0x0301, kRouterBias = 0x0302, kGateUp = 0x0501,
                            kDown = 0x0502, kSharedGate = 0x0601, kSharedUp = 0x0602,
                            kSharedDown = 0x0603;

  static RankLayerWeights load(const NativeRankFile& file, const MoeGeometry& g, int16_t layer,
                               uint64_t stream) {
    const uint64_t E = g.experts, H = g.hidden, Ir = g.local_intermediate,
                   Is = g.shared_intermediate;
    RankLayerWeights w;
    std::vector<uint8_t> codec(E, 0);
    for (uint64_t e = 0; e < E; ++e) {
      const std::vector<size_t> gu = file.find(kGateUp, layer, int16_t(e));
      if (!gu.empty() && file.tensor(gu[0]).codec_id == GLMAXX_CODEC_EXL3_SOURCE) codec[e] = 1;
    }
    const bool any_exl3 = std::count(codec.begin(), codec.end(), 1) > 0;
    const bool any_nvfp4 = std::count(codec.begin(), codec.end(), 0) > 0;
    w.router_ = NativeBuffer::allocate(E * H * 2);
    w.bias_ = NativeBuffer::allocate(E * 4);
    if (any_nvfp4) {
      w.w13v_ = NativeBuffer::allocate(E * 2 * Ir * H / 2);
      w.w13s_ = NativeBuffer::allocate(E * 2 * Ir * H / 16);
      w.w2v_ = NativeBuffer::allocate(E * H * Ir / 2);
      w.w2s_ = NativeBuffer::allocate(E * H * Ir / 16);
      const std::vector<float> ones(E, 1.0f);  // EXL3 experts' NVFP4 global scale
      w.w13g_ = NativeBuffer::upload(ones.data(), E * 4, stream);
      w.w2g_ = NativeBuffer::upload(ones.data(), E * 4, stream);
      if (any_exl3)
        for (const NativeBuffer* b : {&w.w13v_, &w.w13s_, &w.w2v_, &w.w2s_}) b->zero(stream);
    }
    const uint64_t words = (H / 16) * (Ir / 16) * 48;  // per projection; K*N/16*3 halves
    if (any_exl3) {
      for (NativeBuffer* b : {&w.gate_tr_, &w.up_tr_, &w.down_tr_}) *b = NativeBuffer::allocate(E * words * 2);
      for (NativeBuffer* b : {&w.gate_suh_, &w.up_suh_, &w.down_svh_}) *b = NativeBuffer::allocate(E * H * 2);
      for (NativeBuffer* b : {&w.gate_svh_, &w.up_svh_, &w.down_suh_}) *b = NativeBuffer::allocate(E * Ir * 2);
      if (any_nvfp4) {
        w.codec_ = NativeBuffer::upload(codec.data(), E, stream);
        for (NativeBuffer* b : {&w.gate_tr_, &w.up_tr_, &w.down_tr_}) b->zero(stream);
      }
    }
    std::vector<glmaxx_rank_placement> pl;
    pl.reserve(5 + 3 * E);  // put() writes through one()'s pointer before the next push
    auto one = [&](uint16_t role, int16_t expert, uint16_t codec_id, uint64_t n, uint64_t k,
                   uint8_t projection = 0) {
      const std::vector<size_t> idx = file.find(role, layer, expert, projection);
      if (idx.size() != 1) throw KernelError(ErrorKind::Shape, role);
      const glmaxx_rank_tensor_info& t = file.tensor(idx[0]);
      const uint64_t ln = t.logical_shape[0], lk = t.ndim > 1 ? t.logical_shape[1] : 1;
      const uint64_t pn = t.padded_shape[0], pk = t.ndim > 1 ? t.padded_shape[1] : 1;
      if (t.codec_id != codec_id || ln != n || lk != k || pn != n || pk != k)
        throw KernelError(ErrorKind::Shape, role);
      glmaxx_rank_placement p;
      std::memset(&p, 0, sizeof(p));
      p.tensor_index = uint32_t(idx[0]);
      pl.push_back(p);
      return &pl.back();
    };
    auto put = [](glmaxx_rank_placement* p, int j, const NativeBuffer& b, uint64_t offset,
                  uint64_t bytes) {
      p->dst[j] = b.ptr() + offset;
      p->dst_bytes[j] = bytes;
    };
    put(one(kRouterWeight, -1, GLMAXX_CODEC_BF16, E, H), 0, w.router_, 0, E * H * 2);
    put(one(kRouterBias, -1, GLMAXX_CODEC_FP32, E, 1), 0, w.bias_, 0, E * 4);
    for (uint64_t e = 0; e < E; ++e) {
      if (codec[e] == 0) {
        glmaxx_rank_placement* p = one(kGateUp, int16_t(e), GLMAXX_CODEC_NVFP4_1D, 2 * Ir, H);
        put(p, 0, w.w13v_, e * Ir * H, Ir * H);
        put(p, 1, w.w13s_, e * 2 * Ir * H / 16, 2 * Ir * H / 16);
        put(p, 2, w.w13g_, e * 4, 4);
        p = one(kDown, int16_t(e), GLMAXX_CODEC_NVFP4_1D, H, Ir);
        put(p, 0, w.w2v_, e * H * Ir / 2, H * Ir / 2);
        put(p, 1, w.w2s_, e * H * Ir / 16, H * Ir / 16);
        put(p, 2, w.w2g_, e * 4, 4);
      } else {  // EXL3 source projections: descriptor shape [N, K]
        struct Proj {
          uint16_t role;
          uint8_t projection;
          uint64_t n, k;
          const NativeBuffer &tr, &suh, &svh;
        };
        const Proj projs[3] = {{kGateUp, 1, Ir, H, w.gate_tr_, w.gate_suh_, w.gate_svh_},
                               {kGateUp, 2, Ir, H, w.up_tr_, w.up_suh_, w.up_svh_},
                               {kDown, 3, H, Ir, w.down_tr_, w.down_suh_, w.down_svh_}};
        for (const Proj& pr : projs) {
          glmaxx_rank_placement* p =
              one(pr.role, int16_t(e), GLMAXX_CODEC_EXL3_SOURCE, pr.n, pr.k, pr.projection);
          put(p, 0, pr.tr, e * words * 2, words * 2);
          put(p, 1, pr.suh, e * pr.k * 2, pr.k * 2);
          put(p, 2, pr.svh, e * pr.n * 2, pr.n * 2);
        }
      }
    }
    if (Is) {
      w.sh13_ = NativeBuffer::allocate(2 * Is * H * 2);
      w.sh2_ = NativeBuffer::allocate(H * Is * 2);
      put(one(kSharedGate, -1, GLMAXX_CODEC_BF16, Is, H), 0, w.sh13_, 0, Is * H * 2);
      put(one(kSharedUp, -1, GLMAXX_CODEC_BF16, Is, H), 0, w.sh13_, Is * H * 2, Is * H * 2);
      put(one(kSharedDown, -1, GLMAXX_CODEC_BF16, H, Is), 0, w.sh2_, 0, H * Is * 2);
    }
    w.proof_ = file.load(pl, stream, any_exl3 ? GLMAXX_RANK_LOAD_EXL3_SOURCE : 0);
    MoeWeights& m = w.weights_;
    m.router_weight_bf16 = w.router_.ptr();
    m.router_bias_f32 = w.bias_.ptr();
    m.w13_values = w.w13v_.ptr();
    m.w13_scales = w.w13s_.ptr();
    m.w13_global_f32 = w.w13g_.ptr();
    m.w2_values = w.w2v_.ptr();
    m.w2_scales = w.w2s_.ptr();
    m.w2_global_f32 = w.w2g_.ptr();
    m.shared13_bf16 = Is ? w.sh13_.ptr() : 0;
    m.shared2_bf16 = Is ? w.sh2_.ptr() : 0;
    if (any_exl3) {
      // heap-held: the step keeps this host struct's address (MoeWeights::exl3)
      w.exl3_.reset(new glmaxx_moe_exl3_experts());
      glmaxx_moe_exl3_experts& x = *w.exl3_;
      std::memset(&x, 0, sizeof(x));
      x.abi_version = GLMAXX_MOE_EXL3_ABI_VERSION;
      x.struct_bytes = sizeof(x);
      x.bits = 3;
      x.codec_u8 = any_nvfp4 ? w.codec_.ptr() : 0;
      x.gate_trellis_u16 = w.gate_tr_.ptr();
      x.up_trellis_u16 = w.up_tr_.ptr();
      x.down_trellis_u16 = w.down_tr_.ptr();
      x.gate_suh_f16 = w.gate_suh_.ptr();
      x.gate_svh_f16 = w.gate_svh_.ptr();
      x.up_suh_f16 = w.up_suh_.ptr();
      x.up_svh_f16 = w.up_svh_.ptr();
      x.down_suh_f16 = w.down_suh_.ptr();
      x.down_svh_f16 = w.down_svh_.ptr();
      m.exl3 = w.exl3_.get();
    }
    return w;
  }
  const MoeWeights& weights() const { return weights_; }
  const glmaxx_rank_payload_proof& proof() const { return proof_; }
  bool exl3() const { return exl3_ != nullptr; }

 private:
  RankLayerWeights() { std::memset(&proof_, 0, sizeof(proof_)); }
  NativeBuffer router_, bias_, w13v_, w13s_, w13g_, w2v_, w2s_, w2g_, sh13_, sh2_;
  NativeBuffer codec_, gate_tr_, up_tr_, down_tr_, gate_suh_, gate_svh_, up_suh_, up_svh_,
      down_suh_, down_svh_;
  std::unique_ptr<glmaxx_moe_exl3_experts> exl3_;
  MoeWeights weights_;
  glmaxx_rank_payload_proof proof_;
};

}  // namespace host
}  // namespace glmaxx
