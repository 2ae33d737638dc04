// Test program of the C++ host runtime (include/glmaxx_host.hpp), driven by
// tests/test_host_cpp.py.
//
//   host_test cpu            checks that need no device; exit 0 when all pass
//   host_test gpu <dir>      runs one rank's routed-MoE step through RoutedMoeStep and
//                            BucketedMoeGraphs on seeded weights and writes every input
//                            and output to <dir> for the oracle comparison
//   host_test rankfile <dir> NativeRankFile over <dir>/rank{0..3}.g5n (device-free):
//                            set validation, verify, lookup, host placement, errors
//   host_test rankgpu <file> <dir>  RankLayerWeights::load of layer 3 (16 experts, TP4
//                            geometry) and one RoutedMoeStep on it; writes x and out
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

#include "glmaxx_host.hpp"

using namespace glmaxx::host;

namespace {

int failures = 0;
#define EXPECT(cond)                                                         \
  do {                                                                       \
    if (!(cond)) {                                                           \
      std::fprintf(stderr, "FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond); \
      ++failures;                                                            \
    }                                                                        \
  } while (0)

template <typename F>
bool throws_kind(F&& f, ErrorKind kind) {
  try {
    f();
  } catch (const KernelError& e) {
    return e.kind() == kind;
  }
  return false;
}

int run_cpu() {
  // ABI string and the reference workspace formulas
  validate_native_moe_abi(8, 64);
  validate_native_moe_abi(1024, 8192);
  EXPECT(throws_kind([] { validate_native_moe_abi(0, 8); }, ErrorKind::Shape));
  EXPECT(throws_kind([] { validate_native_moe_abi(1, 9); }, ErrorKind::Shape));
  EXPECT(reference_fc1_workspace_bytes(8) == glmaxx_nvfp4_routed_fc1_workspace_bytes(8));
  // row buckets (crates/glm-cli/src/profile.rs:10-11)
  const std::vector<uint32_t> b = reference_buckets();
  EXPECT(b.size() == 13 && b.front() == 1 && b.back() == 3072);
  EXPECT(bucket_for(3, b) == 4 && bucket_for(65, b) == 128 && bucket_for(129, b) == 256);
  EXPECT(bucket_for(3072, b) == 3072);
  EXPECT(throws_kind([&] { bucket_for(3073, b); }, ErrorKind::Shape));
  EXPECT(throws_kind([&] { bucket_for(0, b); }, ErrorKind::Shape));
  // topology rules of the rank context, checked before any device call
  EXPECT(throws_kind([] { NativeRankContext::bind(0, 3); }, ErrorKind::Topology));
  EXPECT(throws_kind([] { NativeRankContext::bind(4, 4); }, ErrorKind::Topology));
  // error objects
  const KernelError w(ErrorKind::Workspace, 1, 100, 50);
  EXPECT(w.required() == 100 && w.provided() == 50 && std::string(w.what()) == "Workspace(1)");
  EXPECT(throws_kind([] { check(-2); }, ErrorKind::Driver));
  EXPECT(throws_kind([] { NativeBuffer::allocate(0); }, ErrorKind::Shape));
  std::printf("host cpu checks: %d failure(s)\n", failures);
  return failures ? 1 : 0;
}

// ------------------------------------------------------------------ seeded data
struct Lcg {
  uint64_t s;
  explicit Lcg(uint64_t seed) : s(seed * 6364136223846793005ull + 1442695040888963407ull) {}
  uint32_t next() {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return uint32_t(s >> 33);
  }
  double uniform() { return (next() + 0.5) / 2147483648.0; }
  double normal() {  // Box-Muller
    const double u1 = uniform(), u2 = uniform();
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
  }
};

uint16_t to_bf16(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return uint16_t((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

template <typename T>
void dump(const std::string& path, const std::vector<T>& v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(v.data()), std::streamsize(v.size() * sizeof(T)));
}

int run_gpu(const std::string& dir) {
  NativeRankContext ctx = NativeRankContext::bind(0, 1);
  const uint64_t s = ctx.stream();
  MoeGeometry g;
  g.max_tokens = 64;
  g.hidden = 6144;
  g.experts = 16;
  g.local_intermediate = 512;
  g.top_k = 8;
  g.groups = 1;
  g.topk_groups = 1;
  g.route_scale = 2.5f;
  g.shared_intermediate = 256;
  const uint64_t H = g.hidden, E = g.experts, I = g.local_intermediate, Is = g.shared_intermediate;
  Lcg rng(7);
  // router (bf16 N(0, 0.02)) and correction bias (N(0, 0.01))
  std::vector<uint16_t> router(E * H);
  for (auto& v : router) v = to_bf16(float(0.02 * rng.normal()));
  std::vector<float> bias(E);
  for (auto& v : bias) v = float(0.01 * rng.normal());
  // NVFP4 experts: random E2M1 codes, E4M3 block scales 0x30..0x3f, global 1/2688
  auto nvfp4 = [&](uint64_t rows, uint64_t k, std::vector<uint8_t>& val, std::vector<uint8_t>& sc) {
    val.resize(E * rows * k / 2);
    sc.resize(E * rows * k / 16);
    for (auto& v : val) v = uint8_t(rng.next());
    for (auto& v : sc) v = uint8_t(0x30 + rng.next() % 16);
  };
  std::vector<uint8_t> w13v, w13s, w2v, w2s;
  nvfp4(2 * I, H, w13v, w13s);
  nvfp4(H, I, w2v, w2s);
  std::vector<float> g13(E, 1.0f / 2688.0f), g2(E, 1.0f / 2688.0f);
  std::vector<uint16_t> sh13(2 * Is * H), sh2(H * Is);
  for (auto& v : sh13) v = to_bf16(float(0.02 * rng.normal()));
  for (auto& v : sh2) v = to_bf16(float(0.02 * rng.normal()));
  const uint32_t T = 40;
  std::vector<uint16_t> x(T * H);
  for (auto& v : x) v = to_bf16(float(rng.normal()));

  NativeBuffer d_router = NativeBuffer::upload(router.data(), router.size() * 2, s);
  NativeBuffer d_bias = NativeBuffer::upload(bias.data(), bias.size() * 4, s);
  NativeBuffer d_w13v = NativeBuffer::upload(w13v.data(), w13v.size(), s);
  NativeBuffer d_w13s = NativeBuffer::upload(w13s.data(), w13s.size(), s);
  NativeBuffer d_g13 = NativeBuffer::upload(g13.data(), g13.size() * 4, s);
  NativeBuffer d_w2v = NativeBuffer::upload(w2v.data(), w2v.size(), s);
  NativeBuffer d_w2s = NativeBuffer::upload(w2s.data(), w2s.size(), s);
  NativeBuffer d_g2 = NativeBuffer::upload(g2.data(), g2.size() * 4, s);
  NativeBuffer d_sh13 = NativeBuffer::upload(sh13.data(), sh13.size() * 2, s);
  NativeBuffer d_sh2 = NativeBuffer::upload(sh2.data(), sh2.size() * 2, s);
  NativeBuffer d_x = NativeBuffer::upload(x.data(), x.size() * 2, s);
  NativeBuffer d_out = NativeBuffer::allocate(uint64_t(T) * H * 4);

  MoeWeights w;
  w.router_weight_bf16 = d_router.ptr();
  w.router_bias_f32 = d_bias.ptr();
  w.w13_values = d_w13v.ptr();
  w.w13_scales = d_w13s.ptr();
  w.w13_global_f32 = d_g13.ptr();
  w.w2_values = d_w2v.ptr();
  w.w2_scales = d_w2s.ptr();
  w.w2_global_f32 = d_g2.ptr();
  w.shared13_bf16 = d_sh13.ptr();
  w.shared2_bf16 = d_sh2.ptr();
  RoutedMoeStep step(ctx, g, w);

  // an eager step on T rows
  step.launch(d_x.ptr(), d_out.ptr(), T, s);
  step.check_device_status(s);
  std::vector<float> out(uint64_t(T) * H);
  d_out.download_at(out.data(), out.size() * 4, 0, s);
  std::vector<uint16_t> re(uint64_t(T) * g.top_k);
  std::vector<float> rw(uint64_t(T) * g.top_k);
  check(glmaxx_memcpy_d2h(re.data(), step.route_experts_u16(), re.size() * 2, s));
  check(glmaxx_memcpy_d2h(rw.data(), step.route_weights_f32(), rw.size() * 4, s));
  ctx.synchronize();

  // the same rows through a bucket graph (bucket 64): bit-identical rows
  BucketedMoeGraphs graphs(step, {4, 64});
  const uint64_t o1 = graphs.run(d_x.ptr(), T, s);
  std::vector<float> out_b(uint64_t(T) * H);
  check(glmaxx_memcpy_d2h(out_b.data(), o1, out_b.size() * 4, s));
  // fewer rows in a smaller bucket after a larger one: padding zeroed
  const uint64_t o2 = graphs.run(d_x.ptr(), 3, s);
  std::vector<float> out_c(3 * H);
  check(glmaxx_memcpy_d2h(out_c.data(), o2, out_c.size() * 4, s));
  step.launch(d_x.ptr(), d_out.ptr(), 3, s);
  std::vector<float> out_3(3 * H);
  d_out.download_at(out_3.data(), out_3.size() * 4, 0, s);
  ctx.synchronize();
  EXPECT(std::memcmp(out_b.data(), out.data(), out.size() * 4) == 0);
  EXPECT(std::memcmp(out_c.data(), out_3.data(), out_3.size() * 4) == 0);
  EXPECT(graphs.captured() == 2);
  // an out-of-range token count is refused before any launch
  EXPECT(throws_kind([&] { step.launch(d_x.ptr(), d_out.ptr(), 65, s); }, ErrorKind::Shape));

  dump(dir + "/x.bin", x);
  dump(dir + "/router.bin", router);
  dump(dir + "/bias.bin", bias);
  dump(dir + "/w13v.bin", w13v);
  dump(dir + "/w13s.bin", w13s);
  dump(dir + "/g13.bin", g13);
  dump(dir + "/w2v.bin", w2v);
  dump(dir + "/w2s.bin", w2s);
  dump(dir + "/g2.bin", g2);
  dump(dir + "/sh13.bin", sh13);
  dump(dir + "/sh2.bin", sh2);
  dump(dir + "/route_experts.bin", re);
  dump(dir + "/route_weights.bin", rw);
  dump(dir + "/out.bin", out);
  std::printf("host gpu run: %d failure(s), T=%u, workspace %llu bytes\n", failures, T,
              static_cast<unsigned long long>(step.workspace_bytes()));
  return failures ? 1 : 0;
}

std::vector<uint8_t> read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

template <typename F>
std::string rank_error_kind(F&& f) {
  try {
    f();
  } catch (const RankFileError& e) {
    return e.kind();
  }
  return "none";
}

int run_rankfile(const std::string& dir) {
  std::vector<NativeRankFile> files;
  for (int r = 0; r < 4; ++r) files.push_back(NativeRankFile::open(dir + "/rank" + std::to_string(r) + ".g5n"));
  NativeRankFile::validate_set({&files[0], &files[1], &files[2], &files[3]});
  EXPECT(rank_error_kind([&] {
           NativeRankFile::validate_set({&files[1], &files[0], &files[2], &files[3]});
         }) == std::string("RankSet"));
  for (int r = 0; r < 4; ++r) {
    const NativeRankFile& f = files[r];
    EXPECT(f.info().rank == uint32_t(r) && f.tensor_count() == 3);
    EXPECT(f.tensor_name(1) == "model.test.nvfp4.weight");
    EXPECT(f.manifest() == "{\"rank\":" + std::to_string(r) + ",\"schema\":\"reader-test\"}");
    EXPECT(f.find(0x0501, 3, 0).size() == 1 && f.find(0x0501, 78, 0, 1).size() == 1);
    EXPECT(f.codec_metadata(1).size() == 128 && f.codec_metadata(2).size() == 96);
    const glmaxx_rank_payload_proof v = f.verify();
    EXPECT(v.tensor_count == 3 && std::memcmp(v.payload_sha256, f.info().payload_sha256, 32) == 0);
    // the plain tensor placed in host memory equals its bytes in the file
    const glmaxx_rank_tensor_info& t = f.tensor(0);
    std::vector<uint8_t> dst(t.payload_bytes, 0xAB);
    glmaxx_rank_placement p;
    std::memset(&p, 0, sizeof(p));
    p.tensor_index = 0;
    p.dst[0] = reinterpret_cast<uint64_t>(dst.data());
    p.dst_bytes[0] = dst.size();
    f.load({p}, 0, GLMAXX_RANK_LOAD_HOST_DESTINATIONS);
    const std::vector<uint8_t> bytes = read_file(dir + "/rank" + std::to_string(r) + ".g5n");
    EXPECT(std::memcmp(dst.data(), bytes.data() + t.payload_offset, dst.size()) == 0);
    p.dst_bytes[0] = dst.size() - 1;  // a destination one byte short
    EXPECT(rank_error_kind([&] { f.load({p}, 0, GLMAXX_RANK_LOAD_HOST_DESTINATIONS); }) ==
           std::string("Argument"));
  }
  EXPECT(rank_error_kind([&] { NativeRankFile::open(dir + "/truncated.g5n"); }) ==
         std::string("Truncated"));
  EXPECT(rank_error_kind([&] { NativeRankFile::open(dir + "/missing.g5n"); }) == std::string("Io"));
  std::printf("host rankfile checks: %d failure(s)\n", failures);
  return failures ? 1 : 0;
}

int run_rankgpu(const std::string& file, const std::string& dir) {
  NativeRankContext ctx = NativeRankContext::bind(0, 1);
  const uint64_t s = ctx.stream();
  MoeGeometry g;
  g.max_tokens = 64;
  g.experts = 16;
  g.groups = 1;
  g.topk_groups = 1;
  g.local_intermediate = 512;
  g.shared_intermediate = 512;
  const NativeRankFile f = NativeRankFile::open(file);
  const RankLayerWeights w = RankLayerWeights::load(f, g, 3, s);
  EXPECT(w.proof().payload_bytes == f.info().payload_bytes);
  std::printf("layer codec: %s\n", w.exl3() ? "exl3/hybrid" : "nvfp4");
  RoutedMoeStep step(ctx, g, w.weights());
  const uint32_t T = 40;
  Lcg rng(11);
  std::vector<uint16_t> x(uint64_t(T) * g.hidden);
  for (auto& v : x) v = to_bf16(float(rng.normal()));
  NativeBuffer d_x = NativeBuffer::upload(x.data(), x.size() * 2, s);
  NativeBuffer d_out = NativeBuffer::allocate(uint64_t(T) * g.hidden * 4);
  step.launch(d_x.ptr(), d_out.ptr(), T, s);
  step.check_device_status(s);
  std::vector<float> out(uint64_t(T) * g.hidden);
  d_out.download_at(out.data(), out.size() * 4, 0, s);
  ctx.synchronize();
  dump(dir + "/x.bin", x);
  dump(dir + "/out.bin", out);
  std::printf("host rankgpu run: %d failure(s)\n", failures);
  return failures ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "cpu";
  try {
    if (mode == "cpu") return run_cpu();
    if (mode == "gpu" && argc > 2) return run_gpu(argv[2]);
    if (mode == "rankfile" && argc > 2) return run_rankfile(argv[2]);
    if (mode == "rankgpu" && argc > 3) return run_rankgpu(argv[2], argv[3]);
  } catch (const KernelError& e) {
    std::fprintf(stderr, "KernelError %s\n", e.what());
    return 2;
  } catch (const RankFileError& e) {
    std::fprintf(stderr, "RankFileError %s\n", e.what());
    return 3;
  }
  std::fprintf(stderr, "usage: host_test cpu | gpu <dir> | rankfile <dir> | rankgpu <file> <dir>\n");
  return 64;
}
