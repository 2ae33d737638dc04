// NVFP4 tensor-core throughput of this GPU, measured with this library's own
// tcgen05 code: one CTA per SM issues back-to-back block-scaled MMAs
// (tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16, M = 128, K = 64
// per instruction) on operands resident in shared memory and scale factors
// resident in TMEM.  Optional scale-factor copies (tcgen05.cp) between the MMAs
// price the copies the grouped GEMMs issue per K-block.  The prefill roofline
// uses the MMA-only rate as its measured NVFP4 peak.
//
//   shapes: N = 128 or 256 tokens per MMA; dual = two MMAs per K-block that
//   share the B tile (the FC1 gate/up pattern, N = 128 only).
//   copies: kind 1 = tcgen05.cp.32x128b.warpx4 (one 512-byte scale atom, to all
//   four lane quarters), kind 2 = tcgen05.cp.128x256b (4 KB lane-major block);
//   kind | 4: the copies of a 4-K-block stage are issued together before its
//   first MMA (the grouped GEMMs' pattern) instead of before each K-block.
//
// Operand bytes are a fixed pseudo-random pattern (finite E2M1 codes, E4M3
// scales near 1), so the tensor pipe does representative switching work.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/glmaxx_kernel.h"
#include "device.cuh"
#include "runtime.h"

namespace glmaxx {
namespace {

constexpr int kPeakThreads = 128;
constexpr uint32_t kSfBase = 256;    // TMEM column of the resident scale factors
constexpr uint32_t kCpBase = 320;    // TMEM columns the timed copies write (cycled)
constexpr uint32_t kCpSlots = 16;    // 16 slots of 8 columns

template <int N, bool DUAL>
struct PeakShape {
  static constexpr int kABytes = 128 * 128;  // 128 rows x 128 bytes (K = 256 per row)
  static constexpr int kBBytes = N * 128;
  static constexpr int kSmemA = kABytes * (DUAL ? 2 : 1);
  static constexpr int kSfBytes = 8192;      // scale staging (atoms and lane-major blocks)
  static constexpr int kUsed = kSmemA + kBBytes + kSfBytes + 1024 /* align */ + 64;
  // at least 120 KB, so that one CTA (holding all 512 TMEM columns) runs per SM
  static constexpr int kSmem = kUsed > 120 * 1024 ? kUsed : 120 * 1024;
  static constexpr int kNJ = N / 128;        // SFB atoms along N
  static_assert(!DUAL || N == 128, "dual MMAs use N = 128 (TMEM budget)");
};

__device__ __forceinline__ uint32_t mix32(uint32_t i) {
  i ^= i >> 16;
  i *= 0x7feb352dU;
  i ^= i >> 15;
  i *= 0x846ca68bU;
  i ^= i >> 16;
  return i;
}

template <int N, bool DUAL, int CP_KIND, bool BATCH>
__global__ void __launch_bounds__(kPeakThreads, 1)
    nvfp4_mma_peak_kernel(uint32_t iters, uint32_t copies, uint32_t* status,
                          unsigned long long* cycles) {
  using S = PeakShape<N, DUAL>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + S::kSmemA;
  uint8_t* ssf = sb + S::kBBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(ssf + S::kSfBytes);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar + 1);
  const int warp = threadIdx.x >> 5;

  // operands: pseudo-random E2M1 bytes; scales: E4M3 codes 0x30..0x3f (0.5 .. 1.9)
  for (uint32_t i = threadIdx.x; i < uint32_t(S::kSmemA + S::kBBytes) / 4; i += kPeakThreads)
    reinterpret_cast<uint32_t*>(sa)[i] = mix32(i + 977u * blockIdx.x) & 0x77777777u;
  for (uint32_t i = threadIdx.x; i < uint32_t(S::kSfBytes) / 4; i += kPeakThreads)
    reinterpret_cast<uint32_t*>(ssf)[i] = (mix32(i ^ 0x5bd1e995u) & 0x0f0f0f0fu) | 0x30303030u;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  fence_proxy_async_smem();
  if (warp == 0) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t d0 = tmem, d1 = tmem + 128;  // accumulators (d1: dual only)
  const uint32_t sfa0 = tmem + kSfBase, sfa1 = tmem + kSfBase + 16;
  const uint32_t sfb = tmem + kSfBase + 32;   // 4 K-blocks x kNJ atoms x 4 columns

  unsigned long long t0 = 0, t1 = 0;
  if (threadIdx.x == 0) {
    // resident scale factors: one atom per (operand, K-block, N block)
    for (int kb = 0; kb < 4; ++kb) {
      tc_cp_sf(sfa0 + kb * 4, smem_desc_sf(ssf + kb * 512));
      if (DUAL) tc_cp_sf(sfa1 + kb * 4, smem_desc_sf(ssf + 2048 + kb * 512));
      for (int j = 0; j < S::kNJ; ++j)
        tc_cp_sf(sfb + kb * 4 * S::kNJ + j * 4, smem_desc_sf(ssf + 4096 + (j * 4 + kb) * 512));
    }
    const uint32_t idesc = idesc_mxf4nvf4(N);
    const uint64_t a0 = smem_desc_sw128(sa);
    const uint64_t a1 = smem_desc_sw128(sa + (DUAL ? S::kABytes : 0));
    const uint64_t bd = smem_desc_sw128(sb);
    t0 = clock64();
    uint32_t slot = 0;
    for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        if (CP_KIND != 0 && (!BATCH || kb == 0)) {
          for (uint32_t c = 0; c < (BATCH ? 4 * copies : copies); ++c) {
            const uint32_t dst = tmem + kCpBase + (slot % kCpSlots) * 8;
            if (CP_KIND == 1)
              tc_cp_sf(dst, smem_desc_sf(ssf + (slot % 16) * 512));
            else
              tc_cp_sf_pair(dst, smem_desc_sf_pair(ssf + (slot & 1) * 4096));
            ++slot;
          }
        }
        const uint32_t acc = (it | kb) != 0;
        mma_fp4(d0, a0 + 2 * kb, bd + 2 * kb, idesc, acc, sfa0 + kb * 4, sfb + kb * 4 * S::kNJ);
        if (DUAL)
          mma_fp4(d1, a1 + 2 * kb, bd + 2 * kb, idesc, acc, sfa1 + kb * 4, sfb + kb * 4 * S::kNJ);
      }
    }
    tc_commit(bar);
  }
  __syncwarp();
  // every thread waits for the MMAs (bounded: a loop of at most 200,000
  // iterations takes well under the bound); a timeout is reported
  const bool done = mbar_wait(bar, 0, nullptr);
  if (threadIdx.x == 0) {
    t1 = clock64();
    if (!done) atomicOr(status, kStatusWaitTimeout);
    if (cycles) cycles[blockIdx.x] = t1 - t0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <int N, bool DUAL, int CP_KIND, bool BATCH = false>
cudaError_t launch_peak(uint32_t iters, uint32_t copies, uint32_t ctas, uint32_t* status,
                        unsigned long long* cycles, cudaStream_t stream) {
  using S = PeakShape<N, DUAL>;
  auto kern = nvfp4_mma_peak_kernel<N, DUAL, CP_KIND, BATCH>;
  cudaError_t st = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem);
  if (st != cudaSuccess) return st;
  kern<<<ctas, kPeakThreads, S::kSmem, stream>>>(iters, copies, status, cycles);
  return cudaPeekAtLastError();
}

}  // namespace
}  // namespace glmaxx

extern "C" int32_t glmaxx_nvfp4_mma_peak_launch(uint32_t n, uint32_t dual, uint32_t copy_kind,
                                                uint32_t copies_per_kblock, uint32_t iters,
                                                uint32_t ctas, uint32_t* status_u32,
                                                unsigned long long* cycles_u64,
                                                void* cuda_stream) {
  using namespace glmaxx;
  if (status_u32 == nullptr) return GLMAXX_ERR_NULL;
  const uint32_t form = copy_kind & 3u;
  const bool batch = (copy_kind & 4u) != 0;
  if (!(n == 128 || n == 256) || (dual && n != 128) || copy_kind > 6 || form == 3 ||
      (form == 0) != (copies_per_kblock == 0) || (batch && form == 0) || copies_per_kblock > 16 ||
      iters == 0 || iters > 200000 || ctas == 0 || ctas > 4096)
    return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
  cudaError_t st = cudaErrorInvalidValue;
#define GLMAXX_PEAK(N_, D_, K_, B_) \
  st = launch_peak<N_, D_, K_, B_>(iters, copies_per_kblock, ctas, status_u32, cycles_u64, s)
#define GLMAXX_PEAK_FORMS(N_, D_)                    \
  do {                                               \
    if (form == 0) GLMAXX_PEAK(N_, D_, 0, false);    \
    else if (form == 1 && !batch) GLMAXX_PEAK(N_, D_, 1, false); \
    else if (form == 1) GLMAXX_PEAK(N_, D_, 1, true);            \
    else if (!batch) GLMAXX_PEAK(N_, D_, 2, false);              \
    else GLMAXX_PEAK(N_, D_, 2, true);                           \
  } while (0)
  if (n == 128 && dual) GLMAXX_PEAK_FORMS(128, true);
  else if (n == 128) GLMAXX_PEAK_FORMS(128, false);
  else GLMAXX_PEAK_FORMS(256, false);
#undef GLMAXX_PEAK_FORMS
#undef GLMAXX_PEAK
  return st == cudaSuccess ? 0 : int32_t(st);
}
