// Exhaustive checks of the NVFP4 encode.  First, the hardware conversions against this library's
// restatement of the reference codec (crates/glm-format/src/float.rs:15-73):
// every fp32 bit pattern with a finite value goes through e2m1_cvt and
// e2m1_encode, and every positive finite one through e4m3_cvt_pos and
// e4m3_encode_pos.  The quantisation kernels use the hardware forms, so a zero
// mismatch count makes their codes the reference's codes for every input.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/glmaxx_kernel.h"
#include "device.cuh"
#include "runtime.h"

namespace glmaxx {
namespace {

// out: [0] E2M1 mismatches, [1] E4M3 mismatches, [2] a mismatching E2M1 input's
// bits + 1 (0 = none), [3] the same for E4M3
__global__ void codec_selfcheck_kernel(unsigned long long* out) {
  unsigned long long bad2 = 0, bad3 = 0;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t u = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; u < (1ull << 32);
       u += stride) {
    const uint32_t bits = static_cast<uint32_t>(u);
    const float f = __uint_as_float(bits);
    if (!isfinite(f)) continue;
    if (e2m1_cvt(f) != e2m1_encode(f)) {
      ++bad2;
      atomicCAS(&out[2], 0ull, static_cast<unsigned long long>(bits) + 1);
    }
    if (f > 0.0f && e4m3_cvt_pos(f) != e4m3_encode_pos(f)) {
      ++bad3;
      atomicCAS(&out[3], 0ull, static_cast<unsigned long long>(bits) + 1);
    }
  }
  if (bad2) atomicAdd(&out[0], bad2);
  if (bad3) atomicAdd(&out[1], bad3);
}

// Every finite fp32 value v against each divisor in decs: the code that
// nvfp4_block's quotient path gives (e2m1x8_quotient, fast path where the
// divisor allows it) against the code of the exactly rounded quotient
// fl(v / dec).  out: [0] mismatches, [1] a mismatching (divisor index << 32 | v
// bits) + 1, [2] values that took the fast path, [3] values checked.
__global__ void quotient_selfcheck_kernel(const float* __restrict__ decs, uint32_t n_decs,
                                          unsigned long long* out) {
  unsigned long long bad = 0, fast_hits = 0, checked = 0;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint32_t d = 0; d < n_decs; ++d) {
    const float dec = decs[d];
    const bool fast = quotient_fast_ok(dec);
    const float rdec = fast ? __frcp_rn(dec) : 0.0f;
    for (uint64_t u = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; u < (1ull << 32);
         u += stride) {
      const uint32_t bits = static_cast<uint32_t>(u);
      const float f = __uint_as_float(bits);
      if (!isfinite(f)) continue;
      const float v[8] = {f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const uint32_t got = e2m1x8_quotient(v, dec, rdec, fast) & 0xfu;
      const uint32_t want = f == 0.0f ? 0u : e2m1_cvt(__fdiv_rn(f, dec));
      ++checked;
      if (fast) {
        const float q = __fmul_rn(f, rdec);
        if (f == 0.0f || e2m1_cvt(__fmul_rn(q, 0.99999904632568359375f)) ==
                             e2m1_cvt(__fmul_rn(q, 1.00000095367431640625f)))
          ++fast_hits;
      }
      if (got != want) {
        ++bad;
        atomicCAS(&out[1], 0ull, ((static_cast<unsigned long long>(d) << 32) | bits) + 1);
      }
    }
  }
  if (bad) atomicAdd(&out[0], bad);
  atomicAdd(&out[2], fast_hits);
  atomicAdd(&out[3], checked);
}

}  // namespace
}  // namespace glmaxx

extern "C" int32_t glmaxx_nvfp4_quotient_selfcheck_launch(const float* decs, uint32_t n_decs,
                                                          unsigned long long* result_u64x4,
                                                          void* cuda_stream) {
  using namespace glmaxx;
  if (result_u64x4 == nullptr || decs == nullptr) return GLMAXX_ERR_NULL;
  if (n_decs == 0 || n_decs > 4096) return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
  cudaError_t st = cudaMemsetAsync(result_u64x4, 0, 4 * sizeof(unsigned long long), s);
  if (st != cudaSuccess) return int32_t(st);
  quotient_selfcheck_kernel<<<info.sms * 8, 256, 0, s>>>(decs, n_decs, result_u64x4);
  return int32_t(cudaPeekAtLastError());
}

extern "C" int32_t glmaxx_nvfp4_codec_selfcheck_launch(unsigned long long* result_u64x4,
                                                       void* cuda_stream) {
  using namespace glmaxx;
  if (result_u64x4 == nullptr) return GLMAXX_ERR_NULL;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
  cudaError_t st = cudaMemsetAsync(result_u64x4, 0, 4 * sizeof(unsigned long long), s);
  if (st != cudaSuccess) return int32_t(st);
  codec_selfcheck_kernel<<<info.sms * 8, 256, 0, s>>>(result_u64x4);
  return int32_t(cudaPeekAtLastError());
}
