// EXL3 3-bit trellis projection (reference ABI glmaxx_exl3_projection_launch,
// kernels/sm120/exl3_projection_control.cu:286-337), bit-exact with the CPU
// definition Exl3Trellis::matmul_reference_f16 (crates/glm-format/src/
// exl3.rs:404-453): x*suh -> fp16 -> H128 -> fp16, ascending-k fp32
// projection of the decoded fp16 weights -> fp16, H128 -> *svh -> fp16.
//
// Weight decode (exl3.rs:471-513): the 16-bit window ending at bit
// (lane*8 + weight + 257) * bits of the tile's circular bitstream, multiplied
// by the MCG constant, masked/xored into two fp16 halves that are summed.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/glmaxx_kernel.h"
#include "device.cuh"
#include "runtime.h"

namespace glmaxx {
namespace {

__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }

__device__ __forceinline__ uint16_t decode_3inst(uint32_t window) {
  const uint32_t value = window * 0xCBAC1FEDu;
  const uint32_t packed = (value & 0x8FFF8FFFu) ^ 0x3B603B60u;
  return f2h(__fadd_rn(h2f(uint16_t(packed)), h2f(uint16_t(packed >> 16))));
}

__device__ __forceinline__ uint16_t decode_at(const uint16_t* __restrict__ trellis, uint32_t n,
                                              uint32_t bits, uint32_t row, uint32_t col) {
  const uint32_t tile_halves = 16 * bits, tile_words = 8 * bits;
  const uint64_t tile = uint64_t(row / 16) * (n / 16) + col / 16;
  const uint16_t* base = trellis + tile * tile_halves;
  const uint32_t lr = row & 15, lc = col & 15;
  const uint32_t lane = ((lc >> 1) & 3) * 8 + (lc & 1) * 4 + ((lr & 7) >> 1);
  const uint32_t weight = (lc >= 8 ? 4 : 0) + (lr >= 8 ? 2 : 0) + (lr & 1);
  const uint32_t end_bit = (lane * 8 + weight + 257) * bits;
  const uint32_t first = (end_bit - 16) / 32, last = (end_bit - 1) / 32;
  const uint32_t shift = (last + 1) * 32 - end_bit;
  auto word = [&](uint32_t i) {
    const uint32_t h = (i % tile_words) * 2;
    return uint32_t(base[h]) | (uint32_t(base[h + 1]) << 16);
  };
  const uint64_t merged = (uint64_t(word(first)) << 32) | word(last);
  return decode_3inst(uint32_t((merged >> shift) & 0xffff));
}

// H128 of one 128-block held in shared memory, as exl3.rs:515-531: each output
// is the ascending-column sum of +-input, times 1/sqrt(128).
__device__ __forceinline__ float hadamard_row(const float* in, uint32_t r, float norm) {
  float sum = 0.f;
  for (uint32_t c = 0; c < 128; ++c) {
    const float v = (__popc(r & c) & 1) ? -in[c] : in[c];
    sum = __fadd_rn(sum, v);
  }
  return __fmul_rn(sum, norm);
}

// grid (K/128, rows), 128 threads
__global__ void exl3_rotate_in(const uint16_t* __restrict__ x, const uint16_t* __restrict__ suh,
                               uint16_t* __restrict__ rotated, uint32_t K) {
  __shared__ float blk[128];
  const uint32_t r = blockIdx.y, b = blockIdx.x, i = threadIdx.x;
  const uint64_t idx = uint64_t(r) * K + b * 128 + i;
  blk[i] = h2f(f2h(__fmul_rn(h2f(x[idx]), h2f(suh[b * 128 + i]))));
  __syncthreads();
  const float norm = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
  rotated[idx] = f2h(hadamard_row(blk, i, norm));
}

// grid (N/128, rows), 128 threads: one output column per thread, ascending k.
__global__ void exl3_project(const uint16_t* __restrict__ rotated,
                             const uint16_t* __restrict__ trellis, uint16_t* __restrict__ projected,
                             uint32_t K, uint32_t N, uint32_t bits) {
  const uint32_t r = blockIdx.y, col = blockIdx.x * 128 + threadIdx.x;
  const uint16_t* src = rotated + uint64_t(r) * K;
  float acc = 0.f;
  for (uint32_t k = 0; k < K; ++k)
    acc = __fadd_rn(acc, __fmul_rn(h2f(src[k]), h2f(decode_at(trellis, N, bits, k, col))));
  projected[uint64_t(r) * N + col] = f2h(acc);
}

// grid (N/128, rows), 128 threads
__global__ void exl3_rotate_out(const uint16_t* __restrict__ projected,
                                const uint16_t* __restrict__ svh, uint16_t* __restrict__ out,
                                uint32_t N) {
  __shared__ float blk[128];
  const uint32_t r = blockIdx.y, b = blockIdx.x, i = threadIdx.x;
  const uint64_t idx = uint64_t(r) * N + b * 128 + i;
  blk[i] = h2f(projected[idx]);
  __syncthreads();
  const float norm = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
  out[idx] = f2h(__fmul_rn(hadamard_row(blk, i, norm), h2f(svh[b * 128 + i])));
}

bool valid_exl3(const glmaxx_exl3_descriptor& d) {
  if (d.abi_version != GLMAXX_EXL3_ABI_VERSION || d.struct_bytes != sizeof(d) || d.flags) return false;
  for (uint64_t r : d.reserved)
    if (r) return false;
  if (d.projection < GLMAXX_EXL3_GATE || d.projection > GLMAXX_EXL3_DOWN) return false;
  if (d.bits != 3 || d.rows == 0 || d.rows > 3072) return false;
  if (d.logical_k == 0 || d.logical_n == 0 || d.logical_k % 128 || d.logical_n % 128) return false;
  return d.input_f16 && d.trellis_u16 && d.suh_f16 && d.svh_f16 && d.rotated_input_f16 &&
         d.projected_f16 && d.output_f16 && d.validation_error_u32;
}

}  // namespace
}  // namespace glmaxx

extern "C" int32_t glmaxx_exl3_projection_launch(const glmaxx_exl3_descriptor* descriptor,
                                                 void* cuda_stream, int32_t* asynchronous_error) {
  using namespace glmaxx;
  if (descriptor == nullptr || cuda_stream == nullptr || asynchronous_error == nullptr)
    return GLMAXX_ERR_NULL;
  *asynchronous_error = 0;
  const glmaxx_exl3_descriptor& d = *descriptor;
  if (!valid_exl3(d) ||
      d.workspace_bytes < glmaxx_exl3_projection_workspace_bytes(d.rows, d.logical_k, d.logical_n))
    return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(cuda_stream);
  cudaError_t st = cudaMemsetAsync(reinterpret_cast<void*>(d.validation_error_u32), 0, 4, s);
  if (st != cudaSuccess) return int32_t(st);
  exl3_rotate_in<<<dim3(d.logical_k / 128, d.rows), 128, 0, s>>>(
      reinterpret_cast<const uint16_t*>(d.input_f16), reinterpret_cast<const uint16_t*>(d.suh_f16),
      reinterpret_cast<uint16_t*>(d.rotated_input_f16), d.logical_k);
  exl3_project<<<dim3(d.logical_n / 128, d.rows), 128, 0, s>>>(
      reinterpret_cast<const uint16_t*>(d.rotated_input_f16),
      reinterpret_cast<const uint16_t*>(d.trellis_u16),
      reinterpret_cast<uint16_t*>(d.projected_f16), d.logical_k, d.logical_n, d.bits);
  exl3_rotate_out<<<dim3(d.logical_n / 128, d.rows), 128, 0, s>>>(
      reinterpret_cast<const uint16_t*>(d.projected_f16), reinterpret_cast<const uint16_t*>(d.svh_f16),
      reinterpret_cast<uint16_t*>(d.output_f16), d.logical_n);
  return int32_t(cudaPeekAtLastError());
}
