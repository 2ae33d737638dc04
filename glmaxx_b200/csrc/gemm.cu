// Host launchers for the tcgen05 grouped GEMM variants: TMA tensor-map
// encoding (driver entry point fetched at run time, no libcuda link) and
// persistent launches of one CTA per SM.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "moe.h"

namespace glmaxx {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q{};
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Byte-element 3-D map over [experts][rows][row_bytes], box 128 B x 128 rows x 1.
cudaError_t encode_a(CUtensorMap* m, const void* base, uint32_t experts, uint32_t rows,
                     uint32_t row_bytes) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[3] = {row_bytes, rows, experts};
  cuuint64_t strides[2] = {row_bytes, uint64_t(row_bytes) * rows};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Byte-element 2-D map over [rows][row_bytes], box 128 B x nt rows.
cudaError_t encode_b(CUtensorMap* m, const void* base, uint32_t rows, uint32_t row_bytes,
                     uint32_t nt) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {128, nt};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <bool FP4, bool DUAL, int NT, int STAGES, int EPI>
cudaError_t run(const GemmLaunch& g, int num_sms, cudaStream_t stream) {
  static_assert(gemm_smem_bytes<FP4, DUAL, NT, STAGES, EPI>() <= 227 * 1024, "smem budget");
  auto kernel = grouped_gemm_kernel<FP4, DUAL, NT, STAGES, EPI>;
  constexpr int smem = gemm_smem_bytes<FP4, DUAL, NT, STAGES, EPI>();
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (st != cudaSuccess) return st;
    configured[dev] = true;
  }
  if (g.a_row_bytes % 128 != 0 || g.b_row_bytes != g.a_row_bytes) return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  cudaError_t st = encode_a(&ta, g.a, g.a_experts, g.a_rows, g.a_row_bytes);
  if (st != cudaSuccess) return st;
  st = encode_b(&tb, g.b, g.b_rows, g.b_row_bytes, NT);
  if (st != cudaSuccess) return st;
  kernel<<<num_sms, GemmShape<FP4, DUAL, NT>::kThreads, smem, stream>>>(ta, tb, g.args);
  return cudaPeekAtLastError();
}

}  // namespace

void choose_k_splits(uint32_t tiles, uint32_t k_chunks, int sms, uint32_t max_splits,
                     uint32_t* splits, uint32_t* kc_per) {
  uint32_t want = tiles >= uint32_t(sms) ? 1u : uint32_t(sms) / (tiles ? tiles : 1);
  if (want > max_splits) want = max_splits;
  if (want > k_chunks) want = k_chunks;
  if (want < 1) want = 1;
  const uint32_t per = (k_chunks + want - 1) / want;
  *kc_per = per;
  *splits = (k_chunks + per - 1) / per;  // every slice has at least one chunk
}

int gemm_tile_rows(GemmVariant v) {
  switch (v) {
    case kFc1DecodeFp4:
    case kFc2DecodeFp4:
    case kFc2DecodeFp4Pair:
    case kFc2DecodeFp4Store:
      return 32;
    case kShared1Bf16N64:
    case kShared2Bf16N64:
    case kShared1Bf16N64Split:
    case kShared2Bf16N64Split:
      return 64;
    default:
      return 128;
  }
}

cudaError_t launch_gemm(GemmVariant v, const GemmLaunch& g, int num_sms, cudaStream_t stream) {
  switch (v) {
    case kFc1DecodeFp4:
      return run<true, true, 32, 5, kEpiSwiGLU>(g, num_sms, stream);
    case kFc2DecodeFp4:
      return run<true, false, 32, 8, kEpiRoutedPlane>(g, num_sms, stream);
    case kFc2DecodeFp4Pair:
      return run<true, true, 32, 5, kEpiRoutedPlane>(g, num_sms, stream);
    case kFc2DecodeFp4Store:
      return run<true, false, 32, 8, kEpiStoreF32>(g, num_sms, stream);
    case kFc1PrefillFp4:
      return run<true, true, 128, 3, kEpiSwiGLU>(g, num_sms, stream);
    case kFc2PrefillFp4:
      return run<true, false, 128, 4, kEpiRoutedAtomic>(g, num_sms, stream);
    case kFc2PrefillFp4Store:
      return run<true, false, 128, 4, kEpiStoreF32>(g, num_sms, stream);
    case kFc2PrefillFp4PairPlane:
      return run<true, true, 128, 3, kEpiRoutedPlane>(g, num_sms, stream);
    case kFc2PrefillFp4PairAtomic:
      return run<true, true, 128, 3, kEpiRoutedAtomic>(g, num_sms, stream);
    case kShared1Bf16N64:
      return run<false, true, 64, 5, kEpiSwiGLU>(g, num_sms, stream);
    case kShared2Bf16N64:
      return run<false, false, 64, 8, kEpiStoreF32>(g, num_sms, stream);
    case kShared1Bf16N128:
      return run<false, true, 128, 4, kEpiSwiGLU>(g, num_sms, stream);
    case kShared2Bf16N128:
      return run<false, false, 128, 6, kEpiStoreF32>(g, num_sms, stream);
    case kShared1Bf16N64Split:
      return run<false, true, 64, 5, kEpiStorePartial>(g, num_sms, stream);
    case kShared2Bf16N64Split:
      return run<false, false, 64, 8, kEpiStorePartial>(g, num_sms, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace glmaxx
