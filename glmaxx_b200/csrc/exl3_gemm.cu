// EXL3 experts with many rows per expert (prefill, continuous batches): a
// tcgen05 fp16 GEMM whose A operand -- the expert's weights -- is decoded from
// the 3-bit trellis straight into shared memory, so the weights cross HBM once,
// in their 3-bit form, and never exist as fp16 in global memory.
//
//   warp 0      TMA: the stage's token rows (B, rotated fp16 inputs) and the
//               stage's trellis bytes (4 k-tile rows x 8 n-tiles x 96 B)
//   warp 1      tcgen05.mma.kind::f16 (fp16 x fp16 -> fp32 in TMEM), 4 per stage
//   warps 2-5   epilogue: TMEM -> fp16 projection P[row][n]
//   warps 6-13  decoders: 32 trellis tiles per stage -> fp16 in the 128-byte
//               swizzled K-major layout the MMA reads
//
// Output: P = f16(sum_k x[row][k] W[k][n]) with fp32 tensor-core accumulation;
// the decode is the reference 3INST (exl3.rs:471-513), the accumulation order is
// not the reference's sequential one (the decode-fused GEMV keeps that order for
// experts with few rows).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "device.cuh"
#include "exl3.cuh"
#include "moe.h"
#include "runtime.h"

namespace glmaxx {
namespace {

constexpr int kXNT = 128;                    // token rows per tile (MMA N)
constexpr int kXStages = 4;
constexpr int kXAccBufs = 2;
constexpr int kXABytes = 128 * 128;          // 128 weight rows x 64 fp16 (128 B of K)
constexpr int kXBBytes = kXNT * 128;         // 128 token rows x 128 B of K
constexpr int kXTrellisRowBytes = 8 * 96;    // 8 consecutive n-tiles of one k-tile row
constexpr int kXTBytes = 4 * kXTrellisRowBytes;
constexpr int kXStageBytes = kXABytes + kXBBytes + kXTBytes;  // 35,840 (a multiple of 1024)
constexpr int kXDecoders = 16;              // decoder warps: n-tile dw % 8, k-tile half dw / 8
constexpr int kXKtPerDecoder = 4 * 8 / kXDecoders;  // k-tiles of the stage per decoder
constexpr int kXThreads = (6 + kXDecoders) * 32;
constexpr int kXSmem = kXStageBytes * kXStages + 1024 + 512;
static_assert(kXStageBytes % 1024 == 0, "stage alignment");

__host__ __device__ constexpr uint32_t idesc_f16(uint32_t n) {
  // kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, K-major, M = 128
  return (1u << 4) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

struct Exl3TcArgs {
  const uint16_t* trellis;   // expert g's trellis at trellis + g * trellis_stride (halves)
  uint64_t trellis_stride;
  const NTile* tiles;        // (expert, row_start, rows) of the EXL3 experts with many rows
  const uint32_t* tile_count;
  uint32_t m_tiles;          // Nproj / 128
  uint32_t k_chunks;         // K / 64
  uint32_t Nproj;            // the projection's output width
  uint16_t* out;             // [rows][Nproj] f16
  uint32_t* status;
};

__global__ void __launch_bounds__(kXThreads, 1)
    exl3_tc_kernel(const __grid_constant__ CUtensorMap tmap_b, const Exl3TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kXStageBytes * kXStages);
  uint64_t* full_tb = bars;                 // trellis + B landed (TMA)
  uint64_t* full_a = bars + kXStages;       // decoders wrote A
  uint64_t* empty_bar = bars + 2 * kXStages;
  uint64_t* tfull = bars + 3 * kXStages;
  uint64_t* tempty = tfull + kXAccBufs;
  uint64_t* drain_bar = tempty + kXAccBufs;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kXStages; ++s) {
      mbar_init(&full_tb[s], 1);
      mbar_init(&full_a[s], kXDecoders);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < kXAccBufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain_bar, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch(&tmap_b);
  if (warp == 1) {
    tmem_alloc(s_tmem, kXAccBufs * kXNT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  const uint32_t items = *args.tile_count * args.m_tiles;
  auto stage_a = [&](int s) { return smem + s * kXStageBytes; };
  auto stage_b = [&](int s) { return smem + s * kXStageBytes + kXABytes; };
  auto stage_t = [&](int s) { return smem + s * kXStageBytes + kXABytes + kXBBytes; };
  auto fail = [&](uint32_t bit) {
    *s_abort = 1;
    if (args.status) atomicOr(args.status, bit);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (uint32_t item = blockIdx.x; ok && item < items; item += gridDim.x) {
        const NTile t = args.tiles[item / args.m_tiles];
        const uint32_t i = item % args.m_tiles;
        const uint8_t* tr = reinterpret_cast<const uint8_t*>(args.trellis +
                                                             uint64_t(t.expert) * args.trellis_stride);
        for (uint32_t kc = 0; kc < args.k_chunks; ++kc) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, s_abort)) {
            fail(kStatusWaitTimeout);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_tb[stage], kXBBytes + kXTBytes);
          tma_load_2d(stage_b(stage), &tmap_b, &full_tb[stage], int32_t(kc * 128),
                      int32_t(t.row_start));
#pragma unroll
          for (int kt = 0; kt < 4; ++kt) {
            const uint64_t tile = uint64_t(kc * 4 + kt) * (args.Nproj / 16) + i * 8;
            bulk_load(stage_t(stage) + kt * kXTrellisRowBytes, tr + tile * 96, kXTrellisRowBytes,
                      &full_tb[stage]);
          }
          ++issued;
          if (++stage == kXStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      const uint32_t pending = issued < kXStages ? issued : kXStages;
      for (uint32_t b = 0; b < pending; ++b) {
        stage = (stage == 0) ? kXStages - 1 : stage - 1;
        if (stage == kXStages - 1) phase ^= 1;
        if (!mbar_wait(&full_tb[stage], phase, nullptr)) fail(kStatusWaitTimeout);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_f16(kXNT);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (uint32_t item = blockIdx.x; ok && item < items; item += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, s_abort)) {
          fail(kStatusWaitTimeout);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * kXNT;
        for (uint32_t kc = 0; kc < args.k_chunks; ++kc) {
          if (!mbar_wait(&full_tb[stage], phase, s_abort) ||
              !mbar_wait(&full_a[stage], phase, s_abort)) {
            fail(kStatusWaitTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = smem_desc_sw128(stage_a(stage));
          const uint64_t bd = smem_desc_sw128(stage_b(stage));
#pragma unroll
          for (int kb = 0; kb < 4; ++kb)  // 16 fp16 of K (32 bytes) per MMA
            mma_bf16(d, ad + 2 * kb, bd + 2 * kb, kIdesc, (kc > 0 || kb > 0) ? 1u : 0u);
          tc_commit(&empty_bar[stage]);
          if (++stage == kXStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        if (++acc == kXAccBufs) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      tc_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0, nullptr)) fail(kStatusTmemTimeout);
    }
  } else if (warp >= 6) {
    // ------------------------------------------------------------ decoders
    // Decoder dw writes n-tile dw % 8 of the 128-row A tile for k-tiles
    // kXKtPerDecoder * (dw / 8) .. of the stage's four (two decoders per n-tile,
    // so that twice the warps hide the decode's latency chains).  Lane l owns
    // weights 8l..8l+7 of a tile: rows (k) lrb + (w&1) +
    // 8((w>>1)&1), column (n) lcb + 8((w>>2)&1); weights w and w+1 are k, k+1 of
    // one n, one 4-byte store into the swizzled row n.  The decoder's trellis
    // words of the stage are read before any decode, so their latencies overlap.
    const uint32_t dw = (warp - 6) % 8, kt0 = (warp - 6) / 8 * kXKtPerDecoder;
    const Exl3LaneWindow lw = exl3_lane_window(lane);
    const uint32_t lcb = 2 * ((lane >> 3) & 3) + ((lane >> 2) & 1);
    const uint32_t lrb = 2 * (lane & 3);
    uint32_t widx[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) widx[j] = (lw.word0 + j) % 24;
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    for (uint32_t item = blockIdx.x; ok && item < items; item += gridDim.x) {
      for (uint32_t kc = 0; kc < args.k_chunks; ++kc) {
        if (!mbar_wait(&full_tb[stage], phase, s_abort)) {
          fail(kStatusWaitTimeout);
          ok = false;
          break;
        }
        const uint32_t* ts = reinterpret_cast<const uint32_t*>(stage_t(stage));
        uint8_t* a = stage_a(stage);
        uint32_t wd[kXKtPerDecoder][3];
#pragma unroll
        for (int kk = 0; kk < kXKtPerDecoder; ++kk)
#pragma unroll
          for (int j = 0; j < 3; ++j)
            wd[kk][j] = ts[((kt0 + kk) * kXTrellisRowBytes + dw * 96) / 4 + widx[j]];
#pragma unroll
        for (int kk = 0; kk < kXKtPerDecoder; ++kk) {
          const uint32_t ktl = kt0 + kk;
          uint32_t wp[4];
          exl3_decode_span_pairs(wd[kk], lw.off, wp);
#pragma unroll
          for (int w = 0; w < 8; w += 2) {
            const uint32_t n = dw * 16 + lcb + 8 * ((w >> 2) & 1);
            const uint32_t k = ktl * 16 + lrb + 8 * ((w >> 1) & 1);  // even
            const uint32_t byte = 2 * k;
            uint8_t* dst = a + n * 128 + ((((byte >> 4) ^ (n & 7)) << 4) | (byte & 15));
            *reinterpret_cast<uint32_t*>(dst) = wp[w / 2];
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[stage]);
        if (++stage == kXStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const uint32_t m = quarter * 32 + lane;
    uint32_t acc = 0, acc_phase = 0;
    for (uint32_t item = blockIdx.x; item < items; item += gridDim.x) {
      const NTile t = args.tiles[item / args.m_tiles];
      const uint32_t i = item % args.m_tiles;
      if (!mbar_wait(&tfull[acc], acc_phase, s_abort)) {
        fail(kStatusWaitTimeout);
        break;
      }
      tc_fence_after();
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kXNT;
      for (uint32_t c0 = 0; c0 < t.rows; c0 += 32) {
        uint32_t v[32];
        tmem_ld32_async(lane_base + c0, v);
        tmem_wait_ld();
        reg_fence(v);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (c0 + j >= t.rows) break;
          args.out[uint64_t(t.row_start + c0 + j) * args.Nproj + i * 128 + m] =
              __half_as_ushort(__float2half_rn(__uint_as_float(v[j])));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == kXAccBufs) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kXAccBufs * kXNT);
}

// Tiles of 128 rows for every EXL3 expert (codec null or 1) with at least
// min_rows rows; single CTA.  Tile order does not affect results.
__global__ void exl3_tc_tiles_kernel(const uint32_t* __restrict__ offsets, uint32_t E,
                                     const uint8_t* __restrict__ codec, uint32_t min_rows,
                                     NTile* __restrict__ tiles, uint32_t* __restrict__ tile_count) {
  __shared__ uint32_t base;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  for (uint32_t e0 = 0; e0 < E; e0 += blockDim.x) {
    const uint32_t e = e0 + threadIdx.x;
    uint32_t rows = e < E ? offsets[e + 1] - offsets[e] : 0;
    if (rows < min_rows || (codec != nullptr && e < E && codec[e] != 1)) rows = 0;
    const uint32_t nt = (rows + kXNT - 1) / kXNT;
    const uint32_t off = nt ? atomicAdd(&base, nt) : 0;
    for (uint32_t j = 0; j < nt; ++j) {
      NTile t;
      t.expert = e;
      t.row_start = offsets[e] + j * kXNT;
      t.sf_row_start = 0;
      t.rows = min(uint32_t(kXNT), rows - j * kXNT);
      tiles[off + j] = t;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *tile_count = base;
}

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

}  // namespace

cudaError_t launch_exl3_tc_tiles(const uint32_t* offsets, uint32_t E, const uint8_t* codec,
                                 uint32_t min_rows, NTile* tiles, uint32_t* tile_count,
                                 cudaStream_t stream) {
  exl3_tc_tiles_kernel<<<1, 256, 0, stream>>>(offsets, E, codec, min_rows, tiles, tile_count);
  return cudaPeekAtLastError();
}

cudaError_t launch_exl3_tc(const uint16_t* x, uint32_t x_rows, uint32_t K, const uint16_t* trellis,
                           uint64_t trellis_stride, const NTile* tiles, const uint32_t* tile_count,
                           uint32_t Nproj, uint16_t* out, uint32_t* status, int num_sms,
                           cudaStream_t stream) {
  if (K % 64 || Nproj % 128 || x_rows == 0) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t st = cudaFuncSetAttribute(exl3_tc_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kXSmem);
    if (st != cudaSuccess) return st;
    configured[dev] = true;
  }
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  CUtensorMap tb;
  cuuint64_t dims[2] = {uint64_t(K) * 2, x_rows};
  cuuint64_t strides[1] = {uint64_t(K) * 2};
  cuuint32_t box[2] = {128, kXNT};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint16_t*>(x), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  Exl3TcArgs a{};
  a.trellis = trellis;
  a.trellis_stride = trellis_stride;
  a.tiles = tiles;
  a.tile_count = tile_count;
  a.m_tiles = Nproj / 128;
  a.k_chunks = K / 64;
  a.Nproj = Nproj;
  a.out = out;
  a.status = status;
  exl3_tc_kernel<<<num_sms, kXThreads, kXSmem, stream>>>(tb, a);
  return cudaPeekAtLastError();
}

}  // namespace glmaxx
