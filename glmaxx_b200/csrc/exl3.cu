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
#include "exl3.cuh"
#include "moe.h"
#include "runtime.h"

namespace glmaxx {
namespace {

__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
// the two fp16 halves of a 32-bit word (low half = the lower k)
__device__ __forceinline__ void exl3_halves(uint32_t v, uint16_t& lo, uint16_t& hi) {
  asm("mov.b32 {%0, %1}, %2;" : "=h"(lo), "=h"(hi) : "r"(v));
}
// c + a*b in fp32 with one rounding, a and b fp16
__device__ __forceinline__ float exl3_fma_f16(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }


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

// ---------------------------------------------------------------------------
// Decode-fused EXL3 GEMV/GEMM: P[row][n] = f16( sum_k x[row][k] * W[k][n] ) with
// the reference's arithmetic (exl3.rs:404-453: fp32, multiply then add, k
// ascending from 0, one chain per output), so results are bit-identical to
// the CPU definition.  x and W are fp16, so every product x*w is exact in fp32
// (11 x 11 significant bits, exponents far inside fp32's range): rounding it
// is the identity, and round(round(x*w) + acc) = round(x*w + acc), one fused
// multiply-add.  The fma takes the fp16 factors as they are
// (fma.rn.f32.f16), so neither x nor the weights are widened first.  One warp owns 32 output columns (two 16x16 trellis tile
// columns); every 16 k it decodes its two tiles cooperatively -- lane l holds
// weights l*8 .. l*8+7 of a tile's 256-weight circular bitstream, the 4x2
// block (k, n) = (2(l&3) + (w&1) + 8((w>>1)&1), 2((l>>3)&3) + ((l>>2)&1) +
// 8((w>>2)&1)) -- transposes them through shared memory, and each lane then
// extends the chains of its column for RB rows.  Work items are (group = one
// weight matrix, block of RB rows of that group).
// ---------------------------------------------------------------------------
constexpr uint32_t kExl3KChunk = 256;                  // x staged per 256 k

struct Exl3GemvArgs {
  const uint16_t* x;             // [rows][K] f16, row r of group g at x + r*K
  const uint16_t* trellis;       // group g's trellis at trellis + g * trellis_stride (halves)
  uint64_t trellis_stride;
  const uint32_t* group_rows;    // [groups + 1] row offsets (exclusive prefix), or null:
                                 // one group of implicit_rows rows
  const uint32_t* items;         // [n_items] (group << 16 | row block), device list
  const uint32_t* n_items;       // device count of items
  uint32_t implicit_rows;
  uint16_t* out;                 // [rows][N] f16
  uint32_t K, N;
  // optional second projection of the same rows, shape and item list (the up
  // projection beside gate): blocks N/32 .. 2N/32 - 1 take x2 / trellis2 / out2,
  // so one launch holds twice the work units and its last wave is relatively
  // shorter; null: one projection
  const uint16_t* x2;
  const uint16_t* trellis2;
  uint16_t* out2;
};

template <int RB>
__global__ void __launch_bounds__(32) exl3_gemv_kernel(Exl3GemvArgs a) {
  // decoded 16 k x 32 columns, column-major (column c's 16 k values contiguous);
  // 40-half pitch keeps the 16-byte column reads and the 4-byte row-pair writes
  // of a warp on distinct banks
  constexpr int kPitch = 40;
  __shared__ __align__(16) uint16_t ws[32 * kPitch];
  __shared__ __align__(16) uint16_t xs[RB][kExl3KChunk]; // x of this item's rows (fp16)
  const uint32_t lane = threadIdx.x;
  const Exl3LaneWindow lw = exl3_lane_window(lane);
  const uint32_t ncw = a.N / 32;                         // column warps per projection
  const bool second = blockIdx.x >= ncw;                 // block-uniform
  const uint16_t* __restrict__ xin = second ? a.x2 : a.x;
  const uint16_t* __restrict__ trellis = second ? a.trellis2 : a.trellis;
  uint16_t* __restrict__ out = second ? a.out2 : a.out;
  const uint32_t c0 = (blockIdx.x - (second ? ncw : 0)) * 32;  // first column of this warp
  const uint32_t nt0 = c0 / 16;                          // first tile column
  const uint32_t lcb = 2 * ((lane >> 3) & 3) + ((lane >> 2) & 1);
  const uint32_t lrb = 2 * (lane & 3);
  const bool listed = a.group_rows != nullptr;
  const uint32_t count = listed ? *a.n_items : (a.implicit_rows + RB - 1) / RB;
  for (uint32_t it = blockIdx.y; it < count; it += gridDim.y) {
    const uint32_t item = listed ? a.items[it] : it;
    const uint32_t g = listed ? item >> 16 : 0, blk = listed ? item & 0xffff : item;
    const uint32_t r0 = (listed ? a.group_rows[g] : 0) + blk * RB;
    const uint32_t rend = listed ? a.group_rows[g + 1] : a.implicit_rows;
    const uint32_t nr = min(uint32_t(RB), rend - r0);
    const uint16_t* tr = trellis + uint64_t(g) * a.trellis_stride;
    float acc[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) acc[r] = 0.f;
    for (uint32_t kc = 0; kc < a.K; kc += kExl3KChunk) {
      const uint32_t kn = min(kExl3KChunk, a.K - kc);  // a multiple of 16
      __syncwarp();
      for (uint32_t i = lane; i < nr * kExl3KChunk; i += 32) {  // only this item's rows
        const uint32_t r = i / kExl3KChunk, k = i % kExl3KChunk;
        xs[r][k] = k < kn ? xin[uint64_t(r0 + r) * a.K + kc + k] : uint16_t(0);
      }
      __syncwarp();
      uint32_t span[2][3];
      auto tile_ptr = [&](uint32_t k, int j) {
        return tr + (uint64_t(k / 16) * (a.N / 16) + nt0 + j) * kExl3TileHalves;
      };
      exl3_load_span(tile_ptr(kc, 0), lw, span[0]);
      exl3_load_span(tile_ptr(kc, 1), lw, span[1]);
      for (uint32_t k16 = 0; k16 < kn; k16 += 16) {
        uint32_t wp[2][4];
        exl3_decode_span_pairs(span[0], lw.off, wp[0]);
        exl3_decode_span_pairs(span[1], lw.off, wp[1]);
        if (k16 + 16 < kn) {  // next step's words are in flight during this step
          exl3_load_span(tile_ptr(kc + k16 + 16, 0), lw, span[0]);
          exl3_load_span(tile_ptr(kc + k16 + 16, 1), lw, span[1]);
        }
        // weights w and w+1 are rows lr, lr+1 of one column: one 4-byte store
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int w = 0; w < 8; w += 2) {
            const uint32_t lr = lrb + 8 * ((w >> 1) & 1);
            const uint32_t lc = lcb + 8 * ((w >> 2) & 1);
            *reinterpret_cast<uint32_t*>(&ws[(16 * j + lc) * kPitch + lr]) = wp[j][w / 2];
          }
        __syncwarp();
        const uint4 c01 = *reinterpret_cast<const uint4*>(&ws[lane * kPitch]);
        const uint4 c23 = *reinterpret_cast<const uint4*>(&ws[lane * kPitch + 8]);
        const uint32_t cw[8] = {c01.x, c01.y, c01.z, c01.w, c23.x, c23.y, c23.z, c23.w};
        uint16_t wl[8], wh[8];  // weights k16 + 2q (low half) and k16 + 2q + 1 (high half)
#pragma unroll
        for (int q = 0; q < 8; ++q) exl3_halves(cw[q], wl[q], wh[q]);
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (r >= static_cast<int>(nr)) break;  // nr is the same for the whole warp
          const uint4 x01 = *reinterpret_cast<const uint4*>(&xs[r][k16]);
          const uint4 x23 = *reinterpret_cast<const uint4*>(&xs[r][k16 + 8]);
          const uint32_t xw[8] = {x01.x, x01.y, x01.z, x01.w, x23.x, x23.y, x23.z, x23.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint16_t xl, xh;
            exl3_halves(xw[q], xl, xh);
            acc[r] = exl3_fma_f16(xl, wl[q], acc[r]);
            acc[r] = exl3_fma_f16(xh, wh[q], acc[r]);
          }
        }
        __syncwarp();
      }
    }
#pragma unroll
    for (int r = 0; r < RB; ++r)
      if (r < static_cast<int>(nr)) out[uint64_t(r0 + r) * a.N + c0 + lane] = f2h(acc[r]);
  }
}

// Work list: one item per (group, block of rb rows) of every group with rows
// whose codec is EXL3 (codec == null: every group); single CTA.  Item order
// does not affect results (every item computes its own outputs).
__global__ void exl3_items_kernel(const uint32_t* __restrict__ group_rows, uint32_t groups,
                                  const uint8_t* __restrict__ codec, uint32_t rb, uint32_t max_rows,
                                  uint32_t* __restrict__ items, uint32_t* __restrict__ n_items) {
  __shared__ uint32_t base;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  for (uint32_t g0 = 0; g0 < groups; g0 += blockDim.x) {
    const uint32_t g = g0 + threadIdx.x;
    uint32_t rows = g < groups ? group_rows[g + 1] - group_rows[g] : 0;
    if (codec != nullptr && g < groups && codec[g] != 1) rows = 0;
    if (max_rows != 0 && rows >= max_rows) rows = 0;  // left to the tensor-core path
    const uint32_t nb = (rows + rb - 1) / rb;
    const uint32_t off = nb ? atomicAdd(&base, nb) : 0;
    for (uint32_t b = 0; b < nb; ++b) items[off + b] = (g << 16) | b;
    __syncthreads();
  }
  if (threadIdx.x == 0) *n_items = base;
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

// ---------------------------------------------------------------------------
// Per-assignment-row stages of the EXL3 experts (rows in compacted order,
// expert e owns rows offsets[e] .. offsets[e+1]; rows of NVFP4 experts are left
// alone).  Each CTA handles one 128-wide block of one row.
// ---------------------------------------------------------------------------
struct Exl3RowMap {
  const uint32_t* offsets;  // [E + 1]
  const uint8_t* codec;     // [E] or null (every expert EXL3)
  uint32_t E;
};

// Expert owning row r, or -1 when r is past the last row or the expert is not EXL3.
__device__ __forceinline__ int exl3_row_expert(const Exl3RowMap& m, uint32_t r) {
  if (r >= m.offsets[m.E]) return -1;
  uint32_t lo = 0, hi = m.E;  // offsets[lo] <= r < offsets[hi]
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (m.offsets[mid] <= r) lo = mid; else hi = mid;
  }
  if (m.codec != nullptr && m.codec[lo] != 1) return -1;
  return static_cast<int>(lo);
}

// H128 of one 128-element block held by a warp (lane owns elements lane + 32j,
// j = 0..3), times 1/sqrt(128).  exact: each output is the reference's
// ascending-column sum of +-input (exl3.rs:515-531), from the block staged in
// `blk`; otherwise a fast Walsh-Hadamard transform (same Sylvester matrix,
// butterflies through shuffles), for rows whose projection is not bit-exact
// anyway (the tensor-core path).
__device__ __forceinline__ void exl3_h128_warp(float (&v)[4], bool exact, float* blk,
                                               uint32_t lane) {
  const float norm = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
  if (exact) {
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) blk[lane + 32 * j] = v[j];
    __syncwarp();
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (uint32_t c = 0; c < 128; ++c) {
      const float x = blk[c];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t i = lane + 32 * j;
        acc[j] = __fadd_rn(acc[j], (__popc(i & c) & 1) ? -x : x);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(acc[j], norm);
    return;
  }
#pragma unroll
  for (uint32_t h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float o = __shfl_xor_sync(0xffffffffu, v[j], h);
      v[j] = (lane & h) ? __fsub_rn(o, v[j]) : __fadd_rn(v[j], o);
    }
  }
  // h = 32 and 64: partners in the lane's own registers (j bit 0 and bit 1)
  float w0 = __fadd_rn(v[0], v[1]), w1 = __fsub_rn(v[0], v[1]);
  float w2 = __fadd_rn(v[2], v[3]), w3 = __fsub_rn(v[2], v[3]);
  v[0] = __fmul_rn(__fadd_rn(w0, w2), norm);
  v[1] = __fmul_rn(__fadd_rn(w1, w3), norm);
  v[2] = __fmul_rn(__fsub_rn(w0, w2), norm);
  v[3] = __fmul_rn(__fsub_rn(w1, w3), norm);
}

// True when expert e's rows use the exact (reference-order) projection chain.
__device__ __forceinline__ bool exl3_exact_rows(const Exl3RowMap& m, int e, uint32_t tc_min_rows) {
  return tc_min_rows == 0 || m.offsets[e + 1] - m.offsets[e] < tc_min_rows;
}

// Input rotation (exl3.rs:404-453 steps 1-2): out[r][k] = f16(H128(f16(x[r][k] *
// suh[e][k]))).  x is either the bf16 token row row_token[r] of the layer
// input (converted to fp16 first) or the fp16 row r of `src`.  One CTA per
// row, 8 warps over its 128-blocks.
__global__ void __launch_bounds__(256) exl3_rows_rotate_in(
    Exl3RowMap m, const uint16_t* __restrict__ x_bf16, const uint32_t* __restrict__ row_token,
    const uint16_t* __restrict__ src_f16, const uint16_t* __restrict__ suh, uint32_t K,
    uint16_t* __restrict__ out, uint32_t tc_min_rows) {
  __shared__ float blk[8][128];
  __shared__ int s_e;
  const uint32_t r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) s_e = exl3_row_expert(m, r);
  __syncthreads();
  const int e = s_e;
  if (e < 0) return;
  const bool exact = exl3_exact_rows(m, e, tc_min_rows);
  const uint64_t xrow = x_bf16 != nullptr ? uint64_t(row_token[r]) * K : uint64_t(r) * K;
  for (uint32_t b = warp; b < K / 128; b += 8) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t k = b * 128 + lane + 32 * j;
      const float xv = x_bf16 != nullptr ? h2f(f2h(__uint_as_float(uint32_t(x_bf16[xrow + k]) << 16)))
                                         : h2f(src_f16[xrow + k]);
      v[j] = h2f(f2h(__fmul_rn(xv, h2f(suh[uint64_t(e) * K + k]))));
    }
    exl3_h128_warp(v, exact, blk[warp], lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) out[uint64_t(r) * K + b * 128 + lane + 32 * j] = f2h(v[j]);
  }
}

// Output rotation (steps 4-5): y = f16(H128(p) * svh[e]).  With `plane` set the
// routing-weighted fp32 value w * y goes to plane[token][slot][n] (the operand
// of the expert-order combine); otherwise y replaces p in place.
__global__ void __launch_bounds__(256) exl3_rows_rotate_out(
    Exl3RowMap m, uint16_t* __restrict__ p, const uint16_t* __restrict__ svh, uint32_t N,
    float* __restrict__ plane, const uint32_t* __restrict__ row_token,
    const uint32_t* __restrict__ row_slot, const float* __restrict__ row_weight, uint32_t top_k,
    uint32_t tc_min_rows) {
  __shared__ float blk[8][128];
  __shared__ int s_e;
  const uint32_t r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) s_e = exl3_row_expert(m, r);
  __syncthreads();
  const int e = s_e;
  if (e < 0) return;
  const bool exact = exl3_exact_rows(m, e, tc_min_rows);
  const uint64_t dst = plane != nullptr ? uint64_t(row_token[r]) * top_k + row_slot[r] : 0;
  const float wgt = plane != nullptr ? row_weight[r] : 0.f;
  for (uint32_t b = warp; b < N / 128; b += 8) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = h2f(p[uint64_t(r) * N + b * 128 + lane + 32 * j]);
    exl3_h128_warp(v, exact, blk[warp], lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t n = b * 128 + lane + 32 * j;
      const uint16_t y = f2h(__fmul_rn(v[j], h2f(svh[uint64_t(e) * N + n])));
      if (plane != nullptr)
        plane[dst * N + n] = __fmul_rn(wgt, h2f(y));
      else
        p[uint64_t(r) * N + n] = y;
    }
  }
}

// SwiGLU between the EXL3 projections: h = f16(silu(g) * u) with silu(v) =
// v / (1 + exp(-v)) (CUDA's expf and an IEEE division).
__global__ void exl3_rows_swiglu(Exl3RowMap m, const uint16_t* __restrict__ g,
                                 const uint16_t* __restrict__ u, uint32_t I,
                                 uint16_t* __restrict__ h) {
  __shared__ int s_e;
  const uint32_t r = blockIdx.y;
  if (threadIdx.x == 0) s_e = exl3_row_expert(m, r);
  __syncthreads();
  if (s_e < 0) return;
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= I) return;
  const uint64_t idx = uint64_t(r) * I + c;
  const float gv = h2f(g[idx]);
  const float sv = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
  h[idx] = f2h(__fmul_rn(sv, h2f(u[idx])));
}

// Rows per grouped work item: every item decodes its expert's whole projection,
// so an expert with 3-4 rows decodes once instead of twice (rows >= 8 take the
// tensor-core path); the multiply-add work follows the item's real row count.
constexpr int kExl3GroupRowBlock = 4;

}  // namespace

template <int RB>
cudaError_t run_exl3_gemv(const Exl3GemvArgs& a, uint32_t max_items, cudaStream_t stream) {
  dim3 grid((a.x2 != nullptr ? 2 : 1) * (a.N / 32), max_items < 4096 ? max_items : 4096);
  exl3_gemv_kernel<RB><<<grid, 32, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

cudaError_t launch_exl3_gemv_single(const uint16_t* x, const uint16_t* trellis, uint32_t rows,
                                    uint32_t K, uint32_t N, uint16_t* out, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  if (K % 16 || N % 32) return cudaErrorInvalidValue;
  Exl3GemvArgs a{};
  a.x = x;
  a.trellis = trellis;
  a.out = out;
  a.K = K;
  a.N = N;
  a.implicit_rows = rows;
  // rows per item: the FMA work of a block is RB chains per decoded weight
  if (rows == 1) return run_exl3_gemv<1>(a, 1, stream);
  if (rows == 2) return run_exl3_gemv<2>(a, 1, stream);
  if (rows <= 4) return run_exl3_gemv<4>(a, 1, stream);
  return run_exl3_gemv<8>(a, (rows + 7) / 8, stream);
}

cudaError_t launch_exl3_items(const uint32_t* group_rows, uint32_t groups, const uint8_t* codec,
                              uint32_t max_rows, uint32_t* items, uint32_t* n_items,
                              cudaStream_t stream) {
  if (groups >= 65536) return cudaErrorInvalidValue;
  exl3_items_kernel<<<1, 256, 0, stream>>>(group_rows, groups, codec, kExl3GroupRowBlock,
                                           max_rows, items, n_items);
  return cudaPeekAtLastError();
}

// Grouped projection over the item list of launch_exl3_items; with x2 set, a
// second projection of the same shape (x2, trellis2 -> out2) in the same launch.
cudaError_t launch_exl3_gemv_grouped(const uint16_t* x, const uint16_t* trellis,
                                     uint64_t trellis_stride, const uint32_t* group_rows,
                                     uint32_t max_items, const uint32_t* items,
                                     const uint32_t* n_items, uint32_t K, uint32_t N, uint16_t* out,
                                     cudaStream_t stream, const uint16_t* x2 = nullptr,
                                     const uint16_t* trellis2 = nullptr,
                                     uint16_t* out2 = nullptr) {
  if (K % 16 || N % 32) return cudaErrorInvalidValue;
  Exl3GemvArgs a{};
  a.x = x;
  a.trellis = trellis;
  a.trellis_stride = trellis_stride;
  a.group_rows = group_rows;
  a.items = items;
  a.n_items = n_items;
  a.out = out;
  a.K = K;
  a.N = N;
  a.x2 = x2;
  a.trellis2 = trellis2;
  a.out2 = out2;
  return run_exl3_gemv<kExl3GroupRowBlock>(a, max_items, stream);
}

// Experts with at least this many rows take the tensor-core projection
// (exl3_gemm.cu); the others the bit-exact decode-fused GEMV.
constexpr uint32_t kExl3TcMinRows = 8;

uint64_t exl3_experts_workspace_bytes(uint32_t A, uint32_t H, uint32_t I, uint32_t E) {
  const uint64_t wide = H > I ? H : I;
  const uint64_t max_tiles = (uint64_t(A) + 127) / 128 + E;
  return 4 * uint64_t(A) * wide * 2 + uint64_t(A) * I * 2 + (uint64_t(E) + A + 2) * 4 +
         max_tiles * sizeof(NTile) + 16 + 9 * 256;
}

cudaError_t launch_exl3_experts(const Exl3ExpertsLaunch& L, cudaStream_t stream) {
  const uint32_t A = L.A, H = L.H, I = L.I;
  if (H % 128 || I % 128 || A == 0) return cudaErrorInvalidValue;
  // workspace: xr [A][max(H,I)], p0, p1, p2 [A][max(H,I)], h [A][I], items
  const uint64_t wide = H > I ? H : I;
  uint8_t* w = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(L.workspace) + 255) & ~uintptr_t(255));
  auto take = [&](uint64_t bytes) {
    uint8_t* q = w;
    w += (bytes + 255) / 256 * 256;
    return q;
  };
  uint16_t* xr = reinterpret_cast<uint16_t*>(take(uint64_t(A) * wide * 2));
  uint16_t* p0 = reinterpret_cast<uint16_t*>(take(uint64_t(A) * wide * 2));
  uint16_t* p1 = reinterpret_cast<uint16_t*>(take(uint64_t(A) * wide * 2));
  uint16_t* p2 = reinterpret_cast<uint16_t*>(take(uint64_t(A) * wide * 2));
  uint16_t* h = reinterpret_cast<uint16_t*>(take(uint64_t(A) * I * 2));
  uint32_t* n_items = reinterpret_cast<uint32_t*>(take(16));
  uint32_t* items = reinterpret_cast<uint32_t*>(take((uint64_t(L.E) + A) * 4));
  const uint64_t max_tiles = (uint64_t(A) + 127) / 128 + L.E;
  NTile* tc_tiles = reinterpret_cast<NTile*>(take(max_tiles * sizeof(NTile)));
  uint32_t* tc_count = reinterpret_cast<uint32_t*>(take(16));
  const uint32_t max_items = L.E + (A + kExl3GroupRowBlock - 1) / kExl3GroupRowBlock;
  Exl3RowMap m{L.offsets, L.codec, L.E};
  const uint64_t gate_stride = uint64_t(H) * I * kExl3Bits / 16;  // halves per expert
#define X3(expr)                              \
  do {                                        \
    cudaError_t _st = (expr);                 \
    if (_st != cudaSuccess) return _st;       \
  } while (0)
  X3(launch_exl3_items(L.offsets, L.E, L.codec, kExl3TcMinRows, items, n_items, stream));
  X3(launch_exl3_tc_tiles(L.offsets, L.E, L.codec, kExl3TcMinRows, tc_tiles, tc_count, stream));
  // gate / up: rotate the token rows with each projection's suh (gate into xr,
  // up into p2, which holds nothing until the down projection), project both in
  // one decode-fused launch, then each projection's tensor-core rows, rotate out
  uint16_t* xr_up = p2;
  for (int proj = 0; proj < 2; ++proj) {
    exl3_rows_rotate_in<<<A, 256, 0, stream>>>(m, L.x_bf16, L.row_token, nullptr,
                                                proj ? L.up_suh : L.gate_suh, H,
                                                proj ? xr_up : xr, kExl3TcMinRows);
    X3(cudaPeekAtLastError());
  }
  X3(launch_exl3_gemv_grouped(xr, L.gate_trellis, gate_stride, L.offsets, max_items, items,
                              n_items, H, I, p0, stream, xr_up, L.up_trellis, p1));
  for (int proj = 0; proj < 2; ++proj) {
    const uint16_t* tr = proj ? L.up_trellis : L.gate_trellis;
    uint16_t* pout = proj ? p1 : p0;
    X3(launch_exl3_tc(proj ? xr_up : xr, A, H, tr, gate_stride, tc_tiles, tc_count, I, pout,
                      L.status, L.num_sms, stream));
    exl3_rows_rotate_out<<<A, 256, 0, stream>>>(m, pout, proj ? L.up_svh : L.gate_svh, I, nullptr,
                                                 nullptr, nullptr, nullptr, 0, kExl3TcMinRows);
    X3(cudaPeekAtLastError());
  }
  exl3_rows_swiglu<<<dim3((I + 255) / 256, A), 256, 0, stream>>>(m, p0, p1, I, h);
  X3(cudaPeekAtLastError());
  // down: rotate h, project to hidden, rotate out into the weighted plane
  exl3_rows_rotate_in<<<A, 256, 0, stream>>>(m, nullptr, nullptr, h, L.down_suh, I, xr,
                                              kExl3TcMinRows);
  X3(cudaPeekAtLastError());
  X3(launch_exl3_gemv_grouped(xr, L.down_trellis, gate_stride, L.offsets, max_items, items,
                              n_items, I, H, p2, stream));
  X3(launch_exl3_tc(xr, A, I, L.down_trellis, gate_stride, tc_tiles, tc_count, H, p2, L.status,
                    L.num_sms, stream));
  exl3_rows_rotate_out<<<A, 256, 0, stream>>>(m, p2, L.down_svh, H, L.plane, L.row_token,
                                               L.row_slot, L.row_weight, L.top_k, kExl3TcMinRows);
  X3(cudaPeekAtLastError());
#undef X3
  return cudaSuccess;
}

namespace {

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
  st = launch_exl3_gemv_single(reinterpret_cast<const uint16_t*>(d.rotated_input_f16),
                               reinterpret_cast<const uint16_t*>(d.trellis_u16), d.rows,
                               d.logical_k, d.logical_n, reinterpret_cast<uint16_t*>(d.projected_f16),
                               s);
  if (st != cudaSuccess) return int32_t(st);
  exl3_rotate_out<<<dim3(d.logical_n / 128, d.rows), 128, 0, s>>>(
      reinterpret_cast<const uint16_t*>(d.projected_f16), reinterpret_cast<const uint16_t*>(d.svh_f16),
      reinterpret_cast<uint16_t*>(d.output_f16), d.logical_n);
  return int32_t(cudaPeekAtLastError());
}

extern "C" int32_t glmaxx_exl3_gemv_launch(uint64_t input_f16, uint64_t trellis_u16, uint32_t rows,
                                           uint32_t logical_k, uint32_t logical_n, uint32_t bits,
                                           uint64_t output_f16, void* cuda_stream) {
  using namespace glmaxx;
  if (!input_f16 || !trellis_u16 || !output_f16 || cuda_stream == nullptr) return GLMAXX_ERR_NULL;
  if (bits != 3 || rows == 0 || logical_k == 0 || logical_n == 0 || logical_k % 16 ||
      logical_n % 32)
    return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  return int32_t(launch_exl3_gemv_single(
      reinterpret_cast<const uint16_t*>(input_f16), reinterpret_cast<const uint16_t*>(trellis_u16),
      rows, logical_k, logical_n, reinterpret_cast<uint16_t*>(output_f16),
      reinterpret_cast<cudaStream_t>(cuda_stream)));
}
