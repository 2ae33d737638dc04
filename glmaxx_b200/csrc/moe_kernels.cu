// Routing, compaction, NVFP4 quantisation and combine kernels of the routed
// MoE step (everything around the two grouped GEMMs).
//
// Data flow of one rank-local step (T tokens, H hidden, E experts, I local
// intermediate, K = top_k):
//   router_logits  x[T,H] bf16, Wr[E,H] bf16  -> partial[8][T][E] f32
//   router_select  partial, bias              -> experts[T,K] u16, weights[T,K] f32,
//                                                bitmap[E][ceil(T/32)] (token-in-expert bits)
//   compact        bitmap                     -> counts, offsets, padded offsets, word
//                                                prefixes, GEMM n-tile list
//   quant_scatter  x, routes, prefixes        -> per-assignment NVFP4 rows in expert-
//                                                contiguous, 128-padded "row space"
//   (FC1 GEMM)                                -> h[row, I] bf16 (SwiGLU applied)
//   fc2_quant      h                          -> NVFP4 rows of h
//   (FC2 GEMM)                                -> plane[T][K][H] or atomics into out[T,H]
//   combine        plane (+ shared expert)    -> out[T,H] f32
//
// Assignment order inside an expert is ascending token, i.e. the reference's
// stable (expert, token, slot) compaction (crates/glm-reference/src/
// routed_fc1.rs:20-58): a token's rank inside expert e is the number of
// smaller tokens routed to e, read from the bitmap with popcounts.
#include <cuda_runtime.h>

#include <cstdint>

#include "device.cuh"
#include "moe.h"

namespace glmaxx {

// ---------------------------------------------------------------------------
// Router logits.  Canonical order (shared with the CPU restatement):
//   logit[t][e] = ((s_0 + s_1) + ...) + s_7,  s_c = fma-chain over the c-th
//   eighth of H in ascending k from 0.
// Both kernels split the grid's z over the 8 chunks, and the first kernel of a
// step also clears the token-in-expert bitmap.
// ---------------------------------------------------------------------------
// Small-T kernel: CTA tile 32 tokens x 32 experts x one K chunk, 8 warps of
// 16 tokens x 8 experts; lane (tp = lane % 8, ep = lane / 8) of warp w owns
// tokens tp and tp + 8 and experts ep and ep + 4 of its warp's tile: four
// independent fma-chains, each in ascending k, two warps per scheduler.
// K advances in phases of 128 elements.  The kernel is bound by the latency of
// its global loads unless most of a CTA's 96 KB are in flight at once, so the
// raw bf16 rows of up to kRbRing phases are requested by cp.async at the start
// (a ring of phase buffers, refilled kRbRing - 1 phases ahead).  Each phase is
// then widened to fp32 into one of two compute buffers ([row][k], 528-byte
// pitch: 16 mod 128, so the 16-byte loads of 8 consecutive rows fall on
// distinct banks).  Per 4 k a thread loads 4 x 16 bytes for 16 fmas, and a
// warp's load touches 8 (tokens) or 4 (experts) rows: one wavefront each.
constexpr uint32_t kRbTile = 32;              // tokens (and experts) per CTA
constexpr uint32_t kRbThreads = 256;
constexpr uint32_t kRbPhaseK = 128;           // k per phase
constexpr uint32_t kRbRows = 2 * kRbTile;     // x rows then w rows
constexpr uint32_t kRbRing = 6;               // bf16 phase buffers (H = 6144: the whole chunk)
constexpr uint32_t kRbRawPitch = kRbPhaseK * 2 + 16;       // bytes per bf16 row
constexpr uint32_t kRbRawBytes = kRbRows * kRbRawPitch;    // one bf16 phase buffer
constexpr uint32_t kRbPitch = kRbPhaseK + 4;               // floats per fp32 row
constexpr uint32_t kRbBufFloats = kRbRows * kRbPitch;      // one fp32 compute buffer
constexpr uint32_t kRbSmem = kRbRing * kRbRawBytes + 2 * kRbBufFloats * 4;
constexpr uint32_t kRbPieces = kRbRows * kRbPhaseK / 8 / kRbThreads;  // 16-byte pieces per thread

__global__ void __launch_bounds__(kRbThreads) router_logits_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, float* __restrict__ partial,
    uint32_t T, uint32_t H, uint32_t E, uint32_t* __restrict__ bitmap, uint32_t bitmap_words) {
  extern __shared__ __align__(16) uint8_t rb_smem[];
  uint8_t* raw = rb_smem;                                              // [kRbRing][rows][pitch]
  float* fbuf = reinterpret_cast<float*>(rb_smem + kRbRing * kRbRawBytes);  // [2][rows][pitch]
  const uint32_t chunk = H / 8;  // multiple of 32 (H % 256 == 0)
  const uint32_t e0 = blockIdx.x * kRbTile, t0 = blockIdx.y * kRbTile, c = blockIdx.z;
  const uint32_t tid = threadIdx.x;
  {
    const uint64_t lin = (uint64_t(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    const uint64_t nthreads = uint64_t(gridDim.x) * gridDim.y * gridDim.z * blockDim.x;
    for (uint64_t i = lin * blockDim.x + tid; i < bitmap_words; i += nthreads) bitmap[i] = 0;
  }
  const uint32_t phases = (chunk + kRbPhaseK - 1) / kRbPhaseK;
  // piece i of a phase: row i / 16 (x rows 0..31, then w rows), k 8 * (i % 16);
  // rows past T or E, and k past the chunk, are zero
  auto fill = [&](uint32_t p) {
    if (p < phases) {
      uint8_t* buf = raw + (p % kRbRing) * kRbRawBytes;
      const uint32_t k0 = p * kRbPhaseK;
#pragma unroll
      for (int j = 0; j < int(kRbPieces); ++j) {
        const uint32_t i = tid + kRbThreads * j, r = i / 16, kk = (i % 16) * 8;
        const bool is_x = r < kRbTile;
        const uint32_t row = (is_x ? t0 : e0) + (r % kRbTile);
        uint8_t* dst = buf + r * kRbRawPitch + kk * 2;
        if (row < (is_x ? T : E) && k0 + kk < chunk)
          cp_async_16(dst, (is_x ? x : w) + uint64_t(row) * H + uint64_t(c) * chunk + k0 + kk);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();  // one group per phase slot, empty past the last phase
  };
  auto widen = [&](uint32_t p) {
    const uint8_t* src = raw + (p % kRbRing) * kRbRawBytes;
    float* dst = fbuf + (p & 1) * kRbBufFloats;
#pragma unroll
    for (int j = 0; j < int(kRbPieces); ++j) {
      const uint32_t i = tid + kRbThreads * j, r = i / 16, kk = (i % 16) * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(src + r * kRbRawPitch + kk * 2);
      const uint32_t v[4] = {u.x, u.y, u.z, u.w};
      float4* d = reinterpret_cast<float4*>(dst + r * kRbPitch + kk);
      d[0] = make_float4(__uint_as_float(v[0] << 16), __uint_as_float(v[0] & 0xffff0000u),
                         __uint_as_float(v[1] << 16), __uint_as_float(v[1] & 0xffff0000u));
      d[1] = make_float4(__uint_as_float(v[2] << 16), __uint_as_float(v[2] & 0xffff0000u),
                         __uint_as_float(v[3] << 16), __uint_as_float(v[3] & 0xffff0000u));
    }
  };
  for (uint32_t p = 0; p + 1 < kRbRing; ++p) fill(p);
  const uint32_t warp = tid >> 5, lane = tid & 31;
  const uint32_t tp = lane & 7, ep = lane >> 3;
  const uint32_t xrow = (warp & 1) * 16 + tp;             // and xrow + 8
  const uint32_t wrow = kRbTile + (warp >> 1) * 8 + ep;   // and wrow + 4
  float acc[2][2] = {};
  for (uint32_t p = 0; p < phases; ++p) {
    cp_async_wait<kRbRing - 2>();  // phase p has landed (this thread's copies)
    __syncthreads();               // ... everyone's; phase p - 1's raw buffer is widened
    fill(p + kRbRing - 1);         // into the raw buffer of phase p - 1
    widen(p);
    __syncthreads();
    const float* buf = fbuf + (p & 1) * kRbBufFloats;
    const float* xr = buf + xrow * kRbPitch;
    const float* wr = buf + wrow * kRbPitch;
    const uint32_t kn = min(kRbPhaseK, chunk - p * kRbPhaseK);
    // operands of step k + 4 are loaded before the fmas of step k (the fmas
    // otherwise wait on the shared-memory loads they follow)
    auto ld = [](const float* q) { return *reinterpret_cast<const float4*>(q); };
    float4 xa = ld(xr), xb = ld(xr + 8 * kRbPitch), wa = ld(wr), wb = ld(wr + 4 * kRbPitch);
#pragma unroll 4
    for (uint32_t k = 0; k < kn; k += 4) {
      const uint32_t kk = k + 4 < kn ? k + 4 : k;
      const float4 nxa = ld(xr + kk), nxb = ld(xr + 8 * kRbPitch + kk);
      const float4 nwa = ld(wr + kk), nwb = ld(wr + 4 * kRbPitch + kk);
      const float xv[2][4] = {{xa.x, xa.y, xa.z, xa.w}, {xb.x, xb.y, xb.z, xb.w}};
      const float wv[2][4] = {{wa.x, wa.y, wa.z, wa.w}, {wb.x, wb.y, wb.z, wb.w}};
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 2; ++j) acc[i][j] = fmaf(xv[i][q], wv[j][q], acc[i][j]);
      xa = nxa;
      xb = nxb;
      wa = nwa;
      wb = nwb;
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t t = t0 + xrow + 8 * i;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t e = e0 + (wrow - kRbTile) + 4 * j;
      if (t < T && e < E) partial[(uint64_t(c) * T + t) * E + e] = acc[i][j];
    }
  }
}

// ---------------------------------------------------------------------------
// Router logits for large T (same canonical order as above).  CTA tile: 128
// tokens x 128 experts x one K chunk (blockIdx.z); 256 threads, each owning 8
// tokens x 8 experts (experts tx*4.. and 64+tx*4..).  K advances in 32-wide
// slabs staged in shared memory as fp32 (tokens as duplicated pairs, so that
// one fma.rn.f32x2 applies one x to two experts), double-buffered with the
// next slab's global loads in flight.  fma.rn.f32x2 is two independent
// correctly rounded fmas, so every output is still one ascending fma chain.
constexpr uint32_t kRtSlab = 32;
constexpr uint32_t kRtXPitch = 128 * 2 + 8;  // floats per k row of token pairs
constexpr uint32_t kRtWPitch = 128 + 4;      // floats per k row of experts
constexpr uint32_t kRtBufFloats = kRtSlab * (kRtXPitch + kRtWPitch);
constexpr uint32_t kRouterTiledMinTokens = 256;

__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__global__ void __launch_bounds__(256, 2) router_logits_tiled_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, float* __restrict__ partial,
    uint32_t T, uint32_t H, uint32_t E, uint32_t* __restrict__ bitmap, uint32_t bitmap_words) {
  extern __shared__ __align__(16) float rtsm[];
  const uint32_t tid = threadIdx.x;
  const uint32_t e0 = blockIdx.x * 128, t0 = blockIdx.y * 128, c = blockIdx.z;
  const uint32_t chunk = H / 8;
  {
    const uint64_t lin = (uint64_t(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    const uint64_t nthreads = uint64_t(gridDim.x) * gridDim.y * gridDim.z * blockDim.x;
    for (uint64_t i = lin * blockDim.x + tid; i < bitmap_words; i += nthreads) bitmap[i] = 0;
  }
  // staging: per slab and operand 128 rows x 64 bytes = 512 pieces of 16 bytes, 2 per thread
  uint4 rx[2], rw[2];
  auto gload = [&](uint32_t k0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t p = tid + 256u * i, row = p >> 2, part = p & 3;
      const uint64_t col = uint64_t(c) * chunk + k0 + part * 8;
      rx[i] = t0 + row < T ? *reinterpret_cast<const uint4*>(x + uint64_t(t0 + row) * H + col)
                           : make_uint4(0, 0, 0, 0);
      rw[i] = e0 + row < E ? *reinterpret_cast<const uint4*>(w + uint64_t(e0 + row) * H + col)
                           : make_uint4(0, 0, 0, 0);
    }
  };
  auto sstore = [&](float* buf) {
    float* xs2 = buf;
    float* ws = buf + kRtSlab * kRtXPitch;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t p = tid + 256u * i, row = p >> 2, part = p & 3;
      const uint32_t xv[4] = {rx[i].x, rx[i].y, rx[i].z, rx[i].w};
      const uint32_t wv[4] = {rw[i].x, rw[i].y, rw[i].z, rw[i].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t k = part * 8 + 2 * q;
        const float xl = __uint_as_float(xv[q] << 16), xh = __uint_as_float(xv[q] & 0xffff0000u);
        *reinterpret_cast<float2*>(xs2 + k * kRtXPitch + 2 * row) = make_float2(xl, xl);
        *reinterpret_cast<float2*>(xs2 + (k + 1) * kRtXPitch + 2 * row) = make_float2(xh, xh);
        ws[k * kRtWPitch + row] = __uint_as_float(wv[q] << 16);
        ws[(k + 1) * kRtWPitch + row] = __uint_as_float(wv[q] & 0xffff0000u);
      }
    }
  };
  const uint32_t tx = tid & 15, ty = tid >> 4;
  uint64_t acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0;
  const uint32_t nslab = chunk / kRtSlab;
  gload(0);
  sstore(rtsm);
  __syncthreads();
  for (uint32_t s = 0; s < nslab; ++s) {
    const float* cur = rtsm + (s & 1) * kRtBufFloats;
    if (s + 1 < nslab) gload((s + 1) * kRtSlab);
    const float* xs2 = cur;
    const float* ws = cur + kRtSlab * kRtXPitch;
#pragma unroll 4
    for (uint32_t k = 0; k < kRtSlab; ++k) {
      const ulonglong2* xp = reinterpret_cast<const ulonglong2*>(xs2 + k * kRtXPitch + ty * 16);
      const ulonglong2 x01 = xp[0], x23 = xp[1], x45 = xp[2], x67 = xp[3];
      const uint64_t xi[8] = {x01.x, x01.y, x23.x, x23.y, x45.x, x45.y, x67.x, x67.y};
      const ulonglong2 wa = *reinterpret_cast<const ulonglong2*>(ws + k * kRtWPitch + tx * 4);
      const ulonglong2 wb = *reinterpret_cast<const ulonglong2*>(ws + k * kRtWPitch + 64 + tx * 4);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[i][0] = ffma2(xi[i], wa.x, acc[i][0]);
        acc[i][1] = ffma2(xi[i], wa.y, acc[i][1]);
        acc[i][2] = ffma2(xi[i], wb.x, acc[i][2]);
        acc[i][3] = ffma2(xi[i], wb.y, acc[i][3]);
      }
    }
    if (s + 1 < nslab) sstore(rtsm + ((s + 1) & 1) * kRtBufFloats);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t t = t0 + ty * 8 + i;
    if (t >= T) continue;
    float* row = partial + (uint64_t(c) * T + t) * E + e0;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const uint64_t p0 = acc[i][2 * g], p1 = acc[i][2 * g + 1];
      *reinterpret_cast<float4*>(row + 64 * g + tx * 4) =
          make_float4(__uint_as_float(uint32_t(p0)), __uint_as_float(uint32_t(p0 >> 32)),
                      __uint_as_float(uint32_t(p1)), __uint_as_float(uint32_t(p1 >> 32)));
    }
  }
}

// ---------------------------------------------------------------------------
// Router selection, one warp per token (lane owns experts lane + 32j):
//   s = sigmoid(logit), choice = s + bias; group score = top1 + top2 of choice;
//   keep the best `topk_groups` groups; pick `top_k` experts by choice among
//   them (slot order = descending choice, ties -> lower index);
//   weight = (s / sum_slots s) * route_scale, the sum taken in slot order.
// ---------------------------------------------------------------------------
// Order-preserving 32-bit key of a non-NaN float (larger float -> larger key).
__device__ __forceinline__ uint32_t fkey(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Same selection with lane l owning the 8 consecutive experts 8l .. 8l+7, for
// shapes whose groups are whole runs of lanes (E % 8 == 0, gs = E / groups a
// multiple of 8 with gs / 8 a power of two): a group's top-2 merges over its
// lanes in log2(gs/8) shuffles, every lane ranks its group against the others by
// one shuffle per group, and each top-k round is a lane-local argmax plus two
// warp reductions.  Tie rules are the reference's: the lower group index and the
// lower expert index win, so the result is the same bits as the general kernel.
__global__ void __launch_bounds__(256) router_select_runs_kernel(
    const float* __restrict__ partial, const float* __restrict__ bias, uint32_t T, uint32_t E,
    uint32_t groups, uint32_t topk_groups, uint32_t top_k, float route_scale,
    uint16_t* __restrict__ experts_out, float* __restrict__ weights_out,
    uint32_t* __restrict__ bitmap, uint32_t bitmap_stride, uint32_t* __restrict__ status) {
  constexpr uint32_t kFull = 0xffffffffu;
  constexpr uint32_t kNone = 0u;  // below every finite choice
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t >= T) return;
  const uint32_t e0 = lane * 8;
  const bool mine = e0 < E;  // E % 8 == 0: a lane's experts are all valid or all absent
  // logits: the 8 chunk partials in chunk order, every load in flight first
  float4 p[8][2];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float4* src = reinterpret_cast<const float4*>(partial + (uint64_t(c) * T + t) * E + e0);
    p[c][0] = mine ? src[0] : make_float4(0.f, 0.f, 0.f, 0.f);
    p[c][1] = mine ? src[1] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float bj[8];  // scalar loads: the bias is only required to be 4-byte aligned
#pragma unroll
  for (int j = 0; j < 8; ++j) bj[j] = mine ? bias[e0 + j] : 0.f;
  float L[8] = {p[0][0].x, p[0][0].y, p[0][0].z, p[0][0].w,
                p[0][1].x, p[0][1].y, p[0][1].z, p[0][1].w};
#pragma unroll
  for (int c = 1; c < 8; ++c) {
    const float q[8] = {p[c][0].x, p[c][0].y, p[c][0].z, p[c][0].w,
                        p[c][1].x, p[c][1].y, p[c][1].z, p[c][1].w};
#pragma unroll
    for (int j = 0; j < 8; ++j) L[j] = __fadd_rn(L[j], q[j]);
  }
  float sc[8];
  uint32_t key[8];
  bool bad = false;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sc[j] = 0.f;
    key[j] = kNone;
    if (mine) {
      if (!isfinite(L[j])) bad = true;
      sc[j] = router_sigmoid(L[j]);
      key[j] = fkey(__fadd_rn(sc[j], bj[j]));
    }
  }
  // group score = top1 + top2 of the group's choices (multiset top-2)
  const uint32_t gs = E / groups, lpg = gs / 8;  // lanes per group
  uint32_t k1 = kNone, k2 = kNone;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (key[j] > k1) {
      k2 = k1;
      k1 = key[j];
    } else if (key[j] > k2) {
      k2 = key[j];
    }
  }
  for (uint32_t off = 1; off < lpg; off <<= 1) {
    const uint32_t o1 = __shfl_xor_sync(kFull, k1, off), o2 = __shfl_xor_sync(kFull, k2, off);
    const uint32_t n1 = max(k1, o1), n2 = max(min(k1, o1), max(k2, o2));
    k1 = n1;
    k2 = n2;
  }
  const float gscore = __fadd_rn(fkey_inv(k1), fkey_inv(k2));  // gs >= 8
  // keep the best topk_groups groups (ties -> lower group index)
  const uint32_t g = lane / lpg;
  uint32_t beaten = 0;
  for (uint32_t h = 0; h < groups; ++h) {
    const float other = __shfl_sync(kFull, gscore, h * lpg);
    if (other > gscore || (other == gscore && h < g)) ++beaten;
  }
  const bool kept = mine && beaten < topk_groups;
  // top_k experts by choice among the kept groups (ties -> lower expert index)
  uint32_t taken = 0;
  uint32_t my_e = 0;
  float my_s = 0.f, denom = 0.f;
  for (uint32_t k = 0; k < top_k; ++k) {
    uint32_t bk = kNone, bj_ = 8;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (kept && !((taken >> j) & 1u) && (bj_ == 8 || key[j] > bk)) {
        bk = key[j];
        bj_ = j;
      }
    const uint32_t mk = __reduce_max_sync(kFull, bk);
    const uint32_t wl = __reduce_min_sync(kFull, (bj_ != 8 && bk == mk) ? lane : 32u);
    if (wl == 32u) {
      bad = true;
      continue;
    }
    float s_win = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (uint32_t(j) == bj_) s_win = sc[j];
    const float ws_ = __shfl_sync(kFull, s_win, wl);
    const uint32_t we = wl * 8 + __shfl_sync(kFull, bj_, wl);
    if (lane == wl) taken |= 1u << bj_;
    denom = k == 0 ? ws_ : __fadd_rn(denom, ws_);
    if (lane == k) {
      my_e = we;
      my_s = ws_;
    }
  }
  if (lane < top_k) {
    const float wgt = __fmul_rn(__fdiv_rn(my_s, denom), route_scale);
    experts_out[uint64_t(t) * top_k + lane] = static_cast<uint16_t>(my_e);
    weights_out[uint64_t(t) * top_k + lane] = wgt;
    atomicOr(&bitmap[uint64_t(my_e) * bitmap_stride + t / 32], 1u << (t % 32));
  }
  bad = __any_sync(kFull, bad);
  if (bad && lane == 0 && status) atomicOr(status, kStatusNonFiniteInput);
}

__global__ void __launch_bounds__(256) router_select_kernel(
    const float* __restrict__ partial, const float* __restrict__ bias, uint32_t T, uint32_t E,
    uint32_t groups, uint32_t topk_groups, uint32_t top_k, float route_scale,
    uint16_t* __restrict__ experts_out, float* __restrict__ weights_out,
    uint32_t* __restrict__ bitmap, uint32_t bitmap_stride, uint32_t* __restrict__ status) {
  constexpr uint32_t kFull = 0xffffffffu;
  constexpr uint32_t kNone = 0u;  // key below every finite choice (fkey(-inf) > 0)
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t >= T) return;
  const uint32_t nj = (E + 31) / 32;
  const uint32_t gs = E / groups;
  float s[8];
  uint32_t key[8], gid[8];
  bool bad = false;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t e = lane + 32 * j;
    float L = 0.f;
    const bool valid = j < nj && e < E;
    if (valid) {
      L = partial[uint64_t(t) * E + e];
#pragma unroll
      for (int c = 1; c < 8; ++c) L = __fadd_rn(L, partial[(uint64_t(c) * T + t) * E + e]);
    }
    s[j] = 0.f;
    key[j] = kNone;
    gid[j] = 0xffffffffu;
    if (valid) {
      if (!isfinite(L)) bad = true;
      s[j] = router_sigmoid(L);
      key[j] = fkey(__fadd_rn(s[j], bias[e]));
      gid[j] = e / gs;
    }
  }
  // group score = top1 + top2 of the group's choices
  float gscore[32];
  for (uint32_t g = 0; g < groups; ++g) {
    uint32_t l1 = kNone, l2 = kNone;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (gid[j] == g) {
        if (key[j] > l1) {
          l2 = l1;
          l1 = key[j];
        } else if (key[j] > l2) {
          l2 = key[j];
        }
      }
    }
    const uint32_t m1 = __reduce_max_sync(kFull, l1);
    const uint32_t owner = __reduce_min_sync(kFull, l1 == m1 ? lane : 32u);
    const uint32_t m2 = __reduce_max_sync(kFull, lane == owner ? l2 : l1);
    gscore[g] = gs >= 2 ? __fadd_rn(fkey_inv(m1), fkey_inv(m2)) : fkey_inv(m1);
  }
  // keep the best topk_groups groups (ties -> lower group index)
  uint32_t gmask = 0;
  for (uint32_t r = 0; r < topk_groups; ++r) {
    int best = -1;
    for (uint32_t g = 0; g < groups; ++g)
      if (!((gmask >> g) & 1u) && (best < 0 || gscore[g] > gscore[best])) best = static_cast<int>(g);
    gmask |= 1u << best;
  }
  // top_k experts by choice among the kept groups (ties -> lower expert index)
  uint32_t taken = 0;
  uint32_t my_e = 0;
  float my_s = 0.f, denom = 0.f;
  for (uint32_t k = 0; k < top_k; ++k) {
    uint32_t bk = kNone, be = 0xffffu;
    float bs = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (gid[j] != 0xffffffffu && ((gmask >> gid[j]) & 1u) && !((taken >> j) & 1u) &&
          (be == 0xffffu || key[j] > bk)) {
        bk = key[j];
        be = lane + 32 * j;
        bs = s[j];
      }
    }
    const uint32_t mk = __reduce_max_sync(kFull, bk);
    const uint32_t we = __reduce_min_sync(kFull, (be != 0xffffu && bk == mk) ? be : 0xffffu);
    if (we == 0xffffu) {
      bad = true;
      continue;
    }
    const float ws_ = __shfl_sync(kFull, bs, we & 31u);
    if ((we & 31u) == lane) taken |= 1u << (we >> 5);
    denom = k == 0 ? ws_ : __fadd_rn(denom, ws_);
    if (lane == k) {
      my_e = we;
      my_s = ws_;
    }
  }
  if (lane < top_k) {
    const float wgt = __fmul_rn(__fdiv_rn(my_s, denom), route_scale);
    experts_out[uint64_t(t) * top_k + lane] = static_cast<uint16_t>(my_e);
    weights_out[uint64_t(t) * top_k + lane] = wgt;
    atomicOr(&bitmap[uint64_t(my_e) * bitmap_stride + t / 32], 1u << (t % 32));
  }
  if (bad && lane == 0 && status) atomicOr(status, kStatusNonFiniteInput);
}

// Routes supplied by the caller (dense [T][K]): validate and set bitmap bits.
__global__ void routes_to_bitmap_kernel(const uint16_t* __restrict__ experts,
                                        const float* __restrict__ weights, uint32_t T,
                                        uint32_t E, uint32_t top_k, uint32_t* __restrict__ bitmap,
                                        uint32_t bitmap_stride, uint32_t* __restrict__ status) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * top_k) return;
  const uint32_t t = i / top_k;
  const uint32_t e = experts[i];
  const float w = weights[i];
  uint32_t err = 0;
  if (e >= E) err |= kStatusExpertOutOfRange;
  if (!isfinite(w) || w < 0.f) err |= kStatusRouteWeightNotFinite;
  if (err) {
    atomicOr(status, err);
    return;
  }
  const uint32_t prev = atomicOr(&bitmap[uint64_t(e) * bitmap_stride + t / 32], 1u << (t % 32));
  if (prev & (1u << (t % 32))) atomicOr(status, kStatusDuplicateTokenSlot);
}

__global__ void zero_words_kernel(uint32_t* p, uint64_t n) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n;
       i += uint64_t(gridDim.x) * blockDim.x)
    p[i] = 0;
}

// ---------------------------------------------------------------------------
// Compaction (single CTA, 1024 threads): per-expert counts and word prefixes
// from the bitmap, exclusive offsets (plain and 128-padded), n-tile list.
// ---------------------------------------------------------------------------
// Large T: the per-expert word prefixes and counts, one CTA per expert (the
// experts' scans are independent; a single CTA walking 256 experts x W words
// was a latency chain of ~200 us at T = 8192).  Thread j scans a run of
// consecutive words; the run totals are scanned across the CTA.
constexpr uint32_t kPrefixThreads = 256;
__global__ void __launch_bounds__(kPrefixThreads) compact_prefix_kernel(
    const uint32_t* __restrict__ bitmap, uint32_t W, uint32_t* __restrict__ wprefix,
    uint32_t* __restrict__ counts) {
  __shared__ uint32_t warp_tot[kPrefixThreads / 32];
  const uint32_t e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t per = (W + kPrefixThreads - 1) / kPrefixThreads;  // words per thread (<= 8)
  const uint32_t w0 = tid * per;
  const uint32_t* row = bitmap + uint64_t(e) * W;
  uint32_t pc[8];
  uint32_t tot = 0;
#pragma unroll
  for (uint32_t i = 0; i < 8; ++i) {
    pc[i] = (i < per && w0 + i < W) ? __popc(row[w0 + i]) : 0u;
    tot += pc[i];
  }
  uint32_t incl = tot;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= uint32_t(off)) incl += o;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  uint32_t base = 0;
  for (uint32_t w = 0; w < warp; ++w) base += warp_tot[w];
  uint32_t run = base + incl - tot;  // exclusive prefix of this thread's first word
#pragma unroll
  for (uint32_t i = 0; i < 8; ++i) {
    if (i < per && w0 + i < W) wprefix[uint64_t(e) * W + w0 + i] = run;
    run += pc[i];
  }
  if (tid == kPrefixThreads - 1) {
    uint32_t total = 0;
    for (uint32_t w = 0; w < kPrefixThreads / 32; ++w) total += warp_tot[w];
    counts[e] = total;
  }
}

__global__ void __launch_bounds__(1024) compact_kernel(
    const uint32_t* __restrict__ bitmap, uint32_t W, uint32_t E, uint32_t nt, uint32_t sf_row_cap,
    uint32_t max_tiles, uint32_t* __restrict__ wprefix, uint32_t* __restrict__ counts,
    uint32_t* __restrict__ offsets, uint32_t* __restrict__ poffs, NTile* __restrict__ tiles,
    uint32_t* __restrict__ tile_count, uint32_t* __restrict__ status,
    const uint8_t* __restrict__ no_tiles, bool counts_ready) {
  // no_tiles[e] != 0 (optional): expert e gets rows but no GEMM tiles (an EXL3 expert).
  // counts_ready: compact_prefix_kernel already wrote wprefix and counts.
  __shared__ uint32_t cnt_s[256], toff_s[257], poff_s[257], off_s[257];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (counts_ready) {
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) cnt_s[e] = counts[e];
  } else if (W <= 32 && E <= 256) {
    // T <= 1024: one bitmap word per lane; the warp's 8 experts (warp + 32q) load
    // together and their scans interleave
    uint32_t pc[8], incl[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t e = warp + 32u * q;
      pc[q] = (e < E && lane < W) ? __popc(bitmap[uint64_t(e) * W + lane]) : 0u;
      incl[q] = pc[q];
    }
#pragma unroll
    for (int off = 1; off < 32; off <<= 1)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl[q], off);
        if (lane >= uint32_t(off)) incl[q] += o;
      }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t e = warp + 32u * q;
      if (e < E) {
        if (lane < W) wprefix[uint64_t(e) * W + lane] = incl[q] - pc[q];
        if (lane == 31) cnt_s[e] = incl[q];
      }
    }
  }
  for (uint32_t e = warp; !counts_ready && (W > 32 || E > 256) && e < E; e += 32) {
    uint32_t running = 0;
    for (uint32_t w0 = 0; w0 < W; w0 += 32) {
      const uint32_t w = w0 + lane;
      const uint32_t pc = w < W ? __popc(bitmap[uint64_t(e) * W + w]) : 0;
      uint32_t incl = pc;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      if (w < W) wprefix[uint64_t(e) * W + w] = running + incl - pc;
      running += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) cnt_s[e] = running;
  }
  __syncthreads();
  if (warp == 0) {
    // each lane scans 8 consecutive experts; lane totals scanned across the warp
    const uint32_t per = (E + 31) / 32;
    uint32_t sc = 0, sp = 0, st = 0;
    for (uint32_t q = 0; q < per; ++q) {
      const uint32_t e = lane * per + q;
      if (e < E) {
        sc += cnt_s[e];
        sp += (cnt_s[e] + nt - 1) / nt * 128;
        st += (no_tiles && no_tiles[e]) ? 0 : (cnt_s[e] + nt - 1) / nt;
      }
    }
    uint32_t ic = sc, ip = sp, it = st;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t a = __shfl_up_sync(0xffffffffu, ic, off);
      const uint32_t b = __shfl_up_sync(0xffffffffu, ip, off);
      const uint32_t c = __shfl_up_sync(0xffffffffu, it, off);
      if (lane >= off) {
        ic += a;
        ip += b;
        it += c;
      }
    }
    uint32_t oc = ic - sc, op = ip - sp, ot = it - st;
    for (uint32_t q = 0; q < per; ++q) {
      const uint32_t e = lane * per + q;
      if (e < E) {
        offsets[e] = oc;
        off_s[e] = oc;
        poffs[e] = op;
        poff_s[e] = op;
        toff_s[e] = ot;
        counts[e] = cnt_s[e];
        oc += cnt_s[e];
        op += (cnt_s[e] + nt - 1) / nt * 128;
        ot += (no_tiles && no_tiles[e]) ? 0 : (cnt_s[e] + nt - 1) / nt;
      }
    }
    if (lane == 31) {
      offsets[E] = ic;
      off_s[E] = ic;
      poffs[E] = ip;
      poff_s[E] = ip;
      toff_s[E] = it;
      const bool over = ip > sf_row_cap || it > max_tiles;
      *tile_count = over ? 0u : it;
      if (over && status) atomicOr(status, kStatusCapacityExceeded);
    }
  }
  __syncthreads();
  if (tiles == nullptr || poff_s[E] > sf_row_cap || toff_s[E] > max_tiles) return;
  for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) {
    const uint32_t c = (no_tiles && no_tiles[e]) ? 0 : cnt_s[e];
    for (uint32_t j = 0; j * nt < c; ++j) {
      NTile tl;
      tl.expert = e;
      tl.row_start = off_s[e] + j * nt;
      tl.sf_row_start = poff_s[e] + j * 128;
      tl.rows = min(nt, c - j * nt);
      tiles[toff_s[e] + j] = tl;
    }
  }
}

// ---------------------------------------------------------------------------
// FC1 input: NVFP4-quantise x[t] once (per-row global scale = amax/2688,
// per-16 E4M3 scales, nvfp4.rs:170-273 arithmetic) and write it to each of the
// token's K assignment rows.  One CTA per token, thread = one 64-wide k-block.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float r = lane < (blockDim.x + 31) / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, off));
    if (lane == 0) red[32] = r;
  }
  __syncthreads();
  return red[32];
}

// One CTA per token, one thread per 16-element NVFP4 block (H/16 threads): the
// token's global scale from the block-wide amax, each block encoded by its own
// thread, the four scale bytes of a 64-element k-block gathered by shuffles, and
// the encoded row stored into every slot's compacted row.
__global__ void __launch_bounds__(1024) quant_scatter_kernel(QuantScatterArgs a) {
  __shared__ float red[33];
  __shared__ uint32_t s_row[32], s_prow[32];
  const uint32_t t = blockIdx.x, b16 = threadIdx.x;
  const uint32_t KB = a.H / 64, B16 = a.H / 16;
  const bool active = b16 < B16;
  // the compacted row and scale row of each slot: one thread per slot, its two
  // dependent loads overlapping the row loads below
  if (b16 < a.top_k) {
    const uint32_t slot = b16, i = t * a.top_k + slot;
    const uint32_t e = a.route_experts[i];
    uint32_t row = 0xffffffffu, prow = 0xffffffffu;
    if (e < a.E) {
      const uint32_t W = (a.T + 31) / 32;
      const uint32_t word = a.bitmap[uint64_t(e) * W + t / 32];
      const uint32_t rank =
          a.wprefix[uint64_t(e) * W + t / 32] + __popc(word & ((1u << (t % 32)) - 1u));
      // scale-factor row: every n tile of a.nt rows owns a whole 128-row atom
      prow = a.poffs[e] + (rank / a.nt) * 128 + rank % a.nt;
      row = a.offsets[e] + rank;  // compacted row
      if (prow >= a.sf_row_cap || row >= a.T * a.top_k) row = prow = 0xffffffffu;
    }
    s_row[slot] = row;
    s_prow[slot] = prow;
    if (row != 0xffffffffu) {
      a.row_token[row] = t;
      a.row_slot[row] = slot;
      a.row_weight[row] = a.route_weights[i];
      a.row_prow[row] = prow;
      a.route_row[i] = row;
    }
  }
  float v[16];
  float amax = 0.f;
  bool finite = true;
  if (active) {
    const uint4* src = reinterpret_cast<const uint4*>(a.x + uint64_t(t) * a.H + b16 * 16);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 u = src[q];
      const uint32_t wds[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[q * 8 + h * 2] = __uint_as_float(wds[h] << 16);
        v[q * 8 + h * 2 + 1] = __uint_as_float(wds[h] & 0xffff0000u);
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      finite = finite && isfinite(v[i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
  }
  if (!finite) atomicOr(a.status, kStatusNonFiniteInput);
  amax = block_max(amax, red);  // its barriers also publish s_row / s_prow
  const float gscale = global_scale_of(amax);
  uint2 packed = make_uint2(0, 0);
  uint32_t sc = 0;
  if (active) sc = nvfp4_block(v, gscale, &packed);
  // the 4 scale bytes of k-block b16 / 4 (B16 % 4 == 0, so the 4 threads share a warp)
  const uint32_t lane = threadIdx.x & 31, q0 = lane & ~3u;
  const uint32_t sfw = __shfl_sync(0xffffffffu, sc, q0) | (__shfl_sync(0xffffffffu, sc, q0 + 1) << 8) |
                       (__shfl_sync(0xffffffffu, sc, q0 + 2) << 16) |
                       (__shfl_sync(0xffffffffu, sc, q0 + 3) << 24);
  if (!active) return;
  for (uint32_t slot = 0; slot < a.top_k; ++slot) {
    const uint32_t row = s_row[slot], prow = s_prow[slot];
    if (row == 0xffffffffu) continue;
    reinterpret_cast<uint2*>(a.xq + uint64_t(row) * (a.H / 2))[b16] = packed;
    if ((b16 & 3) == 0)
      *reinterpret_cast<uint32_t*>(a.xsf + sf_offset(prow, b16 / 4, 0, KB)) = sfw;
    if (b16 == 0) a.row_gscale[row] = gscale;
  }
}

// ---------------------------------------------------------------------------
// FC2 input: NVFP4-quantise each assignment's h row (K = I).  One thread per
// 16-element block: a row's R = I/16 threads are consecutive (R = 16..128,
// 128-thread blocks); its amax is a butterfly over min(R, 32) lanes, then over
// the row's warps through shared memory when R > 32.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fc2_quant_kernel(Fc2QuantArgs a) {
  __shared__ float wmax[8];
  const uint32_t R = a.I / 16;
  const uint32_t rows_per_block = blockDim.x / R;
  const uint32_t r_local = threadIdx.x / R, b16 = threadIdx.x % R;
  const uint32_t row = blockIdx.x * rows_per_block + r_local;
  // rows below a.count (the plane's capacity) are readable whatever the live
  // count, so the h loads, the scale row and the count are all in flight at once
  const bool in_plane = row < a.count;
  const uint32_t count = a.count_ptr ? min(*a.count_ptr, a.count) : a.count;
  const uint32_t prow = in_plane ? a.row_prow[row] : 0xffffffffu;
  bool active = row < count;
  if (active && a.skip_codec != nullptr) {
    uint32_t lo = 0, hi = a.E;  // expert of the row: offsets[lo] <= row < offsets[hi]
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) / 2;
      if (a.offsets[mid] <= row) lo = mid; else hi = mid;
    }
    active = a.skip_codec[lo] != 1;
  }
  float v[16];
  float amax = 0.f;
  bool finite = true;
  if (in_plane) {
    const uint4* src = reinterpret_cast<const uint4*>(a.h + uint64_t(row) * a.I + b16 * 16);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 u = src[q];
      const uint32_t wds[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[q * 8 + h * 2] = __uint_as_float(wds[h] << 16);
        v[q * 8 + h * 2 + 1] = __uint_as_float(wds[h] & 0xffff0000u);
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      finite = finite && isfinite(v[i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
  }
  const uint32_t span = R < 32 ? R : 32;
  for (uint32_t off = 1; off < span; off <<= 1)
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if (R > 32) {  // a row spans R/32 warps: combine them
    const uint32_t warp = threadIdx.x >> 5, first = r_local * (R / 32);
    if ((threadIdx.x & 31) == 0) wmax[warp] = amax;
    __syncthreads();
    amax = wmax[first];
    for (uint32_t w = 1; w < R / 32; ++w) amax = fmaxf(amax, wmax[first + w]);
  }
  const float gscale = global_scale_of(amax);
  uint2 packed = make_uint2(0, 0);
  uint32_t sc = 0;
  if (active) sc = nvfp4_block(v, gscale, &packed);
  const uint32_t lane = threadIdx.x & 31, q0 = lane & ~3u;
  const uint32_t sfw = __shfl_sync(0xffffffffu, sc, q0) | (__shfl_sync(0xffffffffu, sc, q0 + 1) << 8) |
                       (__shfl_sync(0xffffffffu, sc, q0 + 2) << 16) |
                       (__shfl_sync(0xffffffffu, sc, q0 + 3) << 24);
  if (!active) return;
  if (!finite && a.status) atomicOr(a.status, kStatusNonFiniteInput);
  if (prow >= a.sf_row_cap) return;
  reinterpret_cast<uint2*>(a.hq + uint64_t(row) * (a.I / 2))[b16] = packed;
  if ((b16 & 3) == 0)
    *reinterpret_cast<uint32_t*>(a.hsf + sf_offset(prow, b16 / 4, 0, a.I / 64)) = sfw;
  if (b16 == 0) a.gscale[row] = gscale;
}

// Compacted-order route arrays (reference ABI) from the device compaction.
__global__ void compact_write_kernel(CompactWriteArgs a) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.T * a.top_k) return;
  const uint32_t t = i / a.top_k, slot = i % a.top_k;
  const uint32_t e = a.route_experts[i];
  if (e >= a.E) return;
  const uint32_t W = (a.T + 31) / 32;
  const uint32_t word = a.bitmap[uint64_t(e) * W + t / 32];
  const uint32_t rank = a.wprefix[uint64_t(e) * W + t / 32] + __popc(word & ((1u << (t % 32)) - 1u));
  const uint32_t c = a.offsets[e] + rank;
  a.comp_token[c] = t;
  a.comp_expert[c] = static_cast<uint16_t>(e);
  a.comp_slot[c] = static_cast<uint8_t>(slot);
  a.comp_weight[c] = a.route_weights[i];
}

// Reference-ABI compacted routes -> padded offsets, per-row padded row, tiles.
// Single CTA; expert_offsets must be non-decreasing with offsets[E] == A.
__global__ void __launch_bounds__(1024) compat_prepare_kernel(CompatPrepareArgs a) {
  __shared__ uint32_t poff_s[257], toff_s[257];
  if (threadIdx.x < 32) {
    const uint32_t lane = threadIdx.x;
    const uint32_t per = (a.E + 31) / 32;
    uint32_t sp = 0, st = 0;
    bool bad = false;
    for (uint32_t q = 0; q < per; ++q) {
      const uint32_t e = lane * per + q;
      if (e < a.E) {
        const uint32_t b0 = a.offsets[e], b1 = a.offsets[e + 1];
        if (b1 < b0 || b1 > a.A) bad = true;
        const uint32_t c = b1 >= b0 ? b1 - b0 : 0;
        sp += (c + a.nt - 1) / a.nt * 128;
        st += (c + a.nt - 1) / a.nt;
      }
    }
    uint32_t ip = sp, it = st;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t b = __shfl_up_sync(0xffffffffu, ip, off);
      const uint32_t c = __shfl_up_sync(0xffffffffu, it, off);
      if (lane >= off) {
        ip += b;
        it += c;
      }
    }
    uint32_t op = ip - sp, ot = it - st;
    for (uint32_t q = 0; q < per; ++q) {
      const uint32_t e = lane * per + q;
      if (e < a.E) {
        const uint32_t b0 = a.offsets[e], b1 = a.offsets[e + 1];
        const uint32_t c = b1 >= b0 ? b1 - b0 : 0;
        a.poffs[e] = op;
        poff_s[e] = op;
        toff_s[e] = ot;
        op += (c + a.nt - 1) / a.nt * 128;
        ot += (c + a.nt - 1) / a.nt;
      }
    }
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 31) {
      a.poffs[a.E] = ip;
      poff_s[a.E] = ip;
      toff_s[a.E] = it;
      const bool over = bad || ip > a.sf_row_cap || it > a.max_tiles || a.offsets[0] != 0 ||
                        a.offsets[a.E] != a.A;
      *a.tile_count = over ? 0u : it;
      if (over && a.status) atomicOr(a.status, kStatusCapacityExceeded);
    }
  }
  __syncthreads();
  if (*a.tile_count == 0) return;
  for (uint32_t e = threadIdx.x; e < a.E; e += blockDim.x) {
    const uint32_t b0 = a.offsets[e], c = a.offsets[e + 1] - b0;
    const bool on = (a.expert_mask[e / 32] >> (e % 32)) & 1u;
    for (uint32_t j = 0; j * a.nt < c; ++j) {
      NTile tl;
      tl.expert = e;
      tl.row_start = b0 + j * a.nt;
      tl.sf_row_start = poff_s[e] + j * 128;
      tl.rows = on ? min(a.nt, c - j * a.nt) : 0;
      a.tiles[toff_s[e] + j] = tl;
    }
  }
  for (uint32_t r = threadIdx.x; r < a.A; r += blockDim.x) {
    const uint32_t e = a.route_experts[r];
    if (e < a.E && r >= a.offsets[e] && r < a.offsets[e + 1]) {
      const uint32_t rank = r - a.offsets[e];
      a.row_prow[r] = poff_s[e] + (rank / a.nt) * 128 + rank % a.nt;
    }
    else {
      a.row_prow[r] = 0xffffffffu;
      if (a.status) atomicOr(a.status, kStatusExpertOutOfRange);
    }
  }
}

// Reference-ABI quantiser, one CTA per compacted row, one thread per 64-wide
// k-block (nvfp4_routed_fc1.cu:76-147 semantics, expert-local scale layout).
__global__ void __launch_bounds__(256) quant_rows_kernel(QuantRowsArgs a) {
  __shared__ float red[33];
  const uint32_t r = blockIdx.x, kb = threadIdx.x;
  const uint32_t KB = a.K / 64;
  const bool active = kb < KB;
  const uint32_t sr = a.src_row ? a.src_row[r] : r;
  const bool in_range = sr < a.src_rows;
  float v[64];
  float amax = 0.f;
  bool finite = true;
  if (active && in_range) {
    const uint4* src = reinterpret_cast<const uint4*>(a.src + uint64_t(sr) * a.K + kb * 64);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 u = src[q];
      const uint32_t wds[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[q * 8 + h * 2] = __uint_as_float(wds[h] << 16);
        v[q * 8 + h * 2 + 1] = __uint_as_float(wds[h] & 0xffff0000u);
      }
    }
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      finite = finite && isfinite(v[i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
  }
  if (!finite && a.status) atomicOr(a.status, kStatusNonFiniteInput);
  amax = block_max(amax, red);
  if (!active || !in_range) return;
  const uint32_t prow = a.row_prow[r];
  if (prow >= a.sf_row_cap) return;
  const float gscale = global_scale_of(amax);
  uint2 packed[4];
  uint32_t sfw = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) sfw |= nvfp4_block(&v[g * 16], gscale, &packed[g]) << (8 * g);
  uint4* dst = reinterpret_cast<uint4*>(a.values + uint64_t(r) * (a.K / 2) + kb * 32);
  dst[0] = make_uint4(packed[0].x, packed[0].y, packed[1].x, packed[1].y);
  dst[1] = make_uint4(packed[2].x, packed[2].y, packed[3].x, packed[3].y);
  *reinterpret_cast<uint32_t*>(a.scales + sf_offset(prow, kb, 0, KB)) = sfw;
  if (kb == 0) a.gscale[r] = gscale;
}

__global__ void slot_table_kernel(SlotArgs a) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.A) return;
  const uint32_t token = a.route_tokens[i], slot = a.route_slots[i];
  uint32_t err = 0;
  if (token >= a.rows) err |= kStatusRouteTokenOutOfRange;
  if (slot >= a.top_k) err |= kStatusRouteSlotOutOfRange;
  if (a.route_experts[i] >= a.E) err |= kStatusExpertOutOfRange;
  if (!isfinite(a.route_weights[i])) err |= kStatusRouteWeightNotFinite;
  if (err) {
    atomicOr(a.status, err);
    return;
  }
  if (atomicCAS(a.slot_assignment + uint64_t(token) * a.top_k + slot, 0xffffffffu, i) != 0xffffffffu)
    atomicOr(a.status, kStatusDuplicateTokenSlot);
}

__global__ void slot_reduce_kernel(SlotArgs a) {
  const uint64_t total = uint64_t(a.rows) * a.H;
  for (uint64_t lin = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t token = static_cast<uint32_t>(lin / a.H), col = static_cast<uint32_t>(lin % a.H);
    float acc = 0.f;
    for (uint32_t slot = 0; slot < a.top_k; ++slot) {
      const uint32_t asg = a.slot_assignment[uint64_t(token) * a.top_k + slot];
      if (asg != 0xffffffffu && asg < a.A)
        acc = fmaf(a.route_weights[asg], a.assignment_down[uint64_t(asg) * a.H + col], acc);
    }
    a.token_output[lin] = acc;
  }
}

// ---------------------------------------------------------------------------
// Deterministic combine: out[t][c] = (sum over the token's slots in ascending
// expert order of plane[t][slot][c]) + shared[t][c].  The ascending-expert
// order is the reference oracle's compacted accumulation order
// (routed_fc2.rs:63-86); routed + shared follows routed_fc2.rs:250-256.
// ---------------------------------------------------------------------------
// Deterministic combine: out[t] = the token's slot rows summed in ascending
// expert order, then the shared expert (its split-K slices summed in slice
// order).  The slot keys (expert << 8 | slot, so equal experts keep slot order)
// are ordered by a 19-comparator sorting network in registers, then the eight
// slot rows load together in that order.  top_k <= 8, shared_splits <= 16.
__device__ __forceinline__ void kswap(uint32_t (&k)[8], int i, int j) {
  const uint32_t lo = min(k[i], k[j]), hi = max(k[i], k[j]);
  k[i] = lo, k[j] = hi;
}

__device__ __forceinline__ void add4(float4& a, const float4& b) {
  a.x = __fadd_rn(a.x, b.x);
  a.y = __fadd_rn(a.y, b.y);
  a.z = __fadd_rn(a.z, b.z);
  a.w = __fadd_rn(a.w, b.w);
}

__global__ void __launch_bounds__(256) combine_kernel(
    const float* __restrict__ plane, const uint16_t* __restrict__ experts,
    const float* __restrict__ shared, uint32_t shared_splits, float* __restrict__ shared_out,
    float* __restrict__ out, uint32_t T, uint32_t H, uint32_t top_k) {
  const uint32_t t = blockIdx.y;
  const uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (t >= T || c >= H) return;
  uint32_t key[8];
#pragma unroll
  for (uint32_t s = 0; s < 8; ++s)
    key[s] = s < top_k ? (uint32_t(experts[uint64_t(t) * top_k + s]) << 8) | s : 0xffffffffu;
  kswap(key, 0, 2), kswap(key, 1, 3), kswap(key, 4, 6), kswap(key, 5, 7);
  kswap(key, 0, 4), kswap(key, 1, 5), kswap(key, 2, 6), kswap(key, 3, 7);
  kswap(key, 0, 1), kswap(key, 2, 3), kswap(key, 4, 5), kswap(key, 6, 7);
  kswap(key, 2, 4), kswap(key, 3, 5);
  kswap(key, 1, 4), kswap(key, 3, 6);
  kswap(key, 1, 2), kswap(key, 3, 4), kswap(key, 5, 6);
  float4 v[8];
#pragma unroll
  for (uint32_t k = 0; k < 8; ++k)
    if (k < top_k)
      v[k] = *reinterpret_cast<const float4*>(plane + (uint64_t(t) * top_k + (key[k] & 0xffu)) * H + c);
  float4 acc = v[0];
#pragma unroll
  for (uint32_t k = 1; k < 8; ++k)
    if (k < top_k) add4(acc, v[k]);
  if (shared) {
    const uint64_t stride = uint64_t(T) * H;
    const float* sp = shared + uint64_t(t) * H + c;
    float4 sum = *reinterpret_cast<const float4*>(sp);
#pragma unroll 4
    for (uint32_t k = 1; k < shared_splits; ++k) add4(sum, *reinterpret_cast<const float4*>(sp + k * stride));
    if (shared_out) *reinterpret_cast<float4*>(shared_out + uint64_t(t) * H + c) = sum;
    add4(acc, sum);
  }
  *reinterpret_cast<float4*>(out + uint64_t(t) * H + c) = acc;
}

// L2 prefetch of two byte ranges: each thread issues one bulk prefetch of up to
// 32 KB (addresses and sizes 16-byte aligned).  No data reaches the SM.
constexpr uint64_t kPrefetchChunk = 32768;
__global__ void l2_prefetch_kernel(const uint8_t* a, uint64_t a_bytes, const uint8_t* b,
                                   uint64_t b_bytes) {
  const uint64_t na = (a_bytes + kPrefetchChunk - 1) / kPrefetchChunk;
  const uint64_t nb = (b_bytes + kPrefetchChunk - 1) / kPrefetchChunk;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < na + nb;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const bool in_a = i < na;
    const uint64_t off = (in_a ? i : i - na) * kPrefetchChunk;
    const uint64_t total = in_a ? a_bytes : b_bytes;
    const uint32_t size = static_cast<uint32_t>(min(kPrefetchChunk, total - off));
    const uint8_t* ptr = (in_a ? a : b) + off;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(size) : "memory");
  }
}

// Shared-expert FC1 finish after split-K: gate/up = sums of the slice partials
// (parts[s][t][0..I) gate, [I..2I) up, slice order), h = bf16(silu(gate) * up).
__global__ void swiglu_finish_kernel(const float* __restrict__ parts, uint32_t splits, uint32_t T,
                                     uint32_t I, uint16_t* __restrict__ h) {
  const uint64_t idx = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x;
  if (idx >= uint64_t(T) * I) return;
  const uint64_t t = idx / I, c = idx % I;
  const uint64_t stride = uint64_t(T) * 2 * I;
  float g = parts[t * 2 * I + c], u = parts[t * 2 * I + I + c];
  for (uint32_t s = 1; s < splits; ++s) {
    g = __fadd_rn(g, parts[s * stride + t * 2 * I + c]);
    u = __fadd_rn(u, parts[s * stride + t * 2 * I + I + c]);
  }
  const __nv_bfloat16 b = __float2bfloat16_rn(__fmul_rn(silu(g), u));
  h[idx] = *reinterpret_cast<const uint16_t*>(&b);
}

// ---------------------------------------------------------------------------
// NVFP4 packer for weights (PackedNvfp4::pack, 1-D codec, nvfp4.rs:170-273) on
// [batch][N][K] f32 or bf16 tensors with N % 128 == 0 and K % 64 == 0: pass 1
// takes each tensor's amax, pass 2 encodes one 64-wide k-block per thread.
// ---------------------------------------------------------------------------
__global__ void pack_amax_kernel(const void* __restrict__ src, int src_bf16, uint64_t per_tensor,
                                 uint32_t* __restrict__ amax_bits, uint32_t* __restrict__ status) {
  const uint32_t b = blockIdx.y;
  float m = 0.f;
  bool finite = true;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < per_tensor;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t j = uint64_t(b) * per_tensor + i;
    const float v = src_bf16 ? bf16_to_f32(reinterpret_cast<const uint16_t*>(src)[j])
                             : reinterpret_cast<const float*>(src)[j];
    finite = finite && isfinite(v);
    m = fmaxf(m, fabsf(v));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) atomicMax(&amax_bits[b], __float_as_uint(m));
  if (!finite) atomicOr(status, kStatusNonFiniteInput);
}

__global__ void pack_encode_kernel(const void* __restrict__ src, int src_bf16, uint32_t N,
                                   uint32_t K, const uint32_t* __restrict__ amax_bits,
                                   uint8_t* __restrict__ values, uint8_t* __restrict__ scales,
                                   float* __restrict__ global_scale,
                                   float* __restrict__ global_amax) {
  const uint32_t b = blockIdx.y;
  const uint32_t KB = K / 64;
  const uint64_t idx = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x;
  if (idx >= uint64_t(N) * KB) return;
  const uint32_t row = static_cast<uint32_t>(idx / KB), kb = static_cast<uint32_t>(idx % KB);
  const float amax = __uint_as_float(amax_bits[b]);
  const float gscale = global_scale_of(amax);
  float v[64];
  const uint64_t base = (uint64_t(b) * N + row) * K + uint64_t(kb) * 64;
#pragma unroll
  for (int i = 0; i < 64; ++i)
    v[i] = src_bf16 ? bf16_to_f32(reinterpret_cast<const uint16_t*>(src)[base + i])
                    : reinterpret_cast<const float*>(src)[base + i];
  uint2 packed[4];
  uint32_t sfw = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) sfw |= nvfp4_block(&v[g * 16], gscale, &packed[g]) << (8 * g);
  uint8_t* vdst = values + uint64_t(b) * N * (K / 2) + uint64_t(row) * (K / 2) + kb * 32;
  uint4* d4 = reinterpret_cast<uint4*>(vdst);
  d4[0] = make_uint4(packed[0].x, packed[0].y, packed[1].x, packed[1].y);
  d4[1] = make_uint4(packed[2].x, packed[2].y, packed[3].x, packed[3].y);
  *reinterpret_cast<uint32_t*>(scales + uint64_t(b) * N * (K / 16) + sf_offset(row, kb, 0, KB)) = sfw;
  if (idx == 0) {
    global_scale[b] = gscale;
    if (global_amax) global_amax[b] = amax;
  }
}

// ------------------------------------------------------------- host launchers
cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* w, float* partial, uint32_t T,
                                 uint32_t H, uint32_t E, uint32_t* bitmap, uint32_t bitmap_words,
                                 cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t st = cudaFuncSetAttribute(router_logits_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(kRbSmem));
    if (st != cudaSuccess) return st;
    configured[dev] = true;
  }
  if (T >= kRouterTiledMinTokens && E % 128 == 0) {
    const size_t tsmem = 2ull * kRtBufFloats * 4;
    static bool tconfigured[64] = {};
    if (!tconfigured[dev]) {
      cudaError_t st = cudaFuncSetAttribute(router_logits_tiled_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(tsmem));
      if (st != cudaSuccess) return st;
      tconfigured[dev] = true;
    }
    dim3 tgrid(E / 128, (T + 127) / 128, 8);
    router_logits_tiled_kernel<<<tgrid, 256, tsmem, stream>>>(x, w, partial, T, H, E, bitmap,
                                                             bitmap_words);
    return cudaPeekAtLastError();
  }
  dim3 grid((E + kRbTile - 1) / kRbTile, (T + kRbTile - 1) / kRbTile, 8);
  router_logits_kernel<<<grid, kRbThreads, kRbSmem, stream>>>(x, w, partial, T, H, E, bitmap,
                                                             bitmap_words);
  return cudaPeekAtLastError();
}

cudaError_t launch_router_select(const float* partial, const float* bias, uint32_t T, uint32_t E,
                                 uint32_t groups, uint32_t topk_groups, uint32_t top_k,
                                 float route_scale, uint16_t* experts, float* weights,
                                 uint32_t* bitmap, uint32_t bitmap_stride, uint32_t* status,
                                 cudaStream_t stream) {
  // two tokens (warps) per CTA: the per-token selection is a latency chain, so
  // tokens are spread over as many SMs as possible
  const uint32_t gs = groups ? E / groups : 0;
  const bool runs = E % 8 == 0 && E <= 256 && gs % 8 == 0 && ((gs / 8) & (gs / 8 - 1)) == 0;
  if (runs)
    router_select_runs_kernel<<<(T + 1) / 2, 64, 0, stream>>>(
        partial, bias, T, E, groups, topk_groups, top_k, route_scale, experts, weights, bitmap,
        bitmap_stride, status);
  else
    router_select_kernel<<<(T + 1) / 2, 64, 0, stream>>>(partial, bias, T, E, groups, topk_groups,
                                                          top_k, route_scale, experts, weights,
                                                          bitmap, bitmap_stride, status);
  return cudaPeekAtLastError();
}

cudaError_t launch_routes_to_bitmap(const uint16_t* experts, const float* weights, uint32_t T,
                                    uint32_t E, uint32_t top_k, uint32_t* bitmap,
                                    uint32_t bitmap_words, uint32_t* status, cudaStream_t stream) {
  zero_words_kernel<<<64, 256, 0, stream>>>(bitmap, bitmap_words);
  const uint32_t n = T * top_k;
  routes_to_bitmap_kernel<<<(n + 255) / 256, 256, 0, stream>>>(experts, weights, T, E, top_k,
                                                               bitmap, (T + 31) / 32, status);
  return cudaPeekAtLastError();
}

cudaError_t launch_compact(const uint32_t* bitmap, uint32_t T, uint32_t E, uint32_t nt,
                           uint32_t sf_row_cap, uint32_t max_tiles, uint32_t* wprefix,
                           uint32_t* counts, uint32_t* offsets, uint32_t* poffs, NTile* tiles,
                           uint32_t* tile_count, uint32_t* status, cudaStream_t stream,
                           const uint8_t* no_tiles) {
  const uint32_t W = (T + 31) / 32;
  // more than one bitmap word per lane (T > 1024): per-expert prefixes on E CTAs first
  const bool wide = W > 32 && W <= 8 * kPrefixThreads && E <= 256;
  if (wide) {
    compact_prefix_kernel<<<E, kPrefixThreads, 0, stream>>>(bitmap, W, wprefix, counts);
    const cudaError_t st = cudaPeekAtLastError();
    if (st != cudaSuccess) return st;
  }
  compact_kernel<<<1, 1024, 0, stream>>>(bitmap, W, E, nt, sf_row_cap, max_tiles, wprefix, counts,
                                         offsets, poffs, tiles, tile_count, status, no_tiles, wide);
  return cudaPeekAtLastError();
}

cudaError_t launch_compact_write(const CompactWriteArgs& a, cudaStream_t stream) {
  const uint32_t n = a.T * a.top_k;
  compact_write_kernel<<<(n + 255) / 256, 256, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

cudaError_t launch_compat_prepare(const CompatPrepareArgs& a, cudaStream_t stream) {
  compat_prepare_kernel<<<1, 1024, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

cudaError_t launch_quant_scatter(const QuantScatterArgs& a, cudaStream_t stream) {
  const uint32_t threads = (a.H / 16 + 31) / 32 * 32;  // H <= 16384
  if (threads > 1024 || a.top_k > 32) return cudaErrorInvalidValue;
  quant_scatter_kernel<<<a.T, threads, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

cudaError_t launch_fc2_quant(const Fc2QuantArgs& a, cudaStream_t stream) {
  // one thread per 16-element block; 128-thread blocks (one row when I = 2048)
  const uint32_t R = a.I / 16;
  if (R < 16 || R > 128 || (R & (R - 1))) return cudaErrorInvalidValue;
  const uint32_t threads = 128;
  const uint32_t rows_per_block = threads / R;
  const uint32_t blocks = (a.count + rows_per_block - 1) / rows_per_block;
  if (blocks == 0) return cudaSuccess;
  fc2_quant_kernel<<<blocks, threads, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

cudaError_t launch_quant_rows(const QuantRowsArgs& a, cudaStream_t stream) {
  if (a.A == 0) return cudaSuccess;
  const uint32_t threads = (a.K / 64 + 31) / 32 * 32;
  quant_rows_kernel<<<a.A, threads, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

cudaError_t launch_slot_table(const SlotArgs& a, cudaStream_t stream) {
  cudaError_t st = cudaMemsetAsync(a.slot_assignment, 0xff, uint64_t(a.rows) * a.top_k * 4, stream);
  if (st != cudaSuccess) return st;
  slot_table_kernel<<<(a.A + 255) / 256, 256, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

cudaError_t launch_slot_reduce(const SlotArgs& a, cudaStream_t stream) {
  const uint64_t total = uint64_t(a.rows) * a.H;
  const uint64_t want = (total + 255) / 256;
  const uint32_t blocks = static_cast<uint32_t>(want < 148 * 8 ? want : 148 * 8);
  slot_reduce_kernel<<<blocks, 256, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

cudaError_t launch_combine(const float* plane, const uint16_t* experts, const float* shared,
                           uint32_t shared_splits, float* shared_out, float* out, uint32_t T,
                           uint32_t H, uint32_t top_k, cudaStream_t stream) {
  if (top_k > 8 || (shared && (shared_splits == 0 || shared_splits > 16)))
    return cudaErrorInvalidValue;
  dim3 grid((H / 4 + 255) / 256, T);
  combine_kernel<<<grid, 256, 0, stream>>>(plane, experts, shared, shared_splits, shared_out, out,
                                           T, H, top_k);
  return cudaPeekAtLastError();
}

cudaError_t launch_l2_prefetch(const void* a, uint64_t a_bytes, const void* b, uint64_t b_bytes,
                               cudaStream_t stream) {
  if (reinterpret_cast<uintptr_t>(a) % 16 || reinterpret_cast<uintptr_t>(b) % 16 || a_bytes % 16 ||
      b_bytes % 16)
    return cudaErrorInvalidValue;
  const uint64_t n = (a_bytes + kPrefetchChunk - 1) / kPrefetchChunk +
                     (b_bytes + kPrefetchChunk - 1) / kPrefetchChunk;
  if (n == 0) return cudaSuccess;
  const uint64_t want = (n + 127) / 128;
  const uint32_t blocks = static_cast<uint32_t>(want < 64 ? want : 64);
  l2_prefetch_kernel<<<blocks, 128, 0, stream>>>(static_cast<const uint8_t*>(a), a_bytes,
                                                static_cast<const uint8_t*>(b), b_bytes);
  return cudaPeekAtLastError();
}

cudaError_t launch_swiglu_finish(const float* parts, uint32_t splits, uint32_t T, uint32_t I,
                                 uint16_t* h, cudaStream_t stream) {
  const uint64_t n = uint64_t(T) * I;
  swiglu_finish_kernel<<<static_cast<uint32_t>((n + 255) / 256), 256, 0, stream>>>(parts, splits,
                                                                                  T, I, h);
  return cudaPeekAtLastError();
}

cudaError_t launch_pack(const void* src, int src_bf16, uint32_t batch, uint32_t N, uint32_t K,
                        uint8_t* values, uint8_t* scales, float* global_scale, float* global_amax,
                        uint32_t* amax_scratch, uint32_t* status, cudaStream_t stream) {
  zero_words_kernel<<<1, 256, 0, stream>>>(amax_scratch, batch);
  dim3 g1(64, batch);
  pack_amax_kernel<<<g1, 256, 0, stream>>>(src, src_bf16, uint64_t(N) * K, amax_scratch, status);
  const uint64_t work = uint64_t(N) * (K / 64);
  dim3 g2(static_cast<uint32_t>((work + 127) / 128), batch);
  pack_encode_kernel<<<g2, 128, 0, stream>>>(src, src_bf16, N, K, amax_scratch, values, scales,
                                             global_scale, global_amax);
  return cudaPeekAtLastError();
}

}  // namespace glmaxx


