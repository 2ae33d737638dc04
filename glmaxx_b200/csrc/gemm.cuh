// Persistent grouped GEMM on sm_100a tensor cores (tcgen05 + TMEM + TMA),
// in "swap-AB" form: the expert's weight rows fill the 128-row MMA M
// dimension and the tokens routed to that expert form the MMA N dimension.
// This lets a decode step with 1-3 tokens per expert stream its weights at
// full HBM rate (N = 32) and lets prefill reuse each weight tile across 128
// tokens (N = 128).
//
// Operands are K-major byte rows (NVFP4: two E2M1 codes per byte; BF16: two
// bytes per element), staged by TMA with 128-byte swizzle, 128 bytes of K per
// pipeline stage (256 NVFP4 or 64 BF16 elements = 4 MMAs).  NVFP4 block
// scales live in the 128x4 atom layout of crates/glm-format/src/nvfp4.rs:493
// (512 bytes per 128 rows x 64 K); that layout is exactly what
// tcgen05.cp.32x128b.warpx4 moves into TMEM for kind::mxf4nvf4, so weights are
// consumed as packed by the reference codec with no repacking.
//
// Warp roles (192 threads): warp 0 issues TMA, warp 1 owns TMEM and issues
// MMAs, warps 2..5 run the epilogue (warp w reads TMEM lanes 32*(w%4)..).
// Every wait is bounded (device.cuh: mbar_wait); a timeout raises the CTA's
// abort flag, sets kStatusWaitTimeout, drains in-flight copies and MMAs with
// bounded waits, frees TMEM and returns.
#pragma once

#include <cuda.h>

#include "device.cuh"

namespace glmaxx {

// One N tile of a grouped GEMM: up to NT consecutive B rows of one expert.
// B values and per-row metadata are in compacted (expert, token, slot) row
// order.  B scale factors live in a padded row space in which every N tile
// owns whole 128-row scale atoms starting at sf_row_start (a multiple of 128),
// so the tile's scales enter TMEM at column 0 of the atom.  With NT = 128 this
// is exactly the reference's expert-local grouped SFA plan
// (crates/glm-cuda/src/abi.rs:44-91).
struct NTile {
  uint32_t expert;        // expert index (A operand slab)
  uint32_t row_start;     // first B row (compacted row space)
  uint32_t sf_row_start;  // same row in the padded scale-factor row space
  uint32_t rows;          // valid rows in this tile (<= NT)
};

enum EpilogueKind : int {
  kEpiSwiGLU = 0,       // out_bf16[row][col] = bf16(silu(g) * u)
  kEpiRoutedPlane = 1,  // plane[token][slot][col] = w * acc (deterministic combine later)
  kEpiRoutedAtomic = 2, // out_f32[token][col] += w * acc
  kEpiStoreF32 = 3,     // out_f32[row][col] = acc
  kEpiStorePartial = 4, // split-K partial: out_f32[ks][row][col] (+ up half at ldo_up)
};

struct GemmArgs {
  const NTile* tiles;         // explicit n-tile list, or null for implicit tiles
  const uint32_t* tile_count; // device count for explicit lists
  uint32_t implicit_rows;     // implicit tiles: q -> rows [q*NT, min(+NT, implicit_rows))
  uint32_t m_tiles;           // M tiles per n tile (pairs of 128-row tiles in dual mode)
  uint32_t k_chunks;          // K bytes / 128
  uint32_t up_row_offset;     // dual: A rows of the second accumulator = first + this
  uint32_t m_stride;          // A rows between consecutive M tiles (0 = 128)
  uint32_t kblocks;           // K / 64: scale atoms along K
  uint32_t ldo;               // output row stride (elements)
  uint32_t top_k;
  uint32_t k_splits;          // K slices per output tile (split-K; kEpiStorePartial only)
  uint32_t kc_per_split;      // k chunks per slice
  uint32_t ldo_up;            // dual split-K: column offset of the up half in out rows
  uint64_t split_stride;      // elements between consecutive K-slice partial planes
  const uint8_t* sfa;         // A scale atoms, expert-major
  uint64_t sfa_expert_bytes;
  const uint8_t* sfb;         // B scale atoms (padded row space, 128-row tiles)
  const float* a_global;      // [experts] per-tensor scale of A, or null
  const float* b_global;      // [rows] per-row scale of B (compacted rows), or null
  void* out;
  const uint32_t* row_token;  // compacted row -> token
  const uint32_t* row_slot;   // compacted row -> slot
  const float* row_weight;    // compacted row -> routing weight
  uint32_t* status;
};

template <bool FP4, bool DUAL, int NT>
struct GemmShape {
  static constexpr int kAcc = DUAL ? 2 : 1;
  static constexpr int kNJ = NT >= 128 ? NT / 128 : 1;              // SFB atoms along N
  // TMEM columns of one stage's scale factors (4 K-blocks x 4 columns per operand).
  static constexpr int kSfSetCols = FP4 ? (kAcc * 16 + 16 * kNJ) : 0;
  // Two scale sets alternate between consecutive stages, so the scale copy of
  // stage s+1 never overwrites columns that the MMAs of stage s still read.
  static constexpr int kSfSets = FP4 ? 2 : 0;
  static constexpr int kSfCols = kSfSets * kSfSetCols;  // TMEM columns for scales
  // Accumulator buffers (up to 4) let the MMA warp run items ahead of the epilogue.
  static constexpr int kAccBufsFit = (512 - kSfCols) / (kAcc * NT);
  static constexpr int kAccBufs = kAccBufsFit >= 4 ? 4 : (kAccBufsFit >= 1 ? kAccBufsFit : 1);
  static constexpr int kUsedCols = kAccBufs * kAcc * NT + kSfCols;
  static constexpr int kTmemCols = kUsedCols <= 32    ? 32
                                   : kUsedCols <= 64  ? 64
                                   : kUsedCols <= 128 ? 128
                                   : kUsedCols <= 256 ? 256
                                                      : 512;
  static constexpr int kABytes = 128 * 128;
  static constexpr int kBBytes = NT * 128;
  // Lane-major scales (128-row N tiles, dual MMAs): each operand's scales of a
  // stage are staged as two 4 KB blocks, one per K-block pair, each [atom kb x4 |
  // atom kb+1 x4], and reach TMEM with two 128x256b copies instead of four
  // 32x128b broadcast copies.  A converter warp writes them; the TMA moves A and B
  // only.  Measured at T = 8192: FC1 (dual) 1.69 ms lane-major vs 1.85 ms with
  // broadcast copies of TMA-loaded atoms; the single-MMA FC2 the other way round,
  // 1.21 vs 1.08 ms, so it takes the atoms.
  static constexpr bool kLaneSf = FP4 && NT == 128 && DUAL;
  static constexpr int kSfaBytes = FP4 ? (kLaneSf ? 8192 : 2048) : 0;
  static constexpr int kSfbBytes = FP4 ? (kLaneSf ? 8192 : 2048 * kNJ) : 0;
  static constexpr int kStageBytes = kAcc * kABytes + kBBytes + kAcc * kSfaBytes + kSfbBytes;
  static constexpr int kTxBytes = kLaneSf ? kAcc * kABytes + kBBytes : kStageBytes;
  static constexpr int kThreads = kLaneSf ? 224 : 192;
  static_assert(kUsedCols <= 512, "TMEM budget");
  static_assert(NT % 32 == 0 && NT <= 128, "tile rows");
  static_assert(kStageBytes % 1024 == 0, "stage alignment");
};

// Per-warp transpose tile of the N=128 epilogues: 16 tokens x 32 columns, rows
// padded so that the 16-byte row reads of 8 lanes hit distinct banks.
template <bool FP4, bool DUAL, int NT, int EPI>
struct EpiTile {
  static constexpr bool kOn = FP4 && NT == 128 && EPI != kEpiStorePartial;
  static constexpr bool kBf16 = EPI == kEpiSwiGLU;
  static constexpr int kPitch = kBf16 ? 80 : 144;
  static constexpr int kWarpBytes = kOn ? 16 * kPitch : 0;
  static constexpr int kBytes = 4 * kWarpBytes;
};

template <bool FP4, bool DUAL, int NT, int STAGES, int EPI>
constexpr int gemm_smem_bytes() {
  return GemmShape<FP4, DUAL, NT>::kStageBytes * STAGES + 1024 /* align slack */ + 512 +
         EpiTile<FP4, DUAL, NT, EPI>::kBytes;
}

template <bool FP4, bool DUAL, int NT, int STAGES, int EPI>
__global__ void __launch_bounds__(GemmShape<FP4, DUAL, NT>::kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b, const GemmArgs args) {
  using S = GemmShape<FP4, DUAL, NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kStageBytes * STAGES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 4;
  uint64_t* drain_bar = bars + 2 * STAGES + 8;
  uint64_t* sfull_bar = bars + 2 * STAGES + 9;  // lane-major scales written (kLaneSf)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 9);
  using ET = EpiTile<FP4, DUAL, NT, EPI>;
  uint8_t* epi_smem = smem + S::kStageBytes * STAGES + 512;  // after the barrier block
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&sfull_bar[s], 1);
    }
    for (int b = 0; b < S::kAccBufs; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4);
    }
    mbar_init(drain_bar, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tmap_a);
    tma_prefetch(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  const uint32_t tiles_total = args.tiles ? *args.tile_count : (args.implicit_rows + NT - 1) / NT;
  const uint32_t splits = args.k_splits ? args.k_splits : 1;
  const uint32_t kc_per = splits > 1 ? args.kc_per_split : args.k_chunks;
  const uint32_t items = tiles_total * args.m_tiles * splits;
  // item -> (n tile q, m tile i, K slice ks); K slice ks covers chunks [ks*kc_per, ...)
  auto item_q = [&](uint32_t item) { return item / splits / args.m_tiles; };
  auto item_i = [&](uint32_t item) { return (item / splits) % args.m_tiles; };
  auto item_kc0 = [&](uint32_t item) { return (item % splits) * kc_per; };
  auto item_kc1 = [&](uint32_t item) { return min(args.k_chunks, (item % splits) * kc_per + kc_per); };
  // Dual mode either pairs gate/up rows for the SwiGLU epilogue (m_stride 128,
  // second tile = up rows) or streams two adjacent 128-row tiles that share the
  // B tile (m_stride 256, up_row_offset 128), which doubles the weight bytes per
  // pipeline stage.
  const uint32_t m_stride = args.m_stride ? args.m_stride : 128;

  auto stage_a = [&](int s, int h) { return stage_base + s * S::kStageBytes + h * S::kABytes; };
  auto stage_b = [&](int s) { return stage_base + s * S::kStageBytes + S::kAcc * S::kABytes; };
  auto stage_sfa = [&](int s, int h) {
    return stage_base + s * S::kStageBytes + S::kAcc * S::kABytes + S::kBBytes + h * S::kSfaBytes;
  };
  auto stage_sfb = [&](int s) {
    return stage_base + s * S::kStageBytes + S::kAcc * S::kABytes + S::kBBytes +
           S::kAcc * S::kSfaBytes;
  };
  auto tile_of = [&](uint32_t q) {
    if (args.tiles) return args.tiles[q];
    NTile t;
    t.expert = 0;
    t.row_start = q * NT;
    t.sf_row_start = q * NT;
    t.rows = min(static_cast<uint32_t>(NT), args.implicit_rows - q * NT);
    return t;
  };
  auto fail = [&](uint32_t bit) {
    *s_abort = 1;
    if (args.status) atomicOr(args.status, bit);
  };

  constexpr uint32_t kTx = S::kTxBytes;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      // The next item's tile descriptor is loaded one item ahead so that its
      // global-memory latency overlaps the current item's copies.
      NTile t_next = blockIdx.x < items ? tile_of(item_q(blockIdx.x)) : NTile{};
      for (uint32_t item = blockIdx.x; ok && item < items; item += gridDim.x) {
        const uint32_t i = item_i(item);
        const NTile t = t_next;
        const uint32_t next = item + gridDim.x;
        if (next < items) t_next = tile_of(item_q(next));
        const uint8_t* sfa_e = FP4 ? args.sfa + uint64_t(t.expert) * args.sfa_expert_bytes : nullptr;
        const uint32_t kc1 = item_kc1(item);
        for (uint32_t kc = item_kc0(item); kc < kc1; ++kc) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, s_abort)) {
            fail(kStatusWaitTimeout);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kTx);
          const int32_t kx = static_cast<int32_t>(kc * 128);
          tma_load_3d(stage_a(stage, 0), &tmap_a, &full_bar[stage], kx, int32_t(i * m_stride),
                      int32_t(t.expert));
          if (DUAL)
            tma_load_3d(stage_a(stage, 1), &tmap_a, &full_bar[stage], kx,
                        int32_t(i * m_stride + args.up_row_offset), int32_t(t.expert));
          tma_load_2d(stage_b(stage), &tmap_b, &full_bar[stage], kx, int32_t(t.row_start));
          if (FP4 && !S::kLaneSf) {
            bulk_load(stage_sfa(stage, 0),
                      sfa_e + 512ull * (uint64_t(i * m_stride / 128) * args.kblocks + kc * 4), 2048,
                      &full_bar[stage]);
            if (DUAL)
              bulk_load(stage_sfa(stage, 1),
                        sfa_e + 512ull * (uint64_t((i * m_stride + args.up_row_offset) / 128) *
                                              args.kblocks +
                                          kc * 4),
                        2048, &full_bar[stage]);
#pragma unroll
            for (int j = 0; j < S::kNJ; ++j)
              bulk_load(stage_sfb(stage) + j * 2048,
                        args.sfb + 512ull * (uint64_t(t.sf_row_start / 128 + j) * args.kblocks + kc * 4),
                        2048, &full_bar[stage]);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: the last min(issued, STAGES) fills must land before the CTA exits.
      const uint32_t pending = issued < STAGES ? issued : STAGES;
      for (uint32_t b = 0; b < pending; ++b) {
        stage = (stage == 0) ? STAGES - 1 : stage - 1;
        if (stage == STAGES - 1) phase ^= 1;
        if (!mbar_wait(&full_bar[stage], phase, nullptr)) fail(kStatusWaitTimeout);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t sf_base0 = tmem + S::kAccBufs * S::kAcc * NT;  // column offset
      uint32_t sf_set = 0;
      constexpr uint32_t kIdesc = FP4 ? idesc_mxf4nvf4(NT) : idesc_bf16(NT);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (uint32_t item = blockIdx.x; ok && item < items; item += gridDim.x) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, s_abort)) {
          fail(kStatusWaitTimeout);
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + acc * (S::kAcc * NT);
        const uint32_t d1 = d0 + NT;
        const uint32_t kc0 = item_kc0(item), kc1 = item_kc1(item);
        for (uint32_t kc = kc0; kc < kc1; ++kc) {
          if (!mbar_wait(&full_bar[stage], phase, s_abort) ||
              (S::kLaneSf && !mbar_wait(&sfull_bar[stage], phase, s_abort))) {
            fail(kStatusWaitTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sf_base = sf_base0 + sf_set * S::kSfSetCols;
          const uint32_t sfa_t0 = sf_base, sfa_t1 = sf_base + 16;
          const uint32_t sfb_t = sf_base + S::kAcc * 16;
          sf_set ^= 1u;
          if (S::kLaneSf) {
            // one 128x256b copy per operand and K-block pair (8 TMEM columns)
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {
              tc_cp_sf_pair(sfa_t0 + pr * 8, smem_desc_sf_pair(stage_sfa(stage, 0) + pr * 4096));
              if (DUAL)
                tc_cp_sf_pair(sfa_t1 + pr * 8, smem_desc_sf_pair(stage_sfa(stage, 1) + pr * 4096));
              tc_cp_sf_pair(sfb_t + pr * 8, smem_desc_sf_pair(stage_sfb(stage) + pr * 4096));
            }
          } else if (FP4) {
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
              tc_cp_sf(sfa_t0 + kb * 4, smem_desc_sf(stage_sfa(stage, 0) + kb * 512));
              if (DUAL) tc_cp_sf(sfa_t1 + kb * 4, smem_desc_sf(stage_sfa(stage, 1) + kb * 512));
#pragma unroll
              for (int j = 0; j < S::kNJ; ++j)
                tc_cp_sf(sfb_t + kb * 4 * S::kNJ + j * 4,
                         smem_desc_sf(stage_sfb(stage) + (j * 4 + kb) * 512));
            }
          }
          const uint64_t a0 = smem_desc_sw128(stage_a(stage, 0));
          const uint64_t a1 = DUAL ? smem_desc_sw128(stage_a(stage, 1)) : 0;
          const uint64_t bd = smem_desc_sw128(stage_b(stage));
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const uint32_t accum = (kc > kc0 || kb > 0) ? 1u : 0u;
            // advancing the start address by 32 bytes steps K by one MMA inside the swizzle atom
            if (FP4) {
              mma_fp4(d0, a0 + 2 * kb, bd + 2 * kb, kIdesc, accum, sfa_t0 + kb * 4,
                      sfb_t + kb * 4 * S::kNJ);
              if (DUAL)
                mma_fp4(d1, a1 + 2 * kb, bd + 2 * kb, kIdesc, accum, sfa_t1 + kb * 4,
                        sfb_t + kb * 4 * S::kNJ);
            } else {
              mma_bf16(d0, a0 + 2 * kb, bd + 2 * kb, kIdesc, accum);
              if (DUAL) mma_bf16(d1, a1 + 2 * kb, bd + 2 * kb, kIdesc, accum);
            }
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&tfull_bar[acc]);
        if (++acc == S::kAccBufs) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Drain all tensor-core work issued by this thread before TMEM is freed.
      tc_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0, nullptr)) fail(kStatusTmemTimeout);
    }
  } else if (warp == 6) {
    // ------------------------------------------------------- scale converter
    // (kLaneSf only) Copies each stage's scale atoms (4 K-blocks x 512 bytes per
    // operand) from global memory four times over into the stage's lane-major
    // blocks -- lane row 32q + r of a 128x256b copy must hold atom row r, whose
    // word q is the scale word of row 32q + r -- with asynchronous 16-byte
    // copies, kConvDepth stages in flight; a stage is published (sfull) once
    // its copies have landed.
    if constexpr (S::kLaneSf) {
      constexpr int kConvDepth = 1;
      constexpr int kOps = S::kAcc + 1;
      uint32_t stage = 0, phase = 0, pending = 0;
      bool ok = true;
      auto publish_oldest = [&]() {
        fence_proxy_async_smem();
        __syncwarp();
        const uint32_t s_old = (stage + STAGES - pending) % STAGES;
        if (lane == 0) mbar_arrive(&sfull_bar[s_old]);
        --pending;
      };
      for (uint32_t item = blockIdx.x; ok && item < items; item += gridDim.x) {
        const uint32_t i = item_i(item);
        const NTile t = tile_of(item_q(item));
        const uint8_t* sfa_e = args.sfa + uint64_t(t.expert) * args.sfa_expert_bytes;
        const uint64_t a0_atom = uint64_t(i * m_stride / 128) * args.kblocks;
        const uint64_t a1_atom = uint64_t((i * m_stride + args.up_row_offset) / 128) * args.kblocks;
        const uint64_t b_atom = uint64_t(t.sf_row_start / 128) * args.kblocks;
        const uint32_t kc1 = item_kc1(item);
        for (uint32_t kc = item_kc0(item); kc < kc1; ++kc) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, s_abort)) {
            fail(kStatusWaitTimeout);
            ok = false;
            break;
          }
#pragma unroll
          for (int o = 0; o < kOps; ++o) {
            const uint8_t* src = (o == kOps - 1)
                                     ? args.sfb + 512ull * (b_atom + kc * 4)
                                     : sfa_e + 512ull * ((o == 0 ? a0_atom : a1_atom) + kc * 4);
            uint8_t* dst = (o == kOps - 1) ? stage_sfb(stage) : stage_sfa(stage, o);
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
              const uint8_t* g = src + 512 * kb + 16 * lane;
              uint8_t* blk = dst + 4096 * (kb / 2) + 2048 * (kb % 2) + 16 * lane;
#pragma unroll
              for (int q = 0; q < 4; ++q) cp_async_16(blk + 512 * q, g);
            }
          }
          cp_async_commit();
          ++pending;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (pending > static_cast<uint32_t>(kConvDepth)) {
            cp_async_wait<kConvDepth>();
            publish_oldest();
          }
        }
      }
      cp_async_wait<0>();
      while (ok && pending > 0) publish_oldest();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Each lane loads the per-row metadata of rows lane, lane+32, ... of the
    // tile before waiting for the accumulator, so those global loads overlap
    // the MMAs; rows are then broadcast with shuffles.
    constexpr int kRowRegs = NT / 32;
    const int quarter = warp & 3;
    const uint32_t m = quarter * 32 + lane;
    uint32_t acc = 0, acc_phase = 0;
    for (uint32_t item = blockIdx.x; item < items; item += gridDim.x) {
      const uint32_t i = item_i(item);
      const NTile t = tile_of(item_q(item));
      const uint64_t split_base = uint64_t(item % splits) * args.split_stride;
      float scale_a = 1.0f;
      if (FP4 && args.a_global) scale_a = args.a_global[t.expert];
      float r_scale[kRowRegs], r_weight[kRowRegs];
      uint32_t r_dst[kRowRegs];
#pragma unroll
      for (int r = 0; r < kRowRegs; ++r) {
        const uint32_t n = r * 32 + lane;
        const uint32_t row = t.row_start + n;
        r_scale[r] = 1.0f;
        r_weight[r] = 0.0f;
        r_dst[r] = row;
        if (n < t.rows) {
          if (FP4 && args.b_global) r_scale[r] = args.b_global[row];
          if (EPI == kEpiRoutedPlane) {
            r_weight[r] = args.row_weight[row];
            r_dst[r] = args.row_token[row] * args.top_k + args.row_slot[row];
          } else if (EPI == kEpiRoutedAtomic) {
            r_weight[r] = args.row_weight[row];
            r_dst[r] = args.row_token[row];
          }
        }
      }
      if (!mbar_wait(&tfull_bar[acc], acc_phase, s_abort)) {
        fail(kStatusWaitTimeout);
        break;
      }
      tc_fence_after();
      const uint32_t col = (EPI == kEpiSwiGLU ? i * 128 : i * m_stride) + m;
      const uint32_t col1 = i * m_stride + args.up_row_offset + m;  // second tile (non-SwiGLU dual)
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
      const uint32_t c_acc = acc * (S::kAcc * NT);
      // 32-column chunks; the TMEM load of chunk ch+1 is in flight while chunk ch
      // is processed.  Chunk ch covers rows 32*ch.. of the tile: register slot ch.
      const uint32_t nch = (t.rows + 31) / 32;
      const uint32_t tbase = lane_base + c_acc;
      // Values of all 32 columns are computed first, branch-free, so that their
      // latency chains (exp, reciprocal) overlap; the stores then skip the rows
      // past the end of the tile.
      auto process = [&](uint32_t ch, uint32_t (&g)[32], uint32_t (&u)[32]) {
        float src_s = r_scale[0], src_w = r_weight[0];
        uint32_t src_d = r_dst[0];
#pragma unroll
        for (int r = 1; r < kRowRegs; ++r) {
          if (r == static_cast<int>(ch)) {
            src_s = r_scale[r];
            src_w = r_weight[r];
            src_d = r_dst[r];
          }
        }
        // columns (token rows) in groups of 8; groups past the tile's last row are
        // skipped (warp-uniform), which at decode -- 1 to 4 rows per expert --
        // removes most of the per-item epilogue work
        const uint32_t live = t.rows - ch * 32;  // > 0 for every processed chunk
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (!ET::kOn && uint32_t(8 * q) >= live) break;
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int j = 8 * q + jj;
            const float s = __fmul_rn(scale_a, __shfl_sync(0xffffffffu, src_s, j));
            const float gj = __fmul_rn(__uint_as_float(g[j]), s);
            const float uj = DUAL ? __fmul_rn(__uint_as_float(u[j]), s) : 0.0f;
            if (EPI == kEpiSwiGLU) {
              g[j] = __float_as_uint(__fmul_rn(silu(gj), DUAL ? uj : 1.0f));
            } else if (EPI == kEpiRoutedPlane || EPI == kEpiRoutedAtomic) {
              const float rw = __shfl_sync(0xffffffffu, src_w, j);
              g[j] = __float_as_uint(__fmul_rn(rw, gj));
              if (DUAL) u[j] = __float_as_uint(__fmul_rn(rw, uj));
            } else {
              g[j] = __float_as_uint(gj);
              if (DUAL) u[j] = __float_as_uint(uj);
            }
          }
        }
        if constexpr (ET::kOn) {
          // Transposed stores: 16 tokens at a time go through this warp's tile, then
          // each lane writes 16-byte pieces of one token row (h rows or output rows).
          uint8_t* tb = epi_smem + quarter * ET::kWarpBytes;
          constexpr int kPasses = (DUAL && !ET::kBf16) ? 2 : 1;
#pragma unroll
          for (int pass = 0; pass < kPasses; ++pass) {
            const uint32_t colbase = (pass ? col1 : col) - lane;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              __syncwarp();
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const uint32_t v = pass ? u[16 * hf + jj] : g[16 * hf + jj];
                if (ET::kBf16)
                  *reinterpret_cast<uint16_t*>(tb + jj * ET::kPitch + 2 * lane) =
                      __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v)));
                else
                  *reinterpret_cast<uint32_t*>(tb + jj * ET::kPitch + 4 * lane) = v;
              }
              __syncwarp();
              if (ET::kBf16) {
                const uint32_t jj = lane & 15, half = lane >> 4;
                const uint32_t rd = __shfl_sync(0xffffffffu, src_d, 16 * hf + jj);
                if (ch * 32 + 16 * hf + jj < t.rows) {
                  const uint8_t* rowp = tb + jj * ET::kPitch;
                  uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(args.out) +
                                                      uint64_t(rd) * args.ldo + colbase + half * 16);
                  o[0] = *reinterpret_cast<const uint4*>(rowp + half * 32);
                  o[1] = *reinterpret_cast<const uint4*>(rowp + half * 32 + 16);
                }
              } else {
                // fp32 rows: each instruction covers 4 token rows, 8 lanes per row
                // writing its 32 columns as one whole 128-byte line (the vector
                // atomics then fill whole L2 sectors)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const uint32_t jj = 4 * q + (lane >> 3), c4 = (lane & 7) * 4;
                  const uint32_t rd = __shfl_sync(0xffffffffu, src_d, 16 * hf + jj);
                  if (ch * 32 + 16 * hf + jj < t.rows) {
                    const float4 f = *reinterpret_cast<const float4*>(tb + jj * ET::kPitch + 4 * c4);
                    float* o = reinterpret_cast<float*>(args.out) + uint64_t(rd) * args.ldo +
                               colbase + c4;
                    if (EPI == kEpiRoutedAtomic)
                      red_add_v4(o, f);
                    else
                      *reinterpret_cast<float4*>(o) = f;
                  }
                }
              }
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (uint32_t(j) >= live) break;  // warp-uniform
            const uint32_t rd = __shfl_sync(0xffffffffu, src_d, j);
            const float v0 = __uint_as_float(g[j]);
            const float v1 = __uint_as_float(u[j]);
            if (EPI == kEpiSwiGLU) {
              reinterpret_cast<__nv_bfloat16*>(args.out)[uint64_t(rd) * args.ldo + col] =
                  __float2bfloat16_rn(v0);
            } else if (EPI == kEpiRoutedAtomic) {
              float* o = reinterpret_cast<float*>(args.out) + uint64_t(rd) * args.ldo;
              atomicAdd(o + col, v0);
              if (DUAL) atomicAdd(o + col1, v1);
            } else if (EPI == kEpiStorePartial) {
              float* o = reinterpret_cast<float*>(args.out) + split_base + uint64_t(rd) * args.ldo;
              o[col] = v0;
              if (DUAL) o[args.ldo_up + col] = v1;
            } else {  // kEpiRoutedPlane, kEpiStoreF32
              float* o = reinterpret_cast<float*>(args.out) + uint64_t(rd) * args.ldo;
              o[col] = v0;
              if (DUAL) o[col1] = v1;
            }
          }
        }
      };
      uint32_t ga[32], ua[32], gb[32], ub[32];
      auto load = [&](uint32_t ch, uint32_t (&g)[32], uint32_t (&u)[32]) {
        tmem_ld32_async(tbase + ch * 32, g);
        if (DUAL) tmem_ld32_async(tbase + NT + ch * 32, u);
      };
      auto settle = [&](uint32_t (&g)[32], uint32_t (&u)[32]) {
        tmem_wait_ld();
        reg_fence(g);
        if (DUAL) reg_fence(u);
      };
      load(0, ga, ua);
      settle(ga, ua);
      for (uint32_t ch = 0; ch < nch; ch += 2) {
        if (ch + 1 < nch) load(ch + 1, gb, ub);
        process(ch, ga, ua);
        settle(gb, ub);
        if (ch + 1 < nch) {
          if (ch + 2 < nch) load(ch + 2, ga, ua);
          process(ch + 1, gb, ub);
          settle(ga, ua);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == S::kAccBufs) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, S::kTmemCols);
}

}  // namespace glmaxx
