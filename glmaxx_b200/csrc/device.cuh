// Device-side primitives for the sm_100a routed-MoE kernels: mbarriers with
// bounded waits, TMA / bulk copies, and the tcgen05 (5th-gen tensor core,
// TMEM accumulator) instruction wrappers.  Hand-written inline PTX; the
// descriptor bit layouts follow the PTX ISA (tcgen05 "shared memory matrix
// descriptor" and "instruction descriptor" tables).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace glmaxx {

// ---------------------------------------------------------------------------
// Status bits written to the device status word (validation_error_u32).
// Bits 0..4 keep the meaning of the reference's FC2 validation word
// (kernels/sm120/nvfp4_routed_fc2.cu:33-39); the rest are new.
enum : uint32_t {
  kStatusRouteTokenOutOfRange = 1u << 0,
  kStatusRouteSlotOutOfRange = 1u << 1,
  kStatusDuplicateTokenSlot = 1u << 2,
  kStatusExpertOutOfRange = 1u << 3,
  kStatusRouteWeightNotFinite = 1u << 4,
  kStatusNonFiniteInput = 1u << 5,
  kStatusCapacityExceeded = 1u << 6,
  kStatusWaitTimeout = 1u << 8,   // a bounded pipeline wait gave up
  kStatusTmemTimeout = 1u << 9,   // drain of in-flight tensor-core work gave up
  kStatusPeerTimeout = 1u << 10,  // a wait on another rank's flag gave up
};

// A bounded wait gives up after this many nanoseconds (%globaltimer).  Every
// pipeline wait in these kernels completes in microseconds when the pipeline
// is healthy; the bound only turns a would-be hang into an error status.
constexpr uint64_t kWaitTimeoutNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_lane0() { return (threadIdx.x & 31) == 0; }

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false if it
// did not complete within `timeout_ns`, or if `abort` was raised meanwhile.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag,
                                          uint64_t timeout_ns = kWaitTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag != nullptr && *abort_flag) return false;
    if (globaltimer() - start > timeout_ns) return false;
  }
}

// ---------------------------------------------------------------- TMA / bulk
__device__ __forceinline__ void tma_prefetch(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Non-tensor bulk copy global -> shared (16-byte aligned, size multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------- tcgen05
// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row core
// groups of 128-byte rows (SBO = 1024 B), version 1, layout type 2.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* smem) {
  const uint64_t addr = smem_u32(smem);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

// Descriptor of a 32-row x 16-byte, unswizzled block (scale-factor atom) for
// tcgen05.cp: 8-row core groups 128 bytes apart, one 16-byte column.
__device__ __forceinline__ uint64_t smem_desc_sf(const void* smem) {
  const uint64_t addr = smem_u32(smem);
  return ((addr >> 4) & 0x3FFFull) | (8ull << 32) | (1ull << 46);
}

// Instruction descriptor: kind::mxf4nvf4, E2M1 x E2M1, UE4M3 scales, K-major
// A and B, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_mxf4nvf4(uint32_t n) {
  return (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

// Instruction descriptor: kind::f16, BF16 x BF16 -> F32, K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_fp4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate, uint32_t sfa_tmem,
                                        uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], "
      "p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// Descriptor of a 128-row x 32-byte block for tcgen05.cp.128x256b: the first
// 16 bytes of every row in one 2 KB half, the second 16 bytes in the next
// (leading byte offset 2 KB), 8-row core groups 128 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sf_pair(const void* smem) {
  return smem_desc_sf(smem) | (uint64_t(2048 >> 4) << 16);
}
__device__ __forceinline__ void tc_cp_sf_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}
// Asynchronous 16-byte global -> shared copy (L1-allocating), its commit group
// and the wait for all but the newest N groups.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(gsrc))
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Four independent float atomic adds to 16 consecutive bytes (one vector
// reduction instruction).
__device__ __forceinline__ void red_add_v4(float* p, float4 v) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (TMA, tcgen05.cp) of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns.
// Asynchronous 32-column TMEM load (32 lanes x 32 columns of 32 bits): the
// registers are valid only after tmem_wait_ld() and reg_fence() on them.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Orders every later use of r after the preceding tmem_wait_ld() (the compiler
// does not know that the load above writes r asynchronously).
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ----------------------------------------------------------------- numerics
// exp(x) by Cody-Waite reduction x = n ln2 + r and the degree-7 Taylor
// polynomial of e^r (Horner, fused multiply-adds), scaled by 2^n; +inf above
// 88, 0 below -87.  The router defines its sigmoid with this function so that
// host restatements can reproduce its bits.
__device__ __forceinline__ float cw_exp(float x) {
  if (isnan(x)) return x;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  if (x < -87.0f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269502f));
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.42860677e-06f, r);
  float p = 1.98412701e-04f;
  p = fmaf(p, r, 1.38888892e-03f);
  p = fmaf(p, r, 8.33333377e-03f);
  p = fmaf(p, r, 4.16666679e-02f);
  p = fmaf(p, r, 1.66666672e-01f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  return __fmul_rn(p, __int_as_float((static_cast<int>(n) + 127) << 23));
}

__device__ __forceinline__ float router_sigmoid(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, cw_exp(-x)));
}

// SiLU of the FC1 epilogue, v / (1 + exp(-v)) with the fast exponential and
// division intrinsics (a few ulp of fp32, far inside the bf16 rounding of h).
__device__ __forceinline__ float silu(float v) {
  return __fdividef(v, 1.0f + __expf(-v));
}

// ------------------------------------------------------------ NVFP4 encode
// E2M1 code of a finite value: nearest of {0,.5,1,1.5,2,3,4,6} with ties to
// the even code (crates/glm-format/src/float.rs:15-36), sign in bit 3; the
// threshold comparisons below select exactly the code the nearest/ties-even
// search selects.
__device__ __forceinline__ uint32_t e2m1_encode(float v) {
  const float m = fabsf(v);
  uint32_t c = (m > 0.25f) + (m >= 0.75f) + (m > 1.25f) + (m >= 1.75f) + (m > 2.5f) +
               (m >= 3.5f) + (m > 5.0f);
  return c | (signbit(v) ? 0x8u : 0u);
}

// E4M3 code of a positive finite value: nearest over codes 0..0x7e, ties to
// the even code (float.rs:52-73).  Round-to-nearest-even on the 3-bit
// mantissa, subnormals m * 2^-9, saturation at 448 (0x7e).
__device__ __forceinline__ uint32_t e4m3_encode_pos(float v) {
  if (!(v > 0.0f)) return 0u;
  if (v >= 448.0f) return 0x7eu;
  const uint32_t bits = __float_as_uint(v);
  const int exp = static_cast<int>((bits >> 23) & 0xff) - 127;
  if (exp < -6) {
    // subnormal grid: q = v * 2^9 rounded to nearest, ties to even (exact scaling)
    const float q = __fmul_rn(v, 512.0f);
    const uint32_t qi = static_cast<uint32_t>(rintf(q));  // 0..8; 8 == 2^-6 == code 0x08
    return qi;
  }
  // normal: keep 3 mantissa bits with RNE on the 20 dropped bits
  const uint32_t mant = bits & 0x7fffff;
  uint32_t m3 = mant >> 20;
  const uint32_t rem = mant & 0xfffff;
  if (rem > 0x80000u || (rem == 0x80000u && (m3 & 1u))) m3 += 1;
  uint32_t e = static_cast<uint32_t>(exp + 7);
  if (m3 == 8) {
    m3 = 0;
    e += 1;
  }
  const uint32_t code = (e << 3) | m3;
  return code > 0x7eu ? 0x7eu : code;
}

__device__ __forceinline__ float e4m3_decode(uint32_t code) {
  const uint32_t e = (code >> 3) & 0xf, m = code & 7;
  float mag;
  if (e == 0)
    mag = __fmul_rn(static_cast<float>(m), 1.953125e-3f);  // m * 2^-9
  else
    mag = __fmul_rn(1.0f + static_cast<float>(m) * 0.125f, __int_as_float((e - 7 + 127) << 23));
  return (code & 0x80) ? -mag : mag;
}

// Hardware conversions with the reference codec's rounding (round to nearest,
// ties to the even code, saturating): cvt.rn.satfinite.e2m1x2.f32 packs two
// E2M1 codes (first operand in the high nibble); cvt.rn.satfinite.e4m3x2.f32
// two E4M3 codes.  For finite inputs they give the codes of e2m1_encode /
// e4m3_encode_pos (the restatement of float.rs:15-73) -- checked over every fp32
// bit pattern by glmaxx_nvfp4_codec_selfcheck_launch (tests/test_gpu_codec.py).
__device__ __forceinline__ uint32_t e2m1x8_cvt(const float (&q)[8]) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(q[0]), "f"(q[1]), "f"(q[2]), "f"(q[3]), "f"(q[4]), "f"(q[5]), "f"(q[6]), "f"(q[7]));
  return out;
}
__device__ __forceinline__ uint32_t e2m1_cvt(float q) {
  uint16_t out;
  asm("{\n\t.reg .b8 b0;\n\tcvt.rn.satfinite.e2m1x2.f32 b0, %1, %1;\n\t"
      "mov.b16 %0, {b0, b0};\n\t}"
      : "=h"(out)
      : "f"(q));
  return out & 0xfu;
}
__device__ __forceinline__ uint32_t e4m3_cvt_pos(float v) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(out) : "f"(v));
  return out & 0xffu;
}

// E2M1 codes of 8 quotients v[i] / dec, each quotient first rounded to fp32 as
// the reference computes it (code(fl(v / dec))); a zero value gives code 0.
// fast (dec and 1/dec normal): q' = fl(v * rdec), rdec = fl(1 / dec), is within
// 3 * 2^-24 (relative) of the exact quotient, and so is its correctly rounded
// value.  fl(q' * (1 - 2^-20)) and fl(q' * (1 + 2^-20)) bracket both with room to
// spare; the E2M1 rounding is monotone in the magnitude, so when the two ends
// have the same code every value between them -- the rounded quotient included
// -- has it too.  Otherwise (an E2M1 midpoint lies within ~8 ulp) the quotients
// are divided exactly.  The bracket is checked for 8 codes at once.
__device__ __forceinline__ uint32_t e2m1x8_quotient(const float* v, float dec, float rdec,
                                                    bool fast) {
  constexpr float kDown = 0.99999904632568359375f;  // 1 - 2^-20
  constexpr float kUp = 1.00000095367431640625f;    // 1 + 2^-20
  if (fast) {
    float lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float q = __fmul_rn(v[i], rdec);
      lo[i] = v[i] == 0.0f ? 0.0f : __fmul_rn(q, kDown);
      hi[i] = v[i] == 0.0f ? 0.0f : __fmul_rn(q, kUp);
    }
    const uint32_t a = e2m1x8_cvt(lo), b = e2m1x8_cvt(hi);
    if (a == b) return a;
  }
  float q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = v[i] == 0.0f ? 0.0f : __fdiv_rn(v[i], dec);
  return e2m1x8_cvt(q);
}

// Whether e2m1x8_quotient may take its fast path for this divisor.
__device__ __forceinline__ bool quotient_fast_ok(float dec) {
  return dec >= 0x1p-122f && dec <= 0x1p122f;
}

// Quantise one 16-element block (nvfp4.rs:567-608): scale code from the block
// amax, then each value divided by decode(scale) * global.  Returns the scale
// code; writes the 16 codes as 8 bytes (even element in the low nibble).  A zero
// value or a zero scale gives code 0 (not the E2M1 code of -0), as the reference.
__device__ __forceinline__ uint32_t nvfp4_block(const float* v, float global_scale,
                                                uint2* packed) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  uint32_t sc = 0;
  if (amax != 0.0f) sc = e4m3_cvt_pos(__fdiv_rn(__fdiv_rn(amax, 6.0f), global_scale));
  if (sc == 0) {
    *packed = make_uint2(0, 0);
    return 0;
  }
  const float dec = __fmul_rn(e4m3_decode(sc), global_scale);
  const bool fast = quotient_fast_ok(dec);
  const float rdec = fast ? __frcp_rn(dec) : 0.0f;
  packed->x = e2m1x8_quotient(v, dec, rdec, fast);
  packed->y = e2m1x8_quotient(v + 8, dec, rdec, fast);
  return sc;
}

__device__ __forceinline__ float global_scale_of(float amax) {
  return amax == 0.0f ? 1.0f : __fdiv_rn(amax, 2688.0f);
}

// Byte offset of scale (row, k-block kb, group-in-block g) in the 128x4 atom
// layout (crates/glm-format/src/nvfp4.rs:493-521), for a tensor whose K spans
// `kblocks` 64-element blocks.
__host__ __device__ __forceinline__ uint64_t sf_offset(uint64_t row, uint64_t kb, uint32_t g,
                                                       uint64_t kblocks) {
  return 512ull * ((row / 128) * kblocks + kb) + 16ull * (row % 32) + 4ull * ((row % 128) / 32) +
         g;
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

}  // namespace glmaxx
