// Sparse-layer finish: the MoeTpReduce + MoeResidual steps of the reference's
// frozen sparse-layer order (crates/glm-reference/src/routed_fc2.rs:93-109), in
// the summation order of finish_sparse_layer_oracle (routed_fc2.rs:214-258):
// output = residual, then += attention[r] for r in rank order, then += partial[r]
// for r in rank order, one fp32 round-to-nearest add each.
//
// Two forms run the same arithmetic, so their bits agree:
//  * local (glmaxx_moe_finish_launch): every partial is readable by this GPU;
//  * peer (glmaxx_moe_finish_peer_launch): every rank launches the kernel at the
//    same point of its stream over partial buffers that all ranks map (CUDA IPC),
//    in place of an NCCL all-reduce followed by the finish.  A flag barrier on entry
//    says every rank's partial is complete; one on exit says no peer still reads
//    this rank's partial and, in the two-shot form, every peer's rows have landed.
//    One-shot: every rank sums every element, reading the N partials over NVLink.
//    Two-shot: rank r sums the r-th slice (rows when the RMSNorm is on) and stores
//    the result into every rank's outputs, so each element crosses NVLink twice
//    instead of N-1 times.  Plain loads and stores only: no TMA, no multicast.
//
// The optional RMSNorm output (unit weight, for stacked layers) takes one cluster
// of C CTAs per row.  The sum of squares is reduced in a fixed order (per thread,
// an xor tree over the warp, warps in order, CTAs in cluster order through
// distributed shared memory), and C depends only on (rows, hidden), so the norm too
// is the same bits in every form and on every rank.
//
// Signal buffer of each rank, 32-bit words: ready[ranks], done[ranks], epoch,
// arrive, depart (zeroed once).  The epoch lives in device memory because kernel
// arguments are frozen inside a CUDA graph.  Every wait gives up after
// kWaitTimeoutNs and raises kStatusPeerTimeout instead of hanging; the group's
// epochs are then out of step and the signal buffers must be zeroed on every rank
// (after a host barrier) before the next launch.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/glmaxx_kernel.h"
#include "device.cuh"
#include "moe.h"
#include "runtime.h"

namespace glmaxx {
namespace {

constexpr uint32_t kFinishThreads = 256;
constexpr uint32_t kMaxRanks = 8;
constexpr uint32_t kNormMaxPer = 4;  // float4 per thread and row chunk

struct FinishDest {
  float* f32;
  uint16_t* bf16;
  uint16_t* norm;
};

struct FinishKernelArgs {
  const float* residual_f32;
  const uint16_t* residual_bf16;
  const float* attention_f32;  // [ranks][elements] or null
  const float* partials[kMaxRanks];
  FinishDest dest[kMaxRanks];  // dest[0] only, unless two-shot (rank order)
  uint32_t* signals[kMaxRanks];
  uint32_t* status;
  uint64_t elements;
  uint64_t lo, hi;             // float4 range, or row range with the RMSNorm
  uint32_t ranks, rank, dests, hidden;
  float eps;
};

// ------------------------------------------------------------ peer barrier
// Ordering without system-scope fences (each costs microseconds on B200):
//  * a partial was written by kernels that completed before this launch, so it
//    sits in its GPU's L2, which serves peer reads too: the ready flag needs no
//    fence before it;
//  * every load of a peer's partial has returned (its value was stored) before
//    the CTA counts itself out, so the done flag needs no fence either;
//  * only two-shot stores into peers' memory must be complete before the done
//    flag: there each CTA fences at system scope once, before counting out.
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until sig[base + p] >= e (epoch order, wrapping) for every p < ranks.
__device__ bool wait_flags(const uint32_t* sig, uint32_t base, uint32_t ranks, uint32_t e) {
  const uint64_t start = globaltimer();
  for (uint32_t p = 0; p < ranks; ++p) {
    while (static_cast<int32_t>(ld_relaxed_sys(sig + base + p) - e) < 0) {
      if (globaltimer() - start > kWaitTimeoutNs) return false;
    }
  }
  return true;
}

// Entry: the first CTA of this launch to run publishes ready[rank] = e on every
// rank; every CTA waits for all ready flags.  Returns the epoch; *ok says whether
// the wait completed (uniform within the CTA).
__device__ uint32_t peer_enter(const FinishKernelArgs& a, uint32_t* s_epoch, uint32_t* s_ok) {
  const uint32_t N = a.ranks;
  uint32_t* own = a.signals[a.rank];
  if (threadIdx.x == 0) {
    // the epoch word changes only after every CTA of this launch has arrived
    const uint32_t e = ld_relaxed_gpu(own + 2 * N) + 1;
    if (atomicAdd(own + 2 * N + 1, 1u) == 0)
      for (uint32_t p = 0; p < N; ++p) st_relaxed_sys(a.signals[p] + a.rank, e);
    const bool ok = wait_flags(own, 0, N, e);
    if (!ok && a.status) atomicOr(a.status, kStatusPeerTimeout);
    *s_epoch = e;
    *s_ok = ok ? 1u : 0u;
  }
  __syncthreads();
  return *s_epoch;
}

// Exit: the last CTA to leave publishes done[rank] = e on every rank once every
// CTA's loads and stores are complete, waits for every done flag, and advances
// the epoch.
__device__ void peer_exit(const FinishKernelArgs& a, uint32_t e) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  const uint32_t N = a.ranks;
  uint32_t* own = a.signals[a.rank];
  if (a.dests > 1) fence_acq_rel_sys();  // two-shot: stores into peers' outputs landed
  if (atomicAdd(own + 2 * N + 2, 1u) != gridDim.x - 1) return;
  own[2 * N + 1] = 0;  // every CTA has arrived and left
  own[2 * N + 2] = 0;
  for (uint32_t p = 0; p < N; ++p) st_relaxed_sys(a.signals[p] + N + a.rank, e);
  if (!wait_flags(own, N, N, e) && a.status) atomicOr(a.status, kStatusPeerTimeout);
  *reinterpret_cast<volatile uint32_t*>(own + 2 * N) = e;
}

// ------------------------------------------------------------ arithmetic
// U float4 groups at once, every load in flight before the first add; R >= ranks.
template <uint32_t U, uint32_t R>
__device__ __forceinline__ void finish_u(const FinishKernelArgs& a, const uint64_t (&v)[U],
                                         const bool (&in)[U], float (&o)[U][4]) {
#pragma unroll
  for (uint32_t u = 0; u < U; ++u) {
    o[u][0] = o[u][1] = o[u][2] = o[u][3] = 0.0f;
    if (!in[u]) continue;
    if (a.residual_f32) {
      const float4 r = __ldcg(reinterpret_cast<const float4*>(a.residual_f32) + v[u]);
      o[u][0] = r.x, o[u][1] = r.y, o[u][2] = r.z, o[u][3] = r.w;
    } else if (a.residual_bf16) {
      const uint2 r = __ldcg(reinterpret_cast<const uint2*>(a.residual_bf16) + v[u]);
      o[u][0] = __uint_as_float(r.x << 16), o[u][1] = __uint_as_float(r.x & 0xffff0000u);
      o[u][2] = __uint_as_float(r.y << 16), o[u][3] = __uint_as_float(r.y & 0xffff0000u);
    }
  }
  if (a.attention_f32)
#pragma unroll
    for (uint32_t u = 0; u < U; ++u)
      if (in[u])
        for (uint32_t r = 0; r < a.ranks; ++r) {
          const float4 t =
              __ldcg(reinterpret_cast<const float4*>(a.attention_f32 + r * a.elements) + v[u]);
          o[u][0] = __fadd_rn(o[u][0], t.x), o[u][1] = __fadd_rn(o[u][1], t.y);
          o[u][2] = __fadd_rn(o[u][2], t.z), o[u][3] = __fadd_rn(o[u][3], t.w);
        }
  float4 t[U][R];
#pragma unroll
  for (uint32_t u = 0; u < U; ++u)
#pragma unroll
    for (uint32_t r = 0; r < R; ++r)
      if (in[u] && r < a.ranks) t[u][r] = __ldcg(reinterpret_cast<const float4*>(a.partials[r]) + v[u]);
#pragma unroll
  for (uint32_t u = 0; u < U; ++u)
#pragma unroll
    for (uint32_t r = 0; r < R; ++r)
      if (in[u] && r < a.ranks) {
        o[u][0] = __fadd_rn(o[u][0], t[u][r].x), o[u][1] = __fadd_rn(o[u][1], t[u][r].y);
        o[u][2] = __fadd_rn(o[u][2], t[u][r].z), o[u][3] = __fadd_rn(o[u][3], t[u][r].w);
      }
}

__device__ __forceinline__ uint2 pack_bf16x4(const float (&o)[4]) {
  uint32_t b[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) b[j] = __bfloat16_as_ushort(__float2bfloat16_rn(o[j]));
  return make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
}

__device__ __forceinline__ void store4(const FinishKernelArgs& a, uint64_t v, const float (&o)[4]) {
  const uint2 b = pack_bf16x4(o);
  for (uint32_t d = 0; d < a.dests; ++d) {
    if (a.dest[d].f32)
      reinterpret_cast<float4*>(a.dest[d].f32)[v] = make_float4(o[0], o[1], o[2], o[3]);
    if (a.dest[d].bf16) reinterpret_cast<uint2*>(a.dest[d].bf16)[v] = b;
  }
}

// R: ranks rounded up to 2, 4 or 8; U: float4 groups per thread and iteration
// (U * R loads in flight)
template <bool kPeer, uint32_t R, uint32_t U>
__global__ void __launch_bounds__(kFinishThreads) finish_elems_kernel(FinishKernelArgs a) {
  __shared__ uint32_t s_epoch, s_ok;
  uint32_t e = 0;
  bool ok = true;
  if constexpr (kPeer) {
    e = peer_enter(a, &s_epoch, &s_ok);
    ok = s_ok != 0;
  }
  if (ok)
    for (uint64_t v0 = a.lo + blockIdx.x * uint64_t(kFinishThreads * U) + threadIdx.x; v0 < a.hi;
         v0 += uint64_t(gridDim.x) * kFinishThreads * U) {
      uint64_t v[U];
      bool in[U];
#pragma unroll
      for (uint32_t u = 0; u < U; ++u) {
        v[u] = v0 + u * kFinishThreads;
        in[u] = v[u] < a.hi;
      }
      float o[U][4];
      finish_u<U, R>(a, v, in, o);
#pragma unroll
      for (uint32_t u = 0; u < U; ++u)
        if (in[u]) store4(a, v[u], o[u]);
    }
  if constexpr (kPeer) peer_exit(a, e);
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ float ld_cluster_f32(const float* smem, uint32_t cta) {
  uint32_t addr;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(addr) : "r"(smem_u32(smem)), "r"(cta));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// One cluster of C CTAs per row (grid-stride over the row range); CTA c of the
// cluster owns float4 columns [c*q, (c+1)*q) of the row, q = hidden/4/C <= 256*kPer.
template <bool kPeer, uint32_t R, uint32_t kPer>
__global__ void __launch_bounds__(kFinishThreads) finish_norm_kernel(FinishKernelArgs a) {
  __shared__ uint32_t s_epoch, s_ok;
  __shared__ float warp_ss[kFinishThreads / 32];
  __shared__ float cta_ss;
  uint32_t e = 0;
  bool ok = true;
  if constexpr (kPeer) {
    e = peer_enter(a, &s_epoch, &s_ok);
    ok = s_ok != 0;
  }
  const uint32_t C = cluster_nctarank(), c = cluster_ctarank();
  const uint32_t h4 = a.hidden / 4, q = h4 / C;
  const uint64_t ncl = gridDim.x / C;
  // every CTA of a cluster runs the same rows, so the cluster barriers match even
  // when a peer wait failed (then nothing is loaded or stored)
  for (uint64_t row = a.lo + blockIdx.x / C; row < a.hi; row += ncl) {
    float o[kPer][4];
    float ss = 0.0f;
    const uint64_t base = row * h4 + uint64_t(c) * q;
    uint64_t v[kPer];
    bool in[kPer];
#pragma unroll
    for (uint32_t k = 0; k < kPer; ++k) {
      const uint32_t j = threadIdx.x + k * kFinishThreads;
      v[k] = base + j;
      in[k] = ok && j < q;
    }
    // at most 8 partial loads in flight per thread (registers)
    constexpr uint32_t kChunk = (8 / R) < kPer ? (8 / R) : kPer;
#pragma unroll
    for (uint32_t k0 = 0; k0 < kPer; k0 += kChunk) {
      uint64_t vv[kChunk];
      bool ii[kChunk];
      float oo[kChunk][4];
#pragma unroll
      for (uint32_t c = 0; c < kChunk; ++c) vv[c] = v[k0 + c], ii[c] = in[k0 + c];
      finish_u<kChunk, R>(a, vv, ii, oo);
#pragma unroll
      for (uint32_t c = 0; c < kChunk; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[k0 + c][i] = oo[c][i];
    }
#pragma unroll
    for (uint32_t k = 0; k < kPer; ++k)
      if (in[k]) {
        store4(a, v[k], o[k]);
#pragma unroll
        for (int i = 0; i < 4; ++i) ss = __fmaf_rn(o[k][i], o[k][i], ss);
      }
#pragma unroll
    for (uint32_t off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
    if ((threadIdx.x & 31) == 0) warp_ss[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.0f;
#pragma unroll
      for (uint32_t w = 0; w < kFinishThreads / 32; ++w) s = __fadd_rn(s, warp_ss[w]);
      cta_ss = s;
    }
    cluster_sync_all();
    float total = 0.0f;
    for (uint32_t i = 0; i < C; ++i) total = __fadd_rn(total, ld_cluster_f32(&cta_ss, i));
    cluster_sync_all();  // every CTA has read cta_ss before the next row rewrites it
    const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, float(a.hidden)), a.eps));
#pragma unroll
    for (uint32_t k = 0; k < kPer; ++k)
      if (in[k]) {
        float n[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) n[i] = __fmul_rn(o[k][i], inv);
        const uint2 b = pack_bf16x4(n);
        for (uint32_t d = 0; d < a.dests; ++d) reinterpret_cast<uint2*>(a.dest[d].norm)[v[k]] = b;
      }
  }
  if constexpr (kPeer) peer_exit(a, e);
}

// Cluster size of the RMSNorm kernel: a function of (rows, hidden) only.
uint32_t norm_cluster(uint64_t rows, uint32_t hidden) {
  const uint32_t want = rows < 2 * 148 ? 8u : 2u;
  for (uint32_t C = want; C > 1; C >>= 1)
    if ((hidden / 4) % C == 0 && hidden / 4 / C <= kFinishThreads * kNormMaxPer) return C;
  return 1;
}

// CTAs of `kernel` (kFinishThreads threads) resident on the current device at
// once, cached per device.
template <typename Kernel>
uint32_t resident_ctas(Kernel kernel) {
  static int cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int sms = 0, per = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, kFinishThreads, 0);
    cache[dev] = (per > 0 ? per : 1) * (sms > 0 ? sms : 148);
  }
  return uint32_t(cache[dev]);
}

template <bool kPeer, uint32_t R, uint32_t kPer>
cudaError_t launch_norm_t(const FinishKernelArgs& a, uint32_t C, uint32_t clusters,
                          cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(clusters * C);
  cfg.blockDim = dim3(kFinishThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, finish_norm_kernel<kPeer, R, kPer>, a);
}

// clusters: one per row up to one resident wave
template <bool kPeer, uint32_t R, uint32_t kPer>
cudaError_t launch_norm_r(const FinishKernelArgs& a, uint32_t C, uint64_t rows,
                          cudaStream_t stream) {
  const uint32_t resident = resident_ctas(finish_norm_kernel<kPeer, R, kPer>);
  uint64_t clusters = rows < resident / C ? rows : resident / C;
  if (clusters == 0) clusters = 1;  // a peer rank with no rows still joins the barrier
  return launch_norm_t<kPeer, R, kPer>(a, C, uint32_t(clusters), stream);
}

template <bool kPeer, uint32_t R, uint32_t U>
cudaError_t launch_elems(const FinishKernelArgs& a, cudaStream_t stream) {
  const uint64_t n = a.hi - a.lo;
  uint64_t want = (n + kFinishThreads * U - 1) / (kFinishThreads * U);
  const uint32_t resident = resident_ctas(finish_elems_kernel<kPeer, R, U>);
  if (want > resident) want = resident;  // one wave: every CTA waits on the peers once
  if (want == 0) want = 1;  // a peer rank with an empty slice still joins the barrier
  finish_elems_kernel<kPeer, R, U><<<static_cast<uint32_t>(want), kFinishThreads, 0, stream>>>(a);
  return cudaPeekAtLastError();
}

template <bool kPeer>
cudaError_t launch_finish_any(FinishKernelArgs a, uint64_t rows, cudaStream_t stream) {
  const bool norm = a.dest[0].norm != nullptr;
  if (!norm) {
    if (a.ranks <= 2) return launch_elems<kPeer, 2, 4>(a, stream);
    if (a.ranks <= 4) return launch_elems<kPeer, 4, 2>(a, stream);
    return launch_elems<kPeer, 8, 2>(a, stream);
  }
  const uint32_t C = norm_cluster(rows, a.hidden);
  const uint32_t q = a.hidden / 4 / C;
  if (q > kFinishThreads * kNormMaxPer) return cudaErrorInvalidValue;
  const uint64_t range = a.hi - a.lo;
  const uint32_t per = (q + kFinishThreads - 1) / kFinishThreads;
  if (a.ranks <= 2) {
    if (per <= 1) return launch_norm_r<kPeer, 2, 1>(a, C, range, stream);
    if (per <= 2) return launch_norm_r<kPeer, 2, 2>(a, C, range, stream);
    return launch_norm_r<kPeer, 2, 4>(a, C, range, stream);
  }
  if (a.ranks <= 4) {
    if (per <= 1) return launch_norm_r<kPeer, 4, 1>(a, C, range, stream);
    if (per <= 2) return launch_norm_r<kPeer, 4, 2>(a, C, range, stream);
    return launch_norm_r<kPeer, 4, 4>(a, C, range, stream);
  }
  if (per <= 1) return launch_norm_r<kPeer, 8, 1>(a, C, range, stream);
  if (per <= 2) return launch_norm_r<kPeer, 8, 2>(a, C, range, stream);
  return launch_norm_r<kPeer, 8, 4>(a, C, range, stream);
}

FinishKernelArgs kernel_args(const FinishArgs& f) {
  FinishKernelArgs a{};
  a.residual_f32 = f.residual_f32;
  a.residual_bf16 = f.residual_bf16;
  a.attention_f32 = f.attention_f32;
  for (uint32_t r = 0; r < f.ranks; ++r) a.partials[r] = f.partials[r];
  a.dest[0] = FinishDest{f.output_f32, f.output_bf16, f.norm_bf16};
  a.dests = 1;
  a.elements = f.elements;
  a.ranks = f.ranks;
  a.hidden = f.hidden;
  a.eps = f.eps;
  return a;
}

}  // namespace

cudaError_t launch_finish(const FinishArgs& f, cudaStream_t stream) {
  FinishKernelArgs a = kernel_args(f);
  if (f.norm_bf16 != nullptr) {
    if (f.hidden == 0 || f.hidden % 4 || f.elements % f.hidden) return cudaErrorInvalidValue;
    const uint64_t rows = f.elements / f.hidden;
    a.lo = 0, a.hi = rows;
    return launch_finish_any<false>(a, rows, stream);
  }
  a.lo = 0, a.hi = f.elements / 4;
  if (a.hi == 0) return cudaSuccess;
  return launch_finish_any<false>(a, 0, stream);
}

cudaError_t launch_finish_peer(const FinishArgs& f, const FinishPeer& p, cudaStream_t stream) {
  FinishKernelArgs a = kernel_args(f);
  a.rank = p.rank;
  a.status = p.status;
  for (uint32_t r = 0; r < f.ranks; ++r) a.signals[r] = p.signals[r];
  if (p.two_shot) {
    a.dests = f.ranks;
    for (uint32_t r = 0; r < f.ranks; ++r)
      a.dest[r] = FinishDest{p.outputs_f32[r], p.outputs_bf16[r], p.norms_bf16[r]};
  }
  uint64_t units, rows = 0;
  if (f.norm_bf16 != nullptr) {
    if (f.hidden == 0 || f.hidden % 4 || f.elements % f.hidden) return cudaErrorInvalidValue;
    units = rows = f.elements / f.hidden;
  } else {
    units = f.elements / 4;
  }
  a.lo = 0, a.hi = units;
  if (p.two_shot) {
    a.lo = units * p.rank / f.ranks;
    a.hi = units * (p.rank + 1) / f.ranks;
  }
  return launch_finish_any<true>(a, rows, stream);
}

}  // namespace glmaxx

// ------------------------------------------------------------------ C ABI
using glmaxx::FinishArgs;
using glmaxx::FinishPeer;

namespace {

// Validation shared by both forms; `peer` allows a missing residual (a plain
// all-reduce of the partials).
int32_t finish_args(const glmaxx_moe_finish_descriptor& d, bool peer, FinishArgs* a) {
  if (d.abi_version != GLMAXX_MOE_FINISH_ABI_VERSION || d.struct_bytes != sizeof(d) || d.flags)
    return GLMAXX_ERR_DESCRIPTOR;
  for (uint64_t v : d.reserved)
    if (v) return GLMAXX_ERR_DESCRIPTOR;
  if (d.ranks == 0 || d.ranks > 8 || d.elements == 0 || d.elements % 4) return GLMAXX_ERR_DESCRIPTOR;
  if (d.residual_f32 != 0 && d.residual_bf16 != 0) return GLMAXX_ERR_DESCRIPTOR;
  if (!peer && d.residual_f32 == 0 && d.residual_bf16 == 0) return GLMAXX_ERR_DESCRIPTOR;
  if (d.output_f32 == 0 && d.output_bf16 == 0 && d.norm_bf16 == 0) return GLMAXX_ERR_DESCRIPTOR;
  if (d.norm_bf16 && (d.hidden == 0 || d.hidden % 4 || d.elements % d.hidden || !(d.eps >= 0.0f)))
    return GLMAXX_ERR_DESCRIPTOR;
  if (d.partials_f32 == 0) return GLMAXX_ERR_NULL;
  if (d.residual_f32 % 16 || d.residual_bf16 % 8 || d.attention_f32 % 16 || d.output_f32 % 16 ||
      d.output_bf16 % 8 || d.norm_bf16 % 8)
    return GLMAXX_ERR_DESCRIPTOR;
  *a = FinishArgs{};
  const uint64_t* parts = reinterpret_cast<const uint64_t*>(d.partials_f32);
  for (uint32_t r = 0; r < d.ranks; ++r) {
    if (parts[r] == 0 || parts[r] % 16) return GLMAXX_ERR_DESCRIPTOR;
    a->partials[r] = reinterpret_cast<const float*>(parts[r]);
  }
  a->residual_f32 = reinterpret_cast<const float*>(d.residual_f32);
  a->residual_bf16 = reinterpret_cast<const uint16_t*>(d.residual_bf16);
  a->attention_f32 = reinterpret_cast<const float*>(d.attention_f32);
  a->output_f32 = reinterpret_cast<float*>(d.output_f32);
  a->output_bf16 = reinterpret_cast<uint16_t*>(d.output_bf16);
  a->norm_bf16 = reinterpret_cast<uint16_t*>(d.norm_bf16);
  a->hidden = d.hidden;
  a->eps = d.eps;
  a->elements = d.elements;
  a->ranks = d.ranks;
  return GLMAXX_OK;
}

// Every rank's copy of one output (host array of `ranks` device addresses, rank
// order): present exactly when this rank's output is, aligned, and with this
// rank's entry equal to the descriptor's own output.
template <typename T>
int32_t peer_outputs(uint64_t array, uint64_t own, uint32_t ranks, uint32_t rank, uint32_t align,
                     T** out) {
  if (own == 0) {
    if (array != 0) return GLMAXX_ERR_DESCRIPTOR;
    for (uint32_t r = 0; r < ranks; ++r) out[r] = nullptr;
    return GLMAXX_OK;
  }
  if (array == 0) return GLMAXX_ERR_NULL;
  const uint64_t* p = reinterpret_cast<const uint64_t*>(array);
  for (uint32_t r = 0; r < ranks; ++r) {
    if (p[r] == 0 || p[r] % align) return GLMAXX_ERR_DESCRIPTOR;
    out[r] = reinterpret_cast<T*>(p[r]);
  }
  return p[rank] == own ? GLMAXX_OK : GLMAXX_ERR_DESCRIPTOR;
}

}  // namespace

extern "C" {

int32_t glmaxx_moe_finish_launch(const glmaxx_moe_finish_descriptor* descriptor,
                                 void* cuda_stream) {
  if (descriptor == nullptr) return GLMAXX_ERR_NULL;
  FinishArgs a;
  const int32_t v = finish_args(*descriptor, false, &a);
  if (v != GLMAXX_OK) return v;
  glmaxx::DeviceInfo info;
  const int32_t arch = glmaxx::current_device_info(&info);
  if (arch != 0) return arch;
  return int32_t(glmaxx::launch_finish(a, reinterpret_cast<cudaStream_t>(cuda_stream)));
}

uint64_t glmaxx_moe_peer_signal_bytes(uint32_t ranks) {
  return ranks == 0 || ranks > 8 ? 0 : 256;
}

int32_t glmaxx_moe_finish_peer_launch(const glmaxx_moe_finish_descriptor* descriptor,
                                      const glmaxx_moe_peer_descriptor* peer,
                                      void* cuda_stream) {
  if (descriptor == nullptr || peer == nullptr) return GLMAXX_ERR_NULL;
  FinishArgs a;
  int32_t v = finish_args(*descriptor, true, &a);
  if (v != GLMAXX_OK) return v;
  const glmaxx_moe_peer_descriptor& p = *peer;
  if (p.abi_version != GLMAXX_MOE_PEER_ABI_VERSION || p.struct_bytes != sizeof(p))
    return GLMAXX_ERR_DESCRIPTOR;
  for (uint64_t r : p.reserved)
    if (r) return GLMAXX_ERR_DESCRIPTOR;
  const uint32_t mode = p.flags;
  if (mode != GLMAXX_MOE_PEER_ONE_SHOT && mode != GLMAXX_MOE_PEER_TWO_SHOT)
    return GLMAXX_ERR_DESCRIPTOR;
  const uint32_t N = a.ranks;
  if (p.rank >= N) return GLMAXX_ERR_DESCRIPTOR;
  if (p.signals_u32 == 0) return GLMAXX_ERR_NULL;
  FinishPeer fp{};
  fp.rank = p.rank;
  fp.two_shot = mode == GLMAXX_MOE_PEER_TWO_SHOT;
  fp.status = reinterpret_cast<uint32_t*>(p.status_u32);
  if (p.status_u32 % 4) return GLMAXX_ERR_DESCRIPTOR;
  const uint64_t* sig = reinterpret_cast<const uint64_t*>(p.signals_u32);
  for (uint32_t r = 0; r < N; ++r) {
    if (sig[r] == 0 || sig[r] % 16) return GLMAXX_ERR_DESCRIPTOR;
    fp.signals[r] = reinterpret_cast<uint32_t*>(sig[r]);
  }
  if (fp.two_shot) {
    if ((v = peer_outputs(p.outputs_f32, descriptor->output_f32, N, p.rank, 16, fp.outputs_f32)) ||
        (v = peer_outputs(p.outputs_bf16, descriptor->output_bf16, N, p.rank, 8, fp.outputs_bf16)) ||
        (v = peer_outputs(p.norms_bf16, descriptor->norm_bf16, N, p.rank, 8, fp.norms_bf16)))
      return v;
  } else if (p.outputs_f32 || p.outputs_bf16 || p.norms_bf16) {
    return GLMAXX_ERR_DESCRIPTOR;
  }
  glmaxx::DeviceInfo info;
  const int32_t arch = glmaxx::current_device_info(&info);
  if (arch != 0) return arch;
  return int32_t(glmaxx::launch_finish_peer(a, fp, reinterpret_cast<cudaStream_t>(cuda_stream)));
}

}  // extern "C"
