// Shared device helpers for the sm_100a quaternion linear kernels: element
// conversion, the device error word, bounded mbarrier waits, TMA loads and
// the tcgen05 (UMMA / TMEM) instructions, all as inline PTX.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>
#include <stdint.h>

namespace qlin {

// ---------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Four fp32 values -> four 16-bit values packed in 8 bytes (round to nearest even).
// Output rows of the column-partitioned layer's other ranks: the same
// [M, ld] layout, already offset to this rank's columns (peer memory mapped
// through CUDA IPC; plain stores over NVLink, no multicast), or, when mc is
// set, the multicast address of every rank's full output (one multimem
// store through NVSwitch reaches all ranks, this one included).
constexpr int kMaxPeers = 7;
struct PeerOut {
  void* y[kMaxPeers] = {};
  int n = 0;
  void* mc = nullptr;
};
__host__ __device__ __forceinline__ bool has_peers(const PeerOut& p) { return p.n > 0 || p.mc != nullptr; }

// Stores through an NVLink multicast address (multimem.st: NVSwitch writes
// the bytes into the same offset of every member's memory).  The data are
// raw 16-bit pairs moved as .f32 words (the form the instruction takes).
__device__ __forceinline__ void multimem_st8(void* p, uint2 v) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};"
               ::"l"(p), "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y))
               : "memory");
}
__device__ __forceinline__ void multimem_st16(void* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
               ::"l"(p), "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}

// Stores four 16-bit outputs (8 bytes) at element offset off of y and, for
// kernels built with peer outputs, of every peer's output -- or once through
// the multicast address (a compile-time choice: the runtime loop alone cost
// 8% of a prefill call).
template <typename T, bool PEERS>
__device__ __forceinline__ void store_out(T* y, const PeerOut& peers, int64_t off, uint2 v) {
  if constexpr (PEERS) {
    if (peers.mc) {
      multimem_st8(reinterpret_cast<T*>(peers.mc) + off, v);
      return;
    }
  }
  *reinterpret_cast<uint2*>(y + off) = v;
  if constexpr (PEERS) {
    for (int p = 0; p < peers.n; ++p) *reinterpret_cast<uint2*>(reinterpret_cast<T*>(peers.y[p]) + off) = v;
  }
}

// 16-byte global loads that stay in program order with the dependency wait
// (griddepcontrol.wait) and with mbarrier waits: volatile asm with a memory
// clobber, L2 only (.cg).  A plain __ldg of a const __restrict__ pointer may
// be scheduled above the dependency wait and read what the previous kernel of
// the stream has not finished writing.
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}
__device__ __forceinline__ float4 ld_cg_f4(const void* p) {
  float4 r;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p)
               : "memory");
  return r;
}

// Orders this thread's earlier stores (peer memory included) before any
// later signal at system scope.
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Dot product of two vectors of eight 16-bit elements (16 bytes each), fp32.
template <typename T>
__device__ __forceinline__ float dot8(uint4 a, uint4 b) {
  const T* pa = reinterpret_cast<const T*>(&a);
  const T* pb = reinterpret_cast<const T*>(&b);
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    s0 = fmaf(to_f32(pa[i]), to_f32(pb[i]), s0);
    s1 = fmaf(to_f32(pa[i + 1]), to_f32(pb[i + 1]), s1);
  }
  return s0 + s1;
}

template <typename T> __device__ __forceinline__ uint2 pack4(float a, float b, float c, float d);
template <> __device__ __forceinline__ uint2 pack4<__nv_bfloat16>(float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}
template <> __device__ __forceinline__ uint2 pack4<__half>(float a, float b, float c, float d) {
  __half2 lo = __floats2half2_rn(a, b), hi = __floats2half2_rn(c, d);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

// ---------------------------------------------------------------------------
// device error word (status codes from qlin_b200.h); bounded waits set it
// ---------------------------------------------------------------------------
// Defined here: the library is one translation unit (qlin_abi.cu).
__device__ int g_device_error = 0;

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Longest any single wait may take before the kernel gives up (2 s); real
// waits in these kernels last microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ---------------------------------------------------------------------------
// shared memory / mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
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
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, for at most
// limit_ns.  Returns false (and records QLIN_ERR_TIMEOUT = 7) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) {
      record_error(7);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// TMA (tensor maps are kernel parameters: __grid_constant__ CUtensorMap)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Plain bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses, size a multiple of 16), completing on an mbarrier.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue/commit, TMEM -> register loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
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

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16/f16 in, fp32 acc).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;  // no output lanes disabled
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate),
        "r"(m0), "r"(m1), "r"(m2), "r"(m3));
}

// Arrive (once) on an mbarrier when all previously issued tcgen05.mma of
// this thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor, K-major operand tile whose rows are 64 bytes
// (32 x 16-bit elements) written by TMA with 64-byte swizzling: eight rows
// form a 512-byte group (stride byte offset), the leading byte offset is not
// used by swizzled K-major layouts, version 1 (sm_100), layout code 4.
__device__ __forceinline__ uint64_t smem_desc_sw64(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;          // start address, 16-byte units
  d |= 1ull << 16;                       // leading byte offset (unused)
  d |= (uint64_t)(512 >> 4) << 32;       // stride byte offset: 8 rows * 64 B
  d |= 1ull << 46;                       // descriptor version
  d |= 4ull << 61;                       // 64-byte swizzle
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation, both operands
// K-major.  ab_fmt: 0 = f16, 1 = bf16.  negate_a flips the sign of A.
__host__ __device__ constexpr uint32_t make_idesc_f16(int m, int n, uint32_t ab_fmt, bool negate_a) {
  return (1u << 4)                    // D format f32
         | (ab_fmt << 7)              // A format
         | (ab_fmt << 10)             // B format
         | ((negate_a ? 1u : 0u) << 13)
         | ((uint32_t)(n >> 3) << 17) // N / 8
         | ((uint32_t)(m >> 4) << 24);// M / 16
}

// ---------------------------------------------------------------------------
// clusters / distributed shared memory
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
__device__ __forceinline__ uint32_t map_peer_smem(uint32_t local_addr, uint32_t peer) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(peer));
  return r;
}
// Split cluster barrier (all threads of every CTA of the cluster).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from this CTA's shared memory into another CTA's of the cluster, counted as
// transaction bytes on that CTA's mbarrier (dst and bar: shared::cluster
// addresses).  The source must stay untouched, and its CTA alive, until the
// destination's barrier has completed.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                  uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst_cluster), "r"(src_cta), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's memory before reading it.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

}  // namespace qlin
