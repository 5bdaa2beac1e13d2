// Shared device helpers for the sm_100a kernels of nanovllm_b200.
//
// Everything here is written for Blackwell (sm_100a): mbarrier-tracked TMA (cp.async.bulk.tensor), tcgen05
// tensor-memory allocation / MMA / loads, and bounded waits.  Every spin on an mbarrier or a flag reads
// %globaltimer and gives up after a wall-clock limit: it then records an error code in a global error word that
// the host reads, so a protocol bug ends the kernel with a status instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define NV_DEVICE __device__ __forceinline__

namespace nvb {

// ------------------------------------------------------------------------------------------ error word
// Error codes written into the per-device error word (host: nanovllm_b200.ops.check_device_errors()).
enum DeviceError : int {
  kErrNone = 0,
  kErrMbarTimeout = 1,    // an mbarrier wait gave up
  kErrFlagTimeout = 2,    // a peer-flag wait gave up
  kErrBadArgument = 3,    // a kernel saw an argument it cannot handle (e.g. an index out of range)
};

// Wall-clock budget of one bounded wait.  A healthy pipeline completes a stage in microseconds; after this
// long the wait gives up, records an error code and the kernel winds down instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

NV_DEVICE uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------------ programmatic launch
// Every kernel starts with pdl_wait(): it returns once the preceding kernel on the stream has completed and its
// memory is visible (immediately when the kernel was launched without the programmatic-serialization
// attribute).  pdl_trigger() lets the next kernel's CTAs be scheduled while this one is still running, so their
// prologue (barrier set-up, TMEM allocation, weight prefetch) overlaps this kernel's tail.  Nothing before
// pdl_wait() may read data an earlier kernel writes or write data an earlier kernel reads.
NV_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
NV_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

NV_DEVICE void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------------------------------------ small math
NV_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
NV_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

NV_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

NV_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------------------------------------------------ mbarrier
NV_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
NV_DEVICE void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
NV_DEVICE void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

NV_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
NV_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

NV_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Bounded wait.  Returns false (and records kErrMbarTimeout) when the time limit is reached or when another
// role of the CTA already aborted (``abort_flag`` in shared memory non-zero).
NV_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_error(err, kErrMbarTimeout);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------ TMA
NV_DEVICE void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled TMA load (no multicast) into shared memory, completion counted on ``bar``.
NV_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Prefetch a 2-D tile into L2 (no shared-memory destination, no completion tracking, no multicast).
NV_DEVICE void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// 3-D tiled TMA load (no multicast).
NV_DEVICE void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Offset in bytes of 16-byte chunk ``chunk`` of row ``row`` inside a TMA SWIZZLE_128B tile whose rows are
// 128 bytes (the tile base must be 1024-byte aligned).
NV_DEVICE uint32_t swz128(uint32_t row, uint32_t chunk) { return row * 128u + ((chunk ^ (row & 7u)) << 4); }

// ------------------------------------------------------------------------------------------ ldmatrix / mma.sync
NV_DEVICE void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
NV_DEVICE void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
NV_DEVICE void mma_bf16_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------------------------------ tcgen05
NV_DEVICE void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
NV_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;"); }
NV_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
NV_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
NV_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16 inputs, fp32 accumulate), one CTA.
NV_DEVICE void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on ``bar`` once all previously issued tcgen05.mma of this thread have completed.
NV_DEVICE void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
NV_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
NV_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Registers written by asynchronous tcgen05.ld become valid at tcgen05.wait::ld; routing them through an empty
// volatile asm after the wait keeps the compiler from moving their first use above it.
template <int N>
NV_DEVICE void reg_fence(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i])::"memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte swizzle that TMA
// SWIZZLE_128B produces: rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N.
//   bits  0-13 start address >> 4 | 16-29 leading byte offset >> 4 (unused for swizzled K-major, 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups) | bits 46-47 version = 1
//   bits 61-63 layout: 2 = SWIZZLE_128B
NV_DEVICE uint64_t sdesc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both operands K-major.
//   bits 4-5 D format (1 = f32) | 7-9 A format (1 = bf16) | 10-12 B format (1 = bf16)
//   bit 15/16 A/B major (0 = K) | bits 17-22 N >> 3 | bits 24-28 M >> 4
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------------------------------ clusters / DSMEM
NV_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Full cluster barrier (release on arrive, acquire on wait); every thread of every CTA of the cluster executes it.
NV_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
// Shared-memory address of the same variable in CTA ``rank`` of this cluster.
NV_DEVICE uint32_t map_peer(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
NV_DEVICE void st_dsmem_f32(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}
NV_DEVICE float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

}  // namespace nvb
