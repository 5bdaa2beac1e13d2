// Sequence-parallel (SP) collectives over NVLink peer memory, fused into the decode GEMMs of a TP layer.
//
// Layout between the tensor-parallel regions (Megatron-style SP): the residual stream of a step with T tokens is
// sharded by rows, rank r owns rows [r*per, min(T, (r+1)*per)) with per = ceil(T / R).  A row-parallel GEMM
// (o_proj, down_proj, and the vocab-parallel embedding) produces a partial sum [T, H] on every rank; the next
// column-parallel GEMM (qkv, gate_up, LM head) needs RMSNorm(residual + sum of partials) for ALL T rows.  The
// reference names this decomposition (nano-vllm-java/.../layers/Linear.java:269-405, VocabParallelEmbedding.java
// 21-253) but never shards; here it is two fused halves:
//
//   RS (in the producer's epilogue)  every CTA pushes the rows of its output tile to their owners' receive
//        buffers -- recv[owner][src = this rank][row - owner*per][:] -- with peer stores, then publishes one
//        flag per (this rank, CTA) on every rank: bar.sync, then st.release.sys of the forward's epoch by one
//        thread per rank (the release is cumulative over the CTA's stores that the barrier ordered before it,
//        so no full system fence -- measured at 7-9 us per publish -- is needed).
//   AG (in the consumer's prologue)  the owner waits for the R x n_prod flags of its slot, sums the R partial
//        rows in rank order (every owner rounds identically), adds the residual slice, writes it back, applies
//        RMSNorm and stores the normalised row into EVERY rank's gather buffer (peer stores), then flags each
//        row on every rank.  The GEMM's TMA producer first streams the weight tiles (they depend on nothing),
//        then waits for the T row flags of its own rank and TMA-loads the activation tiles from its LOCAL gather
//        buffer: remote data reaches local memory before any TMA touches it (no multicast, no peer TMA).
//
// Flags are epoch-valued (the epoch is bumped once per forward by sp_begin_kernel), and every call site of a
// forward has its own flag slot, so graph replays need no host-side state and no flag is ever reset.  Buffer
// reuse across call sites is safe by causality: rank A can only write a slot-k+1 buffer after it has passed a
// wait that required rank B to be done reading the slot-k contents.  Every wait is bounded (``wait_ns``); on
// expiry the kernel records kErrFlagTimeout in the error word and winds down instead of hanging.
#pragma once
#include "common.cuh"

namespace nvb {
namespace sp {

constexpr int kMaxRanks = 8;
constexpr int kMaxProd = 256;     // producer CTAs per rank per slot (flag array width)
constexpr int kMaxRows = 256;     // tokens of one SP step (decode buckets)
constexpr int kMaxChunks = 8;     // 16-byte chunks per thread in the row kernels: H <= 128 * 8 * 8 = 8192
constexpr int kRowCtas = 128;     // CTAs that reduce rows: always co-resident (one per SM, 148 SMs)

struct Args {
  int mode;        // 0 off, 1 AG + RMSNorm prologue (consumer), 2 RS epilogue (producer)
  int rank, R, T, per, per_max, H;
  int n_prod;      // consumer: producer CTAs per rank of the slot it consumes
  int has_res, norm_mode;
  float eps;
  uint64_t wait_ns;
  const uint32_t* epoch;        // local: forward epoch
  uint32_t* split_flag;         // local, producer with split K: [kMaxProd] (one per CTA) of this slot
  const __nv_bfloat16* my_recv; // local RS receive buffer [R][per_max][H]
  const uint32_t* my_rs_flag;   // local RS flags of this slot [R][kMaxProd]
  __nv_bfloat16* residual;      // local SP residual slice [per_max][H]
  const __nv_bfloat16* norm_w;  // [H] (null for the weightless norm)
  __nv_bfloat16* recv[kMaxRanks];     // every rank's RS receive buffer
  uint32_t* rs_flag[kMaxRanks];       // every rank's RS flags of this slot
  __nv_bfloat16* gather[kMaxRanks];   // every rank's gather buffer [kMaxRows][H]
  uint32_t* ag_flag[kMaxRanks];       // every rank's AG row flags of this slot [kMaxRows]
  unsigned long long* trace;          // optional: %globaltimer stamps of CTA 0's phases (null = off)
};

// Phase stamps for profiling the fused kernels (CTA 0, one thread): slot ``k`` of the call's trace row.
NV_DEVICE void stamp(const Args& a, int k) {
  if (a.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) a.trace[k] = global_timer_ns();
}

NV_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
NV_DEVICE uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
NV_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
NV_DEVICE void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Generic-proxy writes that this thread has observed (through an acquire) become visible to its subsequent
// async-proxy (TMA) reads of global memory.
NV_DEVICE void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Bounded wait until *p == v (flags only ever move forward to the current epoch).  Returns false on timeout,
// or as soon as the error word shows that some kernel of this device already gave up (a failed step then
// winds down in microseconds instead of paying every later wait's full limit).
template <bool SYS>
NV_DEVICE bool wait_eq(const uint32_t* p, uint32_t v, uint64_t t0, uint64_t wait_ns, const int* err) {
  for (uint32_t i = 0;; ++i) {
    if ((SYS ? ld_acquire_sys(p) : ld_acquire_gpu(p)) == v) return true;
    if ((i & 63u) == 63u) {
      if (global_timer_ns() - t0 > wait_ns) return false;
      if (err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0) return false;
    }
  }
}
NV_DEVICE bool wait_eq_sys(const uint32_t* p, uint32_t v, uint64_t t0, uint64_t wait_ns, const int* err) {
  return wait_eq<true>(p, v, t0, wait_ns, err);
}
NV_DEVICE bool wait_eq_gpu(const uint32_t* p, uint32_t v, uint64_t t0, uint64_t wait_ns, const int* err) {
  return wait_eq<false>(p, v, t0, wait_ns, err);
}

NV_DEVICE void unpack8(const uint4& raw, float (&f)[8]) {
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = __bfloat162float(e[j]);
}
NV_DEVICE uint4 pack8(const float (&f)[8]) {
  uint4 r;
  uint32_t* p = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) p[j] = pack_bf16x2(f[2 * j], f[2 * j + 1]);
  return r;
}

NV_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
  return s;
}

// Rows this rank reduces: its SP slice [rank*per, ...).  CTA ``cta`` of ``ncta`` handles local rows cta,
// cta + ncta, ...
__host__ __device__ __forceinline__ int row0_of(const Args& a) { return a.rank * a.per; }
__host__ __device__ __forceinline__ int owned_rows(const Args& a) {
  const int r0 = a.rank * a.per;
  const int r1 = a.T < r0 + a.per ? a.T : r0 + a.per;
  return r1 > r0 ? r1 - r0 : 0;
}

// ---------------------------------------------------------------------------------------------------- RS wait
// Every thread of the CTA takes part; returns false (error recorded) if a flag did not arrive in time.
NV_DEVICE bool wait_rs_flags(const Args& a, int* err) {
  const uint32_t ep = *a.epoch;
  const uint64_t t0 = global_timer_ns();
  int ok = 1;
  const int n = a.R * a.n_prod;
  for (int i = threadIdx.x; i < n && ok; i += blockDim.x) {
    const int src = i / a.n_prod, c = i % a.n_prod;
    if (!wait_eq_sys(a.my_rs_flag + src * kMaxProd + c, ep, t0, a.wait_ns, err)) {
      record_error(err, kErrFlagTimeout);
      ok = 0;
    }
  }
  return __syncthreads_and(ok) != 0;
}

// ------------------------------------------------------------------------------- AG: reduce, norm, broadcast
// CTA ``cta`` of ``ncta`` reduces its owned rows: residual' = bf16(sum_src recv[src][i] (+ residual[i])),
// out = RMSNorm(residual') -> every rank's gather buffer, row rank*per + i; then flags the rows on every rank.
// blockDim.x threads, H % 8 == 0, H <= blockDim.x * 8 * kMaxChunks.
NV_DEVICE void ag_norm_rows(const Args& a, int cta, int ncta, float* red) {
  const uint32_t ep = *a.epoch;
  const int n_own = owned_rows(a);
  const int H = a.H;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int r0 = row0_of(a);
  for (int i = cta; i < n_own; i += ncta) {
    const int t = r0 + i;
    float v[kMaxChunks][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxChunks; ++j) {
      const int c = (j * nt + tid) * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
      if (c < H) {
        uint4 raw[kMaxRanks];
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s)
          if (s < a.R)
            raw[s] = __ldcg(reinterpret_cast<const uint4*>(a.my_recv + ((size_t)s * a.per_max + i) * H + c));
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s) {  // rank order: every owner rounds the same way
          if (s < a.R) {
            float f[8];
            unpack8(raw[s], f);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[j][e] += f[e];
          }
        }
        __nv_bfloat16* res = a.residual + (size_t)i * H + c;
        if (a.has_res) {
          float r[8];
          unpack8(__ldcg(reinterpret_cast<const uint4*>(res)), r);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[j][e] += r[e];
        }
        const uint4 packed = pack8(v[j]);
        *reinterpret_cast<uint4*>(res) = packed;
        unpack8(packed, v[j]);  // continue from the rounded residual, as the unfused path does
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += v[j][e] * v[j][e];
      }
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)H + a.eps);
#pragma unroll
    for (int j = 0; j < kMaxChunks; ++j) {
      const int c = (j * nt + tid) * 8;
      if (c >= H) continue;
      float g[8];
      if (a.norm_mode == 2 || a.norm_w == nullptr) {
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = 1.f;
      } else {
        unpack8(*reinterpret_cast<const uint4*>(a.norm_w + c), g);
        if (a.norm_mode == 1)
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] += 1.f;
      }
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[j][e] * inv * g[e];
      const uint4 packed = pack8(o);
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < a.R) *reinterpret_cast<uint4*>(a.gather[p] + (size_t)t * H + c) = packed;
    }
  }
  __syncthreads();  // every thread's stores precede the flags below (release is cumulative)
  if (tid < a.R) {
    for (int i = cta; i < n_own; i += ncta) st_release_sys(a.ag_flag[tid] + r0 + i, ep);
  }
}

// Wait (bounded) until all T rows of this step are flagged in this rank's gather buffer; one warp polls.
// Returns false (error recorded) on timeout.  After it the caller's TMA may read the gather buffer.
NV_DEVICE bool wait_ag_rows_warp(const Args& a, int* err) {
  const uint32_t ep = *a.epoch;
  const int lane = threadIdx.x & 31;
  const uint64_t t0 = global_timer_ns();
  int ok = 1;
  const uint32_t* flags = a.ag_flag[a.rank];
  for (int t = lane; t < a.T && ok; t += 32)
    if (!wait_eq_sys(flags + t, ep, t0, a.wait_ns, err)) {
      record_error(err, kErrFlagTimeout);
      ok = 0;
    }
  ok = __all_sync(0xffffffffu, ok);
  fence_proxy_async_global();
  return ok != 0;
}

// ---------------------------------------------------------------------------------------------- RS publish
// After this CTA's pushes: one flag per (this rank, CTA) on every rank.  Called by all threads.
NV_DEVICE void rs_publish(const Args& a, int cta) {
  __syncthreads();
  if ((int)threadIdx.x < a.R) st_release_sys(a.rs_flag[threadIdx.x] + a.rank * kMaxProd + cta, *a.epoch);
}

// Push a bf16 tile held in shared memory -- rows = tokens [t0, t1), 128 features starting at feature f0,
// row stride ``ld`` elements -- to the owners' receive buffers (16-byte peer stores).
NV_DEVICE void rs_push_tile(const Args& a, const __nv_bfloat16* tile, int ld, int t0, int t1, int f0) {
  const int chunks = 16;  // 128 features = 16 x 8
  const int n = (t1 - t0) * chunks;
  for (int idx = threadIdx.x; idx < n; idx += blockDim.x) {
    const int t = t0 + idx / chunks, ch = idx % chunks;
    if (f0 + ch * 8 >= a.H) continue;  // the last 128-row weight tile may overhang H
    const uint4 v = *reinterpret_cast<const uint4*>(tile + (size_t)(t - t0) * ld + ch * 8);
    const int owner = t / a.per, local = t - owner * a.per;
    *reinterpret_cast<uint4*>(a.recv[owner] + ((size_t)a.rank * a.per_max + local) * a.H + f0 + ch * 8) = v;
  }
}

}  // namespace sp
}  // namespace nvb
