// Seeded, deterministic sampler: temperature -> softmax -> top-k -> top-p -> exponential race draw.
//
// Reference semantics: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/Sampler.java:69-134:
//   top_k == 1 -> argmax (no randomness); otherwise p = softmax(x / T); keep the k most probable (stable
//   order: value descending, index ascending); keep the shortest prefix of that order whose cumulative
//   probability reaches top_p (the first token is always kept); draw argmax p_i / (-log u_i).
// The reference sorts the whole vocabulary per row; here a CTA per row finds the top-k and top-p cut-offs with
// an MSB-first radix select over order-preserving 32-bit keys of the logits (4 passes of 8 bits).  Masses for
// top-p are accumulated as 2^40-scaled integers so the cut-off is bit-reproducible.  Uniforms come from
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers: As Easy as 1, 2, 3", SC'11) keyed by
// the request seed and counted by (token index, decode step, sequence id): reruns with the same seeds give
// the same tokens.  An optional final-logit soft-cap cap * tanh(x / cap) (Gemma4) is applied first.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "launch.h"

namespace {
using bf16 = __nv_bfloat16;
constexpr int kThreads = 1024;
constexpr int kSub = 8;  // top-p mass sub-histograms of the fast path

struct Philox {
  // Philox4x32 round constants and Weyl key increments as published by Salmon et al. (SC'11).
  static constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  __device__ static uint4 gen(uint4 ctr, uint2 key) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
      const uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
      const uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
      ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
      key.x += W0;
      key.y += W1;
    }
    return ctr;
  }
};

__device__ __forceinline__ uint32_t okey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
__device__ __forceinline__ float ld_logit(const T* p, long i);
template <>
__device__ __forceinline__ float ld_logit<float>(const float* p, long i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_logit<bf16>(const bf16* p, long i) { return __bfloat162float(p[i]); }

__device__ __forceinline__ float capped(float x, float cap) { return cap > 0.f ? cap * tanhf(x / cap) : x; }

struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ ArgMax block_argmax(ArgMax a, ArgMax* sh) {
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, b);
  }
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = a;
  __syncthreads();
  ArgMax r = sh[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) r = better(r, sh[i]);
  return r;
}

__device__ float block_max(float v, float* sh) {
  v = nvb::warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = sh[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) r = fmaxf(r, sh[i]);
  return r;
}

// Exclusive prefix over threads of a per-thread count (block of kThreads).
__device__ int block_excl_scan(int v, int* sh, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  __syncthreads();
  if (lane == 31) sh[w] = incl;
  __syncthreads();
  int base = 0, tot = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
    if (i < w) base += sh[i];
    tot += sh[i];
  }
  *total = tot;
  return base + incl - v;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) sample_kernel(const T* __restrict__ logits, long ld, int V,
                                                          const float* __restrict__ temps, const int* __restrict__ topk,
                                                          const float* __restrict__ topp,
                                                          const int64_t* __restrict__ seeds,
                                                          const int64_t* __restrict__ seq_ids,
                                                          const int* __restrict__ steps, float softcap,
                                                          int64_t* __restrict__ out) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ ArgMax sh_am[32];
  __shared__ float sh_f[32];
  __shared__ int sh_i[32];
  __shared__ unsigned int hist_c[256];
  __shared__ unsigned long long hist_m[256];
  __shared__ uint32_t sel_key;
  __shared__ long long sel_before;
  __shared__ unsigned long long sel_mass_before;
  const int row = blockIdx.x;
  const T* x = logits + row * ld;
  const int tid = threadIdx.x;
  const int k = topk[row];
  // bf16 rows that start 16-byte aligned are streamed 8 logits per load, four loads in flight per thread
  const bool vec = sizeof(T) == 2 && (V & 7) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  if (k == 1) {
    ArgMax a{-INFINITY, 0x7fffffff};
    if (vec) {
      const uint4* x4 = reinterpret_cast<const uint4*>(x);
      const int n4 = V >> 3;
#pragma unroll 4
      for (int i = tid; i < n4; i += blockDim.x) {
        const uint4 raw = x4[i];
        const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) a = better(a, ArgMax{capped(__bfloat162float(e[j]), softcap), i * 8 + j});
      }
    } else {
      for (int i = tid; i < V; i += blockDim.x) a = better(a, ArgMax{capped(ld_logit(x, i), softcap), i});
    }
    a = block_argmax(a, sh_am);
    if (tid == 0) out[row] = a.i == 0x7fffffff ? 0 : a.i;
    return;
  }
  const float invT = 1.f / temps[row];
  const float p = topp[row];
  float mx = -INFINITY;
  if (vec) {
    const uint4* x4 = reinterpret_cast<const uint4*>(x);
    const int n4 = V >> 3;
#pragma unroll 4
    for (int i = tid; i < n4; i += blockDim.x) {
      const uint4 raw = x4[i];
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, capped(__bfloat162float(e[j]), softcap) * invT);
    }
  } else {
    for (int i = tid; i < V; i += blockDim.x) mx = fmaxf(mx, capped(ld_logit(x, i), softcap) * invT);
  }
  mx = block_max(mx, sh_f);
  auto mass = [&](float xv) -> unsigned long long {
    const float e = __expf(xv * invT - mx);  // in (0, 1]
    return (unsigned long long)(e * 1099511627776.0f);  // 2^40 fixed point
  };

  // ---------------- top-k cut-off: key Kk with count(>Kk) < k <= count(>=Kk)
  uint32_t kk_key = 0;  // 0 = keep everything
  int kk_eq_keep = 0x7fffffff;
  if (k > 0 && k < V) {
    uint32_t prefix = 0, mask = 0;
    long long before = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += blockDim.x) hist_c[b] = 0;
      __syncthreads();
      for (int i = tid; i < V; i += blockDim.x) {
        const uint32_t key = okey(capped(ld_logit(x, i), softcap));
        if ((key & mask) == prefix) atomicAdd(&hist_c[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        long long cum = before;
        int b = 255;
        for (; b > 0; --b) {
          if (cum + hist_c[b] >= k) break;
          cum += hist_c[b];
        }
        sel_key = prefix | ((uint32_t)b << shift);
        sel_before = cum;
      }
      __syncthreads();
      prefix = sel_key;
      before = sel_before;
      mask |= 255u << shift;
    }
    kk_key = prefix;
    kk_eq_keep = (int)(k - before);  // how many keys equal to the cut-off stay (lowest indices first)
  }

  // ---------------- rank of each element among those equal to a key, in index order (chunked ownership)
  const int chunk = (V + blockDim.x - 1) / blockDim.x;
  const int c0 = tid * chunk, c1 = min(V, c0 + chunk);
  auto eq_rank_base = [&](uint32_t key) -> int {
    int cnt = 0;
    for (int i = c0; i < c1; ++i) cnt += okey(capped(ld_logit(x, i), softcap)) == key;
    int total;
    return block_excl_scan(cnt, sh_i, &total);
  };
  auto in_topk_pre = [&](uint32_t key) -> bool { return key > kk_key; };

  // mass of the top-k set (fixed point)
  int topk_rank0 = 0;
  if (kk_key != 0) topk_rank0 = eq_rank_base(kk_key);
  unsigned long long zk = 0;
  {
    int r = topk_rank0;
    for (int i = c0; i < c1; ++i) {
      const float xv = capped(ld_logit(x, i), softcap);
      const uint32_t key = okey(xv);
      bool keep = in_topk_pre(key) || kk_key == 0;
      if (!keep && key == kk_key) keep = (r++ < kk_eq_keep);
      if (keep) zk += mass(xv);
    }
  }
  __syncthreads();
  for (int b = tid; b < 256; b += blockDim.x) hist_m[b] = 0;
  __syncthreads();
  {
    // block sum of zk (integers: order independent)
    atomicAdd(&hist_m[0], zk);
    __syncthreads();
    zk = hist_m[0];
    __syncthreads();
  }

  // ---------------- top-p cut-off over the top-k set: key Kp with mass(>Kp) < P <= mass(>=Kp)
  uint32_t kp_key = 0;
  long long kp_eq_keep = 0x7fffffffffffLL;
  if (p < 1.f) {
    const unsigned long long P = (unsigned long long)((double)zk * (double)p);
    uint32_t prefix = 0, mask = 0;
    unsigned long long mbefore = 0;
    const int rank0 = topk_rank0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += blockDim.x) hist_m[b] = 0;
      __syncthreads();
      int r = rank0;
      for (int i = c0; i < c1; ++i) {
        const float xv = capped(ld_logit(x, i), softcap);
        const uint32_t key = okey(xv);
        bool keep = kk_key == 0 || key > kk_key;
        if (!keep && key == kk_key) keep = (r++ < kk_eq_keep);
        if (keep && (key & mask) == prefix) atomicAdd(&hist_m[(key >> shift) & 255u], mass(xv));
      }
      __syncthreads();
      if (tid == 0) {
        unsigned long long cum = mbefore;
        int b = 255;
        for (; b > 0; --b) {
          if (hist_m[b] > 0 && cum + hist_m[b] >= P) break;
          cum += hist_m[b];
        }
        sel_key = prefix | ((uint32_t)b << shift);
        sel_mass_before = cum;
      }
      __syncthreads();
      prefix = sel_key;
      mbefore = sel_mass_before;
      mask |= 255u << shift;
    }
    kp_key = prefix;
    // equal keys have equal mass m_eq: keep while mbefore + r * m_eq < P (at least one kept)
    // m_eq is recomputed from any element with that key
    unsigned long long m_eq = 0;
    for (int i = tid; i < V; i += blockDim.x) {
      const float xv = capped(ld_logit(x, i), softcap);
      if (okey(xv) == kp_key) m_eq = mass(xv);
    }
    __syncthreads();
    if (tid == 0) hist_m[0] = 0;
    __syncthreads();
    if (m_eq) atomicMax(&hist_m[0], m_eq);
    __syncthreads();
    m_eq = hist_m[0];
    if (m_eq > 0 && P > mbefore) kp_eq_keep = (long long)((P - mbefore + m_eq - 1) / m_eq);
    else kp_eq_keep = 1;
    if (kp_eq_keep < 1) kp_eq_keep = 1;
  }

  // ---------------- draw: argmax mass_i / E_i over the kept set
  const uint2 key2 = make_uint2((uint32_t)seeds[row], (uint32_t)((uint64_t)seeds[row] >> 32));
  const uint32_t step = (uint32_t)steps[row];
  const uint32_t sid = (uint32_t)seq_ids[row];
  int rk = kk_key != 0 ? eq_rank_base(kk_key) : 0;
  int rp = (kp_key != 0) ? eq_rank_base(kp_key) : 0;
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int i = c0; i < c1; ++i) {
    const float xv = capped(ld_logit(x, i), softcap);
    const uint32_t key = okey(xv);
    bool keep = kk_key == 0 || key > kk_key;
    if (!keep && key == kk_key) keep = (rk < kk_eq_keep);
    if (kk_key != 0 && key == kk_key) ++rk;
    if (keep && kp_key != 0) {
      if (key < kp_key) keep = false;
      else if (key == kp_key) keep = (rp < kp_eq_keep);
    }
    if (kp_key != 0 && key == kp_key) ++rp;
    if (!keep) continue;
    const uint4 r4 = Philox::gen(make_uint4((uint32_t)i, step, sid, 0x6e76u), key2);
    const float u = (float)(r4.x >> 8) * (1.0f / 16777216.0f);
    const float g = -__logf(fmaxf(1e-10f, u));
    const float pr = __expf(xv * invT - mx);
    best = better(best, ArgMax{pr / fmaxf(1e-10f, g), i});
  }
  best = block_argmax(best, sh_am);
  if (tid == 0) out[row] = best.i == 0x7fffffff ? 0 : best.i;
}


// ------------------------------------------------------------------------------------------------ fast path
// bf16 rows with V % 8 == 0 starting on a 16-byte boundary: every pass streams the row with coalesced 16-byte
// loads.  Index order (needed for the "first k of equal keys" ties) comes from warp-contiguous segments: warp w
// owns elements [w * SEG, (w + 1) * SEG), lanes cover 8 consecutive elements each per 256-element step, and a
// tie's rank is (ties in earlier warps) + (ties earlier in this warp's segment) -- the same ranks the chunked
// slow path computes, so both paths pick the same token.
constexpr int kWarps = kThreads / 32;

struct WarpSeg {
  int lo, hi;
};
__device__ __forceinline__ WarpSeg warp_seg(int V) {
  const int per = ((V + 255) / 256 + kWarps - 1) / kWarps * 256;
  const int lo = min(V, (int)(threadIdx.x >> 5) * per);
  return {lo, min(V, lo + per)};
}

struct Row8 {
  float v[8];
  uint32_t k[8];  // 0 marks "no element" (no real logit maps to key 0)
};
__device__ __forceinline__ Row8 load8(const bf16* x, int i0, int hi, float softcap) {
  Row8 r;
  if (i0 < hi) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + i0);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      r.v[j] = capped(__bfloat162float(e[j]), softcap);
      r.k[j] = okey(r.v[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      r.v[j] = -INFINITY;
      r.k[j] = 0;
    }
  }
  return r;
}

__device__ __forceinline__ int warp_excl(int v, int* total) {
  const int lane = threadIdx.x & 31;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  *total = __shfl_sync(0xffffffffu, incl, 31);
  return incl - v;
}

// Per-element ranks among elements equal to key1 / key2 (index order), advancing the warp's running counts.
__device__ __forceinline__ void step_ranks(const Row8& r, uint32_t key1, uint32_t key2, int& run1, int& run2,
                                           int (&r1)[8], int (&r2)[8]) {
  if (key1 == 0 && key2 == 0) {  // no tie key (block-uniform): ranks are unused, skip the warp scans
#pragma unroll
    for (int j = 0; j < 8; ++j) r1[j] = r2[j] = 0;
    return;
  }
  int c1 = 0, c2 = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c1 += (key1 != 0 && r.k[j] == key1);
    c2 += (key2 != 0 && r.k[j] == key2);
  }
  int t1, t2;
  int a1 = run1 + warp_excl(c1, &t1), a2 = run2 + warp_excl(c2, &t2);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    r1[j] = a1;
    r2[j] = a2;
    a1 += (key1 != 0 && r.k[j] == key1);
    a2 += (key2 != 0 && r.k[j] == key2);
  }
  run1 += t1;
  run2 += t2;
}

// Ties in earlier warps: every warp counts its own, then each thread sums the counts of the warps before it.
__device__ __forceinline__ void warp_tie_bases(const bf16* x, int V, float softcap, uint32_t key1, uint32_t key2,
                                               int* sh1, int* sh2, int& base1, int& base2) {
  base1 = base2 = 0;
  if (key1 == 0 && key2 == 0) return;  // no tie key (block-uniform): no pass over the row
  const WarpSeg sg = warp_seg(V);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int c1 = 0, c2 = 0;
  for (int b0 = sg.lo; b0 < sg.hi; b0 += 256) {
    const Row8 r = load8(x, b0 + lane * 8, sg.hi, softcap);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c1 += (key1 != 0 && r.k[j] == key1);
      c2 += (key2 != 0 && r.k[j] == key2);
    }
  }
  c1 = __reduce_add_sync(0xffffffffu, c1);
  c2 = __reduce_add_sync(0xffffffffu, c2);
  __syncthreads();
  if (lane == 0) {
    sh1[w] = c1;
    sh2[w] = c2;
  }
  __syncthreads();
  base1 = base2 = 0;
  for (int i = 0; i < w; ++i) {
    base1 += sh1[i];
    base2 += sh2[i];
  }
}

__global__ void __launch_bounds__(kThreads) sample_fast_kernel(const bf16* __restrict__ logits, long ld, int V,
                                                               const float* __restrict__ temps,
                                                               const int* __restrict__ topk,
                                                               const float* __restrict__ topp,
                                                               const int64_t* __restrict__ seeds,
                                                               const int64_t* __restrict__ seq_ids,
                                                               const int* __restrict__ steps, float softcap,
                                                               int64_t* __restrict__ out,
                                                               const int* __restrict__ ids) {
  // ids (optional, [B][V]): the row holds candidate logits, column c standing for vocabulary id ids[c] (ids
  // ascending along the row, so position order is id order); uniforms are keyed and the result reported by id
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ ArgMax sh_am[32];
  __shared__ float sh_f[32];
  __shared__ int sh_a[32], sh_b[32];
  __shared__ unsigned int hist_c[256];
  // top-p mass histograms: with no top-k cut every element adds its mass, so 8 sub-histograms (warp & 7) take
  // the 64-bit atomics and are summed into sub-histogram 0 after each pass (3.6x faster on a 64 x 262144 T 0.7 /
  // top-p 0.9 batch); after a top-k cut only the kept elements add and one histogram is cheaper
  __shared__ unsigned long long hist_m8[kSub][256];
  unsigned long long* hist_m = hist_m8[0];
  __shared__ uint32_t sel_key;
  __shared__ long long sel_before;
  __shared__ unsigned long long sel_mass_before;
  const int row = blockIdx.x;
  const bf16* x = logits + row * ld;
  const int tid = threadIdx.x, lane = tid & 31;
  const int k = topk[row];
  const WarpSeg sg = warp_seg(V);
  const uint4* x4 = reinterpret_cast<const uint4*>(x);
  const int n4 = V >> 3;
  if (k == 1) {
    ArgMax a{-INFINITY, 0x7fffffff};
#pragma unroll 4
    for (int i = tid; i < n4; i += blockDim.x) {
      const uint4 raw = x4[i];
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) a = better(a, ArgMax{capped(__bfloat162float(e[j]), softcap), i * 8 + j});
    }
    a = block_argmax(a, sh_am);
    if (tid == 0) out[row] = a.i == 0x7fffffff ? 0 : (ids != nullptr ? ids[(long)row * V + a.i] : a.i);
    return;
  }
  const float invT = 1.f / temps[row];
  const float p = topp[row];
  float mx = -INFINITY;
#pragma unroll 4
  for (int i = tid; i < n4; i += blockDim.x) {
    const uint4 raw = x4[i];
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) mx = fmaxf(mx, capped(__bfloat162float(e[j]), softcap) * invT);
  }
  mx = block_max(mx, sh_f);
  auto mass = [&](float xv) -> unsigned long long {
    const float e = __expf(xv * invT - mx);  // in (0, 1]
    return (unsigned long long)(e * 1099511627776.0f);  // 2^40 fixed point
  };

  // ---------------- top-k cut-off: key Kk with count(>Kk) < k <= count(>=Kk)
  uint32_t kk_key = 0;
  int kk_eq_keep = 0x7fffffff;
  if (k > 0 && k < V) {
    uint32_t prefix = 0, mask = 0;
    long long before = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += blockDim.x) hist_c[b] = 0;
      __syncthreads();
      for (int b0 = sg.lo; b0 < sg.hi; b0 += 256) {
        const Row8 r = load8(x, b0 + lane * 8, sg.hi, softcap);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (r.k[j] != 0 && (r.k[j] & mask) == prefix) atomicAdd(&hist_c[(r.k[j] >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        long long cum = before;
        int b = 255;
        for (; b > 0; --b) {
          if (cum + hist_c[b] >= k) break;
          cum += hist_c[b];
        }
        sel_key = prefix | ((uint32_t)b << shift);
        sel_before = cum;
      }
      __syncthreads();
      prefix = sel_key;
      before = sel_before;
      mask |= 255u << shift;
    }
    kk_key = prefix;
    kk_eq_keep = (int)(k - before);
  }

  // ---------------- mass of the top-k set (fixed point, order independent sum)
  int kb1, kb2;
  warp_tie_bases(x, V, softcap, kk_key, 0, sh_a, sh_b, kb1, kb2);
  unsigned long long zk = 0;
  {
    int run1 = kb1, run2 = 0;
    for (int b0 = sg.lo; b0 < sg.hi; b0 += 256) {
      const Row8 r = load8(x, b0 + lane * 8, sg.hi, softcap);
      int r1[8], r2[8];
      step_ranks(r, kk_key, 0, run1, run2, r1, r2);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (r.k[j] == 0) continue;
        bool keep = kk_key == 0 || r.k[j] > kk_key;
        if (!keep && r.k[j] == kk_key) keep = r1[j] < kk_eq_keep;
        if (keep) zk += mass(r.v[j]);
      }
    }
  }
  __syncthreads();
  for (int b = tid; b < 256; b += blockDim.x) hist_m[b] = 0;
  __syncthreads();
  atomicAdd(&hist_m[0], zk);
  __syncthreads();
  zk = hist_m[0];
  __syncthreads();

  // ---------------- top-p cut-off over the top-k set: key Kp with mass(>Kp) < P <= mass(>=Kp)
  uint32_t kp_key = 0;
  long long kp_eq_keep = 0x7fffffffffffLL;
  if (p < 1.f) {
    const unsigned long long P = (unsigned long long)((double)zk * (double)p);
    uint32_t prefix = 0, mask = 0;
    unsigned long long mbefore = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      const int nsub = kk_key == 0 ? kSub : 1;  // block-uniform
      for (int b = tid; b < nsub * 256; b += blockDim.x) (&hist_m8[0][0])[b] = 0;
      __syncthreads();
      unsigned long long* hm = hist_m8[(tid >> 5) & (nsub - 1)];
      int run1 = kb1, run2 = 0;
      for (int b0 = sg.lo; b0 < sg.hi; b0 += 256) {
        const Row8 r = load8(x, b0 + lane * 8, sg.hi, softcap);
        int r1[8], r2[8];
        step_ranks(r, kk_key, 0, run1, run2, r1, r2);
        uint32_t cb = 0xFFFFFFFFu;  // runs of equal buckets among a thread's 8 neighbours add once
        unsigned long long cm = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (r.k[j] == 0) continue;
          bool keep = kk_key == 0 || r.k[j] > kk_key;
          if (!keep && r.k[j] == kk_key) keep = r1[j] < kk_eq_keep;
          if (keep && (r.k[j] & mask) == prefix) {
            const uint32_t bk = (r.k[j] >> shift) & 255u;
            const unsigned long long m = mass(r.v[j]);
            if (bk == cb) {
              cm += m;
            } else {
              if (cm) atomicAdd(&hm[cb], cm);
              cb = bk;
              cm = m;
            }
          }
        }
        if (cm) atomicAdd(&hm[cb], cm);
      }
      __syncthreads();
      if (nsub > 1) {
        for (int b = tid; b < 256; b += blockDim.x) {
          unsigned long long t = 0;
#pragma unroll
          for (int w = 0; w < kSub; ++w) t += hist_m8[w][b];
          hist_m[b] = t;
        }
        __syncthreads();
      }
      if (tid == 0) {
        unsigned long long cum = mbefore;
        int b = 255;
        for (; b > 0; --b) {
          if (hist_m[b] > 0 && cum + hist_m[b] >= P) break;
          cum += hist_m[b];
        }
        sel_key = prefix | ((uint32_t)b << shift);
        sel_mass_before = cum;
      }
      __syncthreads();
      prefix = sel_key;
      mbefore = sel_mass_before;
      mask |= 255u << shift;
    }
    kp_key = prefix;
    // equal keys have equal mass m_eq: keep while mbefore + r * m_eq < P (at least one kept)
    unsigned long long m_eq = 0;
#pragma unroll 4
    for (int i = tid; i < n4; i += blockDim.x) {
      const uint4 raw = x4[i];
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xv = capped(__bfloat162float(e[j]), softcap);
        if (okey(xv) == kp_key) m_eq = mass(xv);
      }
    }
    __syncthreads();
    if (tid == 0) hist_m[0] = 0;
    __syncthreads();
    if (m_eq) atomicMax(&hist_m[0], m_eq);
    __syncthreads();
    m_eq = hist_m[0];
    if (m_eq > 0 && P > mbefore) kp_eq_keep = (long long)((P - mbefore + m_eq - 1) / m_eq);
    else kp_eq_keep = 1;
    if (kp_eq_keep < 1) kp_eq_keep = 1;
  }

  // ---------------- draw: argmax mass_i / E_i over the kept set
  const uint2 key2 = make_uint2((uint32_t)seeds[row], (uint32_t)((uint64_t)seeds[row] >> 32));
  const uint32_t step = (uint32_t)steps[row];
  const uint32_t sid = (uint32_t)seq_ids[row];
  int db1, db2;
  warp_tie_bases(x, V, softcap, kk_key, kp_key, sh_a, sh_b, db1, db2);
  ArgMax best{-INFINITY, 0x7fffffff};
  {
    int run1 = db1, run2 = db2;
    for (int b0 = sg.lo; b0 < sg.hi; b0 += 256) {
      const Row8 r = load8(x, b0 + lane * 8, sg.hi, softcap);
      int r1[8], r2[8];
      step_ranks(r, kk_key, kp_key, run1, run2, r1, r2);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t key = r.k[j];
        if (key == 0) continue;
        bool keep = kk_key == 0 || key > kk_key;
        if (!keep && key == kk_key) keep = r1[j] < kk_eq_keep;
        if (keep && kp_key != 0) {
          if (key < kp_key) keep = false;
          else if (key == kp_key) keep = r2[j] < kp_eq_keep;
        }
        if (!keep) continue;
        const int i = b0 + lane * 8 + j;
        const uint32_t gi = ids != nullptr ? (uint32_t)ids[(long)row * V + i] : (uint32_t)i;
        const uint4 r4 = Philox::gen(make_uint4(gi, step, sid, 0x6e76u), key2);
        const float u = (float)(r4.x >> 8) * (1.0f / 16777216.0f);
        const float g = -__logf(fmaxf(1e-10f, u));
        const float pr = __expf(r.v[j] * invT - mx);
        best = better(best, ArgMax{pr / fmaxf(1e-10f, g), i});
      }
    }
  }
  best = block_argmax(best, sh_am);
  if (tid == 0) out[row] = best.i == 0x7fffffff ? 0 : (ids != nullptr ? ids[(long)row * V + best.i] : best.i);
}
}  // namespace

void sample_cuda(torch::Tensor logits, torch::Tensor temps, torch::Tensor topk, torch::Tensor topp, torch::Tensor seeds,
                 torch::Tensor seq_ids, torch::Tensor steps, double softcap, torch::Tensor out,
                 c10::optional<torch::Tensor> ids) {
  const int B = logits.size(0), V = logits.size(1);
  TORCH_CHECK(logits.stride(1) == 1, "logits rows must be contiguous");
  if (B == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
#define ARGS                                                                                                    \
  logits.stride(0), V, temps.data_ptr<float>(), topk.data_ptr<int>(), topp.data_ptr<float>(),                   \
      seeds.data_ptr<int64_t>(), seq_ids.data_ptr<int64_t>(), steps.data_ptr<int>(), (float)softcap,            \
      out.data_ptr<int64_t>()
  const bool aligned = logits.scalar_type() == at::kBFloat16 && V % 8 == 0 && logits.stride(0) % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(logits.data_ptr()) & 15) == 0;
  if (ids.has_value()) {
    // candidate rows (distributed sampling under tensor parallelism): bf16, padded to a multiple of 8 columns
    TORCH_CHECK(aligned, "candidate sampling needs 16-byte aligned bf16 rows with a multiple of 8 columns");
    TORCH_CHECK(ids->is_cuda() && ids->scalar_type() == at::kInt && ids->is_contiguous() && ids->size(0) == B &&
                    ids->size(1) == V,
                "candidate ids must be contiguous int32 [B, V]");
    C10_CUDA_CHECK(nvb::launch(sample_fast_kernel, dim3(B), dim3(kThreads), 0, stream,
                               reinterpret_cast<const bf16*>(logits.data_ptr()), logits.stride(0), V,
                               temps.data_ptr<float>(), topk.data_ptr<int>(), topp.data_ptr<float>(),
                               seeds.data_ptr<int64_t>(), seq_ids.data_ptr<int64_t>(), steps.data_ptr<int>(),
                               (float)softcap, out.data_ptr<int64_t>(), (const int*)ids->data_ptr<int>()));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const bool fast = aligned && std::getenv("NVB_SAMPLER_SLOW") == nullptr;
  if (logits.scalar_type() == at::kFloat)
    C10_CUDA_CHECK(nvb::launch(sample_kernel<float>, dim3(B), dim3(kThreads), 0, stream, logits.data_ptr<float>(), ARGS));
  else if (fast)
    C10_CUDA_CHECK(nvb::launch(sample_fast_kernel, dim3(B), dim3(kThreads), 0, stream,
                               reinterpret_cast<const bf16*>(logits.data_ptr()), ARGS, (const int*)nullptr));
  else
    C10_CUDA_CHECK(nvb::launch(sample_kernel<bf16>, dim3(B), dim3(kThreads), 0, stream, reinterpret_cast<const bf16*>(logits.data_ptr()), ARGS));
#undef ARGS
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
