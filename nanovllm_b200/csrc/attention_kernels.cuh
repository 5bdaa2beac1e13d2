// Kernel templates of the paged attention family (decode split-KV, combine, prefill, generic fallback).
// Included by attention.cu (torch launchers) and decode_noalloc.cu (allocation-free C entry point);
// every including translation unit instantiates its own copies (internal linkage).
#pragma once
#include "common.cuh"

namespace {

constexpr int KT = 64;  // keys per tile
constexpr float kLog2e = 1.4426950408889634f;
using bf16 = __nv_bfloat16;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// byte offset of (row, dim) inside a K/V tile made of HD/64 swizzled boxes of KT rows x 128 B
template <int HD>
__device__ __forceinline__ uint32_t tile_off(int row, int dim) {
  return (uint32_t)(dim >> 6) * (KT * 128) + nvb::swz128(row, (dim & 63) >> 3);
}

__device__ __forceinline__ float apply_cap(float x, float softcap) {
  return softcap > 0.f ? softcap * tanhf(x / softcap) : x;
}

struct TileAddr {
  int paged;
  // paged: row index into the [num_blocks * nkv * block_size, hd] view
  // contiguous: 3-D coordinates (dim, head, token) into the packed qkv view
};

template <int HD>
__device__ __forceinline__ void issue_tile(uint8_t* k_dst, uint8_t* v_dst, const CUtensorMap* kmap,
                                           const CUtensorMap* vmap, uint64_t* bar, bool paged, int row, int khead,
                                           int vhead, int token) {
  constexpr int NBOX = HD / 64;
  nvb::mbar_arrive_expect_tx(bar, 2 * KT * HD * 2);
#pragma unroll
  for (int j = 0; j < NBOX; ++j) {
    if (paged) {
      nvb::tma_load_2d(k_dst + j * KT * 128, kmap, bar, j * 64, row);
      nvb::tma_load_2d(v_dst + j * KT * 128, vmap, bar, j * 64, row);
    } else {
      nvb::tma_load_3d(k_dst + j * KT * 128, kmap, bar, j * 64, khead, token);
      nvb::tma_load_3d(v_dst + j * KT * 128, vmap, bar, j * 64, vhead, token);
    }
  }
}

// ============================================================================================ decode
// Split-KV finish inside the decode kernel: every split CTA of (sequence b, kv head) announces itself on a
// per-(b, kv head) counter once its partials are written; the last one to arrive merges the splits (fixed
// split order, so the result does not depend on which CTA finishes last) and resets the counter for the next
// launch.  Without a counter array (nullptr) the separate attn_combine_kernel does the merge.
template <int HD>
__device__ __forceinline__ void decode_arrive_and_combine(int* counters, const float* part_o, const float* part_lse,
                                                          bf16* out, int b, int kvh, int nq, int nkv, int G,
                                                          int nsplit, int ctx, int window, int part_tiles) {
  __shared__ int s_last;
  __threadfence();  // this CTA's partials are visible device-wide before it is counted
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&counters[b * nkv + kvh], 1);
    s_last = old == nsplit - 1;
    if (s_last) counters[b * nkv + kvh] = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int ntiles = (ctx + KT - 1) / KT;
  const int win_start = window > 0 ? max(0, ctx - window) : 0;
  const int s_lo = (win_start / KT) / part_tiles;
  const int s_hi = min(nsplit, (ntiles + part_tiles - 1) / part_tiles);
  for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
    const int row = idx / HD, d = idx % HD;
    const int qh = kvh * G + row;
    const long base = ((long)b * nq + qh) * nsplit;
    float M = -INFINITY;
    for (int sp = s_lo; sp < s_hi; ++sp) M = fmaxf(M, __ldcg(part_lse + base + sp));
    float num = 0.f, den = 0.f;
    if (M != -INFINITY)
      for (int sp = s_lo; sp < s_hi; ++sp) {
        const float w = exp2f(__ldcg(part_lse + base + sp) - M);
        num += w * __ldcg(part_o + (base + sp) * HD + d);
        den += w;
      }
    out[((long)b * nq + qh) * HD + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
  }
}

template <int HD, int STAGES>
__global__ void __launch_bounds__(128) paged_decode_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ q,
    const int* __restrict__ block_tables, int bt_stride, const int* __restrict__ ctx_lens, bf16* __restrict__ out,
    float* __restrict__ part_o, float* __restrict__ part_lse, int nq, int nkv, int block_size, float scale,
    float softcap, int window, int part_tiles, int* err, int* combine_counters = nullptr) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  constexpr int TILE = KT * HD * 2;
  constexpr int QP = HD + 8;  // padded Q row (elements)
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int nsplit = gridDim.x;
  const int G = nq / nkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ctx = ctx_lens[b];
  if ((long)ctx > (long)nsplit * part_tiles * KT || (long)ctx > (long)bt_stride * block_size) {
    // more keys than the split grid or the block-table row covers: skip the sequence (every split CTA of it
    // takes this branch, so the split-merge counter stays consistent) and report instead of truncating
    if (tid == 0 && split == 0) nvb::record_error(err, nvb::kErrBadArgument);
    return;
  }
  const int ntiles = (ctx + KT - 1) / KT;
  const int win_start = window > 0 ? max(0, ctx - window) : 0;
  const int t_begin = max(split * part_tiles, win_start / KT);
  const int t_end = min((split + 1) * part_tiles, ntiles);
  const bool fused_combine = combine_counters != nullptr && nsplit > 1;
  if (t_begin >= t_end) {  // the combine step skips splits without keys
    if (fused_combine)
      decode_arrive_and_combine<HD>(combine_counters, part_o, part_lse, out, b, kvh, nq, nkv, G, nsplit, ctx, window,
                                    part_tiles);
    return;
  }
  const int nt = t_end - t_begin;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* ring = smem;
  bf16* qs = reinterpret_cast<bf16*>(smem + STAGES * 2 * TILE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(qs + 16 * QP);
  __shared__ int abort_flag;

  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) nvb::mbar_init(&bars[s], 1);
    nvb::fence_mbar_init();
  }
  for (int idx = tid; idx < 16 * (HD / 8); idx += blockDim.x) {
    const int r = idx / (HD / 8), c = idx % (HD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G) v = *reinterpret_cast<const uint4*>(q + ((long)b * nq + kvh * G + r) * HD + c * 8);
    *reinterpret_cast<uint4*>(qs + r * QP + c * 8) = v;
  }
  __syncthreads();
  const int* bt = block_tables + (long)b * bt_stride;
  auto tile_row = [&](int t) {
    const int tok = t * KT;
    return (bt[tok / block_size] * nkv + kvh) * block_size + (tok % block_size);
  };
  if (tid == 0) {
    nvb::tma_prefetch_desc(&kmap);
    nvb::tma_prefetch_desc(&vmap);
    for (int i = 0; i < STAGES && i < nt; ++i)
      issue_tile<HD>(ring + i * 2 * TILE, ring + i * 2 * TILE + TILE, &kmap, &vmap, &bars[i], true,
                     tile_row(t_begin + i), 0, 0, 0);
  }

  const int g = lane >> 2, c4 = lane & 3;
  float o[HD / 8][4];
#pragma unroll
  for (int d = 0; d < HD / 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const uint32_t qs_addr = nvb::smem_u32(qs);
  bool aborted = false;

  for (int i = 0; i < nt; ++i) {
    const int st = i % STAGES;
    const bool ok = nvb::mbar_wait(&bars[st], (uint32_t)((i / STAGES) & 1), err, &abort_flag);
    if (__syncthreads_or(!ok)) { aborted = true; break; }
    const uint32_t kb = nvb::smem_u32(ring + st * 2 * TILE);
    const uint32_t vb = kb + TILE;
    const int key0 = warp * 16;  // this warp's keys inside the tile
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t a[4];
      nvb::ldmatrix_x4(a[0], a[1], a[2], a[3], qs_addr + ((lane & 15) * QP + kk * 16 + (lane >> 4) * 8) * 2);
      const int mi = lane >> 3, r = lane & 7;
      const int key = key0 + r + (mi >> 1) * 8;
      const int dim = kk * 16 + (mi & 1) * 8;
      uint32_t b0, b1, b2, b3;
      nvb::ldmatrix_x4(b0, b1, b2, b3, kb + tile_off<HD>(key, dim));
      nvb::mma_bf16_16816(s[0], a, b0, b1);
      nvb::mma_bf16_16816(s[1], a, b2, b3);
    }
    // scale, cap, mask; rows g (e<2) and g+8 (e>=2)
    const int tok0 = (t_begin + i) * KT + key0;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = g + (e >> 1) * 8;
        const int key = tok0 + j * 8 + 2 * c4 + (e & 1);
        float x = apply_cap(s[j][e] * scale, softcap) * kLog2e;
        if (row >= G || key >= ctx || key < win_start) x = -INFINITY;
        s[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float nm = fmaxf(m_run[h], mx[h]);
      corr[h] = (nm == -INFINITY) ? 1.f : exp2f(m_run[h] - nm);
      m_run[h] = nm;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float p = (m_run[h] == -INFINITY) ? 0.f : exp2f(s[j][e] - m_run[h]);
        s[j][e] = p;
        rs[h] += p;
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) l_run[h] = l_run[h] * corr[h] + rs[h];
#pragma unroll
    for (int d = 0; d < HD / 8; ++d) {
      o[d][0] *= corr[0];
      o[d][1] *= corr[0];
      o[d][2] *= corr[1];
      o[d][3] *= corr[1];
    }
    uint32_t pa[4];
    pa[0] = nvb::pack_bf16x2(s[0][0], s[0][1]);
    pa[1] = nvb::pack_bf16x2(s[0][2], s[0][3]);
    pa[2] = nvb::pack_bf16x2(s[1][0], s[1][1]);
    pa[3] = nvb::pack_bf16x2(s[1][2], s[1][3]);
#pragma unroll
    for (int dp = 0; dp < HD / 16; ++dp) {
      const int mi = lane >> 3, r = lane & 7;
      const int key = key0 + r + (mi & 1) * 8;
      const int dim = dp * 16 + (mi >> 1) * 8;
      uint32_t b0, b1, b2, b3;
      nvb::ldmatrix_x4_trans(b0, b1, b2, b3, vb + tile_off<HD>(key, dim));
      nvb::mma_bf16_16816(o[2 * dp], pa, b0, b1);
      nvb::mma_bf16_16816(o[2 * dp + 1], pa, b2, b3);
    }
    __syncthreads();
    if (tid == 0 && i + STAGES < nt)
      issue_tile<HD>(ring + st * 2 * TILE, ring + st * 2 * TILE + TILE, &kmap, &vmap, &bars[st], true,
                     tile_row(t_begin + i + STAGES), 0, 0, 0);
  }
  if (aborted) {
    // drain copies still in flight (bounded) before the CTA exits
    if (tid == 0)
      for (int s = 0; s < STAGES; ++s) nvb::mbar_wait(&bars[s], 0, nullptr, nullptr);
    if (fused_combine)  // keep the counters consistent; the error word already reports the failure
      decode_arrive_and_combine<HD>(combine_counters, part_o, part_lse, out, b, kvh, nq, nkv, G, nsplit, ctx, window,
                                    part_tiles);
    return;
  }
  // merge the four warps' partial softmax states through shared memory (the ring is free now)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  float* comb = reinterpret_cast<float*>(ring);  // [4][16][HD]
  float* cm = comb + 4 * 16 * HD;                // [4][16]
  float* cl = cm + 64;                           // [4][16]
#pragma unroll
  for (int d = 0; d < HD / 8; ++d)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = g + (e >> 1) * 8, dim = d * 8 + 2 * c4 + (e & 1);
      comb[(warp * 16 + row) * HD + dim] = o[d][e];
    }
  if (c4 == 0) {
    cm[warp * 16 + g] = m_run[0];
    cm[warp * 16 + g + 8] = m_run[1];
    cl[warp * 16 + g] = l_run[0];
    cl[warp * 16 + g + 8] = l_run[1];
  }
  __syncthreads();
  for (int idx = tid; idx < G * HD; idx += blockDim.x) {
    const int row = idx / HD, dim = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, cm[w * 16 + row]);
    float L = 0.f, acc = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(cm[w * 16 + row] - M);
        L += cl[w * 16 + row] * f;
        acc += comb[(w * 16 + row) * HD + dim] * f;
      }
    }
    const float val = L > 0.f ? acc / L : 0.f;
    const int qh = kvh * G + row;
    if (nsplit == 1) {
      out[((long)b * nq + qh) * HD + dim] = __float2bfloat16(val);
    } else {
      const long slot = ((long)b * nq + qh) * nsplit + split;
      part_o[slot * HD + dim] = val;
      if (dim == 0) part_lse[slot] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
  if (fused_combine)
    decode_arrive_and_combine<HD>(combine_counters, part_o, part_lse, out, b, kvh, nq, nkv, G, nsplit, ctx, window,
                                  part_tiles);
}

__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                    const int* __restrict__ ctx_lens, bf16* __restrict__ out, int nq, int nsplit,
                                    int HD, int part_tiles, int window) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const int qh = blockIdx.x, b = blockIdx.y;
  const int ctx = ctx_lens[b];
  const int ntiles = (ctx + KT - 1) / KT;
  const int win_start = window > 0 ? max(0, ctx - window) : 0;
  const int s_lo = (win_start / KT) / part_tiles;
  const int s_hi = min(nsplit, (ntiles + part_tiles - 1) / part_tiles);
  const long base = ((long)b * nq + qh) * nsplit;
  float M = -INFINITY;
  for (int s = s_lo; s < s_hi; ++s) M = fmaxf(M, part_lse[base + s]);
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    if (M != -INFINITY)
      for (int s = s_lo; s < s_hi; ++s) {
        const float w = exp2f(part_lse[base + s] - M);
        num += w * part_o[(base + s) * HD + d];
        den += w;
      }
    out[((long)b * nq + qh) * HD + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
  }
}

// ============================================================================================ prefill
template <int HD, int STAGES>
__global__ void __launch_bounds__(128) prefill_attn_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ q,
    long q_tok_stride, bf16* __restrict__ out, long o_tok_stride, const int* __restrict__ cu_q,
    const int* __restrict__ cu_k, const int* __restrict__ block_tables, int bt_stride, int paged, int nq, int nkv,
    int block_size, float scale, float softcap, int window, int causal, int* err) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  constexpr int TILE = KT * HD * 2;
  constexpr int QP = HD + 8;
  const int qtile = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int G = nq / nkv;
  const int TPT = 64 / G;  // tokens per q tile
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = cu_q[seq], qlen = cu_q[seq + 1] - q0;
  const int k0 = cu_k[seq], klen = cu_k[seq + 1] - k0;
  const int tok_begin = qtile * TPT;
  if (tok_begin >= qlen) return;
  const int tok_end = min(tok_begin + TPT, qlen);
  const int pos_lo = klen - qlen + tok_begin, pos_hi = klen - qlen + tok_end - 1;
  const int key_end = causal ? min(klen, pos_hi + 1) : klen;
  const int key_begin = (window > 0 && causal) ? max(0, pos_lo - window + 1) : 0;
  const int t_begin = key_begin / KT, t_end = (key_end + KT - 1) / KT;
  const int nt = t_end - t_begin;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* ring = smem;
  bf16* qs = reinterpret_cast<bf16*>(smem + STAGES * 2 * TILE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(qs + 64 * QP);
  __shared__ int abort_flag;
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) nvb::mbar_init(&bars[s], 1);
    nvb::fence_mbar_init();
  }
  for (int idx = tid; idx < 64 * (HD / 8); idx += blockDim.x) {
    const int r = idx / (HD / 8), c = idx % (HD / 8);
    const int j = tok_begin + r / G;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (j < qlen) v = *reinterpret_cast<const uint4*>(q + (long)(q0 + j) * q_tok_stride + (kvh * G + r % G) * HD + c * 8);
    *reinterpret_cast<uint4*>(qs + r * QP + c * 8) = v;
  }
  __syncthreads();
  const int* bt = block_tables != nullptr ? block_tables + (long)seq * bt_stride : nullptr;
  auto issue = [&](int t, int st) {
    const int tok = t * KT;
    int row = 0;
    if (paged) row = (bt[tok / block_size] * nkv + kvh) * block_size + (tok % block_size);
    issue_tile<HD>(ring + st * 2 * TILE, ring + st * 2 * TILE + TILE, &kmap, &vmap, &bars[st], paged != 0, row,
                   nq + kvh, nq + nkv + kvh, k0 + tok);
  };
  if (tid == 0) {
    nvb::tma_prefetch_desc(&kmap);
    nvb::tma_prefetch_desc(&vmap);
    for (int i = 0; i < STAGES && i < nt; ++i) issue(t_begin + i, i);
  }
  const int g = lane >> 2, c4 = lane & 3;
  // absolute positions of this thread's two rows
  int rpos[2], rvalid[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = warp * 16 + g + h * 8;
    const int j = tok_begin + r / G;
    rvalid[h] = j < qlen;
    rpos[h] = klen - qlen + j;
  }
  float o[HD / 8][4];
#pragma unroll
  for (int d = 0; d < HD / 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const uint32_t qs_addr = nvb::smem_u32(qs);
  bool aborted = false;

  for (int i = 0; i < nt; ++i) {
    const int st = i % STAGES;
    const bool ok = nvb::mbar_wait(&bars[st], (uint32_t)((i / STAGES) & 1), err, &abort_flag);
    if (__syncthreads_or(!ok)) { aborted = true; break; }
    const uint32_t kb = nvb::smem_u32(ring + st * 2 * TILE);
    const uint32_t vb = kb + TILE;
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t a[4];
      nvb::ldmatrix_x4(a[0], a[1], a[2], a[3],
                       qs_addr + ((warp * 16 + (lane & 15)) * QP + kk * 16 + (lane >> 4) * 8) * 2);
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int key = np * 16 + r + (mi >> 1) * 8;
        const int dim = kk * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        nvb::ldmatrix_x4(b0, b1, b2, b3, kb + tile_off<HD>(key, dim));
        nvb::mma_bf16_16816(s[2 * np], a, b0, b1);
        nvb::mma_bf16_16816(s[2 * np + 1], a, b2, b3);
      }
    }
    const int tok0 = (t_begin + i) * KT;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int key = tok0 + n * 8 + 2 * c4 + (e & 1);
        float x = apply_cap(s[n][e] * scale, softcap) * kLog2e;
        bool valid = rvalid[h] && key < klen;
        if (causal) valid = valid && key <= rpos[h] && (window <= 0 || key > rpos[h] - window);
        if (!valid) x = -INFINITY;
        s[n][e] = x;
        mx[h] = fmaxf(mx[h], x);
      }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float nm = fmaxf(m_run[h], mx[h]);
      corr[h] = (nm == -INFINITY) ? 1.f : exp2f(m_run[h] - nm);
      m_run[h] = nm;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float p = (m_run[h] == -INFINITY) ? 0.f : exp2f(s[n][e] - m_run[h]);
        s[n][e] = p;
        rs[h] += p;
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) l_run[h] = l_run[h] * corr[h] + rs[h];
#pragma unroll
    for (int d = 0; d < HD / 8; ++d) {
      o[d][0] *= corr[0];
      o[d][1] *= corr[0];
      o[d][2] *= corr[1];
      o[d][3] *= corr[1];
    }
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t pa[4];
      pa[0] = nvb::pack_bf16x2(s[2 * ks][0], s[2 * ks][1]);
      pa[1] = nvb::pack_bf16x2(s[2 * ks][2], s[2 * ks][3]);
      pa[2] = nvb::pack_bf16x2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      pa[3] = nvb::pack_bf16x2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        const int key = ks * 16 + r + (mi & 1) * 8;
        const int dim = dp * 16 + (mi >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        nvb::ldmatrix_x4_trans(b0, b1, b2, b3, vb + tile_off<HD>(key, dim));
        nvb::mma_bf16_16816(o[2 * dp], pa, b0, b1);
        nvb::mma_bf16_16816(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();
    if (tid == 0 && i + STAGES < nt) issue(t_begin + i + STAGES, st);
  }
  if (aborted) {
    if (tid == 0)
      for (int s = 0; s < STAGES; ++s) nvb::mbar_wait(&bars[s], 0, nullptr, nullptr);
    return;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (!rvalid[h]) continue;
    const int r = warp * 16 + g + h * 8;
    const int j = tok_begin + r / G;
    const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
    bf16* dst = out + (long)(q0 + j) * o_tok_stride + (kvh * G + r % G) * HD;
#pragma unroll
    for (int d = 0; d < HD / 8; ++d)
      *reinterpret_cast<uint32_t*>(dst + d * 8 + 2 * c4) = nvb::pack_bf16x2(o[d][2 * h] * inv, o[d][2 * h + 1] * inv);
  }
}

// ============================================================================================ fallback
// CUDA-core path for head dims the tensor-core kernels do not instantiate (Gemma4 global layers use 512):
// one warp per (query token, head), online softmax over the keys.
__global__ void attn_generic_kernel(const bf16* __restrict__ q, long q_tok_stride, bf16* __restrict__ out,
                                    long o_tok_stride, const bf16* __restrict__ kc, const bf16* __restrict__ vc,
                                    long kv_tok_stride, const int* __restrict__ cu_q, const int* __restrict__ cu_k,
                                    const int* __restrict__ block_tables, int bt_stride, int paged, int nseq, int nq,
                                    int nkv, int HD, int block_size, float scale, float softcap, int window,
                                    int causal, int total_q) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= total_q * nq) return;
  const int tq = warp_global / nq, h = warp_global % nq;
  int seq = 0;
  while (seq + 1 < nseq && cu_q[seq + 1] <= tq) ++seq;
  const int q0 = cu_q[seq], qlen = cu_q[seq + 1] - q0;
  const int k0 = cu_k[seq], klen = cu_k[seq + 1] - k0;
  const int j = tq - q0;
  const int pos = klen - qlen + j;
  const int kvh = h / (nq / nkv);
  const int key_end = causal ? pos + 1 : klen;
  const int key_begin = (causal && window > 0) ? max(0, pos - window + 1) : 0;
  float qv[16], acc[16];
  const int per = (HD + 31) / 32;  // dims per lane; lanes past HD idle when HD < 32
  for (int i = 0; i < per; ++i) {
    const int dim = lane + 32 * i;
    qv[i] = dim < HD ? __bfloat162float(q[(long)tq * q_tok_stride + h * HD + dim]) : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int key = key_begin; key < key_end; ++key) {
    const bf16 *kr, *vr;
    if (paged) {
      const int blk = block_tables[(long)seq * bt_stride + key / block_size];
      const long off = (((long)blk * nkv + kvh) * block_size + key % block_size) * HD;
      kr = kc + off;
      vr = vc + off;
    } else {
      kr = kc + (long)(k0 + key) * kv_tok_stride + kvh * HD;
      vr = vc + (long)(k0 + key) * kv_tok_stride + kvh * HD;
    }
    float d = 0.f;
    for (int i = 0; i < per; ++i)
      if (lane + 32 * i < HD) d += qv[i] * __bfloat162float(kr[lane + 32 * i]);
    d = nvb::warp_sum(d);
    const float x = apply_cap(d * scale, softcap);
    const float nm = fmaxf(m, x);
    const float corr = expf(m - nm), p = expf(x - nm);
    l = l * corr + p;
    for (int i = 0; i < per; ++i)
      if (lane + 32 * i < HD) acc[i] = acc[i] * corr + p * __bfloat162float(vr[lane + 32 * i]);
    m = nm;
  }
  for (int i = 0; i < per; ++i)
    if (lane + 32 * i < HD)
      out[(long)tq * o_tok_stride + h * HD + lane + 32 * i] = __float2bfloat16(l > 0.f ? acc[i] / l : 0.f);
}

template <int HD, int STAGES>
size_t decode_smem() {
  return 1024 + STAGES * 2 * KT * HD * 2 + 16 * (HD + 8) * 2 + STAGES * 8 + 64;
}
template <int HD, int STAGES>
size_t prefill_smem() {
  return 1024 + STAGES * 2 * KT * HD * 2 + 64 * (HD + 8) * 2 + STAGES * 8 + 64;
}

}  // namespace
