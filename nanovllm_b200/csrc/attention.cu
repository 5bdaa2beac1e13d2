// Paged attention for sm_100a: split-KV flash decoding and varlen (paged or contiguous) prefill.
//
// Reference semantics: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/Attention.java:245-396
// (online-softmax over paged slots; causal end kLen - qLen + qi + 1; optional sliding-window start
// absQ - W + 1; GQA head mapping kvh = h / (nq / nkv); score = dot(q, k) * scale) and
// BidirectionalAttention.java:71-145 (no mask).  Logit soft-capping cap * tanh(s / cap) is applied to the
// scaled score when ``softcap > 0``.
//
// Data movement: K/V tiles of 64 keys x head_dim are fetched by TMA (cp.async.bulk.tensor, no multicast) with
// the 128-byte swizzle into a multi-stage ring tracked by mbarriers; one thread issues the copies.  The
// cache layout is [num_blocks, nkv, block_size, hd], so a 64-key tile of one head is one contiguous
// 64 x hd box.  The contractions run on mma.sync m16n8k16 (bf16 in, fp32 accumulate): decode attention is
// bound by HBM bytes, not by the tensor pipe, and the register-resident online softmax keeps the whole tile
// in registers.
//
// Decode: one CTA per (kv-split, kv head, sequence); the G = nq / nkv query heads of the group are the
// 16-row M tile; the four warps split the 64 keys of each tile and merge their (max, sum, O) at the end.
// Splits write fp32 partials + log2-sum-exp to a scratch buffer that attn_combine merges.
// Prefill: one CTA per (64-row q tile, kv head, sequence); rows are (token, head-in-group) pairs so the K/V
// tile is shared by all G heads; each warp owns 16 rows.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "tma_host.h"

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
template <int HD, int STAGES>
__global__ void __launch_bounds__(128) paged_decode_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ q,
    const int* __restrict__ block_tables, int bt_stride, const int* __restrict__ ctx_lens, bf16* __restrict__ out,
    float* __restrict__ part_o, float* __restrict__ part_lse, int nq, int nkv, int block_size, float scale,
    float softcap, int window, int part_tiles, int* err) {
  constexpr int TILE = KT * HD * 2;
  constexpr int QP = HD + 8;  // padded Q row (elements)
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int nsplit = gridDim.x;
  const int G = nq / nkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ctx = ctx_lens[b];
  const int ntiles = (ctx + KT - 1) / KT;
  const int win_start = window > 0 ? max(0, ctx - window) : 0;
  const int t_begin = max(split * part_tiles, win_start / KT);
  const int t_end = min((split + 1) * part_tiles, ntiles);
  if (t_begin >= t_end) return;  // the combine step skips splits without keys
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
}

__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                    const int* __restrict__ ctx_lens, bf16* __restrict__ out, int nq, int nsplit,
                                    int HD, int part_tiles, int window) {
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
  const int per = HD / 32;
  for (int i = 0; i < per; ++i) {
    qv[i] = __bfloat162float(q[(long)tq * q_tok_stride + h * HD + lane + 32 * i]);
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
    for (int i = 0; i < per; ++i) d += qv[i] * __bfloat162float(kr[lane + 32 * i]);
    d = nvb::warp_sum(d);
    const float x = apply_cap(d * scale, softcap);
    const float nm = fmaxf(m, x);
    const float corr = expf(m - nm), p = expf(x - nm);
    l = l * corr + p;
    for (int i = 0; i < per; ++i) acc[i] = acc[i] * corr + p * __bfloat162float(vr[lane + 32 * i]);
    m = nm;
  }
  for (int i = 0; i < per; ++i)
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

int* err_ptr(c10::optional<torch::Tensor>& e) { return e.has_value() ? e->data_ptr<int>() : nullptr; }

void check_kv(const torch::Tensor& c, int64_t nkv, int64_t hd) {
  TORCH_CHECK(c.is_cuda() && c.scalar_type() == at::kBFloat16 && c.is_contiguous(), "cache must be contiguous bf16");
  TORCH_CHECK(c.dim() == 4 && c.size(1) == nkv && c.size(3) == hd, "cache must be [num_blocks, nkv, block, hd]");
  TORCH_CHECK(c.size(2) % KT == 0, "block size must be a multiple of 64");
}

}  // namespace

// q [B, nq, hd]; caches [num_blocks, nkv, block, hd]; out [B, nq, hd]; part_o [B, nq, nsplit, hd] fp32;
// part_lse [B, nq, nsplit] fp32 (unused when nsplit == 1).
void paged_decode_cuda(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                       torch::Tensor ctx_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_lse,
                       double scale, double softcap, int64_t window, int64_t part_tiles, int64_t nsplit,
                       c10::optional<torch::Tensor> err) {
  const int B = q.size(0), nq = q.size(1), hd = q.size(2);
  const int nkv = k_cache.size(1), block_size = k_cache.size(2);
  TORCH_CHECK(q.is_contiguous() && out.is_contiguous(), "q/out must be contiguous");
  TORCH_CHECK(nq % nkv == 0 && nq / nkv <= 16, "GQA group must be <= 16");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt, "int32 metadata");
  check_kv(k_cache, nkv, hd);
  check_kv(v_cache, nkv, hd);
  if (B == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (hd != 64 && hd != 128 && hd != 256) {
    // generic path: treat each sequence as a 1-token query
    auto cu_q = torch::arange(0, B + 1, ctx_lens.options());
    auto cu_k = torch::zeros({B + 1}, ctx_lens.options());
    cu_k.slice(0, 1).copy_(torch::cumsum(ctx_lens, 0));
    const int total = B * nq;
    attn_generic_kernel<<<(total * 32 + 127) / 128, 128, 0, stream>>>(
        reinterpret_cast<const bf16*>(q.data_ptr()), (long)nq * hd, reinterpret_cast<bf16*>(out.data_ptr()),
        (long)nq * hd, reinterpret_cast<const bf16*>(k_cache.data_ptr()),
        reinterpret_cast<const bf16*>(v_cache.data_ptr()), 0, cu_q.data_ptr<int>(), cu_k.data_ptr<int>(),
        block_tables.data_ptr<int>(), block_tables.size(1), 1, B, nq, nkv, hd, block_size, (float)scale,
        (float)softcap, (int)window, 1, B);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const uint64_t rows = (uint64_t)k_cache.size(0) * nkv * block_size;
  CUtensorMap km = nvb::make_tmap_2d_bf16(k_cache.data_ptr(), rows, hd, hd, KT);
  CUtensorMap vm = nvb::make_tmap_2d_bf16(v_cache.data_ptr(), rows, hd, hd, KT);
  dim3 grid((unsigned)nsplit, nkv, B);
  auto* qp = reinterpret_cast<const bf16*>(q.data_ptr());
  auto* op = reinterpret_cast<bf16*>(out.data_ptr());
  float* po = nsplit > 1 ? part_o.data_ptr<float>() : nullptr;
  float* pl = nsplit > 1 ? part_lse.data_ptr<float>() : nullptr;
  int* e = err_ptr(err);
#define LAUNCH_DEC(HD_, ST_)                                                                                     \
  {                                                                                                              \
    auto kern = paged_decode_kernel<HD_, ST_>;                                                                   \
    size_t sm = decode_smem<HD_, ST_>();                                                                         \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);                            \
    kern<<<grid, 128, sm, stream>>>(km, vm, qp, block_tables.data_ptr<int>(), block_tables.size(1),              \
                                    ctx_lens.data_ptr<int>(), op, po, pl, nq, nkv, block_size, (float)scale,     \
                                    (float)softcap, (int)window, (int)part_tiles, e);                            \
  }
  if (hd == 64) LAUNCH_DEC(64, 4)
  else if (hd == 128) LAUNCH_DEC(128, 3)
  else LAUNCH_DEC(256, 2)
#undef LAUNCH_DEC
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (nsplit > 1) {
    attn_combine_kernel<<<dim3(nq, B), hd < 128 ? hd : 128, 0, stream>>>(
        po, pl, ctx_lens.data_ptr<int>(), op, nq, (int)nsplit, hd, (int)part_tiles, (int)window);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// Varlen prefill.  paged: K/V from the caches through block_tables.  contiguous (paged == false): K/V are
// heads nq..nq+2nkv of the packed qkv tensor ``kv_src`` [T, (nq + 2 nkv) * hd] (BERT, no cache).
void prefill_attention_cuda(torch::Tensor q, torch::Tensor out, torch::Tensor cu_q, torch::Tensor cu_k,
                            int64_t max_q, c10::optional<torch::Tensor> k_cache, c10::optional<torch::Tensor> v_cache,
                            c10::optional<torch::Tensor> block_tables, c10::optional<torch::Tensor> kv_src,
                            int64_t nq, int64_t nkv, int64_t hd, double scale, double softcap, int64_t window,
                            bool causal, c10::optional<torch::Tensor> err) {
  const int nseq = cu_q.size(0) - 1;
  if (nseq <= 0 || max_q <= 0) return;
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1, "q/out inner dim must be contiguous");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && cu_k.scalar_type() == at::kInt, "cu_seqlens must be int32");
  const bool paged = k_cache.has_value();
  const long q_stride = q.dim() == 3 ? q.stride(0) : q.stride(0);
  const long o_stride = out.dim() == 3 ? out.stride(0) : out.stride(0);
  auto stream = at::cuda::getCurrentCUDAStream();
  int* e = err_ptr(err);
  const int G = nq / nkv;
  TORCH_CHECK(nq % nkv == 0 && 64 % G == 0, "GQA group must divide 64");
  int block_size = 1;
  const int* bt = nullptr;
  int bt_stride = 0;
  if (paged) {
    check_kv(*k_cache, nkv, hd);
    check_kv(*v_cache, nkv, hd);
    TORCH_CHECK(block_tables.has_value(), "block tables required for paged prefill");
    block_size = k_cache->size(2);
    bt = block_tables->data_ptr<int>();
    bt_stride = block_tables->size(1);
  } else {
    TORCH_CHECK(kv_src.has_value() && kv_src->stride(-1) == 1, "kv_src required for contiguous prefill");
  }
  if (hd != 64 && hd != 128 && hd != 256) {
    const int total_q = q.size(0);
    const bf16* kc = paged ? reinterpret_cast<const bf16*>(k_cache->data_ptr())
                           : reinterpret_cast<const bf16*>(kv_src->data_ptr()) + nq * hd;
    const bf16* vc = paged ? reinterpret_cast<const bf16*>(v_cache->data_ptr())
                           : reinterpret_cast<const bf16*>(kv_src->data_ptr()) + (nq + nkv) * hd;
    const long kvs = paged ? 0 : kv_src->stride(0);
    attn_generic_kernel<<<((long)total_q * nq * 32 + 127) / 128, 128, 0, stream>>>(
        reinterpret_cast<const bf16*>(q.data_ptr()), q_stride, reinterpret_cast<bf16*>(out.data_ptr()), o_stride, kc,
        vc, kvs, cu_q.data_ptr<int>(), cu_k.data_ptr<int>(), bt, bt_stride, paged ? 1 : 0, nseq, nq, nkv, hd,
        block_size, (float)scale, (float)softcap, (int)window, causal ? 1 : 0, total_q);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  CUtensorMap km, vm;
  if (paged) {
    const uint64_t rows = (uint64_t)k_cache->size(0) * nkv * block_size;
    km = nvb::make_tmap_2d_bf16(k_cache->data_ptr(), rows, hd, hd, KT);
    vm = nvb::make_tmap_2d_bf16(v_cache->data_ptr(), rows, hd, hd, KT);
  } else {
    const uint64_t T = kv_src->size(0);
    const uint64_t heads = nq + 2 * nkv;
    uint64_t dims[3] = {(uint64_t)hd, heads, T};
    uint64_t strides[2] = {(uint64_t)hd * 2, (uint64_t)kv_src->stride(0) * 2};
    uint32_t box[3] = {64, 1, KT};
    km = nvb::make_tmap(kv_src->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box);
    vm = km;
  }
  const int TPT = 64 / G;
  dim3 grid((unsigned)((max_q + TPT - 1) / TPT), nkv, nseq);
  auto* qp = reinterpret_cast<const bf16*>(q.data_ptr());
  auto* op = reinterpret_cast<bf16*>(out.data_ptr());
#define LAUNCH_PF(HD_, ST_)                                                                                      \
  {                                                                                                              \
    auto kern = prefill_attn_kernel<HD_, ST_>;                                                                   \
    size_t sm = prefill_smem<HD_, ST_>();                                                                        \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);                            \
    kern<<<grid, 128, sm, stream>>>(km, vm, qp, q_stride, op, o_stride, cu_q.data_ptr<int>(),                    \
                                    cu_k.data_ptr<int>(), bt, bt_stride, paged ? 1 : 0, nq, nkv, block_size,     \
                                    (float)scale, (float)softcap, (int)window, causal ? 1 : 0, e);               \
  }
  if (hd == 64) LAUNCH_PF(64, 4)
  else if (hd == 128) LAUNCH_PF(128, 2)
  else LAUNCH_PF(256, 2)
#undef LAUNCH_PF
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
