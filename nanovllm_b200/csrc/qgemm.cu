// GGUF dequant-fused GEMMs for packed weights (decode-sized M on tcgen05, plus a dequant kernel for prefill).
//
// The reference multiplies quantized weights on the CPU by decoding each GGML block inside its matmul loops
// (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/internal/GgufDequant.java:15-90 and the per-type
// kernels it dispatches to).  Here the packed bytes stay packed in HBM -- that is the point: a decode GEMM is a
// weight stream, and 4.5-bit weights stream 3.5x faster than bf16 ones.
//
// Layout (written once at load time by ops/quant.py, a lossless byte permutation of the GGUF blocks): the
// weight is cut into tiles of 128 rows x 256 K elements ("row steps"); within a row step the block fields are
// stored structure-of-arrays (all scales first, then all quant bytes) so every field is 2/4/16-byte aligned
// (FP4 codes are regrouped pair-adjacent: byte t of a block holds elements 2t and 2t+1),
// and the row step is padded to a multiple of 16 bytes (bytes per row step: Q4_0 / IQ4_NL / MXFP4 / NVFP4 /
// Q4_K / IQ4_XS 144, Q4_1 160, Q5_K 176, Q6_K 224, Q8_0 272).  Tiles are stored [N/128][K/256][128 rows]
// [row step], so one row-step tile is ONE contiguous run of 128 * bprs bytes: a single bulk copy
// (cp.async.bulk, no tensor map, no multicast) per pipeline stage, and perfect DRAM streaming.
//
// qgemm_decode_kernel<TYPE, BN> (swap-AB like the bf16 decode GEMM: 128 weight rows = MMA M, tokens = MMA N):
//   warp 0 lane 0   producer: the CTA's activation slice [BN x Krange] is loaded ONCE by TMA and stays
//                   resident in shared memory; the packed weight tiles stream through a ring of row steps;
//   warps 4..11     dequant: first convert the resident activation slice to f16 in place, then two threads per
//                   weight row decode each 64-wide K sub-step into an f16 128 x 64 tile in the UMMA
//                   SWIZZLE_128B K-major layout (FP4: hardware e2m1x2 -> f16x2 conversion times the block scale,
//                   exact; 4/8-bit integer codes: 1024.0-magic f16 halves, one subtract, one fma), then
//                   fence.proxy.async + mbarrier arrive;
//   warp 1 lane 0   tcgen05.mma (kind::f16 with f16 operands, fp32 accumulator in TMEM) on each tile;
//   warps 0..3      epilogue: tcgen05.ld, bf16 output (one split) or fp32 split-K partials [S][M][N] that the
//                   consumer sums exactly like the bf16 decode GEMM's.
// Every wait is bounded (nvb::mbar_wait -> device error word) so a broken pipeline returns instead of hanging.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cuda.h>
#include <cuda_fp16.h>
#include "common.cuh"
#include "launch.h"
#include "tma_host.h"

namespace {

using bf16 = __nv_bfloat16;
constexpr int QBM = 128, QBK = 64, QSTEP = 256;
constexpr int kQXBytes = 128 * 1024;    // resident activation slice budget
constexpr int kQRingBytes = 224 * 1024;  // activation slice + bf16 tiles + packed ring
constexpr int kQAStages = 2;             // dequantized bf16 tiles in flight

// GGML type ids (the GGUF on-disk codes)
constexpr int T_Q4_0 = 2, T_Q4_1 = 3, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ4_NL = 20,
              T_IQ4_XS = 23, T_MXFP4 = 39, T_NVFP4 = 40;

__host__ __device__ constexpr int row_step_bytes(int t) {
  return t == T_Q4_1 ? 160 : t == T_Q8_0 ? 272 : t == T_Q5_K ? 176 : t == T_Q6_K ? 224 : 144;
}

__device__ __forceinline__ float h2f(const uint8_t* p) {
  return __half2float(*reinterpret_cast<const __half*>(p));
}

// value of a ue4m3 scale byte, halved (the FP4 grid below is stored doubled)
__device__ __forceinline__ float ue4m3_half(uint32_t x) {
  if (x == 0 || x == 0x7F) return 0.f;
  const int e = (x >> 3) & 0xF, m = x & 7;
  if (e == 0) return (float)m * 0x1p-10f;
  return (float)(8 + m) * __int_as_float((e - 11 + 127) << 23);
}

// 2^(e - 128): the e8m0 scale, halved
__device__ __forceinline__ float e8m0_half(uint32_t e) {
  if (e >= 2) return __int_as_float((int)(e - 1) << 23);
  return __int_as_float(e == 1 ? (1 << 22) : (1 << 21));
}

struct Luts {
  float fp4[16];   // e2m1 grid doubled
  float iq4[16];   // IQ4_NL non-linear grid
};

__device__ __forceinline__ void load8(const uint8_t* p, uint8_t (&b)[8]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const uint8_t* s = reinterpret_cast<const uint8_t*>(&v);
#pragma unroll
  for (int j = 0; j < 8; ++j) b[j] = s[j];
}

// Decode elements [e0, e0 + 8) (e0 a multiple of 8) of one 256-element row step in the repacked layout.
template <int TYPE>
__device__ __forceinline__ void decode8(const uint8_t* __restrict__ p, int e0, const Luts& L, float (&v)[8]) {
  if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
    const int sb = e0 >> 5, i0 = e0 & 31;
    const float d = h2f(p), dmin = h2f(p + 2);
    const uint8_t* q = p + 4;
    int sc, mn;
    if (sb < 4) {
      sc = q[sb] & 63;
      mn = q[sb + 4] & 63;
    } else {
      sc = (q[sb + 4] & 0xF) | ((q[sb - 4] >> 6) << 4);
      mn = (q[sb + 4] >> 4) | ((q[sb] >> 6) << 4);
    }
    const float ds = d * (float)sc, dm = dmin * (float)mn;
    const uint8_t* qs = p + (TYPE == T_Q4_K ? 16 : 48) + (sb >> 1) * 32 + i0;
    uint8_t b[8];
    load8(qs, b);
    uint8_t h[8];
    if constexpr (TYPE == T_Q5_K) load8(p + 16 + i0, h);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int n = (sb & 1) ? (b[j] >> 4) : (b[j] & 0xF);
      if constexpr (TYPE == T_Q5_K) n += 16 * ((h[j] >> sb) & 1);
      v[j] = ds * (float)n - dm;
    }
  } else if constexpr (TYPE == T_Q6_K) {
    const int hh = e0 >> 7, w = e0 & 127, k = w >> 5, l0 = w & 31;
    uint8_t ql[8], qh[8];
    load8(p + hh * 64 + (k & 1) * 32 + l0, ql);
    load8(p + 128 + hh * 32 + l0, qh);
    const float s = (float)reinterpret_cast<const int8_t*>(p + 192)[hh * 8 + 2 * k + (l0 >> 4)];
    const float d = h2f(p + 208);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int nib = (k >> 1) ? (ql[j] >> 4) : (ql[j] & 0xF);
      const int q = nib | (((qh[j] >> (2 * k)) & 3) << 4);
      v[j] = d * ((float)(q - 32) * s);
    }
  } else if constexpr (TYPE == T_Q8_0) {
    const int b = e0 >> 5, i0 = e0 & 31;
    const float d = h2f(p + 2 * b);
    uint8_t q[8];
    load8(p + 16 + b * 32 + i0, q);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = d * (float)(int8_t)q[j];
  } else if constexpr (TYPE == T_NVFP4) {
    // repacked codes are pair-adjacent: byte t of a 64-element block holds elements 2t (low) and 2t+1 (high)
    const int blk = e0 >> 6, ei = e0 & 63;
    const float d = ue4m3_half(p[blk * 4 + (ei >> 4)]);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p + 16 + blk * 32 + (ei >> 1));
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = d * L.fp4[(w >> (4 * j)) & 0xF];
  } else if constexpr (TYPE == T_MXFP4) {
    const int b = e0 >> 5, ei = e0 & 31;
    const float d = e8m0_half(p[b]);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p + 16 + b * 16 + (ei >> 1));
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = d * L.fp4[(w >> (4 * j)) & 0xF];
  } else {
    // 32-element blocks with 16 quant bytes: elements 0..15 low nibbles, 16..31 high nibbles
    const int b = e0 >> 5, i0 = e0 & 31;
    const int qoff = (TYPE == T_Q4_1) ? 32 : 16;
    uint8_t q[8];
    load8(p + qoff + b * 16 + (i0 & 15), q);
    const bool hi = i0 >= 16;
    if constexpr (TYPE == T_Q4_0) {
      const float d = h2f(p + 2 * b);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = d * (float)((hi ? (q[j] >> 4) : (q[j] & 0xF)) - 8);
    } else if constexpr (TYPE == T_Q4_1) {
      const float d = h2f(p + 2 * b), m = h2f(p + 16 + 2 * b);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = d * (float)(hi ? (q[j] >> 4) : (q[j] & 0xF)) + m;
    } else if constexpr (TYPE == T_IQ4_NL) {
      const float d = h2f(p + 2 * b);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = d * L.iq4[hi ? (q[j] >> 4) : (q[j] & 0xF)];
    } else {  // IQ4_XS
      const float d = h2f(p);
      const uint32_t sh = *reinterpret_cast<const uint16_t*>(p + 2);
      const int ls = ((((int)p[4 + (b >> 1)] >> (4 * (b & 1))) & 0xF) | ((int)((sh >> (2 * b)) & 3) << 4)) - 32;
      const float dl = d * (float)ls;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = dl * L.iq4[hi ? (q[j] >> 4) : (q[j] & 0xF)];
    }
  }
}

__constant__ float c_fp4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
__constant__ float c_iq4[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

// the grids are read with data-dependent indices: shared memory serves 16 distinct words without serialising
__device__ __forceinline__ void init_luts(Luts& L) {
  if (threadIdx.x < 16) {
    L.fp4[threadIdx.x] = c_fp4[threadIdx.x];
    L.iq4[threadIdx.x] = c_iq4[threadIdx.x];
  }
}

// ------------------------------------------------------------------------------------------ f16 chunk decode
// The fused GEMM multiplies in f16 (kind::f16 with f16 A and B): every FP4 value times its ue4m3 scale has at
// most 6 significant bits, so the f16 weights are exact, and the K-quant formula keeps 11 mantissa bits instead
// of bf16's 8.  decode_h8 returns elements [e0, e0 + 8) of a row step as 8 f16 (one 16-byte smem chunk).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// eight e2m1 codes (4 bytes; low nibble -> low half of each f16x2) to four f16x2, hardware conversion
__device__ __forceinline__ void e2m1x8_to_h2(uint32_t w, uint32_t (&d)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]) : "r"(w));
}
__device__ __forceinline__ uint32_t f2_to_h2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ uint32_t h2_bcast(float v) { return f2_to_h2(v, v); }

// per f16 half: 1024.0 with the masked code bits as mantissa, (t & mask) | 0x6400
__device__ __forceinline__ uint32_t nib_pair(uint32_t t, uint32_t mask) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(t), "r"(mask), "r"(0x64006400u));  // (a & b) | c
  return d;
}

template <int TYPE>
__device__ __forceinline__ uint4 decode_h8(const uint8_t* __restrict__ p, int e0, const Luts& L) {
  uint4 o;
  if constexpr (TYPE == T_NVFP4 || TYPE == T_MXFP4) {
    uint32_t w;
    float sc;
    if constexpr (TYPE == T_NVFP4) {
      const int blk = e0 >> 6, ei = e0 & 63;
      w = *reinterpret_cast<const uint32_t*>(p + 16 + blk * 32 + (ei >> 1));
      sc = 2.f * ue4m3_half(p[blk * 4 + (ei >> 4)]);   // cvt yields the true e2m1 value (half the grid)
    } else {
      const int b = e0 >> 5, ei = e0 & 31;
      w = *reinterpret_cast<const uint32_t*>(p + 16 + b * 16 + (ei >> 1));
      sc = 2.f * e8m0_half(p[b]);
    }
    const uint32_t s2 = h2_bcast(sc);
    uint32_t h[4];
    e2m1x8_to_h2(w, h);
    o.x = hmul2(h[0], s2);
    o.y = hmul2(h[1], s2);
    o.z = hmul2(h[2], s2);
    o.w = hmul2(h[3], s2);
  } else if constexpr (TYPE == T_Q4_K) {
    const int sb = e0 >> 5, i0 = e0 & 31;
    const float d = h2f(p), dmin = h2f(p + 2);
    const uint8_t* q = p + 4;
    int sc, mn;
    if (sb < 4) {
      sc = q[sb] & 63;
      mn = q[sb + 4] & 63;
    } else {
      sc = (q[sb + 4] & 0xF) | ((q[sb - 4] >> 6) << 4);
      mn = (q[sb + 4] >> 4) | ((q[sb] >> 6) << 4);
    }
    const bool hi = sb & 1;
    // 1024 + code in each f16 half (high nibbles land 4 bits up: 1024 + 16 code, scale / 16)
    const float ds = d * (float)sc * (hi ? 0.0625f : 1.f);
    const uint32_t s2 = h2_bcast(ds), m2 = h2_bcast(-(dmin * (float)mn));
    const uint32_t mask = hi ? 0x00F000F0u : 0x000F000Fu;
    const uint2 w = *reinterpret_cast<const uint2*>(p + 16 + (sb >> 1) * 32 + i0);
    const uint32_t k1024 = 0x64006400u;
    o.x = hfma2(hsub2(nib_pair(prmt(w.x, 0, 0x4140), mask), k1024), s2, m2);
    o.y = hfma2(hsub2(nib_pair(prmt(w.x, 0, 0x4342), mask), k1024), s2, m2);
    o.z = hfma2(hsub2(nib_pair(prmt(w.y, 0, 0x4140), mask), k1024), s2, m2);
    o.w = hfma2(hsub2(nib_pair(prmt(w.y, 0, 0x4342), mask), k1024), s2, m2);
  } else if constexpr (TYPE == T_Q8_0) {
    const int b = e0 >> 5, i0 = e0 & 31;
    const uint32_t s2 = h2_bcast(h2f(p + 2 * b));
    const uint2 w = *reinterpret_cast<const uint2*>(p + 16 + b * 32 + i0);
    const uint32_t x0 = w.x ^ 0x80808080u, x1 = w.y ^ 0x80808080u;  // two's complement -> offset binary
    const uint32_t k1152 = 0x64806480u;                                 // 1024 + 128
    o.x = hmul2(hsub2(prmt(x0, 0x64646464u, 0x4140), k1152), s2);
    o.y = hmul2(hsub2(prmt(x0, 0x64646464u, 0x4342), k1152), s2);
    o.z = hmul2(hsub2(prmt(x1, 0x64646464u, 0x4140), k1152), s2);
    o.w = hmul2(hsub2(prmt(x1, 0x64646464u, 0x4342), k1152), s2);
  } else {
    float v[8];
    decode8<TYPE>(p, e0, L, v);
    o.x = f2_to_h2(v[0], v[1]);
    o.y = f2_to_h2(v[2], v[3]);
    o.z = f2_to_h2(v[4], v[5]);
    o.w = f2_to_h2(v[6], v[7]);
  }
  return o;
}

// 1-D bulk copy global -> shared (no tensor map, no multicast); completion counted on ``bar``.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          nvb::smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(nvb::smem_u32(bar))
      : "memory");
}

struct QArgs {
  int N, M, K;
  int ksteps;       // K / 256
  int kper;         // row steps per split (the resident activation slice covers kper * 256 columns)
  int S;            // splits
  int ws;           // packed ring stages
  int bprs;         // bytes per row step
  const uint8_t* w; // tile-major packed weight
  bf16* out;
  long out_ld;
  float* partial;
  int* err;
};

__host__ __device__ constexpr uint32_t q_pow2_cols(int n) {
  uint32_t c = 32;
  while (c < (uint32_t)n) c <<= 1;
  return c;
}

// kind::f16 instruction descriptor with f16 A and B, f32 accumulator, both K-major
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

constexpr int kQDequantWarps = 8;
constexpr int kQThreads = 128 + 32 * kQDequantWarps;

template <int TYPE, int BN>
__global__ void __launch_bounds__(kQThreads, 1) qgemm_decode_kernel(const __grid_constant__ CUtensorMap xmap, QArgs a) {
  constexpr uint32_t A_TILE = QBM * QBK * 2;  // 16 KB f16 tile
  constexpr uint32_t X_BOX = BN * QBK * 2;    // one [BN x 64] activation box
  constexpr uint32_t TMEM_COLS = q_pow2_cols(BN);
  constexpr uint32_t IDESC = idesc_f16_f32(QBM, BN);
  const uint32_t stage_bytes = (uint32_t)a.bprs * QBM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xres = smem;                                           // kper * 4 boxes
  uint8_t* atile = xres + (size_t)a.kper * 4 * X_BOX;             // kQAStages f16 tiles (1 KB aligned)
  uint8_t* wring = atile + (size_t)kQAStages * A_TILE;            // ws packed stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(wring + (size_t)a.ws * stage_bytes);
  uint64_t* xbar = bars;
  uint64_t* xready = bars + 1;
  uint64_t* wfull = bars + 2;
  uint64_t* wempty = wfull + a.ws;
  uint64_t* afull = wempty + a.ws;
  uint64_t* aempty = afull + kQAStages;
  uint64_t* tfull = aempty + kQAStages;
  __shared__ Luts luts;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.x / a.S, split = blockIdx.x % a.S;
  const int row0 = group * QBM;
  const int ks0 = split * a.kper;
  const int ks1 = min(a.ksteps, ks0 + a.kper);
  const int nks = ks1 - ks0;

  init_luts(luts);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    nvb::mbar_init(xbar, 1);
    nvb::mbar_init(xready, kQDequantWarps);
    for (int s = 0; s < a.ws; ++s) {
      nvb::mbar_init(&wfull[s], 1);
      nvb::mbar_init(&wempty[s], kQDequantWarps);
    }
    for (int s = 0; s < kQAStages; ++s) {
      nvb::mbar_init(&afull[s], kQDequantWarps);
      nvb::mbar_init(&aempty[s], 1);
    }
    nvb::mbar_init(tfull, 1);
    nvb::fence_mbar_init();
  }
  if (warp == 1) {
    nvb::tmem_alloc(&tmem_base_sh, TMEM_COLS);
    nvb::tmem_relinquish();
  }
  nvb::tc_fence_before();
  __syncthreads();
  nvb::tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  nvb::pdl_trigger();

  const uint8_t* wsrc = a.w + ((size_t)group * a.ksteps + ks0) * stage_bytes;
  if (warp == 0) {
    if (lane == 0) {
      // packed weights are never written by earlier kernels: the first ring streams in before the dependency
      const int pre = nks < a.ws ? nks : a.ws;
      for (int i = 0; i < pre; ++i) {
        nvb::mbar_arrive_expect_tx(&wfull[i], stage_bytes);
        bulk_load(wring + (size_t)i * stage_bytes, wsrc + (size_t)i * stage_bytes, stage_bytes, &wfull[i]);
      }
      nvb::tma_prefetch_desc(&xmap);
      nvb::pdl_wait();
      nvb::mbar_arrive_expect_tx(xbar, (uint32_t)nks * 4 * X_BOX);
      for (int b = 0; b < nks * 4; ++b)
        nvb::tma_load_2d(xres + (size_t)b * X_BOX, &xmap, xbar, ks0 * QSTEP + b * QBK, 0);
      for (int i = pre; i < nks; ++i) {
        const int s = i % a.ws;
        if (!nvb::mbar_wait(&wempty[s], ((i / a.ws) & 1u) ^ 1u, a.err, &abort_flag)) break;
        nvb::mbar_arrive_expect_tx(&wfull[s], stage_bytes);
        bulk_load(wring + (size_t)s * stage_bytes, wsrc + (size_t)i * stage_bytes, stage_bytes, &wfull[s]);
      }
    } else {
      nvb::pdl_wait();
    }
  } else if (warp == 1) {
    nvb::pdl_wait();
    if (lane == 0) {
      bool ok = nvb::mbar_wait(xready, 0, a.err, &abort_flag);
      for (int i = 0; ok && i < nks; ++i) {
        for (int sub = 0; sub < 4; ++sub) {
          const int u = i * 4 + sub, t = u % kQAStages;
          if (!nvb::mbar_wait(&afull[t], (u / kQAStages) & 1u, a.err, &abort_flag)) {
            ok = false;
            break;
          }
          nvb::tc_fence_after();
          const uint32_t a_addr = nvb::smem_u32(atile + (size_t)t * A_TILE);
          const uint32_t b_addr = nvb::smem_u32(xres + (size_t)u * X_BOX);
#pragma unroll
          for (int kk = 0; kk < QBK / 16; ++kk)
            nvb::tc_mma_f16(tmem_base, nvb::sdesc_kmajor_sw128(a_addr + kk * 32), nvb::sdesc_kmajor_sw128(b_addr + kk * 32),
                            IDESC, (u > 0 || kk > 0) ? 1u : 0u);
          nvb::tc_commit(&aempty[t]);
        }
      }
      if (ok) nvb::tc_commit(tfull);
    }
  } else if (warp >= 4) {
    nvb::pdl_wait();
    const int dt = threadIdx.x - 128;       // 0 .. 32 * kQDequantWarps - 1
    bool ok = nvb::mbar_wait(xbar, 0, a.err, &abort_flag);
    if (ok) {
      // the resident activation slice becomes f16 in place (saturating; the layout is elementwise)
      const uint32_t xbytes = (uint32_t)nks * 4 * X_BOX;
      for (uint32_t off = (uint32_t)dt * 16; off < xbytes; off += 32 * kQDequantWarps * 16) {
        uint4 v = *reinterpret_cast<const uint4*>(xres + off);
        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = f2_to_h2(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xFFFF0000u));
        *reinterpret_cast<uint4*>(xres + off) = v;
      }
      nvb::fence_proxy_async();
    }
    __syncwarp();
    if (lane == 0) nvb::mbar_arrive(xready);
    // dequant: thread dt owns row dt % 128 of the tile, chunks [4h, 4h + 4) of each 64-wide sub-step
    const int r = dt & 127, h = dt >> 7;
    const uint32_t swz = (uint32_t)(r & 7);
    for (int i = 0; ok && i < nks; ++i) {
      const int s = i % a.ws;
      if (!nvb::mbar_wait(&wfull[s], (i / a.ws) & 1u, a.err, &abort_flag)) break;
      const uint8_t* p = wring + (size_t)s * stage_bytes + (size_t)r * a.bprs;
      for (int sub = 0; sub < 4; ++sub) {
        const int u = i * 4 + sub, t = u % kQAStages;
        if (u >= kQAStages && !nvb::mbar_wait(&aempty[t], ((u / kQAStages) & 1u) ^ 1u, a.err, &abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* dst = atile + (size_t)t * A_TILE + (size_t)r * 128;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = 4 * h + cc;
          const uint4 o = decode_h8<TYPE>(p, sub * QBK + c * 8, luts);
          *reinterpret_cast<uint4*>(dst + (((uint32_t)c ^ swz) << 4)) = o;
        }
        nvb::fence_proxy_async();  // generic-proxy stores -> visible to the tensor core's async proxy
        __syncwarp();
        if (lane == 0) nvb::mbar_arrive(&afull[t]);
      }
      __syncwarp();
      if (lane == 0) nvb::mbar_arrive(&wempty[s]);
    }
  } else {
    nvb::pdl_wait();  // warps 2, 3: epilogue only
  }

  if (warp < 4) {
    __syncwarp();
    int ok = 0;
    if (lane == 0) ok = nvb::mbar_wait(tfull, 0, a.err, &abort_flag) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    nvb::tc_fence_after();
    if (ok) {
      const int f = row0 + threadIdx.x;  // TMEM lane = weight row
      const uint32_t t_row = tmem_base + ((uint32_t)(warp * 32) << 16);
      constexpr int CH = BN < 64 ? BN : 64;
#pragma unroll 1
      for (int c = 0; c < BN; c += CH) {
        uint32_t v[CH];
#pragma unroll
        for (int q = 0; q < CH; q += 16) nvb::tmem_ld_32x32b_x16(t_row + c + q, v + q);
        nvb::tmem_ld_wait();
        nvb::reg_fence<CH>(v);
        if (f < a.N) {
          if (a.S == 1) {
#pragma unroll
            for (int j = 0; j < CH; ++j)
              if (c + j < a.M) a.out[(long)(c + j) * a.out_ld + f] = __float2bfloat16(__uint_as_float(v[j]));
          } else {
            float* dst = a.partial + (long)split * a.M * a.N + f;
#pragma unroll
            for (int j = 0; j < CH; ++j)
              if (c + j < a.M) dst[(long)(c + j) * a.N] = __uint_as_float(v[j]);
          }
        }
      }
    }
  }
  nvb::tc_fence_before();
  __syncthreads();
  nvb::tc_fence_after();
  if (warp == 1) nvb::tmem_dealloc(tmem_base, TMEM_COLS);
}

// Dense bf16 copy of a tile-major packed weight (prefill path: dequantize, then the tensor-core GEMM).
// One thread per 8 consecutive elements of one row.
template <int TYPE>
__global__ void qdequant_kernel(const uint8_t* __restrict__ w, int N, int K, int bprs, bf16* __restrict__ out) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ Luts luts;
  init_luts(luts);
  __syncthreads();
  const int ksteps = K / QSTEP;
  const long chunks = (long)N * (K / 8);
  for (long c = blockIdx.x * (long)blockDim.x + threadIdx.x; c < chunks; c += (long)gridDim.x * blockDim.x) {
    const int row = (int)(c / (K / 8));
    const int e = (int)(c % (K / 8)) * 8;
    const int ks = e / QSTEP;
    const uint8_t* p = w + (((size_t)(row / QBM) * ksteps + ks) * QBM + (row % QBM)) * bprs;
    float v[8];
    decode8<TYPE>(p, e % QSTEP, luts, v);
    uint4 o;
    o.x = nvb::pack_bf16x2(v[0], v[1]);
    o.y = nvb::pack_bf16x2(v[2], v[3]);
    o.z = nvb::pack_bf16x2(v[4], v[5]);
    o.w = nvb::pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(out + (size_t)row * K + e) = o;
  }
}

struct QPlan {
  int bn, kper, S, ws, bprs;
  size_t smem;
};

int q_num_sms() {
  static int n = -1;
  if (n < 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

bool q_type_supported(int t) {
  return t == T_Q4_0 || t == T_Q4_1 || t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_IQ4_NL ||
         t == T_IQ4_XS || t == T_MXFP4 || t == T_NVFP4;
}

// K split: the resident activation slice (BN x kper*256 bf16) must fit kQXBytes, the splits should give every SM
// a CTA, and the packed ring must keep at least two row steps.
QPlan q_plan(int M, int N, int K, int type, int sms) {
  QPlan p{};
  p.bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  p.bprs = row_step_bytes(type);
  const int ksteps = K / QSTEP, groups = (N + QBM - 1) / QBM;
  const int x_step = p.bn * QSTEP * 2;
  int kper = kQXBytes / x_step;
  if (kper < 1) kper = 1;
  const int s_fill = (sms + groups - 1) / groups;
  const int kper_fill = (ksteps + s_fill - 1) / s_fill;
  if (kper > kper_fill) kper = kper_fill;
  if (kper > ksteps) kper = ksteps;
  if (kper < 1) kper = 1;
  const int stage = QBM * p.bprs;
  int ws = 0;
  for (;;) {
    ws = (kQRingBytes - kper * x_step - kQAStages * QBM * QBK * 2) / stage;
    if (ws >= 2 || kper == 1) break;
    kper = (kper + 1) / 2;
  }
  if (ws > 12) ws = 12;
  p.kper = kper;
  p.S = (ksteps + kper - 1) / kper;
  p.ws = ws;
  p.smem = 1024 + (size_t)kper * x_step + (size_t)kQAStages * QBM * QBK * 2 + (size_t)ws * stage +
           (size_t)(2 + 2 * ws + 2 * kQAStages + 1) * 8 + 64;
  return p;
}

template <int TYPE, int BN>
void q_launch(const CUtensorMap& xm, const QArgs& a, const QPlan& p, cudaStream_t st) {
  auto kern = qgemm_decode_kernel<TYPE, BN>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  const int groups = (a.N + QBM - 1) / QBM;
  C10_CUDA_CHECK(nvb::launch(kern, dim3(groups * a.S), dim3(kQThreads), p.smem, st, xm, a));
}

template <int TYPE>
void q_launch_bn(const CUtensorMap& xm, const QArgs& a, const QPlan& p, cudaStream_t st) {
  switch (p.bn) {
    case 16: q_launch<TYPE, 16>(xm, a, p, st); break;
    case 32: q_launch<TYPE, 32>(xm, a, p, st); break;
    case 64: q_launch<TYPE, 64>(xm, a, p, st); break;
    case 128: q_launch<TYPE, 128>(xm, a, p, st); break;
    default: q_launch<TYPE, 256>(xm, a, p, st); break;
  }
}

template <int TYPE>
void q_dequant_launch(const uint8_t* w, int N, int K, int bprs, bf16* out, cudaStream_t st) {
  const long chunks = (long)N * (K / 8);
  int blocks = (int)((chunks + 255) / 256);
  const int cap = q_num_sms() * 16;
  if (blocks > cap) blocks = cap;
  C10_CUDA_CHECK(nvb::launch(qdequant_kernel<TYPE>, dim3(blocks), dim3(256), 0, st, w, N, K, bprs, out));
}

#define Q_DISPATCH(type, FN, ...)                                        \
  switch (type) {                                                        \
    case T_Q4_0: FN<T_Q4_0>(__VA_ARGS__); break;                         \
    case T_Q4_1: FN<T_Q4_1>(__VA_ARGS__); break;                         \
    case T_Q8_0: FN<T_Q8_0>(__VA_ARGS__); break;                         \
    case T_Q4_K: FN<T_Q4_K>(__VA_ARGS__); break;                         \
    case T_Q5_K: FN<T_Q5_K>(__VA_ARGS__); break;                         \
    case T_Q6_K: FN<T_Q6_K>(__VA_ARGS__); break;                         \
    case T_IQ4_NL: FN<T_IQ4_NL>(__VA_ARGS__); break;                     \
    case T_IQ4_XS: FN<T_IQ4_XS>(__VA_ARGS__); break;                     \
    case T_MXFP4: FN<T_MXFP4>(__VA_ARGS__); break;                       \
    case T_NVFP4: FN<T_NVFP4>(__VA_ARGS__); break;                       \
    default: TORCH_CHECK(false, "packed GEMM: unsupported GGML type ", type); \
  }

void q_check_packed(const torch::Tensor& w, int64_t type, int64_t N, int64_t K) {
  TORCH_CHECK(q_type_supported((int)type), "packed GEMM: unsupported GGML type ", type);
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kByte && w.is_contiguous(), "packed weight: contiguous uint8 on CUDA");
  TORCH_CHECK(K % QSTEP == 0 && N > 0, "packed weight: K must be a multiple of 256");
  const long tiles = (N + QBM - 1) / QBM;
  TORCH_CHECK(w.numel() == tiles * (K / QSTEP) * QBM * (long)row_step_bytes((int)type), "packed weight: size mismatch");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0, "packed weight must be 16-byte aligned");
}

}  // namespace

void splitk_sum_cuda(torch::Tensor parts, torch::Tensor out);  // gemm.cu

int64_t qgemm_splits_cuda(int64_t M, int64_t N, int64_t K, int64_t type) {
  if (M <= 0 || M > 256 || K % QSTEP != 0 || !q_type_supported((int)type)) return 1;
  return q_plan((int)M, (int)N, (int)K, (int)type, q_num_sms()).S;
}

int64_t qgemm_row_step_bytes(int64_t type) { return row_step_bytes((int)type); }

// y[M, N] = x[M, K] @ dequant(w)^T for decode-sized M (<= 256).  With more than one split the fp32 partials go
// to ``parts`` [S, M, N] (S from qgemm_splits) and, unless ``partial_out``, are summed into ``out``.
int64_t qgemm_cuda(torch::Tensor x, torch::Tensor w, int64_t type, int64_t N, int64_t K, torch::Tensor out,
                   c10::optional<torch::Tensor> parts, c10::optional<torch::Tensor> err, bool partial_out) {
  q_check_packed(w, type, N, K);
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.size(1) == K && x.stride(1) == 1,
              "packed GEMM: x must be bf16 [M, K] with contiguous rows");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0,
              "packed GEMM: x rows must be 16-byte aligned");
  const int M = (int)x.size(0);
  TORCH_CHECK(M >= 1 && M <= 256, "packed decode GEMM takes 1..256 rows (dequantize for prefill)");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(-1) == 1 && out.size(0) == M && out.size(1) == N,
              "packed GEMM: out must be bf16 [M, N]");
  const QPlan p = q_plan(M, (int)N, (int)K, (int)type, q_num_sms());
  TORCH_CHECK(p.smem <= 227 * 1024, "packed GEMM shared memory plan");
  QArgs a{};
  a.N = (int)N;
  a.M = M;
  a.K = (int)K;
  a.ksteps = (int)(K / QSTEP);
  a.kper = p.kper;
  a.S = p.S;
  a.ws = p.ws;
  a.bprs = p.bprs;
  a.w = w.data_ptr<uint8_t>();
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.out_ld = out.stride(0);
  a.err = err.has_value() ? err->data_ptr<int>() : nullptr;
  if (p.S > 1) {
    TORCH_CHECK(parts.has_value() && parts->is_cuda() && parts->scalar_type() == at::kFloat && parts->is_contiguous() &&
                    parts->numel() >= (long)p.S * M * N,
                "packed GEMM: fp32 partial buffer [S, M, N] required");
    a.partial = parts->data_ptr<float>();
  }
  CUtensorMap xm = nvb::make_tmap_2d_bf16(x.data_ptr(), M, K, x.stride(0), p.bn);
  auto st = at::cuda::getCurrentCUDAStream();
  Q_DISPATCH((int)type, q_launch_bn, xm, a, p, st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (p.S > 1 && !partial_out)
    splitk_sum_cuda(parts->view(-1).narrow(0, 0, (long)p.S * M * N).view({p.S, (long)M, (long)N}), out);
  return p.S;
}

void qdequant_cuda(torch::Tensor w, int64_t type, int64_t N, int64_t K, torch::Tensor out) {
  q_check_packed(w, type, N, K);
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) == N &&
                  out.size(1) == K,
              "dequant output must be contiguous bf16 [N, K]");
  auto st = at::cuda::getCurrentCUDAStream();
  Q_DISPATCH((int)type, q_dequant_launch, w.data_ptr<uint8_t>(), (int)N, (int)K, row_step_bytes((int)type),
             reinterpret_cast<bf16*>(out.data_ptr()), st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
