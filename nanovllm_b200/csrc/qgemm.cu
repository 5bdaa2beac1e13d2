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
// qgemm_decode_kernel<TYPE, BN> (swap-AB like the bf16 decode GEMM: 128 weight rows = MMA M, tokens = MMA N) is
// persistent: one CTA per SM walks its work units (128-row group, K split) with every ring running across unit
// boundaries, so set-up is paid once per SM and the packed stream never drains between units.
//   warp 0 lane 0   producer: the packed row steps stream through a ring of up to 12 stages (the first ring is
//                   requested before the dependency wait); small token tiles keep one K split per CTA and load
//                   its activation slice [BN x Krange] ONCE by TMA;
//   warps 4..11     dequant: two groups of 4 warps take alternate 256-wide row steps, thread = weight row =
//                   TMEM lane, and write the four f16 64-wide sub-tiles straight from registers into one of 3
//                   TMEM row-step slots (tcgen05.st) -- no shared-memory tile, no proxy fence (FP4: hardware
//                   e2m1x2 -> f16x2 conversion times the block scale, exact; integer codes: 1024.0-magic f16
//                   halves with the code bits placed by prmt/lop3, one subtract, one multiply or fma);
//   warp 1 lane 0   tcgen05.mma kind::f16 with the A operand read from TMEM, B (f16 activations) from shared
//                   memory, fp32 accumulators in TMEM (two, so a unit's epilogue overlaps the next unit);
//   warp 2          for token tiles up to 32: does the MMA issuer's mbarrier waits and hands each row step over
//                   through a named barrier (see mma_handoff);
//   warps 3, 12-14  epilogue: (resident mode) first convert the activation slice to f16 in place; then per unit
//                   tcgen05.ld, bf16 output (one split) or fp32 split-K partials [S][M][N] that the consumer sums
//                   exactly like the bf16 decode GEMM's.
// Token tiles of 64 and more use the streaming mode instead of the resident slice: an f16 copy of the
// activations (q_to_f16_kernel) streams through a ring of row steps, so the K range -- and the number of fp32
// split partials -- is not capped by shared memory.
// Every wait is bounded (nvb::mbar_wait -> device error word) so a broken pipeline returns instead of hanging.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <algorithm>
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
constexpr int kQAStages = 3;             // dequantized f16 row steps in flight (TMEM slots of 4 x 32 columns)
// TMEM column of the first A slot: the accumulators use [0, NACC * NCH * BN); 128 leaves room for 3 row-step slots
__host__ __device__ constexpr uint32_t q_acol0(int bn) { return bn <= 64 ? 128u : 256u; }
__host__ __device__ constexpr int q_aslots(int bn) { return (int)((512u - q_acol0(bn)) / 128u); }
constexpr int kQMaxXS = 4;                // activation ring stages in streaming mode (at most)

// GGML type ids (the GGUF on-disk codes)
constexpr int T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12,
              T_Q5_K = 13, T_Q6_K = 14, T_IQ4_NL = 20, T_IQ4_XS = 23, T_TQ1_0 = 34, T_TQ2_0 = 35, T_MXFP4 = 39,
              T_NVFP4 = 40;

// bytes of one 256-element row step in the repacked layout (a multiple of 16: bulk copies and uint2 loads)
__host__ __device__ constexpr int row_step_bytes(int t) {
  return t == T_Q4_1 ? 160 : t == T_Q8_0 ? 272 : t == T_Q5_K ? 176 : t == T_Q6_K ? 224 : t == T_Q5_0 ? 176
       : t == T_Q5_1 ? 192 : t == T_Q2_K ? 96 : t == T_Q3_K ? 112 : t == T_TQ1_0 ? 64 : t == T_TQ2_0 ? 80 : 144;
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
  } else if constexpr (TYPE == T_Q5_0 || TYPE == T_Q5_1) {
    // d[8] | (m[8]) | qh[8] (u32, bit i = fifth bit of element i) | qs[8][16] (low nibbles 0..15, high 16..31)
    constexpr int kM = TYPE == T_Q5_1 ? 16 : 0;
    const int b = e0 >> 5, i0 = e0 & 31;
    const float d = h2f(p + 2 * b);
    const uint32_t qh = *reinterpret_cast<const uint32_t*>(p + 16 + kM + 4 * b) >> i0;
    uint8_t q[8];
    load8(p + 48 + kM + b * 16 + (i0 & 15), q);
    const bool hi = i0 >= 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = (hi ? (q[j] >> 4) : (q[j] & 0xF)) | (int)(((qh >> j) & 1) << 4);
      if constexpr (TYPE == T_Q5_0) v[j] = d * (float)(n - 16);
      else v[j] = d * (float)n + h2f(p + 16 + 2 * b);
    }
  } else if constexpr (TYPE == T_Q2_K || TYPE == T_Q3_K || TYPE == T_TQ2_0) {
    // 2-bit planes: byte (half * 32 + l) holds elements half * 128 + j * 32 + l at bits 2j (j = 0..3)
    const int half = e0 >> 7, j2 = (e0 >> 5) & 3, l0 = e0 & 31;
    constexpr int kQs = TYPE == T_Q2_K ? 16 : TYPE == T_Q3_K ? 32 : 0;
    uint8_t q[8];
    load8(p + kQs + half * 32 + l0, q);
    if constexpr (TYPE == T_Q2_K) {
      // scales[16] (low nibble scale, high nibble min; one per 16 elements) | qs[64] | d | dmin
      const uint32_t sc = p[half * 8 + j2 * 2 + (l0 >> 4)];
      const float dl = h2f(p + 80) * (float)(sc & 0xF), ml = h2f(p + 82) * (float)(sc >> 4);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = dl * (float)((q[j] >> (2 * j2)) & 3) - ml;
    } else if constexpr (TYPE == T_Q3_K) {
      // hmask[32] | qs[64] | 12 bytes of 6-bit scales (+32 bias) | d; a clear hmask bit subtracts 4
      const int si = half * 8 + j2 * 2 + (l0 >> 4), w = si >> 2, k = si & 3;
      const uint32_t lo = (uint32_t)p[96 + ((w & 1) ? 4 : 0) + k] >> ((w >> 1) * 4);
      const int sc = (int)((lo & 0xF) | ((((uint32_t)p[104 + k] >> (2 * w)) & 3) << 4)) - 32;
      const float dl = h2f(p + 108) * (float)sc;
      uint8_t h[8];
      load8(p + l0, h);
      const int hb = half * 4 + j2;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = dl * (float)((int)((q[j] >> (2 * j2)) & 3) - (((h[j] >> hb) & 1) ? 0 : 4));
    } else {  // TQ2_0: qs[64] | d, value d * (q - 1)
      const float d = h2f(p + 64);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = d * (float)((int)((q[j] >> (2 * j2)) & 3) - 1);
    }
  } else if constexpr (TYPE == T_TQ1_0) {
    // base-3 digits: bytes 0..31 carry 5 digits (elements k * 32 + m), bytes 32..47 carry 5 (160 + k * 16 + m),
    // bytes 48..51 carry 4 (240 + k * 4 + m); digit k of byte x is ((x * 3^k mod 256) * 3) >> 8, minus 1
    const float d = h2f(p + 52);
    int kd[8];
    uint8_t x[8];
    if (e0 < 160) {
      load8(p + (e0 & 31), x);
#pragma unroll
      for (int j = 0; j < 8; ++j) kd[j] = e0 >> 5;
    } else if (e0 < 240) {
      load8(p + 32 + ((e0 - 160) & 15), x);
#pragma unroll
      for (int j = 0; j < 8; ++j) kd[j] = (e0 - 160) >> 4;
    } else {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(p + 48);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int e = e0 - 240 + j;
        kd[j] = e >> 2;
        x[j] = (uint8_t)(w >> (8 * (e & 3)));
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t pw = kd[j] == 0 ? 1u : kd[j] == 1 ? 3u : kd[j] == 2 ? 9u : kd[j] == 3 ? 27u : 81u;
      const uint32_t r = ((uint32_t)x[j] * pw) & 0xFF;
      v[j] = d * (float)((int)((r * 3) >> 8) - 1);
    }
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
  } else if constexpr (TYPE == T_Q4_0 || TYPE == T_Q4_1) {
    // nibble codes as 1024 + q (low) or 1024 + 16 q (high nibble, scale / 16)
    const int b = e0 >> 5, i0 = e0 & 31;
    const bool hi = i0 >= 16;
    const uint32_t mask = hi ? 0x00F000F0u : 0x000F000Fu;
    const float d = h2f(p + 2 * b) * (hi ? 0.0625f : 1.f);
    const uint2 w = *reinterpret_cast<const uint2*>(p + (TYPE == T_Q4_1 ? 32 : 16) + b * 16 + (i0 & 15));
    const uint32_t s2 = h2_bcast(d);
    uint32_t q[4] = {nib_pair(prmt(w.x, 0, 0x4140), mask), nib_pair(prmt(w.x, 0, 0x4342), mask),
                     nib_pair(prmt(w.y, 0, 0x4140), mask), nib_pair(prmt(w.y, 0, 0x4342), mask)};
    if constexpr (TYPE == T_Q4_0) {
      const uint32_t kb = hi ? 0x64806480u : 0x64086408u;  // 1024 + 8 code units
#pragma unroll
      for (int j = 0; j < 4; ++j) q[j] = hmul2(hsub2(q[j], kb), s2);
    } else {
      const uint32_t m2 = h2_bcast(h2f(p + 16 + 2 * b));
#pragma unroll
      for (int j = 0; j < 4; ++j) q[j] = hfma2(hsub2(q[j], 0x64006400u), s2, m2);
    }
    o = make_uint4(q[0], q[1], q[2], q[3]);
  } else if constexpr (TYPE == T_Q5_K) {
    const int sb = e0 >> 5, i0 = e0 & 31;
    const float d = h2f(p), dmin = h2f(p + 2);
    const uint8_t* qq = p + 4;
    int sc, mn;
    if (sb < 4) {
      sc = qq[sb] & 63;
      mn = qq[sb + 4] & 63;
    } else {
      sc = (qq[sb + 4] & 0xF) | ((qq[sb - 4] >> 6) << 4);
      mn = (qq[sb + 4] >> 4) | ((qq[sb] >> 6) << 4);
    }
    const bool hi = sb & 1;
    const float ds = d * (float)sc * (hi ? 0.0625f : 1.f);
    const uint32_t s2 = h2_bcast(ds), m2 = h2_bcast(-(dmin * (float)mn));
    const uint32_t mask = hi ? 0x00F000F0u : 0x000F000Fu;
    // the fifth bit (bit sb of the qh byte) lands at 16 (low nibble) or 256 (high nibble) code units
    const uint32_t hmask = hi ? 0x01000100u : 0x00100010u;
    const int hsh = hi ? 8 : 4;
    const uint2 w = *reinterpret_cast<const uint2*>(p + 48 + (sb >> 1) * 32 + i0);
    const uint2 h = *reinterpret_cast<const uint2*>(p + 16 + i0);
    const uint32_t sel[2] = {0x4140, 0x4342};
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t wq = j < 2 ? w.x : w.y, hq = j < 2 ? h.x : h.y;
      const uint32_t hb = ((prmt(hq, 0, sel[j & 1]) >> sb) << hsh) & hmask;
      r[j] = hfma2(hsub2(nib_pair(prmt(wq, 0, sel[j & 1]), mask) | hb, 0x64006400u), s2, m2);
    }
    o = make_uint4(r[0], r[1], r[2], r[3]);
  } else if constexpr (TYPE == T_Q6_K) {
    const int hh = e0 >> 7, wv = e0 & 127, k = wv >> 5, l0 = wv & 31;
    const uint2 ql = *reinterpret_cast<const uint2*>(p + hh * 64 + (k & 1) * 32 + l0);
    const uint2 qh = *reinterpret_cast<const uint2*>(p + 128 + hh * 32 + l0);
    const float s = (float)reinterpret_cast<const int8_t*>(p + 192)[hh * 8 + 2 * k + (l0 >> 4)];
    const bool hi = k >> 1;
    // 6-bit code q = nibble | 2 high bits << 4, as 1024 + q (low nibble) or 1024 + 16 q (high nibble)
    const uint32_t mask = hi ? 0x00F000F0u : 0x000F000Fu;
    const uint32_t hmask = hi ? 0x03000300u : 0x00300030u;
    const int hsh = hi ? 8 : 4;
    const uint32_t s2 = h2_bcast(h2f(p + 208) * s * (hi ? 0.0625f : 1.f));
    const uint32_t kb = hi ? 0x66006600u : 0x64206420u;  // 1024 + 32 code units
    const uint32_t sel[2] = {0x4140, 0x4342};
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lq = j < 2 ? ql.x : ql.y, hq = j < 2 ? qh.x : qh.y;
      const uint32_t hb = ((prmt(hq, 0, sel[j & 1]) >> (2 * k)) << hsh) & hmask;
      r[j] = hmul2(hsub2(nib_pair(prmt(lq, 0, sel[j & 1]), mask) | hb, kb), s2);
    }
    o = make_uint4(r[0], r[1], r[2], r[3]);
  } else if constexpr (TYPE == T_Q2_K || TYPE == T_Q3_K || TYPE == T_TQ2_0) {
    const int half = e0 >> 7, j2 = (e0 >> 5) & 3, l0 = e0 & 31;
    constexpr int kQs = TYPE == T_Q2_K ? 16 : TYPE == T_Q3_K ? 32 : 0;
    const uint2 w = *reinterpret_cast<const uint2*>(p + kQs + half * 32 + l0);
    uint32_t s2, m2 = 0, kb = 0x64006400u;
    uint2 hm = make_uint2(0, 0);
    int hb = 0;
    if constexpr (TYPE == T_Q2_K) {
      const uint32_t sc = p[half * 8 + j2 * 2 + (l0 >> 4)];
      s2 = h2_bcast(h2f(p + 80) * (float)(sc & 0xF));
      m2 = h2_bcast(-(h2f(p + 82) * (float)(sc >> 4)));
    } else if constexpr (TYPE == T_Q3_K) {
      const int si = half * 8 + j2 * 2 + (l0 >> 4), ww = si >> 2, kk = si & 3;
      const uint32_t lo = (uint32_t)p[96 + ((ww & 1) ? 4 : 0) + kk] >> ((ww >> 1) * 4);
      const int sc = (int)((lo & 0xF) | ((((uint32_t)p[104 + kk] >> (2 * ww)) & 3) << 4)) - 32;
      s2 = h2_bcast(h2f(p + 108) * (float)sc);
      hm = *reinterpret_cast<const uint2*>(p + l0);
      hb = half * 4 + j2;
      kb = 0x64046404u;  // 3-bit code (hmask bit as bit 2) minus 4
    } else {
      s2 = h2_bcast(h2f(p + 64));
      kb = 0x64016401u;  // code - 1
    }
    const uint32_t sel[2] = {0x4140, 0x4342};
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t t = ((prmt(j < 2 ? w.x : w.y, 0, sel[j & 1]) >> (2 * j2)) & 0x00030003u) | 0x64006400u;
      if constexpr (TYPE == T_Q3_K) t |= ((prmt(j < 2 ? hm.x : hm.y, 0, sel[j & 1]) >> hb) << 2) & 0x00040004u;
      t = hsub2(t, kb);
      r[j] = TYPE == T_Q2_K ? hfma2(t, s2, m2) : hmul2(t, s2);
    }
    o = make_uint4(r[0], r[1], r[2], r[3]);
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

// Whole 64-element sub-step of a row (elements [64 sub, 64 sub + 64) of the row step) as 32 f16x2, block scales
// decoded once.  Specialised for the formats of the serving configs; the rest go through decode_h8.
__device__ __forceinline__ void e4m3x4_scales(uint32_t sc, uint32_t (&s2)[4]) {
  // ue4m3 0x7F (NaN in e4m3) reads as 0, like the loader's decoder
  const uint32_t nan = __vcmpeq4(sc, 0x7F7F7F7Fu);
  sc &= ~nan;
  uint32_t h01, h23;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h01), "=r"(h23) : "r"(sc));
  s2[0] = prmt(h01, h01, 0x1010);
  s2[1] = prmt(h01, h01, 0x3232);
  s2[2] = prmt(h23, h23, 0x1010);
  s2[3] = prmt(h23, h23, 0x3232);
}

template <int TYPE>
__device__ __forceinline__ void decode_sub64(const uint8_t* __restrict__ p, int sub, const Luts& L, uint32_t (&v)[32]) {
  if constexpr (TYPE == T_NVFP4) {
    const uint4 q0 = *reinterpret_cast<const uint4*>(p + 16 + sub * 32);
    const uint4 q1 = *reinterpret_cast<const uint4*>(p + 16 + sub * 32 + 16);
    uint32_t s2[4];
    e4m3x4_scales(*reinterpret_cast<const uint32_t*>(p + sub * 4), s2);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t h[4];
      e2m1x8_to_h2(w[k], h);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * k + j] = hmul2(h[j], s2[k >> 1]);
    }
  } else if constexpr (TYPE == T_MXFP4) {
    const uint4 q0 = *reinterpret_cast<const uint4*>(p + 16 + sub * 32);
    const uint4 q1 = *reinterpret_cast<const uint4*>(p + 16 + sub * 32 + 16);
    const uint32_t e0 = p[2 * sub], e1 = p[2 * sub + 1];
    const uint32_t sa = h2_bcast(e0 ? __int_as_float((int)e0 << 23) : 0.f);
    const uint32_t sb = h2_bcast(e1 ? __int_as_float((int)e1 << 23) : 0.f);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t h[4];
      e2m1x8_to_h2(w[k], h);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * k + j] = hmul2(h[j], k < 4 ? sa : sb);
    }
  } else if constexpr (TYPE == T_Q4_K) {
    const float d = h2f(p), dmin = h2f(p + 2);
    const uint8_t* q = p + 4;
    const int sl = 2 * sub, sh = 2 * sub + 1;  // low-nibble and high-nibble sub-blocks of this sub-step
    int sc0, mn0, sc1, mn1;
    if (sl < 4) {
      sc0 = q[sl] & 63;
      mn0 = q[sl + 4] & 63;
      sc1 = q[sh] & 63;
      mn1 = q[sh + 4] & 63;
    } else {
      sc0 = (q[sl + 4] & 0xF) | ((q[sl - 4] >> 6) << 4);
      mn0 = (q[sl + 4] >> 4) | ((q[sl] >> 6) << 4);
      sc1 = (q[sh + 4] & 0xF) | ((q[sh - 4] >> 6) << 4);
      mn1 = (q[sh + 4] >> 4) | ((q[sh] >> 6) << 4);
    }
    const uint32_t s0 = h2_bcast(d * (float)sc0), m0 = h2_bcast(-(dmin * (float)mn0));
    const uint32_t s1 = h2_bcast(d * (float)sc1 * 0.0625f), m1 = h2_bcast(-(dmin * (float)mn1));
    const uint4 q0 = *reinterpret_cast<const uint4*>(p + 16 + sub * 32);
    const uint4 q1 = *reinterpret_cast<const uint4*>(p + 16 + sub * 32 + 16);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t k1024 = 0x64006400u;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t t0 = prmt(w[k], 0, 0x4140), t1 = prmt(w[k], 0, 0x4342);
      v[2 * k] = hfma2(hsub2(nib_pair(t0, 0x000F000Fu), k1024), s0, m0);
      v[2 * k + 1] = hfma2(hsub2(nib_pair(t1, 0x000F000Fu), k1024), s0, m0);
      v[16 + 2 * k] = hfma2(hsub2(nib_pair(t0, 0x00F000F0u), k1024), s1, m1);
      v[16 + 2 * k + 1] = hfma2(hsub2(nib_pair(t1, 0x00F000F0u), k1024), s1, m1);
    }
  } else if constexpr (TYPE == T_Q8_0) {
    const uint32_t dbits = *reinterpret_cast<const uint32_t*>(p + 4 * sub);  // d of blocks 2 sub, 2 sub + 1
    const uint32_t da = prmt(dbits, dbits, 0x1010), db = prmt(dbits, dbits, 0x3232);
    const uint32_t k1152 = 0x64806480u;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const uint4 q = *reinterpret_cast<const uint4*>(p + 16 + sub * 64 + 16 * h);
      const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[8 * h + 2 * k] = hmul2(hsub2(prmt(w[k], 0x64646464u, 0x4140), k1152), h < 2 ? da : db);
        v[8 * h + 2 * k + 1] = hmul2(hsub2(prmt(w[k], 0x64646464u, 0x4342), k1152), h < 2 ? da : db);
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 o = decode_h8<TYPE>(p, sub * QBK + c * 8, L);
      v[4 * c] = o.x;
      v[4 * c + 1] = o.y;
      v[4 * c + 2] = o.z;
      v[4 * c + 3] = o.w;
    }
  }
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
  int groups;       // 128-row groups: ceil(N / 128)
  int per_split;    // resident mode: CTAs per split (the grid is per_split * S)
  int ws;           // packed ring stages
  int xs;           // activation ring stages (row steps); 0 = the CTA's activation slice is resident
  int bprs;         // bytes per row step
  const uint8_t* w; // tile-major packed weight
  bf16* out;
  long out_ld;
  float* partial;
  int* err;
  long long* trace;  // optional per-role clock64 trace of CTA 0: [6 roles][64 steps][4 events]
};

#define QTRACE(role, idx, ev)                                                                   \
  do {                                                                                          \
    if (tr != nullptr) tr[((role) * 64 + min((int)(idx), 63)) * 4 + (ev)] = (long long)clock64(); \
  } while (0)

// D(tmem) (+)= A(tmem) * B(smem desc)^T, kind::f16: the A operand is read from tensor memory (128 lanes = rows,
// each 32-bit column holds two consecutive K elements).
__device__ __forceinline__ void tc_mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns per thread (each thread writes its own lane)
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// kind::f16 instruction descriptor with f16 A and B, f32 accumulator, both K-major
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

constexpr int kQDequantWarps = 8;
// warps: 0 producer, 1 MMA issuer, 2 MMA waiter, 3 and 12-14 epilogue (TMEM lane quarters 3, 0, 1, 2),
// 4-11 dequant
constexpr int kQThreads = 32 * 15;

// Named barrier 1 between the MMA issuer warp and its waiter warp, AND-reducing an ok flag.  The issuer never
// touches shared memory between MMA batches: measured on B200, an mbarrier wait (even on a completed phase) or
// any shared-memory load issued by the thread right after a batch of narrow tcgen05.mma stalls until the
// batch has drained, idling the tensor pipe (16 MMAs of N=16: ~880 cycles of issue, ~3000 with an in-thread
// wait), while a named barrier does not.
__device__ __forceinline__ bool mma_handoff(int ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, 1, 64, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(ok)
      : "memory");
  return r != 0;
}

// Work unit u of a CTA = (row group, K split).  Resident mode keeps one split per CTA (its activation slice is
// loaded once): CTA c takes split c % S and row groups c / S + i * per_split.  Streaming mode deals the units
// out round-robin, split-major.
__device__ __forceinline__ bool q_unit(const QArgs& a, int i, int& group, int& split) {
  if (a.xs == 0) {
    split = (int)blockIdx.x % a.S;
    group = (int)blockIdx.x / a.S + i * a.per_split;
  } else {
    const int u = (int)blockIdx.x + i * (int)gridDim.x;
    group = u % a.groups;
    split = u / a.groups;
    if (split >= a.S) return false;
  }
  return group < a.groups;
}

// Walks a CTA's row steps in order: unit i, step j of the unit's K range.
struct QCursor {
  int i, j, nks, group, split, ks0;
  bool ok;
  __device__ __forceinline__ void load(const QArgs& a) {
    ok = q_unit(a, i, group, split);
    if (ok) {
      ks0 = split * a.kper;
      nks = min(a.ksteps, ks0 + a.kper) - ks0;
    }
  }
  __device__ __forceinline__ void start(const QArgs& a) {
    i = 0;
    j = 0;
    load(a);
  }
  __device__ __forceinline__ void next_step(const QArgs& a) {
    if (++j == nks) next_unit(a);
  }
  __device__ __forceinline__ void next_unit(const QArgs& a) {
    j = 0;
    ++i;
    load(a);
  }
};

template <int TYPE, int BN>
__global__ void __launch_bounds__(kQThreads, 1) qgemm_decode_kernel(const __grid_constant__ CUtensorMap xmap, QArgs a) {
  constexpr uint32_t X_BOX = BN * QBK * 2;    // one [BN x 64] activation box
  constexpr uint32_t TMEM_COLS = 512;         // accumulators [0, NACC * BN) + AS row-step slots of 128 columns
  constexpr uint32_t IDESC = idesc_f16_f32(QBM, BN);
  constexpr int NACC = BN <= 128 ? 2 : 1;     // two accumulators: a unit's epilogue overlaps the next unit's MMAs
  constexpr bool WAITER = BN <= 32;           // warp 2 waits for the MMA issuer (see mma_handoff)
  // independent accumulation chains per unit (summed in the epilogue): narrow MMAs issued back to back into one
  // accumulator serialise on it
  constexpr int NCH = BN <= 16 ? 4 : BN <= 32 ? 2 : 1;
  constexpr uint32_t ACOL0 = q_acol0(BN);
  constexpr int AS = q_aslots(BN);            // 3 (BN <= 128) or 2 row-step slots
  static_assert(NACC * NCH * BN <= (int)ACOL0 && AS <= kQAStages && ACOL0 + 128 * AS <= TMEM_COLS, "TMEM plan");
  const uint32_t stage_bytes = (uint32_t)a.bprs * QBM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // resident mode (xs == 0): the CTA's activation slice (kper row steps of its split), converted to f16 in
  // place once; streaming mode (xs > 0, larger token tiles): a ring of xs row steps of an f16 activation copy
  const bool stream = a.xs > 0;
  const int xslots = stream ? a.xs : a.kper;
  uint8_t* xres = smem;                                           // xslots * 4 boxes
  uint8_t* wring = xres + (size_t)xslots * 4 * X_BOX;             // ws packed stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(wring + (size_t)a.ws * stage_bytes);
  uint64_t* xbar = bars;
  uint64_t* xready = bars + 1;
  uint64_t* wfull = bars + 2;
  uint64_t* wempty = wfull + a.ws;
  uint64_t* afull = wempty + a.ws;
  uint64_t* aempty = afull + kQAStages;
  uint64_t* tfull = aempty + kQAStages;   // [2]
  uint64_t* tempty = tfull + 2;           // [2]
  uint64_t* xfull = tempty + 2;           // streaming mode: [xs]
  uint64_t* xempty = xfull + kQMaxXS;
  __shared__ Luts luts;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long* tr = (blockIdx.x == 0 && lane == 0) ? a.trace : nullptr;

  init_luts(luts);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    nvb::mbar_init(xbar, 1);
    nvb::mbar_init(xready, 4);  // the 4 epilogue warps convert the resident activation slice
    for (int s = 0; s < a.ws; ++s) {
      nvb::mbar_init(&wfull[s], 1);
      nvb::mbar_init(&wempty[s], 4);  // the 4 warps of the dequant group that owns the row step
    }
    for (int s = 0; s < kQAStages; ++s) {
      nvb::mbar_init(&afull[s], 4);
      nvb::mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      nvb::mbar_init(&tfull[b], 1);
      nvb::mbar_init(&tempty[b], 4);  // the 4 epilogue warps
    }
    for (int s = 0; s < a.xs; ++s) {
      nvb::mbar_init(&xfull[s], 1);
      nvb::mbar_init(&xempty[s], 1);
    }
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
  if (threadIdx.x == 0) QTRACE(5, 0, 0);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ producer
      QCursor wc, xc;
      wc.start(a);
      uint32_t wit = 0, xit = 0;
      bool ok = true;
      // packed weights are never written by earlier kernels: the first ring streams in before the dependency
      for (; wc.ok && wit < (uint32_t)a.ws; ++wit, wc.next_step(a)) {
        nvb::mbar_arrive_expect_tx(&wfull[wit], stage_bytes);
        bulk_load(wring + (size_t)wit * stage_bytes,
                  a.w + ((size_t)wc.group * a.ksteps + wc.ks0 + wc.j) * stage_bytes, stage_bytes, &wfull[wit]);
      }
      nvb::tma_prefetch_desc(&xmap);
      nvb::pdl_wait();
      xc.start(a);
      if (!stream) {
        if (xc.ok) {
          nvb::mbar_arrive_expect_tx(xbar, (uint32_t)xc.nks * 4 * X_BOX);
          for (int b = 0; b < xc.nks * 4; ++b)
            nvb::tma_load_2d(xres + (size_t)b * X_BOX, &xmap, xbar, xc.ks0 * QSTEP + b * QBK, 0);
        }
      }
      while (ok && (stream ? xc.ok : wc.ok)) {
        if (stream) {
          // row step xit's activations, then the weight row step ws further on
          const int xsl = xit % a.xs;
          if (xit >= (uint32_t)a.xs &&
              !nvb::mbar_wait(&xempty[xsl], ((xit / a.xs) & 1u) ^ 1u, a.err, &abort_flag)) {
            ok = false;
            break;
          }
          nvb::mbar_arrive_expect_tx(&xfull[xsl], 4 * X_BOX);
          for (int b = 0; b < 4; ++b)
            nvb::tma_load_2d(xres + ((size_t)xsl * 4 + b) * X_BOX, &xmap, &xfull[xsl], (xc.ks0 + xc.j) * QSTEP + b * QBK, 0);
          ++xit;
          xc.next_step(a);
          if (!wc.ok) continue;
        }
        const int s = wit % a.ws;
        if (!nvb::mbar_wait(&wempty[s], ((wit / a.ws) & 1u) ^ 1u, a.err, &abort_flag)) {
          ok = false;
          break;
        }
        QTRACE(0, wit, 0);
        nvb::mbar_arrive_expect_tx(&wfull[s], stage_bytes);
        bulk_load(wring + (size_t)s * stage_bytes, a.w + ((size_t)wc.group * a.ksteps + wc.ks0 + wc.j) * stage_bytes,
                  stage_bytes, &wfull[s]);
        ++wit;
        wc.next_step(a);
      }
      if (!ok) {
        // bounded drain of copies that may still be landing in shared memory
        for (uint32_t j = (wit > (uint32_t)a.ws ? wit - a.ws : 0); j < wit; ++j)
          nvb::mbar_wait(&wfull[j % a.ws], (j / a.ws) & 1u, nullptr, nullptr);
        if (stream)
          for (uint32_t j = (xit > (uint32_t)a.xs ? xit - a.xs : 0); j < xit; ++j)
            nvb::mbar_wait(&xfull[j % a.xs], (j / a.xs) & 1u, nullptr, nullptr);
        else
          nvb::mbar_wait(xbar, 0, nullptr, nullptr);
      }
    } else {
      nvb::pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (lane 0 issues)
    // Narrow token tiles (the MMA floor is per instruction) hand their waits to warp 2 and meet it at a named
    // barrier; wide ones, whose MMAs outlast a wait anyway, wait in lane 0 themselves.
    nvb::pdl_wait();
    // the 16 MMAs of row step ``it`` (step j of its unit) into accumulator d_tm; then release its slots
    auto issue_step = [&](uint32_t it, int j, uint32_t d_tm) {
      const int t = it % AS;
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
        const uint32_t a_tm = tmem_base + ACOL0 + (uint32_t)t * 128 + sub * 32;
        const size_t box = stream ? (size_t)(it % a.xs) * 4 + sub : (size_t)j * 4 + sub;
        const uint32_t b_addr = nvb::smem_u32(xres + box * X_BOX);
#pragma unroll
        for (int kk = 0; kk < QBK / 16; ++kk) {
          const int ch = (sub * 4 + kk) % NCH;
          tc_mma_f16_tmem_a(d_tm + ch * BN, a_tm + kk * 8, nvb::sdesc_kmajor_sw128(b_addr + kk * 32), IDESC,
                            (j > 0 || sub > 0 || kk >= NCH) ? 1u : 0u);
        }
      }
      nvb::tc_commit(&aempty[t]);
      if (stream) nvb::tc_commit(&xempty[it % a.xs]);
    };
    QCursor c;
    c.start(a);
    uint32_t it = 0;
    if constexpr (WAITER) {
      bool ok = mma_handoff(1);  // the waiter has seen the activations
      for (uint32_t unit = 0; ok && c.ok; ++unit, c.next_unit(a)) {
        const uint32_t b = unit % NACC;
        for (int j = 0; j < c.nks; ++j, ++it) {
          ok = mma_handoff(1);  // the waiter has seen this row step's operands
          if (!ok) break;
          nvb::tc_fence_after();
          if (lane == 0) issue_step(it, j, tmem_base + b * (NCH * BN));
          __syncwarp();
        }
        if (!ok) break;
        if (lane == 0) nvb::tc_commit(&tfull[b]);
        __syncwarp();
      }
    } else if (lane == 0) {
      bool ok = stream || nvb::mbar_wait(xready, 0, a.err, &abort_flag);
      for (uint32_t unit = 0; ok && c.ok; ++unit, c.next_unit(a)) {
        const uint32_t b = unit % NACC, use = unit / NACC;
        for (int j = 0; j < c.nks; ++j, ++it) {
          if (j == 0 && !nvb::mbar_wait(&tempty[b], (use & 1u) ^ 1u, a.err, &abort_flag)) ok = false;
          if (ok && stream && !nvb::mbar_wait(&xfull[it % a.xs], (it / a.xs) & 1u, a.err, &abort_flag)) ok = false;
          if (ok && !nvb::mbar_wait(&afull[it % AS], (it / AS) & 1u, a.err, &abort_flag)) ok = false;
          if (!ok) break;
          QTRACE(1, it, 0);
          nvb::tc_fence_after();
          issue_step(it, j, tmem_base + b * (NCH * BN));
          QTRACE(1, it, 1);
        }
        if (ok) nvb::tc_commit(&tfull[b]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ MMA waiter (narrow token tiles)
    // every wait of the MMA issuer, in its order; each step ends with the named-barrier hand-off
    nvb::pdl_wait();
    if constexpr (WAITER) {
      int okl = 1;
      if (lane == 0 && !stream) okl = nvb::mbar_wait(xready, 0, a.err, &abort_flag) ? 1 : 0;
      bool ok = mma_handoff(__shfl_sync(0xffffffffu, okl, 0));
      QCursor c;
      c.start(a);
      uint32_t it = 0;
      for (uint32_t unit = 0; ok && c.ok; ++unit, c.next_unit(a)) {
        const uint32_t b = unit % NACC, use = unit / NACC;
        for (int j = 0; j < c.nks; ++j, ++it) {
          okl = 1;
          if (lane == 0) {
            if (j == 0) okl = nvb::mbar_wait(&tempty[b], (use & 1u) ^ 1u, a.err, &abort_flag) ? 1 : 0;
            if (okl && stream) okl = nvb::mbar_wait(&xfull[it % a.xs], (it / a.xs) & 1u, a.err, &abort_flag) ? 1 : 0;
            if (okl) okl = nvb::mbar_wait(&afull[it % AS], (it / AS) & 1u, a.err, &abort_flag) ? 1 : 0;
            QTRACE(1, it, 0);
          }
          ok = mma_handoff(__shfl_sync(0xffffffffu, okl, 0));
          QTRACE(1, it, 1);
          if (!ok) break;
        }
      }
    }
  } else if (warp >= 4 && warp < 4 + kQDequantWarps) {
    // ------------------------------------------------------------------ dequant
    // reads only the packed weights (never written by earlier kernels) and writes TMEM: no dependency wait
    QCursor c;
    c.start(a);
    bool ok = true;
    // two groups of 4 warps take alternate 256-wide row steps; thread = weight row (its TMEM lane); the f16
    // sub-tiles go straight from registers into a TMEM slot that the MMA reads as its A operand
    const int quarter = warp & 3, r = quarter * 32 + lane, g = (warp - 4) >> 2;
    const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
    for (uint32_t it = 0; ok && c.ok; ++it, c.next_step(a)) {
      if ((int)(it & 1u) != g) continue;
      const int s = it % a.ws, t = it % AS;
      if (!nvb::mbar_wait(&wfull[s], (it / a.ws) & 1u, a.err, &abort_flag)) break;
      if (quarter == 0) QTRACE(2 + g, it, 0);
      if (it >= (uint32_t)AS && !nvb::mbar_wait(&aempty[t], ((it / AS) & 1u) ^ 1u, a.err, &abort_flag)) break;
      if (quarter == 0) QTRACE(2 + g, it, 1);
      nvb::tc_fence_after();
      const uint8_t* p = wring + (size_t)s * stage_bytes + (size_t)r * a.bprs;
#pragma unroll 1
      for (int sub = 0; sub < 4; ++sub) {
        uint32_t v[32];
        decode_sub64<TYPE>(p, sub, luts, v);
        tmem_st_32x32b_x32(lane_base + ACOL0 + (uint32_t)t * 128 + sub * 32, v);
      }
      tmem_st_wait();
      if (quarter == 0) QTRACE(2 + g, it, 2);
      nvb::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        nvb::mbar_arrive(&afull[t]);
        nvb::mbar_arrive(&wempty[s]);  // the packed row step has been read
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 3, 12, 13, 14)
    nvb::pdl_wait();
    const int quarter = warp & 3;
    const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16);
    constexpr int CH = BN < 64 ? BN : 64;
    QCursor c;
    c.start(a);
    if (!stream) {
      // resident mode: the activation slice becomes f16 in place first (saturating; elementwise layout)
      bool okx = !c.ok || nvb::mbar_wait(xbar, 0, a.err, &abort_flag);
      if (okx && c.ok) {
        const uint32_t xbytes = (uint32_t)c.nks * 4 * X_BOX;
        for (uint32_t off = (uint32_t)(quarter * 32 + lane) * 16; off < xbytes; off += 128 * 16) {
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
    }
    for (uint32_t unit = 0; c.ok; ++unit, c.next_unit(a)) {
      const uint32_t b = unit % NACC, use = unit / NACC;
      int ok = 0;
      if (lane == 0) ok = nvb::mbar_wait(&tfull[b], use & 1u, a.err, &abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (quarter == 0) QTRACE(4, unit, 0);
      nvb::tc_fence_after();
      const int f = c.group * QBM + quarter * 32 + lane;  // TMEM lane = weight row
#pragma unroll 1
      for (int col = 0; col < BN; col += CH) {
        uint32_t v[CH];
#pragma unroll
        for (int q = 0; q < CH; q += 16) nvb::tmem_ld_32x32b_x16(t_lane + b * (NCH * BN) + col + q, v + q);
        nvb::tmem_ld_wait();
        nvb::reg_fence<CH>(v);
        if constexpr (NCH > 1) {
#pragma unroll
          for (int ch = 1; ch < NCH; ++ch) {
            uint32_t u[CH];
#pragma unroll
            for (int q = 0; q < CH; q += 16) nvb::tmem_ld_32x32b_x16(t_lane + b * (NCH * BN) + ch * BN + col + q, u + q);
            nvb::tmem_ld_wait();
            nvb::reg_fence<CH>(u);
#pragma unroll
            for (int q = 0; q < CH; ++q) v[q] = __float_as_uint(__uint_as_float(v[q]) + __uint_as_float(u[q]));
          }
        }
        if (f < a.N) {
          if (a.S == 1) {
#pragma unroll
            for (int j = 0; j < CH; ++j)
              if (col + j < a.M) a.out[(long)(col + j) * a.out_ld + f] = __float2bfloat16(__uint_as_float(v[j]));
          } else {
            float* dst = a.partial + (long)c.split * a.M * a.N + f;
#pragma unroll
            for (int j = 0; j < CH; ++j)
              if (col + j < a.M) dst[(long)(col + j) * a.N] = __uint_as_float(v[j]);
          }
        }
      }
      if (quarter == 0) QTRACE(4, unit, 1);
      nvb::tc_fence_before();
      __syncwarp();
      if (lane == 0) nvb::mbar_arrive(&tempty[b]);
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
  int bn, kper, S, ws, xs, bprs, grid, per_split;
  size_t smem;
};

// bf16 -> f16 copy of the activations for the streaming mode (saturating), 8 elements per thread.
__global__ void q_to_f16_kernel(const bf16* __restrict__ x, long ld, int M, int K, uint16_t* __restrict__ y) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long per_row = K / 8, n = (long)M * per_row;
  for (long c = blockIdx.x * (long)blockDim.x + threadIdx.x; c < n; c += (long)gridDim.x * blockDim.x) {
    const long m = c / per_row, k = (c % per_row) * 8;
    uint4 v = *reinterpret_cast<const uint4*>(x + m * ld + k);
    uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = f2_to_h2(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xFFFF0000u));
    *reinterpret_cast<uint4*>(y + m * (long)K + k) = v;
  }
}

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
  return t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_Q5_1 || t == T_Q8_0 || t == T_Q2_K || t == T_Q3_K ||
         t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_IQ4_NL || t == T_IQ4_XS || t == T_TQ1_0 ||
         t == T_TQ2_0 || t == T_MXFP4 || t == T_NVFP4;
}

// Persistent grid of at most one CTA per SM.  The K split S is chosen by a cost model in bytes: the busiest CTA's
// packed row steps times the SM count (time at a fixed per-SM stream rate), plus the fp32 split partials written
// and read back; near ties go to fewer splits.  Resident mode also needs the split's activation slice
// (BN x kper*256) within kQXBytes and at least two packed ring stages beside it.
QPlan q_plan(int M, int N, int K, int type, int sms) {
  QPlan p{};
  p.bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  p.bprs = row_step_bytes(type);
  const int ksteps = K / QSTEP, groups = (N + QBM - 1) / QBM;
  const int x_step = p.bn * QSTEP * 2;
  const int stage = QBM * p.bprs;
  // token tiles of 64 and more stream their activations (an f16 copy) through a ring of row steps: a resident
  // slice would cap the K range at 512 and multiply the splits and their fp32 partials
  p.xs = p.bn >= 64 ? (p.bn >= 256 ? 1 : p.bn >= 128 ? 2 : 3) : 0;
  const int kres = std::max(1, std::min(ksteps, kQXBytes / x_step));
  const int smax = std::max(16, (ksteps + kres - 1) / kres);
  double best = -1.0;
  for (int S = 1; S <= std::min(ksteps, smax); ++S) {
    const int kper = (ksteps + S - 1) / S;
    if ((ksteps + kper - 1) / kper != S) continue;  // the same split as a smaller S
    if (!p.xs && kper > kres) continue;
    const int ring = (kQRingBytes - (p.xs ? p.xs : kper) * x_step) / stage;
    if (ring < 2) continue;
    long per_cta;
    int grid, per_split = 0;
    if (p.xs) {
      const long units = (long)groups * S;
      grid = (int)std::min<long>(units, sms);
      per_cta = (units + grid - 1) / grid * kper;
    } else {
      per_split = std::min(groups, std::max(1, sms / S));
      grid = per_split * S;
      per_cta = (long)((groups + per_split - 1) / per_split) * kper;
    }
    const double cost = (double)per_cta * stage * sms + (S > 1 ? (double)S * M * N * 8.0 : 0.0);
    if (best < 0 || cost < best * 0.97) {
      best = cost;
      p.S = S;
      p.kper = kper;
      p.grid = grid;
      p.per_split = per_split;
      p.ws = std::min(12, ring);
    }
  }
  TORCH_CHECK(best >= 0, "packed GEMM: no K split fits shared memory");
  p.smem = 1024 + (size_t)(p.xs ? p.xs : p.kper) * x_step + (size_t)p.ws * stage +
           (size_t)(2 + 2 * p.ws + 2 * kQAStages + 4 + 2 * kQMaxXS) * 8 + 64;
  return p;
}

template <int TYPE, int BN>
void q_launch(const CUtensorMap& xm, const QArgs& a, const QPlan& p, cudaStream_t st) {
  auto kern = qgemm_decode_kernel<TYPE, BN>;
  static int attr_bytes[64] = {0};  // per device: the dynamic shared-memory limit raised so far
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || attr_bytes[dev] < (int)p.smem) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
    if (dev < 64) attr_bytes[dev] = (int)p.smem;
  }
  C10_CUDA_CHECK(nvb::launch(kern, dim3(p.grid), dim3(kQThreads), p.smem, st, xm, a));
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
    case T_Q5_0: FN<T_Q5_0>(__VA_ARGS__); break;                         \
    case T_Q5_1: FN<T_Q5_1>(__VA_ARGS__); break;                         \
    case T_Q8_0: FN<T_Q8_0>(__VA_ARGS__); break;                         \
    case T_Q2_K: FN<T_Q2_K>(__VA_ARGS__); break;                         \
    case T_Q3_K: FN<T_Q3_K>(__VA_ARGS__); break;                         \
    case T_Q4_K: FN<T_Q4_K>(__VA_ARGS__); break;                         \
    case T_Q5_K: FN<T_Q5_K>(__VA_ARGS__); break;                         \
    case T_Q6_K: FN<T_Q6_K>(__VA_ARGS__); break;                         \
    case T_IQ4_NL: FN<T_IQ4_NL>(__VA_ARGS__); break;                     \
    case T_IQ4_XS: FN<T_IQ4_XS>(__VA_ARGS__); break;                     \
    case T_TQ1_0: FN<T_TQ1_0>(__VA_ARGS__); break;                       \
    case T_TQ2_0: FN<T_TQ2_0>(__VA_ARGS__); break;                       \
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

// Optional clock64 trace of CTA 0 of every following qgemm launch (int64 [6][64][4], see QTRACE); None turns it
// off.  A profiling aid: the per-role timeline of one CTA shows which hand-off paces the pipeline.
namespace {
long long* g_qtrace = nullptr;
}
void qgemm_set_trace(c10::optional<torch::Tensor> t) {
  if (t.has_value()) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kLong && t->numel() >= 6 * 64 * 4, "trace: int64 [6, 64, 4]");
    g_qtrace = reinterpret_cast<long long*>(t->data_ptr<int64_t>());
  } else {
    g_qtrace = nullptr;
  }
}

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
  a.groups = (int)((N + QBM - 1) / QBM);
  a.per_split = p.per_split;
  a.ws = p.ws;
  a.xs = p.xs;
  a.bprs = p.bprs;
  a.w = w.data_ptr<uint8_t>();
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.out_ld = out.stride(0);
  a.err = err.has_value() ? err->data_ptr<int>() : nullptr;
  a.trace = g_qtrace;
  if (p.S > 1) {
    TORCH_CHECK(parts.has_value() && parts->is_cuda() && parts->scalar_type() == at::kFloat && parts->is_contiguous() &&
                    parts->numel() >= (long)p.S * M * N,
                "packed GEMM: fp32 partial buffer [S, M, N] required");
    a.partial = parts->data_ptr<float>();
  }
  auto st = at::cuda::getCurrentCUDAStream();
  torch::Tensor xh;
  const void* xp = x.data_ptr();
  long xld = x.stride(0);
  if (p.xs) {  // streaming mode multiplies an f16 copy of the activations
    xh = torch::empty({M, (long)K}, x.options().dtype(at::kHalf));
    const long chunks = (long)M * (K / 8);
    int blocks = (int)((chunks + 255) / 256);
    if (blocks > q_num_sms() * 4) blocks = q_num_sms() * 4;
    C10_CUDA_CHECK(nvb::launch(q_to_f16_kernel, dim3(blocks), dim3(256), 0, st,
                               reinterpret_cast<const bf16*>(x.data_ptr()), xld, M, (int)K,
                               reinterpret_cast<uint16_t*>(xh.data_ptr())));
    xp = xh.data_ptr();
    xld = K;
  }
  // 2-byte elements either way: the bf16 map describes the f16 copy just as well
  CUtensorMap xm = nvb::make_tmap_2d_bf16(xp, M, K, xld, p.bn);
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
