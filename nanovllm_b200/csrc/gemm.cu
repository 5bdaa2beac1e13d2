// Blackwell tcgen05 GEMM:  C[i, j] = sum_k A[i, k] * B[j, k]   (A [Ma, K], B [Nb, K], both K-major bf16).
//
// Replaces the reference's CPU dense linear (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/tensor/
// MatmulRuntime.java:234-309, a column-split gemv in fp32) for every projection of every model.
//
// Design (sm_100a):
//  * persistent kernel, one CTA per SM, 6 warps:
//      warp 0      TMA producer (one elected lane): A and B tiles of 64 K-elements with the 128-byte swizzle
//                  into a STAGES-deep shared-memory ring tracked by full/empty mbarriers;
//      warp 1      TMEM allocator + MMA issuer (one lane): tcgen05.mma.cta_group::1.kind::f16, M=128, N=BN,
//                  K=16, accumulating in tensor memory; tcgen05.commit frees ring stages and publishes tiles;
//      warps 2..5  epilogue: tcgen05.ld 32x32b of their TMEM lane quadrant, convert, store.
//  * two TMEM accumulators (2 x BN columns) so the epilogue of tile t overlaps the main loop of tile t+1.
//  * prefill-sized M: A = activations, B = weights, bf16 output, optional fused SiLU(gate)*up / GELU(gate)*up
//    on gate/up rows interleaved in 128-row blocks (one 256-wide tile holds 128 gate + 128 up columns).
//  * decode-sized M (<= 256 tokens): gemm_decode_kernel swaps A/B so the weight rows fill the 128-lane MMA M
//    dimension and the tokens are the N dimension; the K range may be split over CTAs so every SM streams
//    weights: the fp32 split partials then go to global memory and the consuming kernel (add+RMSNorm, RoPE,
//    the split-activation or split-sum kernel) adds them in split order (deterministic).  Under tensor
//    parallelism the decode kernel also carries the sequence-parallel collectives (sp_comm.cuh): an all-gather
//    + RMSNorm prologue for column-parallel projections and a reduce-scatter epilogue for row-parallel ones.
// Every mbarrier wait is bounded; on timeout the kernel records an error code and all roles exit, TMEM is
// freed, and the host sees the code through the error word.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "sp_comm.cuh"
#include "launch.h"
#include "tma_host.h"

namespace {

using bf16 = __nv_bfloat16;
constexpr int BM = 128;
constexpr int BK = 64;

enum OutMode : int { kOutBf16 = 0 };
enum Act : int { kActNone = 0, kActSiluMul = 1, kActGeluMul = 2 };

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}

struct GemmArgs {
  int Ma, Nb, K;
  int tiles_m, tiles_n, splits, kblocks;
  int out_mode, act;
  void* out;
  long out_ld;
  int* err;
};

__host__ __device__ constexpr uint32_t tmem_cols_for(int bn) {
  uint32_t need = 2u * bn;
  uint32_t c = 32;
  while (c < need) c <<= 1;
  return c;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap amap,
                                                         const __grid_constant__ CUtensorMap bmap, GemmArgs args) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);
  constexpr uint32_t IDESC = nvb::idesc_bf16_f32(BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;      // [2]
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = args.tiles_m * args.tiles_n * args.splits;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      nvb::mbar_init(&full_bar[s], 1);
      nvb::mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      nvb::mbar_init(&tfull_bar[a], 1);
      nvb::mbar_init(&tempty_bar[a], 4);
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

  // Raster of the units.  When the ~148 tiles in flight span at least two rows of output tiles, tile_n runs
  // fastest: they cover a few A row panels and the B panels those meet, so A and B each come from DRAM about
  // once and concurrent CTAs load different B tiles (measured 8-25 % faster on qkv / o_proj / down prefill
  // shapes).  With many tile columns (a wide fused gate/up, the LM head) tile_m runs fastest instead: A stays in
  // L2 while B streams through once (tile_n fastest measured 18 % slower there).
  const bool n_fast = args.tiles_n * 2 <= (int)gridDim.x;
  auto decode_unit = [&](int u, int& tm, int& tn, int& sp) {
    if (n_fast) {
      tn = u % args.tiles_n;
      const int r = u / args.tiles_n;
      tm = r % args.tiles_m;
      sp = r / args.tiles_m;
    } else {
      tm = u % args.tiles_m;
      const int r = u / args.tiles_m;
      tn = r % args.tiles_n;
      sp = r / args.tiles_n;
    }
  };
  auto k_range = [&](int sp, int& kb0, int& kb1) {
    kb0 = (int)((long)args.kblocks * sp / args.splits);
    kb1 = (int)((long)args.kblocks * (sp + 1) / args.splits);
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      nvb::tma_prefetch_desc(&amap);
      nvb::tma_prefetch_desc(&bmap);
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int tm, tn, sp, kb0, kb1;
        decode_unit(u, tm, tn, sp);
        k_range(sp, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (!nvb::mbar_wait(&empty_bar[s], (round & 1u) ^ 1u, args.err, &abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + s * STAGE_BYTES;
          nvb::mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
          nvb::tma_load_2d(sa, &amap, &full_bar[s], kb * BK, tm * BM);
          nvb::tma_load_2d(sa + A_BYTES, &bmap, &full_bar[s], kb * BK, tn * BN);
        }
      }
      if (!ok) {
        // bounded drain of copies that may still be landing in the ring
        for (uint32_t j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
          nvb::mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1u, nullptr, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++lt) {
        int tm, tn, sp, kb0, kb1;
        decode_unit(u, tm, tn, sp);
        k_range(sp, kb0, kb1);
        const uint32_t acc = lt & 1u, use = lt >> 1;
        if (!nvb::mbar_wait(&tempty_bar[acc], (use & 1u) ^ 1u, args.err, &abort_flag)) { ok = false; break; }
        nvb::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          if (!nvb::mbar_wait(&full_bar[s], (it / STAGES) & 1u, args.err, &abort_flag)) { ok = false; break; }
          nvb::tc_fence_after();
          const uint32_t a_addr = nvb::smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = nvb::sdesc_kmajor_sw128(a_addr + kk * 32);
            const uint64_t bd = nvb::sdesc_kmajor_sw128(b_addr + kk * 32);
            nvb::tc_mma_f16(d_tmem, ad, bd, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          nvb::tc_commit(&empty_bar[s]);
        }
        if (!ok) break;
        nvb::tc_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    uint32_t lt = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++lt) {
      int tm, tn, sp;
      decode_unit(u, tm, tn, sp);
      const uint32_t acc = lt & 1u, use = lt >> 1;
      int ok = 0;
      if (lane == 0) ok = nvb::mbar_wait(&tfull_bar[acc], use & 1u, args.err, &abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      nvb::tc_fence_after();
      const int a_row = tm * BM + row_in_tile;
      const uint32_t t_row = tmem_base + acc * BN + ((uint32_t)(quad * 32) << 16);
      if (args.out_mode == kOutBf16) {
        bf16* out = reinterpret_cast<bf16*>(args.out);
        if (args.act == kActNone) {
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            uint32_t r[16];
            nvb::tmem_ld_32x32b_x16(t_row + c, r);
            nvb::tmem_ld_wait();
            const int col = tn * BN + c;
            if (a_row < args.Ma) {
              bf16* dst = out + (long)a_row * args.out_ld + col;
              if (col + 16 <= args.Nb && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                uint4 v0, v1;
                uint32_t* p0 = reinterpret_cast<uint32_t*>(&v0);
                uint32_t* p1 = reinterpret_cast<uint32_t*>(&v1);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  p0[j] = nvb::pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                  p1[j] = nvb::pack_bf16x2(__uint_as_float(r[8 + 2 * j]), __uint_as_float(r[9 + 2 * j]));
                }
                reinterpret_cast<uint4*>(dst)[0] = v0;
                reinterpret_cast<uint4*>(dst)[1] = v1;
              } else {
                for (int j = 0; j < 16 && col + j < args.Nb; ++j) dst[j] = __float2bfloat16(__uint_as_float(r[j]));
              }
            }
          }
        } else {
          // gate = columns [0,128) of the tile, up = [128,256); output column tn*128 + c
#pragma unroll 1
          for (int c = 0; c < BN / 2; c += 16) {
            uint32_t rg[16], ru[16];
            nvb::tmem_ld_32x32b_x16(t_row + c, rg);
            nvb::tmem_ld_32x32b_x16(t_row + BN / 2 + c, ru);
            nvb::tmem_ld_wait();
            const int col = tn * (BN / 2) + c;
            if (a_row < args.Ma && col < args.Nb / 2) {
              bf16* dst = out + (long)a_row * args.out_ld + col;
              float v[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float gte = __uint_as_float(rg[j]), up = __uint_as_float(ru[j]);
                v[j] = (args.act == kActSiluMul ? silu(gte) : gelu_tanh(gte)) * up;
              }
              uint4 v0, v1;
              uint32_t* p0 = reinterpret_cast<uint32_t*>(&v0);
              uint32_t* p1 = reinterpret_cast<uint32_t*>(&v1);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                p0[j] = nvb::pack_bf16x2(v[2 * j], v[2 * j + 1]);
                p1[j] = nvb::pack_bf16x2(v[8 + 2 * j], v[9 + 2 * j]);
              }
              reinterpret_cast<uint4*>(dst)[0] = v0;
              reinterpret_cast<uint4*>(dst)[1] = v1;
            }
          }
        }
      }
      nvb::tc_fence_before();
      __syncwarp();
      if (lane == 0) nvb::mbar_arrive(&tempty_bar[acc]);
    }
  }
  nvb::tc_fence_before();
  __syncthreads();
  nvb::tc_fence_after();
  if (warp == 1) nvb::tmem_dealloc(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------ decode GEMM
// Decode-sized M (<= 256 tokens), swap-AB: the weight rows fill the 128-lane MMA M dimension and the tokens are
// the MMA N dimension (BN = M rounded up).  Each CTA owns NA (1 or 2) adjacent 128-row weight tiles that share
// one activation tile per K step, so a stage carries NA x 16 KB of weights for BN x 128 B of activations and a
// 1-CTA-per-SM ring keeps ~128 KB of weights in flight -- the decode GEMM is a weight-streaming problem and
// the loaded HBM latency is microseconds.  With the fused activation the two tiles are the gate and up rows of
// one 128-feature block (128-row interleaved layout) and act(gate) * up is formed in the epilogue.  The K range
// may be split over S CTAs; split partials are then written as fp32 [S][M][N] and summed, in a fixed order, by
// the kernel that consumes the output (add+RMSNorm, RoPE) or by splitk_sum_kernel.
//
// SP (tensor-parallel sequence-parallel fusion, protocol in sp_comm.cuh):
//   SP == 1  AG prologue: the weight tiles of the first ring stream in, then the CTAs that own rows of this
//            rank's SP slice wait for the RS flags, reduce + residual + RMSNorm their rows and broadcast them
//            into every rank's gather buffer; the TMA producer waits for all T rows to be flagged locally and
//            only then loads the activation tiles (from the local gather buffer).
//   SP == 2  RS epilogue (NA == 1): the output tile goes to the owners' receive buffers instead of ``out``.
//            With split K the S CTAs of a row group meet on per-CTA flags (all CTAs of a decode grid are
//            co-resident: at most one per SM), then CTA q sums token slice q over the S fp32 partials in split
//            order (L2-resident) and pushes it -- no separate sum kernel and no extra HBM round trip.
struct DecodeArgs {
  int N, M, K, kblocks, S, act;
  bf16* out;
  long out_ld;
  float* partial;
  int* err;
};

// Ring depth: as many stages as fit in 224 KB of shared memory (at most 16).  Under full load the HBM latency
// is several microseconds and a CTA's weight bandwidth is its weight bytes in flight over that latency, so the
// ring is sized by capacity, not by a fixed count.
constexpr int kDecodeRingBytes = 224 * 1024;
__host__ __device__ constexpr int decode_stages2(int na, int bn, int ksub = 1) {
  return kDecodeRingBytes / (ksub * (na * BM * BK * 2 + bn * BK * 2)) > 16
             ? 16
             : kDecodeRingBytes / (ksub * (na * BM * BK * 2 + bn * BK * 2));
}
__host__ __device__ constexpr uint32_t pow2_cols(int n) {
  uint32_t c = 32;
  while (c < (uint32_t)n) c <<= 1;
  return c;
}
constexpr int kSpTileLd = BM + 8;  // padded row (elements) of the bf16 output tile staged for the RS push

// KSUB: 64-wide K boxes per pipeline stage.  Loading KSUB adjacent boxes of the same weight rows back to back
// turns each weight row's 128-byte reads into KSUB * 128 contiguous bytes per stage (better DRAM page use).
template <int BN, int NA, int KSUB, int SP>
__global__ void __launch_bounds__(128, 1) gemm_decode_kernel(const __grid_constant__ CUtensorMap amap,
                                                             const __grid_constant__ CUtensorMap bmap,
                                                             DecodeArgs args, const __grid_constant__ nvb::sp::Args sp) {
  constexpr int STAGES = decode_stages2(NA, BN, KSUB);
  constexpr uint32_t A_SUB = BM * BK * 2;
  constexpr uint32_t A_BYTES = NA * A_SUB;
  constexpr uint32_t SUB_BYTES = A_BYTES + BN * BK * 2;  // one 64-wide K box set: NA weight tiles + activations
  constexpr uint32_t STAGE_BYTES = KSUB * SUB_BYTES;
  constexpr uint32_t TMEM_COLS = pow2_cols(NA * BN);
  constexpr uint32_t IDESC = nvb::idesc_bf16_f32(BM, BN);
  static_assert(SP != 2 || NA == 1, "the RS epilogue handles one 128-row weight tile per CTA");
  static_assert(SP != 2 || (size_t)BN * kSpTileLd * 2 <= (size_t)STAGES * STAGE_BYTES, "RS tile fits the ring");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ float red[32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.x / args.S, split = blockIdx.x % args.S;
  const int row0 = group * (NA * BM);  // first weight row of this CTA
  const int nsuper = args.kblocks / KSUB;  // the host picks KSUB > 1 only when it divides kblocks
  const int kb0 = (int)((long)nsuper * split / args.S);   // in stage (super-block) units
  const int kb1 = (int)((long)nsuper * (split + 1) / args.S);
  const int pre = (kb1 - kb0) < STAGES ? (kb1 - kb0) : STAGES;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      nvb::mbar_init(&full_bar[s], 1);
      nvb::mbar_init(&empty_bar[s], 1);
    }
    nvb::mbar_init(tfull_bar, 1);
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

  if (warp == 0 && lane == 0) {
    nvb::tma_prefetch_desc(&amap);
    nvb::tma_prefetch_desc(&bmap);
    // The weights are never written by earlier kernels: the first ring's weight tiles stream in before the
    // dependency wait (and, with SP == 1, before the collective), overlapping the previous kernel's tail.
    for (int it = 0; it < pre; ++it) {
      uint8_t* sa = smem + it * STAGE_BYTES;
      nvb::mbar_arrive_expect_tx(&full_bar[it], STAGE_BYTES);
#pragma unroll
      for (int ks = 0; ks < KSUB; ++ks)
#pragma unroll
        for (int j = 0; j < NA; ++j)
          nvb::tma_load_2d(sa + ks * SUB_BYTES + j * A_SUB, &amap, &full_bar[it], ((kb0 + it) * KSUB + ks) * BK,
                           row0 + j * BM);
    }
  }
  if constexpr (SP != 0) nvb::sp::stamp(sp, 0);
  nvb::pdl_wait();  // activations (and the outputs this kernel overwrites) belong to earlier kernels
  if constexpr (SP != 0) nvb::sp::stamp(sp, 1);

  if constexpr (SP == 1) {
    // while the collective is in flight, pull this CTA's remaining weight tiles (beyond the first ring) into L2
    if (warp == 0 && lane == 0)
      for (int kb = kb0 + pre; kb < kb1; ++kb)
#pragma unroll
        for (int ks = 0; ks < KSUB; ++ks)
#pragma unroll
          for (int j = 0; j < NA; ++j) nvb::tma_prefetch_l2_2d(&amap, (kb * KSUB + ks) * BK, row0 + j * BM);
    // all-gather + RMSNorm prologue: the first row_ctas CTAs reduce this rank's rows (stride row_ctas).  Only
    // CTAs of the first wave take rows: every CTA waits for all rows below, so a row owned by a CTA that could
    // only start after another exits would never arrive (a grid can exceed one wave, e.g. the LM head).
    const int row_ctas = min((int)gridDim.x, nvb::sp::kRowCtas);
    if ((int)blockIdx.x < min(nvb::sp::owned_rows(sp), row_ctas)) {
      nvb::sp::wait_rs_flags(sp, args.err);  // on timeout the error is recorded and the step runs to its end
      nvb::sp::stamp(sp, 2);
      nvb::sp::ag_norm_rows(sp, blockIdx.x, row_ctas, red);
      nvb::sp::stamp(sp, 3);
    }
    if (warp == 0) nvb::sp::wait_ag_rows_warp(sp, args.err);
    nvb::sp::stamp(sp, 4);
  }

  if (warp == 0 && lane == 0) {
    for (int it = 0; it < pre; ++it)
#pragma unroll
      for (int ks = 0; ks < KSUB; ++ks)
        nvb::tma_load_2d(smem + it * STAGE_BYTES + ks * SUB_BYTES + A_BYTES, &bmap, &full_bar[it],
                         ((kb0 + it) * KSUB + ks) * BK, 0);
    uint32_t it = pre;
    for (int kb = kb0 + pre; kb < kb1; ++kb, ++it) {
      const int s = it % STAGES;
      if (!nvb::mbar_wait(&empty_bar[s], ((it / STAGES) & 1u) ^ 1u, args.err, &abort_flag)) break;
      uint8_t* sa = smem + s * STAGE_BYTES;
      nvb::mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
#pragma unroll
      for (int ks = 0; ks < KSUB; ++ks) {
#pragma unroll
        for (int j = 0; j < NA; ++j)
          nvb::tma_load_2d(sa + ks * SUB_BYTES + j * A_SUB, &amap, &full_bar[s], (kb * KSUB + ks) * BK, row0 + j * BM);
        nvb::tma_load_2d(sa + ks * SUB_BYTES + A_BYTES, &bmap, &full_bar[s], (kb * KSUB + ks) * BK, 0);
      }
    }
  }
  if (warp == 1 && lane == 0) {
    uint32_t it = 0;
    bool ok = true;
    for (int kb = kb0; kb < kb1; ++kb, ++it) {
      const int s = it % STAGES;
      if (!nvb::mbar_wait(&full_bar[s], (it / STAGES) & 1u, args.err, &abort_flag)) { ok = false; break; }
      nvb::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < KSUB; ++ks) {
        const uint32_t a_addr = nvb::smem_u32(smem + s * STAGE_BYTES + ks * SUB_BYTES);
        const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
        for (int j = 0; j < NA; ++j)
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            nvb::tc_mma_f16(tmem_base + j * BN, nvb::sdesc_kmajor_sw128(a_addr + j * A_SUB + kk * 32),
                            nvb::sdesc_kmajor_sw128(b_addr + kk * 32), IDESC,
                            (kb > kb0 || ks > 0 || kk > 0) ? 1u : 0u);
      }
      nvb::tc_commit(&empty_bar[s]);
    }
    if (ok) nvb::tc_commit(tfull_bar);
  }
  __syncwarp();
  int ok = 0;
  if (lane == 0) ok = nvb::mbar_wait(tfull_bar, 0, args.err, &abort_flag) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  nvb::tc_fence_after();
  if constexpr (SP != 0) nvb::sp::stamp(sp, 5);

  const int r = threadIdx.x;  // TMEM lane = row inside each tile
  const uint32_t t_row = tmem_base + ((uint32_t)(warp * 32) << 16);
  if constexpr (SP == 2) {
    // ---------------------------------------------------------------- reduce-scatter epilogue (NA == 1)
    // every thread takes part (block barriers); after a timeout ``ok`` is 0 and the CTA still publishes its
    // flags, so peers do not wait for it (the error word already marks the step as failed)
    bf16* tile = reinterpret_cast<bf16*>(smem);  // the ring is idle: all stages were consumed by the MMAs
    const int f = row0 + r;
    constexpr int CH = BN < 64 ? BN : 64;
    if (args.S == 1) {
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < BN; c += CH) {
          uint32_t v[CH];
#pragma unroll
          for (int q = 0; q < CH; q += 16) nvb::tmem_ld_32x32b_x16(t_row + c + q, v + q);
          nvb::tmem_ld_wait();
          nvb::reg_fence<CH>(v);
#pragma unroll
          for (int j = 0; j < CH; ++j) tile[(c + j) * kSpTileLd + r] = __float2bfloat16(__uint_as_float(v[j]));
        }
      }
      __syncthreads();
      nvb::sp::rs_push_tile(sp, tile, kSpTileLd, 0, args.M, row0);
    } else {
      if (ok && f < args.N) {
        float* dst = args.partial + (long)split * args.M * args.N + f;
#pragma unroll 1
        for (int c = 0; c < BN; c += CH) {
          uint32_t v[CH];
#pragma unroll
          for (int q = 0; q < CH; q += 16) nvb::tmem_ld_32x32b_x16(t_row + c + q, v + q);
          nvb::tmem_ld_wait();
          nvb::reg_fence<CH>(v);
#pragma unroll
          for (int j = 0; j < CH; ++j)
            if (c + j < args.M) dst[(long)(c + j) * args.N] = __uint_as_float(v[j]);
        }
      }
      // meet the other split CTAs of this row group (co-resident: the decode grid has at most one CTA per SM)
      const uint32_t ep = *sp.epoch;
      __syncthreads();  // the CTA's partial stores precede the release below (cumulative)
      if (threadIdx.x == 0) nvb::sp::st_release_gpu(sp.split_flag + blockIdx.x, ep);
      int met = 1;
      if ((int)threadIdx.x < args.S) {
        const uint64_t t0 = nvb::global_timer_ns();
        if (!nvb::sp::wait_eq_gpu(sp.split_flag + group * args.S + threadIdx.x, ep, t0, sp.wait_ns, args.err)) {
          nvb::record_error(args.err, nvb::kErrFlagTimeout);
          met = 0;
        }
      }
      __syncthreads_and(met);
      nvb::sp::stamp(sp, 6);
      // token slice ``split`` of the group: sum the S partials in split order (float4 over 4 features, all loads
      // of an item independent so many are in flight from L2), stage bf16, push
      const int ch = (args.M + args.S - 1) / args.S;
      const int t0 = min(args.M, split * ch), t1 = min(args.M, t0 + ch);
      const int items = (t1 - t0) * (BM / 4);
#pragma unroll 4
      for (int idx = threadIdx.x; idx < items; idx += blockDim.x) {
        const int t = t0 + idx / (BM / 4), q = idx % (BM / 4);
        const int ff = row0 + q * 4;
        if (ff >= args.N) continue;  // N % 4 == 0 (checked on the host): a float4 never straddles N
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < args.S; ++s) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(args.partial + ((long)s * args.M + t) * args.N + ff));
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        uint2 packed = make_uint2(nvb::pack_bf16x2(acc.x, acc.y), nvb::pack_bf16x2(acc.z, acc.w));
        *reinterpret_cast<uint2*>(tile + (t - t0) * kSpTileLd + q * 4) = packed;
      }
      __syncthreads();
      nvb::sp::rs_push_tile(sp, tile, kSpTileLd, t0, t1, row0);
    }
    nvb::sp::stamp(sp, 7);
    nvb::sp::rs_publish(sp, blockIdx.x);
    nvb::sp::stamp(sp, 8);
  } else if (ok) {
    if (args.act != kActNone) {
      // NA == 2: tile 0 = gate rows, tile 1 = up rows of feature block ``group``
      const int f = group * BM + r;
      constexpr int CH = BN < 32 ? BN : 32;  // columns per TMEM round trip (2 x CH registers)
#pragma unroll 1
      for (int c = 0; c < BN; c += CH) {
        uint32_t g[CH], u[CH];
#pragma unroll
        for (int q = 0; q < CH; q += 16) {
          nvb::tmem_ld_32x32b_x16(t_row + c + q, g + q);
          nvb::tmem_ld_32x32b_x16(t_row + BN + c + q, u + q);
        }
        nvb::tmem_ld_wait();
        nvb::reg_fence<CH>(g);
        nvb::reg_fence<CH>(u);
        if (f < args.N / 2)
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            const int t = c + j;
            if (t < args.M) {
              const float gv = __uint_as_float(g[j]), uv = __uint_as_float(u[j]);
              args.out[(long)t * args.out_ld + f] =
                  __float2bfloat16((args.act == kActSiluMul ? silu(gv) : gelu_tanh(gv)) * uv);
            }
          }
      }
    } else {
#pragma unroll
      for (int jt = 0; jt < NA; ++jt) {
        const int f = row0 + jt * BM + r;
        constexpr int CH = BN < 64 ? BN : 64;  // columns per TMEM round trip
#pragma unroll 1
        for (int c = 0; c < BN; c += CH) {
          uint32_t v[CH];
#pragma unroll
          for (int q = 0; q < CH; q += 16) nvb::tmem_ld_32x32b_x16(t_row + jt * BN + c + q, v + q);
          nvb::tmem_ld_wait();
          nvb::reg_fence<CH>(v);
          if (f < args.N) {
            if (args.S == 1) {
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (c + j < args.M) args.out[(long)(c + j) * args.out_ld + f] = __float2bfloat16(__uint_as_float(v[j]));
            } else {
              float* dst = args.partial + (long)split * args.M * args.N + f;
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (c + j < args.M) dst[(long)(c + j) * args.N] = __uint_as_float(v[j]);
            }
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


// Split-K finish of the fused gate/up GEMM: partials [S][M][N] in the 128-row interleaved weight order
// (block b = rows [256b, 256b + 128) gate, [256b + 128, 256b + 256) up); out[m][f] = act(sum gate) * sum up for
// f = 128 b + j, sums in split order.  One thread per 4 consecutive features of one row.
__global__ void splitk_act_kernel(const float* __restrict__ partial, int S, int M, int N, bf16* __restrict__ out,
                                  long out_ld, int act) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const int I = N / 2;
  const long total4 = (long)M * I / 4;
  const long MN = (long)M * N;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total4; i += (long)gridDim.x * blockDim.x) {
    const long e = i * 4;
    const int m = (int)(e / I), f = (int)(e % I);
    const int g = (f >> 7) * 256 + (f & 127);
    const float* pg = partial + (long)m * N + g;
    float4 a = *reinterpret_cast<const float4*>(pg);
    float4 u = *reinterpret_cast<const float4*>(pg + 128);
    for (int s = 1; s < S; ++s) {
      const float4 va = *reinterpret_cast<const float4*>(pg + s * MN);
      const float4 vu = *reinterpret_cast<const float4*>(pg + s * MN + 128);
      a.x += va.x; a.y += va.y; a.z += va.z; a.w += va.w;
      u.x += vu.x; u.y += vu.y; u.z += vu.z; u.w += vu.w;
    }
    const float ga[4] = {a.x, a.y, a.z, a.w}, ua[4] = {u.x, u.y, u.z, u.w};
    uint32_t packed[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float o0 = (act == kActSiluMul ? silu(ga[2 * j]) : gelu_tanh(ga[2 * j])) * ua[2 * j];
      const float o1 = (act == kActSiluMul ? silu(ga[2 * j + 1]) : gelu_tanh(ga[2 * j + 1])) * ua[2 * j + 1];
      packed[j] = nvb::pack_bf16x2(o0, o1);
    }
    *reinterpret_cast<uint2*>(out + (long)m * out_ld + f) = make_uint2(packed[0], packed[1]);
  }
}

// out[m][n] = sum_s partial[s][m][n], fixed order (float4 over n; N % 4 == 0)
__global__ void splitk_sum_kernel(const float* __restrict__ partial, int S, long MN, bf16* __restrict__ out, int N,
                                  long out_ld) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long total4 = MN / 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total4; i += (long)gridDim.x * blockDim.x) {
    float4 acc = reinterpret_cast<const float4*>(partial)[i];
    for (int s = 1; s < S; ++s) {
      const float4 v = reinterpret_cast<const float4*>(partial + (long)s * MN)[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const long e = i * 4;
    const long m = e / N, n = e % N;
    bf16* d = out + m * out_ld + n;
    *reinterpret_cast<uint32_t*>(d) = nvb::pack_bf16x2(acc.x, acc.y);
    *reinterpret_cast<uint32_t*>(d + 2) = nvb::pack_bf16x2(acc.z, acc.w);
  }
}

template <int BN, int NA, int KSUB, int SP>
cudaError_t launch_decode(const CUtensorMap& am, const CUtensorMap& bm, const DecodeArgs& a,
                          const nvb::sp::Args& sp, int groups, cudaStream_t stream) {
  auto kern = gemm_decode_kernel<BN, NA, KSUB, SP>;
  constexpr int ST = decode_stages2(NA, BN, KSUB);
  constexpr size_t sm = 1024 + (size_t)ST * KSUB * (NA * BM * BK * 2 + BN * BK * 2) + (2 * ST + 1) * 8 + 64;
  static_assert(ST >= 1 && sm <= 227 * 1024, "decode gemm shared memory");
  static bool attr_set[64] = {false};  // per device: the attribute is a per-device function property
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (r != cudaSuccess) return r;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  C10_CUDA_CHECK(nvb::launch(kern, dim3(groups * a.S), dim3(128), sm, stream, am, bm, a, sp));
  return cudaGetLastError();
}

template <int NA, int KSUB, int SP>
cudaError_t launch_decode_bn_k(int bn, const CUtensorMap& am, const CUtensorMap& bm, const DecodeArgs& a,
                               const nvb::sp::Args& sp, int groups, cudaStream_t st) {
  switch (bn) {
    case 16: return launch_decode<16, NA, KSUB, SP>(am, bm, a, sp, groups, st);
    case 32: return launch_decode<32, NA, KSUB, SP>(am, bm, a, sp, groups, st);
    case 64: return launch_decode<64, NA, KSUB, SP>(am, bm, a, sp, groups, st);
    case 128: return launch_decode<128, NA, KSUB, SP>(am, bm, a, sp, groups, st);
    default: return launch_decode<256, NA, 1, SP>(am, bm, a, sp, groups, st);  // 256-token tiles: one box per stage
  }
}

template <int NA, int SP>
cudaError_t launch_decode_bn(int bn, int ksub, const CUtensorMap& am, const CUtensorMap& bm, const DecodeArgs& a,
                             const nvb::sp::Args& sp, int groups, cudaStream_t st) {
  return ksub == 2 ? launch_decode_bn_k<NA, 2, SP>(bn, am, bm, a, sp, groups, st)
                   : launch_decode_bn_k<NA, 1, SP>(bn, am, bm, a, sp, groups, st);
}

// 64-wide K boxes per decode pipeline stage (NVB_DECODE_KSUB, 1 or 2; default 1).
int decode_ksub() {
  static int k = -1;
  if (k < 0) {
    const char* e = getenv("NVB_DECODE_KSUB");
    k = (e && atoi(e) == 2) ? 2 : 1;
  }
  return k;
}

// Weight tiles per CTA.  Two 128-row tiles share one activation tile per K step (half the activation traffic);
// one tile per CTA doubles the number of tile groups, which halves the K splits -- and the fp32 split partials
// -- a small-N projection needs to fill the SMs.  The fused activation needs the gate/up pair (2).  Projections
// with N <= NVB_DECODE_NA1_MAXN (default 8192) use one tile.
int decode_na(int N, int act) {
  static int maxn = -1;
  if (maxn < 0) {
    const char* e = getenv("NVB_DECODE_NA1_MAXN");
    maxn = e ? atoi(e) : 8192;
  }
  if (act != kActNone) return 2;
  if (N % 256 != 0) return 1;
  return N <= maxn ? 1 : 2;
}

// K splits: make groups * S a near-multiple of the SM count (one CTA per SM), >= 4 k-blocks per split.
int decode_splits(int groups, int kblocks, int sms) {
  if (groups >= sms) return 1;
  int best = 1;
  double best_eff = (double)groups / (double)sms;
  // one wave only: a second wave repeats the pipeline fill and doubles the fp32 partials for little gain
  for (int s = 2; s <= 16 && s * 4 <= kblocks && groups * s <= sms; ++s) {
    const int u = groups * s;
    const double eff = (double)u / (double)sms;
    if (eff > best_eff + 0.03) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

template <int BN, int STAGES>
constexpr size_t gemm_smem() {
  return 1024 + STAGES * (size_t)(BM * BK * 2 + BN * BK * 2) + (2 * STAGES + 4) * 8 + 64;
}

int num_sms() {
  static int n = -1;
  if (n < 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, int STAGES>
void launch_gemm(const CUtensorMap& am, const CUtensorMap& bm, GemmArgs& a, cudaStream_t stream, int max_ctas) {
  auto kern = gemm_tc_kernel<BN, STAGES>;
  constexpr size_t sm = gemm_smem<BN, STAGES>();
  static_assert(sm <= 227 * 1024, "gemm shared memory budget");
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  const int units = a.tiles_m * a.tiles_n * a.splits;
  int grid = units < max_ctas ? units : max_ctas;
  C10_CUDA_CHECK(nvb::launch(kern, dim3(grid), dim3(192), sm, stream, am, bm, a));
}

// Decode launch shared by gemm_cuda and gemm_sp_cuda.  Returns the K splits used.
int64_t run_decode(torch::Tensor x, torch::Tensor w, bf16* out, long out_ld, int act, float* partial,
                   long partial_cap, int force_splits, int* err, bool partial_out, const nvb::sp::Args& sp,
                   int* grid_out) {
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  const int sms = num_sms();
  const int kblocks = (K + BK - 1) / BK;
  const int bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const int NA = sp.mode == 2 ? 1 : decode_na(N, act);
  DecodeArgs d{};
  d.N = N;
  d.M = M;
  d.K = K;
  d.kblocks = kblocks;
  d.act = act;
  const int groups = (N + NA * BM - 1) / (NA * BM);
  if (force_splits > 0) {
    d.S = force_splits;
  } else {
    d.S = partial != nullptr ? decode_splits(groups, kblocks, sms) : 1;
  }
  if (d.S > kblocks) d.S = kblocks;
  if (sp.mode == 2) {
    TORCH_CHECK(groups * d.S <= sms && groups * d.S <= nvb::sp::kMaxProd,
                "RS epilogue: the split CTAs of a group meet, so the grid must fit one wave");
    TORCH_CHECK(N % 4 == 0, "RS epilogue: N % 4 == 0 (float4 split reduction)");
  }
  // with split K the activation runs after the split sum (splitk_act_kernel), not in the GEMM epilogue
  if (d.S > 1 && act != kActNone) {
    TORCH_CHECK(!partial_out, "partial output is not offered for the fused-activation GEMM");
    TORCH_CHECK(out_ld % 4 == 0, "activation output rows must be 8-byte aligned");
    d.act = kActNone;
  }
  d.out = out;
  d.out_ld = out_ld;
  d.err = err;
  if (d.S > 1) {
    TORCH_CHECK(partial != nullptr && partial_cap >= (long)d.S * M * N,
                "decode gemm: fp32 partial buffer of S*M*N elements required");
    d.partial = partial;
  }
  if (getenv("NVB_GEMM_DEBUG"))
    printf("[gemm decode] M=%d N=%d K=%d bn=%d NA=%d groups=%d S=%d sp=%d\n", M, N, K, bn, NA, groups, d.S, sp.mode);
  CUtensorMap am = nvb::make_tmap_2d_bf16(w.data_ptr(), N, K, w.stride(0), BM);
  CUtensorMap bm = nvb::make_tmap_2d_bf16(x.data_ptr(), M, K, x.stride(0), bn);
  int ksub = decode_ksub();
  if (bn > 128 || kblocks % ksub != 0 || d.S > kblocks / ksub) ksub = 1;
  auto stream = at::cuda::getCurrentCUDAStream();
  cudaError_t r;
  if (sp.mode == 1)
    r = NA == 2 ? launch_decode_bn<2, 1>(bn, ksub, am, bm, d, sp, groups, stream)
                : launch_decode_bn<1, 1>(bn, ksub, am, bm, d, sp, groups, stream);
  else if (sp.mode == 2)
    r = launch_decode_bn<1, 2>(bn, ksub, am, bm, d, sp, groups, stream);
  else
    r = NA == 2 ? launch_decode_bn<2, 0>(bn, ksub, am, bm, d, sp, groups, stream)
                : launch_decode_bn<1, 0>(bn, ksub, am, bm, d, sp, groups, stream);
  TORCH_CHECK(r == cudaSuccess, "decode gemm launch failed: ", cudaGetErrorString(r));
  if (grid_out) *grid_out = groups * d.S;
  if (sp.mode == 2) return d.S;  // the epilogue reduced the splits and pushed the rows
  if (d.S > 1 && act != kActNone) {
    const long work = (long)M * (N / 2) / 4;
    int blocks = (int)((work + 255) / 256);
    if (blocks > sms * 8) blocks = sms * 8;
    C10_CUDA_CHECK(nvb::launch(splitk_act_kernel, dim3(blocks), dim3(256), 0, stream, d.partial, d.S, M, N, d.out,
                               d.out_ld, act));
  } else if (d.S > 1 && partial_out) {
    // the caller consumes the partials itself (fused into its next kernel)
  } else if (d.S > 1) {
    const long MN = (long)M * N;
    int blocks = (int)((MN / 4 + 255) / 256);
    if (blocks > sms * 8) blocks = sms * 8;
    C10_CUDA_CHECK(nvb::launch(splitk_sum_kernel, dim3(blocks), dim3(256), 0, stream, d.partial, d.S, MN, d.out, N,
                               d.out_ld));
  }
  return d.S;
}

void check_gemm_operands(const torch::Tensor& x, const torch::Tensor& w) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "gemm expects bf16 CUDA tensors");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "K must be the contiguous dimension");
  TORCH_CHECK(x.size(1) % 8 == 0, "K must be a multiple of 8 (16-byte TMA rows)");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "row strides must be 16-byte multiples");
}

}  // namespace

// y = x @ w^T (x [M, K] bf16, w [N, K] bf16) with optional activation on 128-interleaved gate/up rows of w.
// ``workspace``: fp32 [S, M, N] split-K partials for decode-sized M (S from gemm_splits_for); with ``partial_out``
// the partials are left for the consumer to sum, otherwise a sum (or split-K activation) kernel follows.
int64_t gemm_cuda(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t act, c10::optional<torch::Tensor> workspace,
                  int64_t force_splits, c10::optional<torch::Tensor> err, bool partial_out) {
  check_gemm_operands(x, w);
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(out.stride(-1) == 1, "output rows must be contiguous");
  if (act != kActNone) TORCH_CHECK(N % 256 == 0, "fused gate/up activation needs N % 256 == 0");
  if (M == 0) return 0;
  int* e = err.has_value() ? err->data_ptr<int>() : nullptr;
  if (M <= 256) {
    float* part = nullptr;
    long cap = 0;
    if (workspace.has_value()) {
      TORCH_CHECK(workspace->scalar_type() == at::kFloat && workspace->is_cuda(), "fp32 workspace");
      part = workspace->data_ptr<float>();
      cap = workspace->numel();
    }
    nvb::sp::Args none{};
    const int64_t s = run_decode(x, w, reinterpret_cast<bf16*>(out.data_ptr()), out.stride(0), (int)act, part, cap,
                                 (int)force_splits, e, partial_out, none, nullptr);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return s;
  }
  constexpr int BN = 256;
  GemmArgs a{};
  a.K = K;
  a.kblocks = (K + BK - 1) / BK;
  a.act = (int)act;
  a.err = e;
  a.Ma = M;
  a.Nb = N;
  a.tiles_m = (M + BM - 1) / BM;
  a.tiles_n = (N + BN - 1) / BN;
  a.splits = 1;
  a.out_mode = kOutBf16;
  a.out = out.data_ptr();
  a.out_ld = out.stride(0);
  CUtensorMap am = nvb::make_tmap_2d_bf16(x.data_ptr(), M, K, x.stride(0), BM);
  CUtensorMap bm = nvb::make_tmap_2d_bf16(w.data_ptr(), N, K, w.stride(0), BN);
  launch_gemm<BN, 4>(am, bm, a, at::cuda::getCurrentCUDAStream(), num_sms());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return 1;
}

// Host view of the sequence-parallel plan built by nanovllm_b200/parallel/sp.py (one int64 per field; device
// addresses as integers; per-rank arrays padded to 8).
nvb::sp::Args sp_args_from(const std::vector<int64_t>& v, double eps) {
  // layout: mode, rank, R, T, per, per_max, H, n_prod, has_res, norm_mode, wait_ns, epoch, split_flag, my_recv,
  //         my_rs_flag, residual, norm_w, recv[8], rs_flag[8], gather[8], ag_flag[8], trace
  TORCH_CHECK(v.size() == 18 + 4 * nvb::sp::kMaxRanks, "bad SP plan");
  nvb::sp::Args a{};
  a.mode = (int)v[0];
  a.rank = (int)v[1];
  a.R = (int)v[2];
  a.T = (int)v[3];
  a.per = (int)v[4];
  a.per_max = (int)v[5];
  a.H = (int)v[6];
  a.n_prod = (int)v[7];
  a.has_res = (int)v[8];
  a.norm_mode = (int)v[9];
  a.wait_ns = v[10] > 0 ? (uint64_t)v[10] : nvb::kWaitLimitNs;
  a.eps = (float)eps;
  a.epoch = reinterpret_cast<const uint32_t*>(v[11]);
  a.split_flag = reinterpret_cast<uint32_t*>(v[12]);
  a.my_recv = reinterpret_cast<const bf16*>(v[13]);
  a.my_rs_flag = reinterpret_cast<const uint32_t*>(v[14]);
  a.residual = reinterpret_cast<bf16*>(v[15]);
  a.norm_w = reinterpret_cast<const bf16*>(v[16]);
  for (int p = 0; p < nvb::sp::kMaxRanks; ++p) {
    a.recv[p] = reinterpret_cast<bf16*>(v[17 + p]);
    a.rs_flag[p] = reinterpret_cast<uint32_t*>(v[25 + p]);
    a.gather[p] = reinterpret_cast<bf16*>(v[33 + p]);
    a.ag_flag[p] = reinterpret_cast<uint32_t*>(v[41 + p]);
  }
  a.trace = reinterpret_cast<unsigned long long*>(v[49]);
  TORCH_CHECK(a.R >= 1 && a.R <= nvb::sp::kMaxRanks && a.rank >= 0 && a.rank < a.R, "bad SP rank / size");
  TORCH_CHECK(a.T >= 1 && a.T <= nvb::sp::kMaxRows && a.per >= 1 && a.per <= a.per_max, "bad SP rows");
  TORCH_CHECK(a.H % 8 == 0 && a.H <= 128 * 8 * nvb::sp::kMaxChunks, "SP rows need H % 8 == 0 and H <= 8192");
  return a;
}

// Sequence-parallel fused decode GEMM.  ``sp_plan[0]`` selects the fusion:
//   1: y = RMSNorm-all-gathered activations @ w^T -- ``x`` must be this rank's gather buffer [T, K]; the prologue
//      reduces the RS slot named in the plan, updates the residual slice, normalises and broadcasts, waits for
//      all rows, then runs the GEMM exactly like gemm_cuda (split-K partials, activation, ``partial_out``);
//   2: y = x @ w^T pushed to the owners' receive buffers (reduce-scatter); ``out`` is unused.
// Returns (K splits used, CTAs launched); the CTA count is the producer count a consumer of mode 2 waits for.
std::vector<int64_t> gemm_sp_cuda(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> out, int64_t act,
                                  c10::optional<torch::Tensor> workspace, c10::optional<torch::Tensor> err,
                                  bool partial_out, std::vector<int64_t> sp_plan, double eps) {
  check_gemm_operands(x, w);
  const int M = x.size(0), N = w.size(0);
  TORCH_CHECK(M >= 1 && M <= 256, "the SP-fused GEMM is the decode path: 1..256 tokens");
  nvb::sp::Args sp = sp_args_from(sp_plan, eps);
  TORCH_CHECK(sp.T == M, "plan rows must equal the GEMM's M");
  TORCH_CHECK(sp.mode == 1 || sp.mode == 2, "SP mode must be 1 (AG prologue) or 2 (RS epilogue)");
  if (sp.mode == 2) TORCH_CHECK(act == kActNone && sp.H == N, "RS epilogue: plain projection onto H features");
  if (sp.mode == 1) TORCH_CHECK(sp.H == x.size(1), "AG prologue: rows of H = K features");
  if (act != kActNone) TORCH_CHECK(N % 256 == 0, "fused gate/up activation needs N % 256 == 0");
  int* e = err.has_value() ? err->data_ptr<int>() : nullptr;
  float* part = nullptr;
  long cap = 0;
  if (workspace.has_value()) {
    TORCH_CHECK(workspace->scalar_type() == at::kFloat && workspace->is_cuda(), "fp32 workspace");
    part = workspace->data_ptr<float>();
    cap = workspace->numel();
  }
  bf16* o = nullptr;
  long ld = 0;
  if (sp.mode == 1) {
    TORCH_CHECK(out.has_value() && out->stride(-1) == 1, "AG GEMM output rows must be contiguous");
    o = reinterpret_cast<bf16*>(out->data_ptr());
    ld = out->stride(0);
  }
  int grid = 0;
  const int64_t s = run_decode(x, w, o, ld, (int)act, part, cap, 0, e, partial_out, sp, &grid);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {s, grid};
}

// K splits (and so the fp32 partial slices of the workspace) the decode path uses for this shape.
int64_t gemm_splits_for(int64_t M, int64_t N, int64_t K, int64_t act) {
  if (M > 256 || M <= 0) return 1;
  const int NA = decode_na((int)N, (int)act);
  const int groups = (int)((N + NA * BM - 1) / (NA * BM));
  const int kblocks = (int)((K + BK - 1) / BK);
  // a split fused-activation GEMM pays an extra fp32 round trip and a finishing kernel: only worth it when
  // at most half the SMs would otherwise hold work
  if (act != 0 && groups * 2 > num_sms()) return 1;
  int s = decode_splits(groups, kblocks, num_sms());
  return s > kblocks ? kblocks : s;
}


// out [M, N] bf16 = sum over splits of parts [S, M, N] fp32 (fixed order).
void splitk_sum_cuda(torch::Tensor parts, torch::Tensor out) {
  TORCH_CHECK(parts.scalar_type() == at::kFloat && parts.is_contiguous() && parts.dim() == 3, "parts [S, M, N] fp32");
  const int S = parts.size(0);
  const long M = parts.size(1), N = parts.size(2);
  TORCH_CHECK(N % 4 == 0 && out.stride(-1) == 1, "N must be a multiple of 4");
  const long MN = M * N;
  if (MN == 0) return;
  int blocks = (int)((MN / 4 + 255) / 256);
  if (blocks > num_sms() * 8) blocks = num_sms() * 8;
  C10_CUDA_CHECK(nvb::launch(splitk_sum_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(), 
      parts.data_ptr<float>(), S, MN, reinterpret_cast<bf16*>(out.data_ptr()), (int)N, out.stride(0)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
