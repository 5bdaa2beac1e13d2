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
//    dimension and the tokens are the N dimension; the K range is split over the CTAs of a thread-block
//    cluster so every SM streams weights, and the split partials are reduced through distributed shared memory
//    in a fixed order (deterministic), with the activation applied there.
// Every mbarrier wait is bounded; on timeout the kernel records an error code and all roles exit, TMEM is
// freed, and the host sees the code through the error word.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
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

  // unit -> (tile_m fastest, then tile_n, then split): concurrently running CTAs share B tiles.
  auto decode_unit = [&](int u, int& tm, int& tn, int& sp) {
    tm = u % args.tiles_m;
    const int r = u / args.tiles_m;
    tn = r % args.tiles_n;
    sp = r / args.tiles_n;
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
struct DecodeArgs {
  int N, M, K, kblocks, S, act;
  int cluster;  // 1: the S split CTAs of a row group form a cluster and reduce through distributed smem
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

// KSUB: 64-wide K boxes per pipeline stage.  Loading KSUB adjacent boxes of the same weight rows back to back
// turns each weight row's 128-byte reads into KSUB * 128 contiguous bytes per stage (better DRAM page use).
template <int BN, int NA, int KSUB>
__global__ void __launch_bounds__(128, 1) gemm_decode_kernel(const __grid_constant__ CUtensorMap amap,
                                                             const __grid_constant__ CUtensorMap bmap,
                                                             DecodeArgs args) {
  constexpr int STAGES = decode_stages2(NA, BN, KSUB);
  constexpr uint32_t A_SUB = BM * BK * 2;
  constexpr uint32_t A_BYTES = NA * A_SUB;
  constexpr uint32_t SUB_BYTES = A_BYTES + BN * BK * 2;  // one 64-wide K box set: NA weight tiles + activations
  constexpr uint32_t STAGE_BYTES = KSUB * SUB_BYTES;
  constexpr uint32_t TMEM_COLS = pow2_cols(NA * BN);
  constexpr uint32_t IDESC = nvb::idesc_bf16_f32(BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.x / args.S, split = blockIdx.x % args.S;
  const int row0 = group * (NA * BM);  // first weight row of this CTA
  const int nsuper = args.kblocks / KSUB;  // the host picks KSUB > 1 only when it divides kblocks
  const int kb0 = (int)((long)nsuper * split / args.S);   // in stage (super-block) units
  const int kb1 = (int)((long)nsuper * (split + 1) / args.S);

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
    // dependency wait, overlapping the previous kernel's tail; the activation tiles follow after it.
    const int pre = (kb1 - kb0) < STAGES ? (kb1 - kb0) : STAGES;
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
    nvb::pdl_wait();
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
  } else {
    nvb::pdl_wait();  // the epilogue writes outputs a previous kernel may still read
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

  if (args.cluster) {
    // Split K reduced inside the cluster: every CTA parks its fp32 tile(s) in its own (now idle) ring memory,
    // then CTA q of the cluster sums token columns [q*ch, (q+1)*ch) over the S peers in rank order (the same
    // result whatever the timing) and writes the bf16 (or activated) output.  No fp32 partials leave the SMs.
    // ``ok`` may differ between CTAs after a timeout: every CTA still joins both cluster barriers.
    const int r = threadIdx.x;
    const uint32_t t_row = tmem_base + ((uint32_t)(warp * 32) << 16);
    float* red = reinterpret_cast<float*>(smem);  // [NA][BN][128] fp32, fits the ring (checked on the host)
    if (ok) {
#pragma unroll
      for (int jt = 0; jt < NA; ++jt) {
        constexpr int CH = BN < 32 ? BN : 32;
#pragma unroll 1
        for (int c = 0; c < BN; c += CH) {
          uint32_t v[CH];
#pragma unroll
          for (int q = 0; q < CH; q += 16) nvb::tmem_ld_32x32b_x16(t_row + jt * BN + c + q, v + q);
          nvb::tmem_ld_wait();
          nvb::reg_fence<CH>(v);
#pragma unroll
          for (int j = 0; j < CH; ++j) red[((size_t)jt * BN + c + j) * BM + r] = __uint_as_float(v[j]);
        }
      }
    }
    nvb::cluster_sync();  // all partial tiles of the cluster are in place
    const int q = split, S = args.S;
    const int ch = (BN + S - 1) / S, t0 = q * ch, t1 = min(args.M, min(BN, t0 + ch));
    const uint32_t red_addr = nvb::smem_u32(red);
    if (ok) {
      if (args.act != kActNone) {
        const int f = group * BM + r;
        for (int t = t0; t < t1; ++t) {
          float gsum = 0.f, usum = 0.f;
          for (int p = 0; p < S; ++p) {
            const uint32_t peer = nvb::map_peer(red_addr, (uint32_t)p);
            gsum += nvb::ld_dsmem_f32(peer + (uint32_t)(((size_t)t * BM + r) * 4));
            usum += nvb::ld_dsmem_f32(peer + (uint32_t)(((size_t)(BN + t) * BM + r) * 4));
          }
          if (f < args.N / 2)
            args.out[(long)t * args.out_ld + f] =
                __float2bfloat16((args.act == kActSiluMul ? silu(gsum) : gelu_tanh(gsum)) * usum);
        }
      } else {
#pragma unroll
        for (int jt = 0; jt < NA; ++jt) {
          const int f = row0 + jt * BM + r;
          for (int t = t0; t < t1; ++t) {
            float sum = 0.f;
            for (int p = 0; p < S; ++p)
              sum += nvb::ld_dsmem_f32(nvb::map_peer(red_addr, (uint32_t)p) +
                                       (uint32_t)(((size_t)(jt * BN + t) * BM + r) * 4));
            if (f < args.N) args.out[(long)t * args.out_ld + f] = __float2bfloat16(sum);
          }
        }
      }
    }
    nvb::cluster_sync();  // no CTA leaves while a peer still reads its shared memory
    ok = 0;               // the tile is written
  }
  if (ok) {
    const int r = threadIdx.x;  // TMEM lane = row inside each tile
    const uint32_t t_row = tmem_base + ((uint32_t)(warp * 32) << 16);
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

// ------------------------------------------------------------------------------------------------ stream-K gate/up
// Decode-sized fused gate/up GEMM (NA = 2: a 256-row group = 128 gate + 128 up rows) when there are fewer groups
// than SMs (Qwen3-8B at TP1: 96 groups of 4096-long rows on 148 SMs, so a one-CTA-per-group grid leaves a third
// of HBM bandwidth unused; opt-in, see gemm_sk_floats for the measurement).  The (group, 64-wide K block) work
// units are laid out group-major and cut into one
// contiguous, equal range per CTA (stream-K); a range covers the tail of one group and the head of the next, so a
// CTA accumulates at most two segments, in two TMEM regions.  A segment that covers a whole group goes straight
// through the act(gate) * up epilogue.  Otherwise the CTA writes its fp32 partial of the group to the workspace
// and bumps the group's arrival counter; the last CTA to arrive (no CTA ever waits for another) adds the group's
// partials in segment order -- fixed, so the result does not depend on timing -- applies the activation, writes
// bf16 and resets the counter for the next launch.
struct SkArgs {
  int N, M, K, kblocks, groups, act;
  bf16* out;
  long out_ld;
  float* ws;       // [groups][kSkMaxSeg][2][BN][128] fp32
  int* counters;   // [groups], zero between launches
  int* err;
};
constexpr int kSkMaxSeg = 3;

__device__ __forceinline__ long sk_start(long units, int P, int c) { return units * c / P; }
// CTA whose unit range contains unit x
__device__ __forceinline__ int sk_owner(long units, int P, long x) {
  int c = (int)((x * P) / units);
  while (c + 1 < P && sk_start(units, P, c + 1) <= x) ++c;
  while (c > 0 && sk_start(units, P, c) > x) --c;
  return c;
}

template <int BN>
__global__ void __launch_bounds__(128, 1) gemm_decode_sk_kernel(const __grid_constant__ CUtensorMap amap,
                                                                const __grid_constant__ CUtensorMap bmap,
                                                                SkArgs args) {
  constexpr int NA = 2;
  constexpr int STAGES = decode_stages2(NA, BN, 1);
  constexpr uint32_t A_SUB = BM * BK * 2;
  constexpr uint32_t A_BYTES = NA * A_SUB;
  constexpr uint32_t STAGE_BYTES = A_BYTES + BN * BK * 2;
  constexpr uint32_t TMEM_COLS = pow2_cols(2 * NA * BN);  // two segments x (gate, up)
  constexpr uint32_t IDESC = nvb::idesc_bf16_f32(BM, BN);
  static_assert(2 * NA * BN <= 512, "two segments of gate/up accumulators must fit TMEM");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ int last_flag[2];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x, cta = blockIdx.x;
  const long units = (long)args.groups * args.kblocks;
  const long u0 = sk_start(units, P, cta), u1 = sk_start(units, P, cta + 1);
  const int g_first = (int)(u0 / args.kblocks);

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
    const long n = u1 - u0;
    const int pre = n < STAGES ? (int)n : STAGES;
    for (int it = 0; it < pre; ++it) {  // weights first, before the dependency wait
      const long u = u0 + it;
      const int g = (int)(u / args.kblocks), kb = (int)(u % args.kblocks);
      uint8_t* sa = smem + it * STAGE_BYTES;
      nvb::mbar_arrive_expect_tx(&full_bar[it], STAGE_BYTES);
#pragma unroll
      for (int j = 0; j < NA; ++j) nvb::tma_load_2d(sa + j * A_SUB, &amap, &full_bar[it], kb * BK, g * (NA * BM) + j * BM);
    }
    nvb::pdl_wait();
    for (int it = 0; it < pre; ++it) {
      const int kb = (int)((u0 + it) % args.kblocks);
      nvb::tma_load_2d(smem + it * STAGE_BYTES + A_BYTES, &bmap, &full_bar[it], kb * BK, 0);
    }
    for (long it = pre; it < n; ++it) {
      const int s = (int)(it % STAGES);
      if (!nvb::mbar_wait(&empty_bar[s], ((it / STAGES) & 1u) ^ 1u, args.err, &abort_flag)) break;
      const long u = u0 + it;
      const int g = (int)(u / args.kblocks), kb = (int)(u % args.kblocks);
      uint8_t* sa = smem + s * STAGE_BYTES;
      nvb::mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
#pragma unroll
      for (int j = 0; j < NA; ++j) nvb::tma_load_2d(sa + j * A_SUB, &amap, &full_bar[s], kb * BK, g * (NA * BM) + j * BM);
      nvb::tma_load_2d(sa + A_BYTES, &bmap, &full_bar[s], kb * BK, 0);
    }
  } else {
    nvb::pdl_wait();  // the epilogue writes outputs a previous kernel may still read
  }
  if (warp == 1 && lane == 0) {
    bool ok = true;
    const long n = u1 - u0;
    for (long it = 0; it < n; ++it) {
      const int s = (int)(it % STAGES);
      if (!nvb::mbar_wait(&full_bar[s], (it / STAGES) & 1u, args.err, &abort_flag)) { ok = false; break; }
      nvb::tc_fence_after();
      const long u = u0 + it;
      const int seg = (int)(u / args.kblocks) - g_first;             // 0 or 1
      const bool first = (it == 0) || (u % args.kblocks == 0);       // first unit of its segment
      const uint32_t a_addr = nvb::smem_u32(smem + s * STAGE_BYTES);
      const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
      for (int j = 0; j < NA; ++j)
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          nvb::tc_mma_f16(tmem_base + (seg * NA + j) * BN, nvb::sdesc_kmajor_sw128(a_addr + j * A_SUB + kk * 32),
                          nvb::sdesc_kmajor_sw128(b_addr + kk * 32), IDESC, (!first || kk > 0) ? 1u : 0u);
      nvb::tc_commit(&empty_bar[s]);
    }
    if (ok) nvb::tc_commit(tfull_bar);
  }
  __syncwarp();
  int ok = 0;
  if (lane == 0) ok = nvb::mbar_wait(tfull_bar, 0, args.err, &abort_flag) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  ok = __syncthreads_and(ok);  // the epilogue has block barriers: every warp takes the same path
  nvb::tc_fence_after();

  const int r = threadIdx.x;  // TMEM lane = row inside each 128-row tile
  const uint32_t t_row = tmem_base + ((uint32_t)(warp * 32) << 16);
  const int nseg = (u1 > u0) ? (int)((u1 - 1) / args.kblocks) - g_first + 1 : 0;
  constexpr int CH = BN < 32 ? BN : 32;
  for (int seg = 0; ok && seg < nseg; ++seg) {
    const int g = g_first + seg;
    const long gs = (long)g * args.kblocks, ge = gs + args.kblocks;
    const int f = g * BM + r;  // output feature
    const bool whole = u0 <= gs && u1 >= ge;
    if (whole) {
#pragma unroll 1
      for (int c = 0; c < BN; c += CH) {
        uint32_t gv[CH], uv[CH];
#pragma unroll
        for (int q = 0; q < CH; q += 16) {
          nvb::tmem_ld_32x32b_x16(t_row + (seg * NA) * BN + c + q, gv + q);
          nvb::tmem_ld_32x32b_x16(t_row + (seg * NA + 1) * BN + c + q, uv + q);
        }
        nvb::tmem_ld_wait();
        nvb::reg_fence<CH>(gv);
        nvb::reg_fence<CH>(uv);
#pragma unroll
        for (int j = 0; j < CH; ++j)
          if (c + j < args.M) {
            const float x = __uint_as_float(gv[j]), y = __uint_as_float(uv[j]);
            args.out[(long)(c + j) * args.out_ld + f] =
                __float2bfloat16((args.act == kActSiluMul ? silu(x) : gelu_tanh(x)) * y);
          }
      }
      continue;
    }
    // partial segment: publish this CTA's fp32 partial, then let the last contributor finish the group
    const int c_first = sk_owner(units, P, gs), c_last = sk_owner(units, P, ge - 1);
    const int my = cta - c_first, nparts = c_last - c_first + 1;
    if (nparts > kSkMaxSeg) {  // the host only picks stream-K when every group has at most kSkMaxSeg parts
      if (threadIdx.x == 0) nvb::record_error(args.err, nvb::kErrBadArgument);
      continue;
    }
    float* slot = args.ws + ((size_t)g * kSkMaxSeg + my) * 2 * BN * BM;
#pragma unroll 1
    for (int c = 0; c < BN; c += CH) {
      uint32_t gv[CH], uv[CH];
#pragma unroll
      for (int q = 0; q < CH; q += 16) {
        nvb::tmem_ld_32x32b_x16(t_row + (seg * NA) * BN + c + q, gv + q);
        nvb::tmem_ld_32x32b_x16(t_row + (seg * NA + 1) * BN + c + q, uv + q);
      }
      nvb::tmem_ld_wait();
      nvb::reg_fence<CH>(gv);
      nvb::reg_fence<CH>(uv);
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        slot[(size_t)(c + j) * BM + r] = __uint_as_float(gv[j]);
        slot[(size_t)(BN + c + j) * BM + r] = __uint_as_float(uv[j]);
      }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_flag[seg] = atomicAdd(&args.counters[g], 1) == nparts - 1;
    __syncthreads();
    if (!last_flag[seg]) continue;
    __threadfence();
    if (threadIdx.x == 0) args.counters[g] = 0;  // ready for the next launch
    const float* base = args.ws + (size_t)g * kSkMaxSeg * 2 * BN * BM;
#pragma unroll 1
    for (int t = 0; t < args.M; ++t) {
      float x = 0.f, y = 0.f;
      for (int k = 0; k < nparts; ++k) {  // segment order
        const float* sl = base + (size_t)k * 2 * BN * BM;
        x += __ldcg(sl + (size_t)t * BM + r);
        y += __ldcg(sl + (size_t)(BN + t) * BM + r);
      }
      args.out[(long)t * args.out_ld + f] = __float2bfloat16((args.act == kActSiluMul ? silu(x) : gelu_tanh(x)) * y);
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

template <int BN, int NA, int KSUB>
cudaError_t launch_decode(const CUtensorMap& am, const CUtensorMap& bm, const DecodeArgs& a, int groups,
                          cudaStream_t stream) {
  auto kern = gemm_decode_kernel<BN, NA, KSUB>;
  constexpr int ST = decode_stages2(NA, BN, KSUB);
  constexpr size_t sm = 1024 + (size_t)ST * KSUB * (NA * BM * BK * 2 + BN * BK * 2) + (2 * ST + 1) * 8 + 64;
  static_assert(ST >= 1 && sm <= 227 * 1024, "decode gemm shared memory");
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (a.cluster) {
    constexpr bool kFits = (size_t)NA * BN * BM * 4 <= (size_t)ST * KSUB * (NA * BM * BK * 2 + BN * BK * 2);
    if constexpr (!kFits) {
      return cudaErrorInvalidValue;  // the host never asks for it (NA * BN <= 256)
    } else {
      C10_CUDA_CHECK(nvb::launch_cluster(kern, dim3(groups * a.S), dim3(128), sm, stream, (unsigned)a.S, am, bm, a));
    }
  } else {
    C10_CUDA_CHECK(nvb::launch(kern, dim3(groups * a.S), dim3(128), sm, stream, am, bm, a));
  }
  return cudaGetLastError();
}

template <int NA, int KSUB>
cudaError_t launch_decode_bn_k(int bn, const CUtensorMap& am, const CUtensorMap& bm, const DecodeArgs& a, int groups,
                               cudaStream_t st) {
  switch (bn) {
    case 16: return launch_decode<16, NA, KSUB>(am, bm, a, groups, st);
    case 32: return launch_decode<32, NA, KSUB>(am, bm, a, groups, st);
    case 64: return launch_decode<64, NA, KSUB>(am, bm, a, groups, st);
    case 128: return launch_decode<128, NA, KSUB>(am, bm, a, groups, st);
    default: return launch_decode<256, NA, 1>(am, bm, a, groups, st);  // 256-token tiles keep one box per stage
  }
}

template <int NA>
cudaError_t launch_decode_bn(int bn, int ksub, const CUtensorMap& am, const CUtensorMap& bm, const DecodeArgs& a,
                             int groups, cudaStream_t st) {
  return ksub == 2 ? launch_decode_bn_k<NA, 2>(bn, am, bm, a, groups, st)
                   : launch_decode_bn_k<NA, 1>(bn, am, bm, a, groups, st);
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

// Split K reduced through distributed shared memory inside a cluster of the split CTAs (NVB_DECODE_CLUSTER=1)
// instead of fp32 partials in global memory summed by the consuming kernel.
constexpr int kDecodeMaxCluster = 8;
bool decode_cluster_enabled() {
  const char* e = getenv("NVB_DECODE_CLUSTER");
  return e && atoi(e) == 1;
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

}  // namespace

// y = x @ w^T (x [M, K] bf16, w [N, K] bf16) with optional activation on 128-interleaved gate/up rows of w.
// ``workspace``: fp32 [S, M, N] split-K partials for decode-sized M (S from gemm_splits_for); with ``partial_out``
// the partials are left for the consumer to sum, otherwise a sum (or split-K activation) kernel follows.
int64_t gemm_cuda(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t act, c10::optional<torch::Tensor> workspace,
                  int64_t force_splits, c10::optional<torch::Tensor> err, bool partial_out) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "gemm expects bf16 CUDA tensors");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "K must be the contiguous dimension");
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(K % 8 == 0, "K must be a multiple of 8 (16-byte TMA rows)");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "row strides must be 16-byte multiples");
  TORCH_CHECK(out.stride(-1) == 1, "output rows must be contiguous");
  if (act != kActNone) TORCH_CHECK(N % 256 == 0, "fused gate/up activation needs N % 256 == 0");
  if (M == 0) return 0;
  int* e = err.has_value() ? err->data_ptr<int>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int sms = num_sms();
  const int kblocks = (K + BK - 1) / BK;
  GemmArgs a{};
  a.K = K;
  a.kblocks = kblocks;
  a.act = (int)act;
  a.err = e;
  int64_t splits_used = 1;
  if (M <= 256) {
    const int bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
    const int NA = decode_na(N, (int)act);
    DecodeArgs d{};
    d.N = N;
    d.M = M;
    d.K = K;
    d.kblocks = kblocks;
    d.act = (int)act;
    const int groups = (N + NA * BM - 1) / (NA * BM);
    const bool clus = decode_cluster_enabled();
    if (force_splits > 0) {
      d.S = (int)force_splits;
    } else if (clus) {
      d.S = decode_splits(groups, kblocks, sms);
      if (act != kActNone && groups * 2 > sms) d.S = 1;
    } else {
      d.S = workspace.has_value() ? decode_splits(groups, kblocks, sms) : 1;
    }
    if (d.S > kblocks) d.S = kblocks;
    if (clus && d.S > kDecodeMaxCluster) d.S = kDecodeMaxCluster;
    d.cluster = (clus && d.S > 1 && NA * bn <= 256) ? 1 : 0;
    if (clus && !d.cluster && d.S > 1 && !workspace.has_value()) d.S = 1;  // no partial buffer to fall back on
    // with split K the activation runs after the split sum (splitk_act_kernel), not in the GEMM epilogue --
    // unless the split CTAs reduce inside their cluster, which applies it there
    if (d.S > 1 && act != kActNone && !d.cluster) {
      TORCH_CHECK(!partial_out, "partial output is not offered for the fused-activation GEMM");
      TORCH_CHECK(out.stride(0) % 4 == 0, "activation output rows must be 8-byte aligned");
      d.act = kActNone;
    }
    splits_used = d.cluster ? 1 : d.S;  // no partials leave a cluster-reduced GEMM
    d.out = reinterpret_cast<bf16*>(out.data_ptr());
    d.out_ld = out.stride(0);
    d.err = e;
    if (d.S > 1 && !d.cluster) {
      TORCH_CHECK(workspace.has_value() && workspace->scalar_type() == at::kFloat &&
                      workspace->numel() >= (long)d.S * M * N,
                  "decode gemm: fp32 partial buffer of S*M*N elements required");
      d.partial = workspace->data_ptr<float>();
    }
    if (getenv("NVB_GEMM_DEBUG"))
      printf("[gemm decode] M=%d N=%d K=%d bn=%d NA=%d groups=%d S=%d\n", M, N, K, bn, NA, groups, d.S);
    CUtensorMap am = nvb::make_tmap_2d_bf16(w.data_ptr(), N, K, w.stride(0), BM);
    CUtensorMap bm = nvb::make_tmap_2d_bf16(x.data_ptr(), M, K, x.stride(0), bn);
    int ksub = decode_ksub();
    if (bn > 128 || kblocks % ksub != 0 || d.S > kblocks / ksub) ksub = 1;
    cudaError_t r = NA == 2 ? launch_decode_bn<2>(bn, ksub, am, bm, d, groups, stream)
                            : launch_decode_bn<1>(bn, ksub, am, bm, d, groups, stream);
    TORCH_CHECK(r == cudaSuccess, "decode gemm launch failed: ", cudaGetErrorString(r));
    if (d.cluster) {
      // reduced (and activated) inside the cluster: out is final
    } else if (d.S > 1 && act != kActNone) {
      const long work = (long)M * (N / 2) / 4;
      int blocks = (int)((work + 255) / 256);
      if (blocks > sms * 8) blocks = sms * 8;
      C10_CUDA_CHECK(nvb::launch(splitk_act_kernel, dim3(blocks), dim3(256), 0, stream, d.partial, d.S, M, N, d.out, d.out_ld, (int)act));
    } else if (d.S > 1 && partial_out) {
      // the caller consumes the partials itself (fused into its next kernel)
    } else if (d.S > 1) {
      const long MN = (long)M * N;
      int blocks = (int)((MN / 4 + 255) / 256);
      if (blocks > sms * 8) blocks = sms * 8;
      C10_CUDA_CHECK(nvb::launch(splitk_sum_kernel, dim3(blocks), dim3(256), 0, stream, d.partial, d.S, MN, d.out, N, d.out_ld));
    }
  } else {
    constexpr int BN = 256;
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
    launch_gemm<BN, 4>(am, bm, a, stream, sms);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return M <= 256 ? splits_used : 1;
}

// K splits (and so the fp32 partial slices of the workspace) the decode path uses for this shape.
int64_t gemm_splits_for(int64_t M, int64_t N, int64_t K, int64_t act) {
  if (decode_cluster_enabled()) return 1;  // split K is reduced inside clusters: callers keep no partials
  // K splits the decode path uses when the caller provides a partial buffer
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

// Stream-K fused gate/up (see gemm_decode_sk_kernel): fp32 workspace floats it needs for this shape, 0 when it is
// off or the shape does not take it (a one-CTA-per-group grid already fills the SMs, or would with a split; or
// too few groups for at most kSkMaxSeg contributors per group; or more than 128 tokens).
// Opt-in (NVB_DECODE_STREAMK=1): measured slower than the one-CTA-per-group kernel on B200 (Qwen3-8B gate_up:
// 205 vs 45 us at 128 tokens, 59 vs 35 us at 16) -- the last contributor's serial fix-up of up to three fp32
// partial tiles (up to 384 KB through one SM) sits on the critical path.
int64_t gemm_sk_floats(int64_t M, int64_t N, int64_t K, int64_t act) {
  const char* e = getenv("NVB_DECODE_STREAMK");
  const bool enabled = e && atoi(e) == 1;
  if (!enabled || act == 0 || M <= 0 || M > 128 || N % 256 != 0) return 0;
  const int sms = num_sms();
  const long groups = N / 256, kblocks = (K + BK - 1) / BK;
  if (groups >= sms || groups * 2 <= sms) return 0;
  const long units = groups * kblocks;
  if (units / sms < (kblocks + 1) / 2) return 0;  // a group would span more than kSkMaxSeg CTAs
  const int bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  return groups * kSkMaxSeg * 2 * (long)bn * BM;
}

template <int BN>
void launch_decode_sk(const CUtensorMap& am, const CUtensorMap& bm, const SkArgs& a, int grid, cudaStream_t stream) {
  auto kern = gemm_decode_sk_kernel<BN>;
  constexpr int ST = decode_stages2(2, BN, 1);
  constexpr size_t sm = 1024 + (size_t)ST * (2 * BM * BK * 2 + BN * BK * 2) + (2 * ST + 1) * 8 + 64;
  static_assert(sm <= 227 * 1024, "stream-K decode gemm shared memory");
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  C10_CUDA_CHECK(nvb::launch(kern, dim3(grid), dim3(128), sm, stream, am, bm, a));
}

// out[M, N/2] = act(x @ gate^T) * (x @ up^T) on 128-row-interleaved gate/up weights, stream-K over all SMs.
void gemm_sk_cuda(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t act, torch::Tensor workspace,
                  torch::Tensor counters, c10::optional<torch::Tensor> err) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "gemm expects bf16 CUDA tensors");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1) && x.stride(1) == 1 && w.stride(1) == 1,
              "shape mismatch");
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0 && K % 8 == 0, "16-byte TMA rows");
  TORCH_CHECK(out.stride(-1) == 1 && out.size(0) == M && out.size(1) == N / 2, "out must be [M, N/2]");
  const int64_t need = gemm_sk_floats(M, N, K, act);
  TORCH_CHECK(need > 0, "stream-K gate/up not planned for this shape");
  TORCH_CHECK(workspace.is_cuda() && workspace.scalar_type() == at::kFloat && workspace.numel() >= need,
              "stream-K workspace too small");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= N / 256,
              "stream-K counters: int32 [N/256], zero between launches");
  SkArgs a{};
  a.N = N;
  a.M = M;
  a.K = K;
  a.kblocks = (K + BK - 1) / BK;
  a.groups = N / 256;
  a.act = (int)act;
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.out_ld = out.stride(0);
  a.ws = workspace.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.err = err.has_value() ? err->data_ptr<int>() : nullptr;
  const int bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  CUtensorMap am = nvb::make_tmap_2d_bf16(w.data_ptr(), N, K, w.stride(0), BM);
  CUtensorMap bm = nvb::make_tmap_2d_bf16(x.data_ptr(), M, K, x.stride(0), bn);
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = num_sms();
  switch (bn) {
    case 16: launch_decode_sk<16>(am, bm, a, grid, stream); break;
    case 32: launch_decode_sk<32>(am, bm, a, grid, stream); break;
    case 64: launch_decode_sk<64>(am, bm, a, grid, stream); break;
    default: launch_decode_sk<128>(am, bm, a, grid, stream); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
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
