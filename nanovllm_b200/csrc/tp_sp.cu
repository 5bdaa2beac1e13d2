// Stand-alone sequence-parallel kernels around the SP-fused decode GEMMs (protocol in sp_comm.cuh).
//
//   sp_begin_kernel      bumps the forward epoch once per SP forward (every flag of the forward carries it);
//   sp_embed_rs_kernel   vocab-parallel embedding gather fused with the reduce-scatter: each rank gathers the
//                        rows of the ids in its vocabulary range (zeros elsewhere) and pushes them to the owners
//                        of the token rows, so the first layer's all-gather + RMSNorm prologue reduces them
//                        (reference: nano-vllm-java/.../layers/VocabParallelEmbedding.java:132-146);
//   sp_rs_push_kernel    reduce-scatter of a locally materialised partial [T, H] (projections without a fused
//                        GEMM epilogue, e.g. GGUF-packed weights);
//   sp_ag_norm_kernel    the all-gather + RMSNorm prologue as its own kernel, for consumers that are not an SP
//                        decode GEMM: it returns only when all T rows are in this rank's gather buffer, so any
//                        later kernel on the stream can read them.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <vector>
#include "common.cuh"
#include "launch.h"
#include "sp_comm.cuh"

namespace {
using bf16 = __nv_bfloat16;

__global__ void sp_begin_kernel(uint32_t* epoch) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  if (threadIdx.x == 0) *epoch += 1u;
}

__global__ void __launch_bounds__(128) sp_embed_rs_kernel(const __grid_constant__ nvb::sp::Args sp,
                                                          const bf16* __restrict__ table, const int64_t* __restrict__ ids,
                                                          float scale, long vstart, long vend) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const int H = sp.H;
  for (int t = blockIdx.x; t < sp.T; t += gridDim.x) {
    const long id = ids[t];
    const bool mine = id >= vstart && id < vend;
    const int owner = t / sp.per, local = t - owner * sp.per;
    const bf16* src = table + (size_t)(mine ? id - vstart : 0) * H;
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (mine) {
        v = *reinterpret_cast<const uint4*>(src + c);
        if (scale != 1.f) {
          float f[8];
          nvb::sp::unpack8(v, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] *= scale;
          v = nvb::sp::pack8(f);
        }
      }
      *reinterpret_cast<uint4*>(sp.recv[owner] + ((size_t)sp.rank * sp.per_max + local) * H + c) = v;
    }
  }
  nvb::sp::rs_publish(sp, blockIdx.x);
}

__global__ void __launch_bounds__(128) sp_rs_push_kernel(const __grid_constant__ nvb::sp::Args sp,
                                                         const bf16* __restrict__ x, long ld) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const int H = sp.H;
  for (int t = blockIdx.x; t < sp.T; t += gridDim.x) {
    const int owner = t / sp.per, local = t - owner * sp.per;
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)t * ld + c);
      *reinterpret_cast<uint4*>(sp.recv[owner] + ((size_t)sp.rank * sp.per_max + local) * H + c) = v;
    }
  }
  nvb::sp::rs_publish(sp, blockIdx.x);
}

__global__ void __launch_bounds__(128) sp_ag_norm_kernel(const __grid_constant__ nvb::sp::Args sp, int* err) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ float red[32];
  if ((int)blockIdx.x < nvb::sp::owned_rows(sp)) {  // grid <= kRowCtas: every CTA is co-resident
    nvb::sp::wait_rs_flags(sp, err);
    nvb::sp::ag_norm_rows(sp, blockIdx.x, gridDim.x, red);
  }
  if (threadIdx.x < 32) nvb::sp::wait_ag_rows_warp(sp, err);  // every CTA: the kernel ends when all rows landed
}

// Distributed greedy sampling over a vocab-parallel LM head (reference semantics: nano-vllm-java/.../layers/
// Sampler.java:38-50, top_k == 1 -> argmax, ties to the lowest token id).  Every rank scores its vocabulary
// slice [col0, col0 + ncols) of each row; phase 1 takes the row's local argmax (after the optional soft-cap,
// which is monotonic but can create ties) and stores (value, id) into every rank's exchange buffer, then flags
// it; phase 2 waits for the R flags of each of its rows and keeps the best pair.  8 bytes per row and rank
// cross NVLink instead of the [T, V] logits.  ``epoch`` comes from the host (one per call, equal on all ranks).
struct ArgmaxPeers {
  uint2* exch[nvb::sp::kMaxRanks];     // each rank's exchange buffer [R][kMaxRows] of (value bits, token id)
  uint32_t* flag[nvb::sp::kMaxRanks];  // each rank's flags [R][kMaxRows]
};

__device__ __forceinline__ bool better_pair(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(1024) sp_argmax_kernel(const bf16* __restrict__ logits, long ld, int T, int ncols,
                                                         long col0, float softcap, int64_t* __restrict__ out,
                                                         int rank, int R, uint32_t epoch, ArgmaxPeers P,
                                                         uint64_t wait_ns, int* err) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    const bf16* row = logits + (size_t)t * ld;
    for (int c = tid; c < ncols; c += blockDim.x) {
      float v = __bfloat162float(row[c]);
      if (softcap > 0.f) v = softcap * tanhf(v / softcap);
      const uint32_t i = (uint32_t)(col0 + c);
      if (better_pair(v, i, bv, bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better_pair(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (better_pair(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
      const uint2 pr = make_uint2(__float_as_uint(bv), bi);
      for (int p = 0; p < R; ++p) P.exch[p][(size_t)rank * nvb::sp::kMaxRows + t] = pr;
    }
    __syncthreads();
  }
  __syncthreads();
  if (tid < R) {
    for (int t = blockIdx.x; t < T; t += gridDim.x)
      nvb::sp::st_release_sys(P.flag[tid] + (size_t)rank * nvb::sp::kMaxRows + t, epoch);
  }
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    if (warp == 0) {
      float bv = -INFINITY;
      uint32_t bi = 0xFFFFFFFFu;
      if (lane < R) {
        const uint64_t t0 = nvb::global_timer_ns();
        if (!nvb::sp::wait_eq_sys(P.flag[rank] + (size_t)lane * nvb::sp::kMaxRows + t, epoch, t0, wait_ns, err))
          nvb::record_error(err, nvb::kErrFlagTimeout);
        const uint2 pr = __ldcg(P.exch[rank] + (size_t)lane * nvb::sp::kMaxRows + t);
        bv = __uint_as_float(pr.x);
        bi = pr.y;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better_pair(ov, oi, bv, bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) out[t] = (int64_t)bi;
    }
  }
}

}  // namespace

nvb::sp::Args sp_args_from(const std::vector<int64_t>& v, double eps);

// tokens[T] = argmax over all ranks' vocabulary slices (see sp_argmax_kernel); exch / flags: one device address
// per rank (rank order).
void sp_argmax_cuda(torch::Tensor logits, int64_t ncols, int64_t col0, double softcap, torch::Tensor out,
                    int64_t rank, std::vector<int64_t> exch, std::vector<int64_t> flags, int64_t epoch,
                    int64_t wait_ns, c10::optional<torch::Tensor> err) {
  const int R = (int)exch.size();
  TORCH_CHECK(R >= 1 && R <= nvb::sp::kMaxRanks && (int)flags.size() == R && rank >= 0 && rank < R, "bad ranks");
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 &&
                  logits.stride(1) == 1, "logits: bf16 [T, V/R] with contiguous rows");
  const int T = (int)logits.size(0);
  TORCH_CHECK(T >= 1 && T <= nvb::sp::kMaxRows && ncols >= 1 && ncols <= logits.size(1), "bad rows / columns");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kLong && out.numel() >= T, "out: int64 [T]");
  ArgmaxPeers P{};
  for (int p = 0; p < R; ++p) {
    P.exch[p] = reinterpret_cast<uint2*>(exch[p]);
    P.flag[p] = reinterpret_cast<uint32_t*>(flags[p]);
  }
  const int grid = T < 148 ? T : 148;
  C10_CUDA_CHECK(nvb::launch(sp_argmax_kernel, dim3(grid), dim3(1024), 0, at::cuda::getCurrentCUDAStream(),
                             reinterpret_cast<const bf16*>(logits.data_ptr()), (long)logits.stride(0), T, (int)ncols,
                             (long)col0, (float)softcap, out.data_ptr<int64_t>(), (int)rank, R, (uint32_t)epoch, P,
                             wait_ns > 0 ? (uint64_t)wait_ns : nvb::kWaitLimitNs,
                             err.has_value() ? err->data_ptr<int>() : nullptr));
}

void sp_begin_cuda(int64_t epoch_ptr) {
  C10_CUDA_CHECK(nvb::launch(sp_begin_kernel, dim3(1), dim3(32), 0, at::cuda::getCurrentCUDAStream(),
                             reinterpret_cast<uint32_t*>(epoch_ptr)));
}

// Returns the CTAs launched (the producer count the consuming prologue waits for).
int64_t sp_embed_rs_cuda(torch::Tensor table, torch::Tensor ids, double scale, int64_t vstart, int64_t vend,
                         std::vector<int64_t> plan) {
  nvb::sp::Args sp = sp_args_from(plan, 0.0);
  TORCH_CHECK(sp.mode == 2, "embedding push is an RS producer");
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kBFloat16 && table.is_contiguous() &&
                  table.size(1) == sp.H, "table: contiguous bf16 [V/R, H]");
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && ids.numel() == sp.T, "ids: int64 [T]");
  const int grid = sp.T < 128 ? sp.T : 128;
  C10_CUDA_CHECK(nvb::launch(sp_embed_rs_kernel, dim3(grid), dim3(128), 0, at::cuda::getCurrentCUDAStream(), sp,
                             reinterpret_cast<const bf16*>(table.data_ptr()), ids.data_ptr<int64_t>(), (float)scale,
                             (long)vstart, (long)vend));
  return grid;
}

int64_t sp_rs_push_cuda(torch::Tensor x, std::vector<int64_t> plan) {
  nvb::sp::Args sp = sp_args_from(plan, 0.0);
  TORCH_CHECK(sp.mode == 2, "RS push is an RS producer");
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.size(0) == sp.T &&
                  x.size(1) == sp.H && x.stride(1) == 1 && x.stride(0) % 8 == 0, "x: bf16 [T, H], 16-byte rows");
  const int grid = sp.T < 128 ? sp.T : 128;
  C10_CUDA_CHECK(nvb::launch(sp_rs_push_kernel, dim3(grid), dim3(128), 0, at::cuda::getCurrentCUDAStream(), sp,
                             reinterpret_cast<const bf16*>(x.data_ptr()), (long)x.stride(0)));
  return grid;
}

void sp_ag_norm_cuda(std::vector<int64_t> plan, double eps, c10::optional<torch::Tensor> err) {
  nvb::sp::Args sp = sp_args_from(plan, eps);
  TORCH_CHECK(sp.mode == 1, "AG + norm is an RS consumer");
  int grid = nvb::sp::owned_rows(sp);
  if (grid > nvb::sp::kRowCtas) grid = nvb::sp::kRowCtas;
  if (grid < 1) grid = 1;
  C10_CUDA_CHECK(nvb::launch(sp_ag_norm_kernel, dim3(grid), dim3(128), 0, at::cuda::getCurrentCUDAStream(), sp,
                             err.has_value() ? err->data_ptr<int>() : nullptr));
}
