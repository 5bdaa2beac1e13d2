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
    bf16* dst = sp.recv[owner] + ((size_t)sp.rank * sp.per_max + local) * H;
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
      *reinterpret_cast<uint4*>(dst + c) = v;
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
    bf16* dst = sp.recv[owner] + ((size_t)sp.rank * sp.per_max + local) * H;
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
      *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(x + (size_t)t * ld + c);
  }
  nvb::sp::rs_publish(sp, blockIdx.x);
}

__global__ void __launch_bounds__(128) sp_ag_norm_kernel(const __grid_constant__ nvb::sp::Args sp, int* err) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ float red[32];
  if ((int)blockIdx.x < nvb::sp::owned_rows(sp)) {
    nvb::sp::wait_rs_flags(sp, err);
    nvb::sp::ag_norm_rows(sp, blockIdx.x, gridDim.x, red);
  }
  if (threadIdx.x < 32) nvb::sp::wait_ag_rows_warp(sp, err);  // every CTA: the kernel ends when all rows landed
}

}  // namespace

nvb::sp::Args sp_args_from(const std::vector<int64_t>& v, double eps);

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
  if (grid < 1) grid = 1;
  C10_CUDA_CHECK(nvb::launch(sp_ag_norm_kernel, dim3(grid), dim3(128), 0, at::cuda::getCurrentCUDAStream(), sp,
                             err.has_value() ? err->data_ptr<int>() : nullptr));
}
