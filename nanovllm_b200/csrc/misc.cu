// Small memory-bound kernels: embedding gather (+ scale, vocab-parallel masking), gated activations,
// GELU, bias add, row gather (LM-head last-token pick) and masked mean-pool + L2 normalisation.
//
// Reference ops: embedding (nano-vllm-java/.../layers/VocabParallelEmbedding.java:132-146), siluAndMul /
// geluPytorchTanhAndMul / gelu (nano-vllm-java/.../tensor/Ops.java:225-281, 348-395), the LM head's last
// prefill-token gather (VocabParallelEmbedding.java:227-252) and BERT mean pooling + L2
// (nano-vllm-java/.../models/internal/BertForEmbedding.java:85-114).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "launch.h"

namespace {
using bf16 = __nv_bfloat16;

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.7071067811865476f)); }

__global__ void embedding_kernel(bf16* __restrict__ out, const bf16* __restrict__ table, const int64_t* __restrict__ ids,
                                 int H, float scale, long vstart, long vend) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long t = blockIdx.x;
  const long id = ids[t];
  const bool inside = id >= vstart && id < vend;
  const bf16* src = table + (inside ? (id - vstart) : 0) * (long)H;
  bf16* dst = out + t * (long)H;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (inside) {
      v = *reinterpret_cast<const uint4*>(src + c);
      if (scale != 1.f) {
        bf16* e = reinterpret_cast<bf16*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = __float2bfloat16(__bfloat162float(e[j]) * scale);
      }
    }
    *reinterpret_cast<uint4*>(dst + c) = v;
  }
}

// act: 1 silu(g)*u, 2 gelu_tanh(g)*u.  layout: 0 = [gate | up] halves, 1 = 128-row interleaved blocks
__global__ void act_mul_kernel(bf16* __restrict__ out, const bf16* __restrict__ x, long rows, int I, long x_ld, int act,
                               int interleaved) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long total = rows * (long)I;
  for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
    const long r = idx / I;
    const int f = idx % I;
    int gi, ui;
    if (interleaved) {
      gi = (f >> 7) * 256 + (f & 127);
      ui = gi + 128;
    } else {
      gi = f;
      ui = f + I;
    }
    const float g = __bfloat162float(x[r * x_ld + gi]), u = __bfloat162float(x[r * x_ld + ui]);
    out[r * I + f] = __float2bfloat16((act == 1 ? silu(g) : gelu_tanh(g)) * u);
  }
}

// y = act(x + bias) in place; act: 0 none, 3 gelu(erf), 4 gelu(tanh)
__global__ void bias_act_kernel(bf16* __restrict__ x, const bf16* __restrict__ bias, long rows, int N, long ld, int act) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long total = rows * (long)N;
  for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
    const long r = idx / N;
    const int c = idx % N;
    float v = __bfloat162float(x[r * ld + c]);
    if (bias != nullptr) v += __bfloat162float(bias[c]);
    if (act == 3) v = gelu_erf(v);
    else if (act == 4) v = gelu_tanh(v);
    x[r * ld + c] = __float2bfloat16(v);
  }
}

__global__ void gather_rows_kernel(bf16* __restrict__ out, const bf16* __restrict__ src, const int64_t* __restrict__ idx,
                                   int H, long src_ld) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long r = blockIdx.x;
  const bf16* s = src + idx[r] * src_ld;
  bf16* d = out + r * (long)H;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
    *reinterpret_cast<uint4*>(d + c) = *reinterpret_cast<const uint4*>(s + c);
}

__global__ void mean_pool_l2_kernel(float* __restrict__ out, const bf16* __restrict__ x, const int* __restrict__ cu,
                                    int H) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  extern __shared__ float acc[];
  __shared__ float red[32];
  const int s = blockIdx.x;
  const int t0 = cu[s], t1 = cu[s + 1];
  float ss = 0.f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float a = 0.f;
    for (int t = t0; t < t1; ++t) a += __bfloat162float(x[(long)t * H + c]);
    a /= (float)max(1, t1 - t0);
    acc[c] = a;
    ss += a * a;
  }
  ss = nvb::warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (blockDim.x + 31) / 32; ++i) tot += red[i];
  const float inv = 1.f / fmaxf(sqrtf(tot), 1e-12f);
  for (int c = threadIdx.x; c < H; c += blockDim.x) out[(long)s * H + c] = acc[c] * inv;
}

int grid_for(long total, int threads) {
  long b = (total + threads - 1) / threads;
  return (int)(b > 148 * 16 ? 148 * 16 : (b < 1 ? 1 : b));
}

}  // namespace

void embedding_cuda(torch::Tensor out, torch::Tensor table, torch::Tensor ids, double scale, int64_t vstart,
                    int64_t vend) {
  TORCH_CHECK(table.scalar_type() == at::kBFloat16 && table.is_contiguous(), "table must be contiguous bf16");
  TORCH_CHECK(ids.scalar_type() == at::kLong, "ids must be int64");
  const long T = ids.numel();
  const int H = table.size(1);
  TORCH_CHECK(H % 8 == 0, "hidden must be a multiple of 8");
  if (T == 0) return;
  int threads = H / 8 < 256 ? ((H / 8 + 31) / 32) * 32 : 256;
  C10_CUDA_CHECK(nvb::launch(embedding_kernel, dim3(T), dim3(threads), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<bf16*>(out.data_ptr()), reinterpret_cast<const bf16*>(table.data_ptr()), ids.data_ptr<int64_t>(),
      H, (float)scale, vstart, vend));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void act_mul_cuda(torch::Tensor out, torch::Tensor x, int64_t act, bool interleaved) {
  const long rows = x.size(0);
  const int I = x.size(1) / 2;
  if (rows == 0) return;
  C10_CUDA_CHECK(nvb::launch(act_mul_kernel, dim3(grid_for(rows * I, 256)), dim3(256), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<bf16*>(out.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()), rows, I, x.stride(0),
      (int)act, interleaved ? 1 : 0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void bias_act_cuda(torch::Tensor x, c10::optional<torch::Tensor> bias, int64_t act) {
  const long rows = x.size(0);
  const int N = x.size(1);
  if (rows == 0) return;
  C10_CUDA_CHECK(nvb::launch(bias_act_kernel, dim3(grid_for(rows * N, 256)), dim3(256), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<bf16*>(x.data_ptr()), bias.has_value() ? reinterpret_cast<const bf16*>(bias->data_ptr()) : nullptr,
      rows, N, x.stride(0), (int)act));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gather_rows_cuda(torch::Tensor out, torch::Tensor src, torch::Tensor idx) {
  const long R = idx.numel();
  const int H = src.size(1);
  TORCH_CHECK(H % 8 == 0 && src.stride(1) == 1, "gather_rows needs 16-byte rows");
  if (R == 0) return;
  C10_CUDA_CHECK(nvb::launch(gather_rows_kernel, dim3(R), dim3(128), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<bf16*>(out.data_ptr()), reinterpret_cast<const bf16*>(src.data_ptr()), idx.data_ptr<int64_t>(), H,
      src.stride(0)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mean_pool_l2_cuda(torch::Tensor out, torch::Tensor x, torch::Tensor cu) {
  const int S = cu.numel() - 1;
  const int H = x.size(1);
  if (S <= 0) return;
  C10_CUDA_CHECK(nvb::launch(mean_pool_l2_kernel, dim3(S), dim3(256), H * sizeof(float), at::cuda::getCurrentCUDAStream(), 
      out.data_ptr<float>(), reinterpret_cast<const bf16*>(x.data_ptr()), cu.data_ptr<int>(), H));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
