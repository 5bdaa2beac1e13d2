// LFM2 gated short convolution with per-sequence recurrent state.
//
// Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/ShortConv.java:102-243 -- in_proj gives
// [B | C | x] (3 x hidden); bx = B * x; a causal depthwise conv of kernel L over bx using the previous L-1 bx rows
// of the sequence (its conv state; zeros for a fresh sequence); y = C * conv(bx).  Prefill walks each sequence's
// token range and leaves its last L-1 bx rows in the state; decode shifts the state by one row.
// One CTA per (128-channel chunk, sequence); each thread owns one channel and keeps the window in registers, so a
// whole chunked-prefill range is processed in order without a second pass.  State arena: fp32
// [rows, width], layer slice [L-1][hidden] starting at ``state_off``.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "launch.h"

namespace {
using bf16 = __nv_bfloat16;
constexpr int kMaxL = 8;

__global__ void shortconv_kernel(const bf16* __restrict__ proj, long proj_ld, const float* __restrict__ weight, int L,
                                 int H, const int* __restrict__ cu, const int64_t* __restrict__ rows,
                                 const bool* __restrict__ fresh, float* __restrict__ state, long state_ld,
                                 long state_off, bf16* __restrict__ out) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  const int s = blockIdx.y;
  if (h >= H) return;
  const int t0 = cu[s], t1 = cu[s + 1];
  if (t1 <= t0) return;
  float w[kMaxL];
#pragma unroll
  for (int k = 0; k < kMaxL; ++k) w[k] = k < L ? weight[(long)h * L + k] : 0.f;
  float win[kMaxL];  // win[0] oldest ... win[L-2] newest previous bx
  float* st = state + rows[s] * state_ld + state_off;
  const bool is_fresh = fresh[s];
#pragma unroll
  for (int k = 0; k < kMaxL; ++k) win[k] = (k < L - 1 && !is_fresh) ? st[(long)k * H + h] : 0.f;
  for (int t = t0; t < t1; ++t) {
    const bf16* p = proj + (long)t * proj_ld;
    const float b = __bfloat162float(p[h]);
    const float c = __bfloat162float(p[H + h]);
    const float x = __bfloat162float(p[2 * H + h]);
    const float bx = b * x;
    float acc = w[L - 1] * bx;
#pragma unroll
    for (int k = 0; k < kMaxL - 1; ++k)
      if (k < L - 1) acc += w[k] * win[k];
#pragma unroll
    for (int k = 0; k < kMaxL - 2; ++k)
      if (k < L - 2) win[k] = win[k + 1];
    if (L >= 2) win[L - 2] = bx;
    out[(long)t * H + h] = __float2bfloat16(c * acc);
  }
#pragma unroll
  for (int k = 0; k < kMaxL - 1; ++k)
    if (k < L - 1) st[(long)k * H + h] = win[k];
}

}  // namespace

// proj [T, 3H] bf16; weight [H, L] fp32; cu [S+1] int32 token ranges; rows [S] int64 arena rows; fresh [S] bool;
// state [R, width] fp32 (layer slice at state_off); out [T, H] bf16
void shortconv_cuda(torch::Tensor proj, torch::Tensor weight, torch::Tensor cu, torch::Tensor rows, torch::Tensor fresh,
                    torch::Tensor state, int64_t state_off, torch::Tensor out) {
  const int H = weight.size(0), L = weight.size(1);
  TORCH_CHECK(L >= 1 && L <= kMaxL, "conv kernel length must be 1..8");
  TORCH_CHECK(proj.size(1) == 3 * H && proj.stride(1) == 1, "proj must be [T, 3H]");
  TORCH_CHECK(weight.scalar_type() == at::kFloat && weight.is_contiguous(), "weight must be fp32 [H, L]");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous(), "state must be fp32");
  const int S = cu.numel() - 1;
  if (S <= 0) return;
  dim3 grid((H + 127) / 128, S);
  C10_CUDA_CHECK(nvb::launch(shortconv_kernel, dim3(grid), dim3(128), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<const bf16*>(proj.data_ptr()), proj.stride(0), weight.data_ptr<float>(), L, H,
      cu.data_ptr<int>(), rows.data_ptr<int64_t>(), fresh.data_ptr<bool>(), state.data_ptr<float>(), state.size(1),
      state_off, reinterpret_cast<bf16*>(out.data_ptr())));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
