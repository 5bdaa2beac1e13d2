// Gemma4 (text, QAT mobile) elementwise kernels.
//
// Reference graph: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/internal/Gemma4ForCausalLM.java
// :303-399 (sandwich norms with "norm, then add into the residual", per-layer input gate, layer_scalar, PLE
// combine) and GemmaQat.java:~95 (SRQ activation fake-quant: round(v / s) clamped to [-128, 127], times s;
// Java's Math.round rounds halves up, i.e. floor(v / s + 0.5)).
//
//  rms_norm_post_add : residual = (residual + rmsnorm(x) * w) * post_scale     one CTA per row
//  ple_combine       : out = (rmsnorm(proj * proj_scale) * w + tok) * out_scale   one warp per (token, layer)
//  gate_act_mul      : out = gelu_tanh(gate) * other   (other may be a column slice of a wider tensor)
//  srq               : x = clamp(floor(x / s + 0.5), -128, 127) * s, in place on a row-strided 2D view
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "launch.h"

namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}

__device__ __forceinline__ float block_sum32(float v, float* red) {
  v = nvb::warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = (blockDim.x + 31) >> 5;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// Each thread owns up to 4 vectors of 8 elements (H <= 32768 with 1024 threads).
__global__ void rms_norm_post_add_kernel(const bf16* __restrict__ x, long x_stride, bf16* __restrict__ residual,
                                         const bf16* __restrict__ w, int H, float eps, int mode, float post_scale) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ float red[32];
  const long row = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x;
  float v[4][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int col = (tid + i * nt) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    if (col < H) {
      uint4 raw = *reinterpret_cast<const uint4*>(x + row * x_stride + col);
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][j] = __bfloat162float(e[j]);
        ss += v[i][j] * v[i][j];
      }
    }
  }
  ss = block_sum32(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int col = (tid + i * nt) * 8;
    if (col >= H) continue;
    float g[8];
    if (mode == 2) {
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = 1.f;
    } else {
      uint4 raw = *reinterpret_cast<const uint4*>(w + col);
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = __bfloat162float(e[j]) + (mode == 1 ? 1.f : 0.f);
    }
    bf16* rp = residual + row * (long)H + col;
    uint4 rraw = *reinterpret_cast<const uint4*>(rp);
    const bf16* re = reinterpret_cast<const bf16*>(&rraw);
    uint4 packed;
    uint32_t* p = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // the normed branch is rounded to bf16 first, as a separate norm launch would store it
      const float n0 = __bfloat162float(__float2bfloat16(v[i][2 * j] * inv * g[2 * j]));
      const float n1 = __bfloat162float(__float2bfloat16(v[i][2 * j + 1] * inv * g[2 * j + 1]));
      p[j] = nvb::pack_bf16x2((__bfloat162float(re[2 * j]) + n0) * post_scale,
                              (__bfloat162float(re[2 * j + 1]) + n1) * post_scale);
    }
    *reinterpret_cast<uint4*>(rp) = packed;
  }
}

// rows = T * L; each row has P elements (P % 32 == 0, P <= 1024).
__global__ void ple_combine_kernel(bf16* __restrict__ out, const bf16* __restrict__ proj, const bf16* __restrict__ tok,
                                   const bf16* __restrict__ w, long rows, int P, float eps, float proj_scale,
                                   float out_scale) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bf16* pr = proj + row * P;
  float v[32];
  const int per = P / 32;
  float ss = 0.f;
  for (int i = 0; i < per; ++i) {
    // the scaled projection is what the reference stores before normalising
    v[i] = __bfloat162float(__float2bfloat16(__bfloat162float(pr[lane + 32 * i]) * proj_scale));
    ss += v[i] * v[i];
  }
  ss = nvb::warp_sum(ss);
  const float inv = rsqrtf(ss / (float)P + eps);
  for (int i = 0; i < per; ++i) {
    const int c = lane + 32 * i;
    const float n = __bfloat162float(__float2bfloat16(v[i] * inv * __bfloat162float(w[c])));
    out[row * P + c] = __float2bfloat16((n + __bfloat162float(tok[row * P + c])) * out_scale);
  }
}

__global__ void gate_act_mul_kernel(bf16* __restrict__ out, const bf16* __restrict__ gate, long g_ld,
                                    const bf16* __restrict__ other, long o_ld, long rows, int cols) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const long r = i / cols;
  const int c = (int)(i % cols);
  const float g = __bfloat162float(gate[r * g_ld + c]);
  out[r * cols + c] = __float2bfloat16(gelu_tanh_f(g) * __bfloat162float(other[r * o_ld + c]));
}

__global__ void srq_kernel(bf16* __restrict__ x, long ld, long rows, int cols, float scale) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const long r = i / cols;
  const int c = (int)(i % cols);
  bf16* p = x + r * ld + c;
  float q = floorf(__bfloat162float(*p) / scale + 0.5f);
  q = fminf(fmaxf(q, -128.f), 127.f);
  *p = __float2bfloat16(q * scale);
}

unsigned blocks_for(long n, int t) { return (unsigned)((n + t - 1) / t); }

void check_bf16(const torch::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, n, " must be a bf16 CUDA tensor");
  TORCH_CHECK(t.stride(-1) == 1, n, " rows must be contiguous");
}

}  // namespace

void rms_norm_post_add_cuda(torch::Tensor x, torch::Tensor residual, c10::optional<torch::Tensor> weight, double eps,
                            int64_t mode, double post_scale) {
  check_bf16(x, "x");
  check_bf16(residual, "residual");
  TORCH_CHECK(residual.is_contiguous(), "residual must be contiguous");
  const int H = x.size(-1);
  TORCH_CHECK(H % 8 == 0 && H == residual.size(-1), "hidden size must match and be a multiple of 8");
  const long rows = x.numel() / H;
  if (rows == 0) return;
  const bf16* w = nullptr;
  if (mode != 2) {
    TORCH_CHECK(weight.has_value(), "weight required");
    check_bf16(*weight, "weight");
    w = reinterpret_cast<const bf16*>(weight->data_ptr());
  }
  int threads = ((H / 8 + 31) / 32) * 32;
  if (threads > 1024) threads = 1024;
  TORCH_CHECK((H / 8 + threads - 1) / threads <= 4, "hidden size too large");
  C10_CUDA_CHECK(nvb::launch(rms_norm_post_add_kernel, dim3(rows), dim3(threads), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<const bf16*>(x.data_ptr()), x.dim() > 1 ? x.stride(-2) : H,
      reinterpret_cast<bf16*>(residual.data_ptr()), w, H, (float)eps, (int)mode, (float)post_scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ple_combine_cuda(torch::Tensor out, torch::Tensor proj, torch::Tensor tok, torch::Tensor weight, double eps,
                      double proj_scale, double out_scale) {
  check_bf16(out, "out");
  check_bf16(proj, "proj");
  check_bf16(tok, "tok");
  check_bf16(weight, "weight");
  TORCH_CHECK(out.is_contiguous() && proj.is_contiguous() && tok.is_contiguous(), "contiguous tensors required");
  const int P = weight.numel();
  TORCH_CHECK(P % 32 == 0 && P <= 1024, "per-layer width must be a multiple of 32 and <= 1024");
  TORCH_CHECK(proj.numel() == tok.numel() && out.numel() == tok.numel() && tok.numel() % P == 0, "shape mismatch");
  const long rows = tok.numel() / P;
  if (rows == 0) return;
  C10_CUDA_CHECK(nvb::launch(ple_combine_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<bf16*>(out.data_ptr()), reinterpret_cast<const bf16*>(proj.data_ptr()),
      reinterpret_cast<const bf16*>(tok.data_ptr()), reinterpret_cast<const bf16*>(weight.data_ptr()), rows, P,
      (float)eps, (float)proj_scale, (float)out_scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gate_act_mul_cuda(torch::Tensor out, torch::Tensor gate, torch::Tensor other) {
  check_bf16(out, "out");
  check_bf16(gate, "gate");
  check_bf16(other, "other");
  TORCH_CHECK(out.is_contiguous() && gate.dim() == 2 && other.dim() == 2, "2D inputs, contiguous out");
  TORCH_CHECK(gate.sizes() == other.sizes() && out.sizes() == gate.sizes(), "shape mismatch");
  const long rows = gate.size(0);
  const int cols = gate.size(1);
  if (rows * cols == 0) return;
  C10_CUDA_CHECK(nvb::launch(gate_act_mul_kernel, dim3(blocks_for(rows * cols, 256)), dim3(256), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<bf16*>(out.data_ptr()), reinterpret_cast<const bf16*>(gate.data_ptr()), gate.stride(0),
      reinterpret_cast<const bf16*>(other.data_ptr()), other.stride(0), rows, cols));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void srq_cuda(torch::Tensor x, double scale) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2, "x must be 2D (a column slice is fine)");
  if (scale == 0.0 || x.numel() == 0) return;
  const long rows = x.size(0);
  const int cols = x.size(1);
  C10_CUDA_CHECK(nvb::launch(srq_kernel, dim3(blocks_for(rows * cols, 256)), dim3(256), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<bf16*>(x.data_ptr()), x.stride(0), rows, cols, (float)scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
