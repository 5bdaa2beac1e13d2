// RMSNorm / fused residual-add + RMSNorm / LayerNorm for bf16 activations, fp32 math.
//
// Reference math: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/tensor/Ops.java:440-576 (rmsNorm,
// addRmsNorm with the (1+w) Gemma variant and the weightless variant) and Ops.java:288-324 (layerNorm).
// One CTA per row; each thread owns 8 consecutive elements per 16-byte vector and keeps them in registers
// between the reduction and the normalisation, so a row is read once and written once.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "launch.h"

namespace {

constexpr int kMaxVecs = 4;  // up to 4 x 8 elements per thread

template <int NV>
__device__ __forceinline__ void load_vecs(const __nv_bfloat16* row, int H, int tid, int nthreads, float (&v)[NV][8]) {
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    int col = (tid + i * nthreads) * 8;
    if (col < H) {
      uint4 raw = *reinterpret_cast<const uint4*>(row + col);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(e[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    }
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = nvb::warp_sum(v);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  int nw = (blockDim.x + 31) >> 5;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// mode: 0 = x*w, 1 = x*(1+w), 2 = weightless
template <int NV>
__global__ void rms_norm_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                                __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w,
                                int H, long x_stride, long out_stride, float eps, int mode,
                                const float* __restrict__ xpart, int nsplit, long part_stride) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ float red[32];
  const long row = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x;
  float v[NV][8];
  if (xpart == nullptr) {
    load_vecs<NV>(x + row * x_stride, H, tid, nt, v);
  } else {
    // x = sum of split-K partials [nsplit][rows][H] (fp32), summed in split order
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int col = (tid + i * nt) * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
      if (col < H) {
        int sp = 0;
        for (; sp + 4 <= nsplit; sp += 4) {  // four splits' loads in flight, still added in split order
          float4 a[4], b[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float4* p = reinterpret_cast<const float4*>(xpart + (sp + u) * part_stride + row * (long)H + col);
            a[u] = p[0];
            b[u] = p[1];
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            v[i][0] += a[u].x; v[i][1] += a[u].y; v[i][2] += a[u].z; v[i][3] += a[u].w;
            v[i][4] += b[u].x; v[i][5] += b[u].y; v[i][6] += b[u].z; v[i][7] += b[u].w;
          }
        }
        for (; sp < nsplit; ++sp) {
          const float4* p = reinterpret_cast<const float4*>(xpart + sp * part_stride + row * (long)H + col);
          const float4 a = p[0], b = p[1];
          v[i][0] += a.x; v[i][1] += a.y; v[i][2] += a.z; v[i][3] += a.w;
          v[i][4] += b.x; v[i][5] += b.y; v[i][6] += b.z; v[i][7] += b.w;
        }
      }
    }
  }
  if (residual != nullptr) {
    float r[NV][8];
    load_vecs<NV>(residual + row * (long)H, H, tid, nt, r);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      int col = (tid + i * nt) * 8;
      if (col < H) {
        uint4 packed;
        uint32_t* p = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[i][j];
#pragma unroll
        for (int j = 0; j < 4; ++j) p[j] = nvb::pack_bf16x2(v[i][2 * j], v[i][2 * j + 1]);
        *reinterpret_cast<uint4*>(residual + row * (long)H + col) = packed;
        // normalise what was stored so the math sees the same rounding as the next layer's residual read
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&packed);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(e[j]);
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    int col = (tid + i * nt) * 8;
    if (col < H) {
      float g[8];
      if (mode == 2) {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = 1.f;
      } else {
        uint4 raw = *reinterpret_cast<const uint4*>(w + col);
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = __bfloat162float(e[j]) + (mode == 1 ? 1.f : 0.f);
      }
      uint4 packed;
      uint32_t* p = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        p[j] = nvb::pack_bf16x2(v[i][2 * j] * inv * g[2 * j], v[i][2 * j + 1] * inv * g[2 * j + 1]);
      *reinterpret_cast<uint4*>(out + row * out_stride + col) = packed;
    }
  }
}

template <int NV>
__global__ void layer_norm_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                                  const __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w,
                                  const __nv_bfloat16* __restrict__ b, int H, float eps) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ float red[32];
  const long row = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x;
  float v[NV][8];
  load_vecs<NV>(x + row * (long)H, H, tid, nt, v);
  if (residual != nullptr) {
    float r[NV][8];
    load_vecs<NV>(residual + row * (long)H, H, tid, nt, r);
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] += r[i][j];
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) s += v[i][j];
  const float mean = block_sum(s, red) / (float)H;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    int col = (tid + i * nt) * 8;
    if (col < H)
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += (v[i][j] - mean) * (v[i][j] - mean);
  }
  const float inv = rsqrtf(block_sum(ss, red) / (float)H + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    int col = (tid + i * nt) * 8;
    if (col < H) {
      uint4 rw = *reinterpret_cast<const uint4*>(w + col);
      uint4 rb = *reinterpret_cast<const uint4*>(b + col);
      const __nv_bfloat16* ew = reinterpret_cast<const __nv_bfloat16*>(&rw);
      const __nv_bfloat16* eb = reinterpret_cast<const __nv_bfloat16*>(&rb);
      uint4 packed;
      uint32_t* p = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a0 = (v[i][2 * j] - mean) * inv * __bfloat162float(ew[2 * j]) + __bfloat162float(eb[2 * j]);
        float a1 = (v[i][2 * j + 1] - mean) * inv * __bfloat162float(ew[2 * j + 1]) + __bfloat162float(eb[2 * j + 1]);
        p[j] = nvb::pack_bf16x2(a0, a1);
      }
      *reinterpret_cast<uint4*>(out + row * (long)H + col) = packed;
    }
  }
}

int pick_threads(int H, int* nv) {
  int vecs = H / 8;
  int threads = ((vecs + 31) / 32) * 32;
  if (threads > 1024) threads = 1024;
  *nv = (vecs + threads - 1) / threads;
  return threads;
}

void check_row_tensor(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
}

}  // namespace

// out = norm(x) or, with residual: residual += x; out = norm(residual).   x may be a row-strided view.
void rms_norm_cuda(torch::Tensor out, torch::Tensor x, c10::optional<torch::Tensor> residual,
                   c10::optional<torch::Tensor> weight, double eps, int64_t mode, c10::optional<torch::Tensor> xpart) {
  check_row_tensor(x, "x");
  check_row_tensor(out, "out");
  const int H = x.size(-1);
  TORCH_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  TORCH_CHECK(x.stride(-1) == 1 && out.stride(-1) == 1, "rows must be contiguous");
  const long rows = x.numel() / H;
  if (rows == 0) return;
  const long xs = x.dim() > 1 ? x.stride(-2) : H;
  const long os = out.dim() > 1 ? out.stride(-2) : H;
  __nv_bfloat16* res = nullptr;
  if (residual.has_value()) {
    check_row_tensor(*residual, "residual");
    TORCH_CHECK(residual->is_contiguous(), "residual must be contiguous");
    res = reinterpret_cast<__nv_bfloat16*>(residual->data_ptr());
  }
  const __nv_bfloat16* w = nullptr;
  if (mode != 2) {
    TORCH_CHECK(weight.has_value(), "weight required");
    check_row_tensor(*weight, "weight");
    w = reinterpret_cast<const __nv_bfloat16*>(weight->data_ptr());
  }
  int nv;
  int threads = pick_threads(H, &nv);
  TORCH_CHECK(nv <= kMaxVecs, "hidden size too large for rms_norm");
  auto stream = at::cuda::getCurrentCUDAStream();
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  auto* xi = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  const float* xp = nullptr;
  int nsplit = 0;
  long pstride = 0;
  if (xpart.has_value()) {
    TORCH_CHECK(xpart->scalar_type() == at::kFloat && xpart->is_contiguous() && xpart->dim() == 3 &&
                    xpart->size(1) == rows && xpart->size(2) == H,
                "xpart must be contiguous fp32 [splits, rows, H]");
    xp = xpart->data_ptr<float>();
    nsplit = xpart->size(0);
    pstride = rows * (long)H;
  }
#define LAUNCH(NVV) C10_CUDA_CHECK(nvb::launch(rms_norm_kernel<NVV>, dim3(rows), dim3(threads), 0, stream, o, xi, res, w, H, xs, os, (float)eps, (int)mode, xp, nsplit, pstride))
  switch (nv) {
    case 1: LAUNCH(1); break;
    case 2: LAUNCH(2); break;
    case 3: LAUNCH(3); break;
    default: LAUNCH(4); break;
  }
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void layer_norm_cuda(torch::Tensor out, torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor weight,
                     torch::Tensor bias, double eps) {
  check_row_tensor(x, "x");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
  const int H = x.size(-1);
  TORCH_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  const long rows = x.numel() / H;
  if (rows == 0) return;
  const __nv_bfloat16* res = residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  int nv;
  int threads = pick_threads(H, &nv);
  TORCH_CHECK(nv <= kMaxVecs, "hidden size too large for layer_norm");
  auto stream = at::cuda::getCurrentCUDAStream();
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  auto* xi = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* w = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  auto* b = reinterpret_cast<const __nv_bfloat16*>(bias.data_ptr());
#define LAUNCH(NVV) C10_CUDA_CHECK(nvb::launch(layer_norm_kernel<NVV>, dim3(rows), dim3(threads), 0, stream, o, xi, res, w, b, H, (float)eps))
  switch (nv) {
    case 1: LAUNCH(1); break;
    case 2: LAUNCH(2); break;
    case 3: LAUNCH(3); break;
    default: LAUNCH(4); break;
  }
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
