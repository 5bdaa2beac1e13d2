// Fused per-head Q/K RMSNorm + NeoX RoPE + paged KV-cache store.
//
// Reference ops: per-head q_norm / k_norm (nano-vllm-java/.../models/internal/Qwen3ForCausalLM.java:224-227),
// NeoX half-split rotation with a cos/sin table (nano-vllm-java/.../layers/Norms.java:171-346; the
// proportional Gemma4 variant is a table whose high frequencies are 0, i.e. cos 1 / sin 0), Gemma4's
// weightless v-norm, and storeKvCache (nano-vllm-java/.../layers/Attention.java:221-240).
// One CTA per token; one warp per head.  Input is the packed qkv GEMM output [T, (nq + 2 nkv) * hd];
// q goes to q_out [T, nq, hd], k and v go to the cache pages [num_blocks, nkv, block_size, hd].
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "launch.h"

namespace {

// norm_mode: -1 none, 0 x*w, 1 x*(1+w), 2 weightless
template <int PAIRS>  // pairs per lane = hd / 64
__global__ void qk_norm_rope_store_kernel(
    const __nv_bfloat16* __restrict__ qkv, long qkv_stride, const int64_t* __restrict__ positions,
    const float* __restrict__ cos_sin, int rot_stride, const __nv_bfloat16* __restrict__ q_w,
    const __nv_bfloat16* __restrict__ k_w, int norm_mode, int v_norm, float eps, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache, const int32_t* __restrict__ slots,
    int nq, int nkv, int block_size, int apply_rope, const float* __restrict__ qkv_part, int nsplit, long part_stride) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  constexpr int HD = PAIRS * 64;
  constexpr int HALF = HD / 2;
  const long t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int64_t pos = positions[t];
  const float* cs = cos_sin + pos * (long)rot_stride;
  const int32_t slot = slots != nullptr ? slots[t] : -1;
  const __nv_bfloat16* row = qkv + t * qkv_stride;
  const int total = nq + 2 * nkv;
  // blockIdx.y picks a chunk of nwarps heads: more CTAs in flight when the input is split-K partials
  const int h_end = min(total, (int)(blockIdx.y + 1) * nwarps);
  for (int h = blockIdx.y * nwarps + warp; h < h_end; h += nwarps) {
    const bool is_q = h < nq, is_k = (h >= nq && h < nq + nkv), is_v = h >= nq + nkv;
    float lo[PAIRS], hi[PAIRS];
    if (qkv_part == nullptr) {
      const __nv_bfloat16* src = row + (long)h * HD;
#pragma unroll
      for (int p = 0; p < PAIRS; ++p) {
        lo[p] = __bfloat162float(src[lane + 32 * p]);
        hi[p] = __bfloat162float(src[lane + 32 * p + HALF]);
      }
    } else {
      // sum of split-K partials [nsplit][T][width] (fp32), in split order
      const float* src = qkv_part + t * (long)total * HD + (long)h * HD;
#pragma unroll
      for (int p = 0; p < PAIRS; ++p) lo[p] = hi[p] = 0.f;
      int sp = 0;
      for (; sp + 4 <= nsplit; sp += 4) {  // four splits' loads in flight, still added in split order
#pragma unroll
        for (int p = 0; p < PAIRS; ++p) {
          float a[4], b[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            a[u] = src[(sp + u) * part_stride + lane + 32 * p];
            b[u] = src[(sp + u) * part_stride + lane + 32 * p + HALF];
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            lo[p] += a[u];
            hi[p] += b[u];
          }
        }
      }
      for (; sp < nsplit; ++sp) {
#pragma unroll
        for (int p = 0; p < PAIRS; ++p) {
          lo[p] += src[sp * part_stride + lane + 32 * p];
          hi[p] += src[sp * part_stride + lane + 32 * p + HALF];
        }
      }
    }
    const int mode = is_v ? (v_norm ? 2 : -1) : norm_mode;
    if (mode >= 0) {
      float ss = 0.f;
#pragma unroll
      for (int p = 0; p < PAIRS; ++p) ss += lo[p] * lo[p] + hi[p] * hi[p];
      ss = nvb::warp_sum(ss);
      const float inv = rsqrtf(ss / (float)HD + eps);
      const __nv_bfloat16* w = is_q ? q_w : k_w;
#pragma unroll
      for (int p = 0; p < PAIRS; ++p) {
        float wl = 1.f, wh = 1.f;
        if (mode != 2) {
          wl = __bfloat162float(w[lane + 32 * p]) + (mode == 1 ? 1.f : 0.f);
          wh = __bfloat162float(w[lane + 32 * p + HALF]) + (mode == 1 ? 1.f : 0.f);
        }
        lo[p] = lo[p] * inv * wl;
        hi[p] = hi[p] * inv * wh;
      }
    }
    if (!is_v && apply_rope) {
#pragma unroll
      for (int p = 0; p < PAIRS; ++p) {
        const int i = lane + 32 * p;
        const float c = cs[i], s = cs[HALF + i];
        const float a = lo[p], b = hi[p];
        lo[p] = a * c - b * s;
        hi[p] = b * c + a * s;
      }
    }
    __nv_bfloat16* dst;
    if (is_q) {
      dst = q_out + (t * nq + h) * (long)HD;
    } else {
      if (slot < 0) continue;
      const int kvh = is_k ? (h - nq) : (h - nq - nkv);
      const long blk = slot / block_size, off = slot % block_size;
      __nv_bfloat16* cache = is_k ? k_cache : v_cache;
      dst = cache + ((blk * nkv + kvh) * (long)block_size + off) * HD;
    }
#pragma unroll
    for (int p = 0; p < PAIRS; ++p) {
      dst[lane + 32 * p] = __float2bfloat16(lo[p]);
      dst[lane + 32 * p + HALF] = __float2bfloat16(hi[p]);
    }
  }
}

}  // namespace

void qk_norm_rope_store_cuda(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                             c10::optional<torch::Tensor> q_w, c10::optional<torch::Tensor> k_w, int64_t norm_mode,
                             bool v_norm, double eps, torch::Tensor q_out, c10::optional<torch::Tensor> k_cache,
                             c10::optional<torch::Tensor> v_cache, c10::optional<torch::Tensor> slots, int64_t nq,
                             int64_t nkv, int64_t head_dim, bool apply_rope, c10::optional<torch::Tensor> qkv_part) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16, "qkv must be bf16 CUDA");
  TORCH_CHECK(qkv.stride(-1) == 1, "qkv rows must be contiguous");
  TORCH_CHECK(positions.scalar_type() == at::kLong, "positions must be int64");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(-1) == head_dim, "cos_sin must be fp32 [pos, hd]");
  TORCH_CHECK(head_dim % 64 == 0 && head_dim <= 512, "head_dim must be a multiple of 64 and <= 512");
  const long T = qkv.size(0);
  if (T == 0) return;
  const __nv_bfloat16* qw = q_w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(q_w->data_ptr()) : nullptr;
  const __nv_bfloat16* kw = k_w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(k_w->data_ptr()) : nullptr;
  if (norm_mode == 0 || norm_mode == 1) TORCH_CHECK(qw && kw, "q/k norm weights required");
  __nv_bfloat16* kc = k_cache.has_value() ? reinterpret_cast<__nv_bfloat16*>(k_cache->data_ptr()) : nullptr;
  __nv_bfloat16* vc = v_cache.has_value() ? reinterpret_cast<__nv_bfloat16*>(v_cache->data_ptr()) : nullptr;
  const int32_t* sl = slots.has_value() ? slots->data_ptr<int32_t>() : nullptr;
  int block_size = 1;
  if (kc != nullptr) {
    TORCH_CHECK(sl != nullptr, "slot mapping required with a cache");
    TORCH_CHECK(k_cache->dim() == 4 && k_cache->size(1) == nkv && k_cache->size(3) == head_dim,
                "k_cache must be [num_blocks, nkv, block_size, hd]");
    block_size = k_cache->size(2);
  } else {
    sl = nullptr;
  }
  const int total = nq + 2 * nkv;
  int warps = total < 8 ? total : 8;
  const float* qp = nullptr;
  int nsplit = 0;
  long pstride = 0;
  if (qkv_part.has_value()) {
    TORCH_CHECK(qkv_part->scalar_type() == at::kFloat && qkv_part->is_contiguous() && qkv_part->dim() == 3 &&
                    qkv_part->size(1) == T && qkv_part->size(2) == (long)total * head_dim,
                "qkv_part must be contiguous fp32 [splits, T, (nq + 2 nkv) * hd]");
    qp = qkv_part->data_ptr<float>();
    nsplit = qkv_part->size(0);
    pstride = T * (long)total * head_dim;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
#define LAUNCH(P)                                                                                                  \
  C10_CUDA_CHECK(nvb::launch(qk_norm_rope_store_kernel<P>, dim3(dim3((unsigned)T, (unsigned)((total + warps - 1) / warps))), dim3(warps * 32), 0, stream,                                                       \
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), positions.data_ptr<int64_t>(),        \
      cos_sin.data_ptr<float>(), (int)cos_sin.size(-1), qw, kw, (int)norm_mode, v_norm ? 1 : 0, (float)eps,         \
      reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), kc, vc, sl, (int)nq, (int)nkv, block_size, apply_rope ? 1 : 0, \
      qp, nsplit, pstride))
  switch (head_dim / 64) {
    case 1: LAUNCH(1); break;
    case 2: LAUNCH(2); break;
    case 4: LAUNCH(4); break;
    case 8: LAUNCH(8); break;
    default: TORCH_CHECK(false, "unsupported head_dim ", head_dim);
  }
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
