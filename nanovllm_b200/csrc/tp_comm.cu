// Tensor-parallel collectives over NVLink peer memory (CUDA IPC mappings), fused with the math around them.
//
// The reference has no GPU or communication backend; its RowParallel linears (nano-vllm-java/.../layers/
// Linear.java:330-405) are followed by an all-reduce in the TP decomposition they name, and the next op is the
// fused residual add + RMSNorm (nano-vllm-java/.../tensor/Ops.java:440-576).  Here that chain is one kernel:
//
//   two-shot all-reduce of the row-parallel partial sums [T, H] (bf16, one buffer per rank):
//     phase A  every rank owns rows [rank*ceil(T/R), ...); it reads those rows from every peer's partial
//              buffer (peer loads over NVLink), sums them in rank order 0..R-1 (so all ranks agree bit for
//              bit), adds the residual, and
//     phase B  writes the new residual rows and the RMS-normalised rows into every rank's residual / output
//              buffers (peer stores), i.e. the all-gather is fused into the norm epilogue;
//   a block-level flag barrier before phase A (all partials written) and after phase B (all stores landed,
//   all peers done reading this rank's partial buffer) keeps producer / consumer kernels ordered across GPUs.
//
// Every flag wait is bounded (kWaitLimitNs unless the caller passes a shorter limit); on expiry the kernel records kErrFlagTimeout in the device error
// word and returns instead of hanging.  Flags carry a per-block epoch kept in device memory, so the kernel can
// be captured in CUDA graphs (every rank replays the same launches in the same order).  No TMA, no multicast.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <vector>
#include "common.cuh"
#include "launch.h"

namespace {

using bf16 = __nv_bfloat16;
constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 1024;

struct PeerPtrs {
  const bf16* in[kMaxRanks];   // row-parallel partial sums [T, H]
  bf16* res[kMaxRanks];        // residual stream [T, H]
  bf16* out[kMaxRanks];        // normalised output [T, H]
  uint32_t* sig[kMaxRanks];    // signal pads [2][kMaxBlocks][kMaxRanks]
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread t < nranks publishes this block's arrival to rank t and waits (bounded) for rank t's arrival.  With
// ``publish_writes`` the block's earlier global stores (peer stores included) are made visible at system scope
// before the flag: bar.sync orders them before the signalling thread's (cumulative) release store.
// ``sync_first`` alone (no fence) publishes "this block is done reading": the loads' values were consumed
// before bar.sync, and the release store orders them before the flag.
__device__ bool block_barrier(const PeerPtrs& P, int rank, int nranks, int phase, uint32_t epoch, int* err,
                              uint64_t wait_ns, bool publish_writes, bool sync_first = false) {
  const int t = threadIdx.x;
  int ok = 1;
  if (publish_writes || sync_first) __syncthreads();
  if (t < nranks) {
    // the release store is cumulative over the block's writes that bar.sync ordered before it: no full system
    // fence (fence.sc.sys cost 7-9 us per barrier on B200)
    st_release_sys(P.sig[t] + ((size_t)(phase * kMaxBlocks + blockIdx.x) * kMaxRanks + rank), epoch);
    const uint32_t* mine = P.sig[rank] + ((size_t)(phase * kMaxBlocks + blockIdx.x) * kMaxRanks + t);
    const uint64_t t0 = nvb::global_timer_ns();
    while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
      if (nvb::global_timer_ns() - t0 > wait_ns) {
        nvb::record_error(err, nvb::kErrFlagTimeout);
        ok = 0;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = nvb::warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
  return s;
}

__device__ __forceinline__ void unpack8(const uint4& raw, float (&f)[8]) {
  const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = __bfloat162float(e[j]);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 r;
  uint32_t* p = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) p[j] = nvb::pack_bf16x2(f[2 * j], f[2 * j + 1]);
  return r;
}

// mode: 0 x*w, 1 x*(1+w), 2 weightless, 3 no norm (plain all-reduce; out = sum (+ residual))
// oneshot: every rank reads ALL rows from every peer and writes only its own residual / output (no peer stores,
// no system fence); the closing barrier then only says "done reading your partials".  Two-shot (oneshot = 0)
// moves (R-1)/R of the bytes instead of R-1 times them and wins once the message is large.
template <int NV>
__global__ void __launch_bounds__(1024) tp_allreduce_norm_kernel(PeerPtrs P, int rank, int nranks, int T, int H,
                                                                 const bf16* __restrict__ w, float eps, int mode,
                                                                 int has_res, uint32_t* counters, int* err,
                                                                 int oneshot, uint64_t wait_ns) {
  nvb::pdl_wait();
  nvb::pdl_trigger();
  __shared__ float red[32];
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = counters[blockIdx.x] + 1;
  const int per = oneshot ? T : (T + nranks - 1) / nranks;
  const int tid = threadIdx.x, nt = blockDim.x;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (!block_barrier(P, rank, nranks, 0, epoch, err, wait_ns, false)) {
    if (threadIdx.x == 0) counters[blockIdx.x] = epoch;
    return;
  }
  const int r0 = oneshot ? 0 : rank * per, r1 = min(T, r0 + per);
  const int p_lo = oneshot ? rank : 0, p_hi = oneshot ? rank + 1 : nranks;  // ranks whose buffers get the result
  for (int row = r0 + blockIdx.x; row < r1; row += gridDim.x) {
    const size_t base = (size_t)row * H;
    float v[NV][8];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int col = (tid + i * nt) * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
      if (col < H) {
        // issue every rank's load before the first use so the NVLink latencies overlap
        uint4 raw[kMaxRanks];
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
          if (p < nranks) raw[p] = *reinterpret_cast<const uint4*>(P.in[p] + base + col);
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p) {  // fixed rank order: every owner sums identically
          if (p < nranks) {
            float f[8];
            unpack8(raw[p], f);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] += f[j];
          }
        }
        if (has_res) {
          float r[8];
          unpack8(*reinterpret_cast<const uint4*>(P.res[rank] + base + col), r);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] += r[j];
          const uint4 packed = pack8(v[i]);
#pragma unroll
          for (int p = 0; p < kMaxRanks; ++p)
            if (p >= p_lo && p < p_hi) *reinterpret_cast<uint4*>(P.res[p] + base + col) = packed;
          unpack8(packed, v[i]);  // continue from the rounded value every rank stores
        }
      }
    }
    if (mode == 3) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int col = (tid + i * nt) * 8;
        if (col >= H) continue;
        const uint4 packed = pack8(v[i]);
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
          if (p >= p_lo && p < p_hi) *reinterpret_cast<uint4*>(P.out[p] + base + col) = packed;
      }
      continue;
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
      const int col = (tid + i * nt) * 8;
      if (col >= H) continue;
      float g[8];
      if (mode == 2) {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = 1.f;
      } else {
        unpack8(*reinterpret_cast<const uint4*>(w + col), g);
        if (mode == 1)
#pragma unroll
          for (int j = 0; j < 8; ++j) g[j] += 1.f;
      }
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * g[j];
      const uint4 packed = pack8(o);
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p >= p_lo && p < p_hi) *reinterpret_cast<uint4*>(P.out[p] + base + col) = packed;
    }
  }
  block_barrier(P, rank, nranks, 1, epoch, err, wait_ns, !oneshot, true);
  if (threadIdx.x == 0) counters[blockIdx.x] = epoch;
}

}  // namespace

// ------------------------------------------------------------------------------------------------ IPC plumbing
// A dedicated cudaMalloc allocation per rank (zeroed), exported as a CUDA IPC handle; peers map it once.
std::vector<torch::Tensor> symm_alloc_cuda(int64_t nbytes) {
  TORCH_CHECK(nbytes > 0, "nbytes must be positive");
  const int dev = at::cuda::current_device();
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, (size_t)nbytes) == cudaSuccess, "symmetric buffer allocation failed");
  TORCH_CHECK(cudaMemset(p, 0, (size_t)nbytes) == cudaSuccess, "symmetric buffer memset failed");
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, p) == cudaSuccess, "cudaIpcGetMemHandle failed");
  auto buf = torch::from_blob(
      p, {nbytes}, [](void* q) { cudaFree(q); },
      torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, dev));
  auto handle = torch::empty({(int64_t)sizeof(h)}, torch::TensorOptions().dtype(torch::kUInt8));
  std::memcpy(handle.data_ptr(), &h, sizeof(h));
  return {buf, handle};
}

int64_t ipc_open_cuda(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && handle.device().is_cpu(), "bad IPC handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  const cudaError_t r = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(r == cudaSuccess, "cudaIpcOpenMemHandle failed: ", cudaGetErrorString(r));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close_cuda(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

// in/res/out/sig: one device address per rank (rank order).  res may be all zeros (no residual).
void tp_allreduce_norm_cuda(std::vector<int64_t> in, std::vector<int64_t> res, std::vector<int64_t> out,
                            std::vector<int64_t> sig, int64_t rank, int64_t T, int64_t H,
                            c10::optional<torch::Tensor> weight, double eps, int64_t mode, torch::Tensor counters,
                            c10::optional<torch::Tensor> err, int64_t max_blocks, int64_t oneshot,
                            int64_t wait_ns) {
  const int R = (int)in.size();
  TORCH_CHECK(R >= 1 && R <= kMaxRanks && (int)out.size() == R && (int)sig.size() == R && (int)res.size() == R,
              "one pointer per rank (at most 8 ranks)");
  TORCH_CHECK(rank >= 0 && rank < R, "bad rank");
  TORCH_CHECK(H % 8 == 0 && H <= 32768, "H must be a multiple of 8 and <= 32768");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= kMaxBlocks,
              "counters must be int32 [>= 1024] on the device");
  if (T <= 0) return;
  PeerPtrs P;
  const bool has_res = res[0] != 0;
  for (int i = 0; i < kMaxRanks; ++i) {
    P.in[i] = i < R ? reinterpret_cast<const bf16*>(in[i]) : nullptr;
    P.res[i] = i < R ? reinterpret_cast<bf16*>(res[i]) : nullptr;
    P.out[i] = i < R ? reinterpret_cast<bf16*>(out[i]) : nullptr;
    P.sig[i] = i < R ? reinterpret_cast<uint32_t*>(sig[i]) : nullptr;
  }
  const bf16* w = nullptr;
  if (mode == 0 || mode == 1) {
    TORCH_CHECK(weight.has_value() && weight->scalar_type() == at::kBFloat16 && weight->numel() == H, "norm weight");
    w = reinterpret_cast<const bf16*>(weight->data_ptr());
  }
  int threads = ((H / 8 + 31) / 32) * 32;
  if (threads > 1024) threads = 1024;
  const int nv = (H / 8 + threads - 1) / threads;
  if (oneshot < 0) oneshot = ((long)(R - 1) * T * H * 2 <= (2l << 20)) ? 1 : 0;  // auto: one-shot up to 2 MiB
  const int per = oneshot ? (int)T : (int)((T + R - 1) / R);
  int grid = per < max_blocks ? per : (int)max_blocks;
  if (grid > kMaxBlocks) grid = kMaxBlocks;
  if (grid < 1) grid = 1;
  int* e = err.has_value() ? err->data_ptr<int>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  uint32_t* cnt = reinterpret_cast<uint32_t*>(counters.data_ptr<int>());
  const uint64_t wait = wait_ns > 0 ? (uint64_t)wait_ns : nvb::kWaitLimitNs;
#define LAUNCH(NV_)                                                                                              \
  C10_CUDA_CHECK(nvb::launch(tp_allreduce_norm_kernel<NV_>, dim3(grid), dim3(threads), 0, stream, P, (int)rank, R, (int)T, (int)H, w, (float)eps, \
                                                              (int)mode, has_res ? 1 : 0, cnt, e, (int)oneshot, wait))
  switch (nv) {
    case 1: LAUNCH(1); break;
    case 2: LAUNCH(2); break;
    case 3: LAUNCH(3); break;
    default: LAUNCH(4); break;
  }
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
