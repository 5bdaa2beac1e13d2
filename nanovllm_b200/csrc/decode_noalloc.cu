// Allocation-free C entry point for paged decode attention.
//
// This entry point has no counterpart in the reference: the Java library has no GPU code and no C interface.
//
// Who it is for.  The regular decode-attention op (paged_decode_cuda, driven from Python) takes its split-KV
// scratch from the framework allocator.  Some callers cannot allocate device memory at the point where they
// run attention: code that drives the GPU from another runtime through a plain C ABI (a JVM or a native
// server calling through FFI has no access to this process's torch caching allocator, and a raw cudaMalloc /
// cudaFree per call would synchronise the device and stall the decode loop), and real-time serving loops whose
// policy forbids allocation after start-up.  For them, ``nvb_paged_decode_noalloc`` runs the same split-KV
// kernels with the scratch taken from a fixed, file-scope device array; the caller passes only its own inputs
// and the output buffer.
//
// Limits and contract:
//  * The scratch is ``g_noalloc_scratch``, kNoallocScratchFloats fp32 values (16 MiB).  Every GPU that loads
//    this library keeps that array resident until the process exits.  A call whose split partials
//    (batch * q_heads * splits * (head_dim + 1) floats) would not fit is rejected with code
//    NVB_NOALLOC_ERR_TOO_LARGE and a message from nvb_noalloc_last_error(); nothing is launched.
//  * In host code the name ``g_noalloc_scratch`` is only a host-side stand-in for the device array, not a
//    device address.  The device address is obtained once per device, with that device current, through
//    cudaGetSymbolAddress; the first call on each device does this set-up, so make that first call before any
//    CUDA stream capture begins.
//  * Every call shares the one array and it keeps the previous call's contents.  The kernels overwrite every
//    partial they later read, so nothing needs clearing except the bounded-wait error word, which each call
//    resets with cudaMemsetAsync on the caller's stream.  Calls whose GPU work overlaps (different streams
//    without ordering between them, or several host threads) race on the array: order them on one stream.
//  * The function calls no cudaMalloc, cudaFree or other allocating routine, and no torch API.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "attention_kernels.cuh"

namespace {

constexpr long kNoallocScratchFloats = 4L * 1024 * 1024;  // 16 MiB of fp32 split partials
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_noalloc_scratch[kNoallocScratchFloats];
__device__ __align__(256) int g_noalloc_err[4];

float* g_scratch_dev[kMaxDevices] = {nullptr};
int* g_err_dev[kMaxDevices] = {nullptr};
std::mutex g_setup_mu;
thread_local char g_last_error[256] = {0};

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn g_encode = nullptr;

int fail(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

// One-time, per-device set-up: resolve the device addresses of the file-scope arrays.
int setup_device(int dev) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_encode == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr)
      return fail(3, "cuTensorMapEncodeTiled is not available from the CUDA driver");
    g_encode = reinterpret_cast<EncodeFn>(p);
  }
  if (g_scratch_dev[dev] != nullptr) return 0;
  void* s = nullptr;
  void* e = nullptr;
  cudaError_t r1 = cudaGetSymbolAddress(&s, g_noalloc_scratch);
  if (r1 != cudaSuccess) return fail(3, cudaGetErrorString(r1));
  cudaError_t r2 = cudaGetSymbolAddress(&e, g_noalloc_err);
  if (r2 != cudaSuccess) return fail(3, cudaGetErrorString(r2));
  g_scratch_dev[dev] = static_cast<float*>(s);
  g_err_dev[dev] = static_cast<int*>(e);
  return 0;
}

bool encode_cache_map(CUtensorMap* m, const void* base, unsigned long long rows, int hd) {
  cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)KT};
  cuuint32_t elem[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD, int STAGES>
cudaError_t launch(const CUtensorMap& km, const CUtensorMap& vm, dim3 grid, cudaStream_t st, const bf16* q,
                   const int* bt, int bt_stride, const int* ctx, bf16* out, float* po, float* pl, int nq, int nkv,
                   int block_size, float scale, float softcap, int window, int part_tiles, int* err) {
  auto kern = paged_decode_kernel<HD, STAGES>;
  const size_t sm = decode_smem<HD, STAGES>();
  cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (r != cudaSuccess) return r;
  kern<<<grid, 128, sm, st>>>(km, vm, q, bt, bt_stride, ctx, out, po, pl, nq, nkv, block_size, scale, softcap, window,
                              part_tiles, err, nullptr);  // split merge by the separate combine kernel below
  return cudaGetLastError();
}

}  // namespace

extern "C" {

enum {
  NVB_NOALLOC_OK = 0,
  NVB_NOALLOC_ERR_ARGS = 1,
  NVB_NOALLOC_ERR_TOO_LARGE = 2,
  NVB_NOALLOC_ERR_CUDA = 3,
};

// Capacity of the shared scratch, in fp32 elements.
long nvb_noalloc_scratch_capacity(void) { return kNoallocScratchFloats; }

// Message of the last failed call on this host thread ("" after a success).
const char* nvb_noalloc_last_error(void) { return g_last_error; }

// Device address of the bounded-wait error word of the current device (0 = no kernel gave up), or null before
// the first call on that device.
int* nvb_noalloc_error_word(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  return g_err_dev[dev];
}

// Paged decode attention (one query token per sequence), same kernels and split rule as the framework op.
//   q            bf16 [B, nq, hd], contiguous
//   k_cache/v_cache bf16 [num_blocks, nkv, block_size, hd], contiguous
//   block_tables int32 [B, bt_stride] physical block ids; ctx_lens int32 [B] keys per sequence
//   out          bf16 [B, nq, hd]
//   max_len      upper bound of ctx_lens (sizes the split grid); stream: cudaStream_t (null = legacy stream)
// Returns NVB_NOALLOC_OK or an error code; see nvb_noalloc_last_error().
int nvb_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                             int bt_stride, const int* ctx_lens, void* out, int B, int nq, int nkv, int hd,
                             int num_blocks, int block_size, float scale, float softcap, int window, int max_len,
                             void* stream) {
  g_last_error[0] = 0;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_tables == nullptr || ctx_lens == nullptr ||
      out == nullptr)
    return fail(NVB_NOALLOC_ERR_ARGS, "null pointer argument");
  if (B <= 0 || nq <= 0 || nkv <= 0 || nq % nkv != 0 || nq / nkv > 16)
    return fail(NVB_NOALLOC_ERR_ARGS, "need B > 0 and nq a multiple of nkv with a group of at most 16");
  if (hd != 64 && hd != 128 && hd != 256) return fail(NVB_NOALLOC_ERR_ARGS, "head_dim must be 64, 128 or 256");
  if (block_size <= 0 || block_size % KT != 0) return fail(NVB_NOALLOC_ERR_ARGS, "block_size must be a multiple of 64");
  if (max_len <= 0 || num_blocks <= 0 || bt_stride <= 0) return fail(NVB_NOALLOC_ERR_ARGS, "bad sizes");
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
    return fail(NVB_NOALLOC_ERR_ARGS, "caches must be 16-byte aligned");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(NVB_NOALLOC_ERR_CUDA, "no current CUDA device");
  if (int rc = setup_device(dev)) return rc;

  // split rule of the framework op: ~4 CTAs per SM, at most 16 tiles per split and 64 splits
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long tiles = (max_len + KT - 1) / KT;
  const long target = 4L * sms;
  long per = (B * (long)nkv * tiles + target - 1) / target;
  if (per < 1) per = 1;
  if (per > 16) per = 16;
  const long per_min = (tiles + 63) / 64;
  if (per < per_min) per = per_min;
  const long nsplit = (tiles + per - 1) / per;
  const long need = nsplit > 1 ? (long)B * nq * nsplit * (hd + 1) : 0;
  if (need > kNoallocScratchFloats) {
    char msg[200];
    std::snprintf(msg, sizeof(msg), "split partials need %ld floats but the fixed scratch holds %ld; lower the batch "
                  "or max_len", need, kNoallocScratchFloats);
    return fail(NVB_NOALLOC_ERR_TOO_LARGE, msg);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = g_err_dev[dev];
  cudaError_t r = cudaMemsetAsync(err, 0, sizeof(int), st);
  if (r != cudaSuccess) return fail(NVB_NOALLOC_ERR_CUDA, cudaGetErrorString(r));

  CUtensorMap km, vm;
  const unsigned long long rows = (unsigned long long)num_blocks * nkv * block_size;
  if (!encode_cache_map(&km, k_cache, rows, hd) || !encode_cache_map(&vm, v_cache, rows, hd))
    return fail(NVB_NOALLOC_ERR_CUDA, "tensor map encoding failed");
  float* po = nsplit > 1 ? g_scratch_dev[dev] : nullptr;
  float* pl = nsplit > 1 ? g_scratch_dev[dev] + (long)B * nq * nsplit * hd : nullptr;
  const dim3 grid((unsigned)nsplit, nkv, B);
  const bf16* qp = static_cast<const bf16*>(q);
  bf16* op = static_cast<bf16*>(out);
  if (hd == 64)
    r = launch<64, 4>(km, vm, grid, st, qp, block_tables, bt_stride, ctx_lens, op, po, pl, nq, nkv, block_size, scale,
                      softcap, window, (int)per, err);
  else if (hd == 128)
    r = launch<128, 3>(km, vm, grid, st, qp, block_tables, bt_stride, ctx_lens, op, po, pl, nq, nkv, block_size,
                       scale, softcap, window, (int)per, err);
  else
    r = launch<256, 2>(km, vm, grid, st, qp, block_tables, bt_stride, ctx_lens, op, po, pl, nq, nkv, block_size,
                       scale, softcap, window, (int)per, err);
  if (r != cudaSuccess) return fail(NVB_NOALLOC_ERR_CUDA, cudaGetErrorString(r));
  if (nsplit > 1) {
    attn_combine_kernel<<<dim3(nq, B), hd < 128 ? hd : 128, 0, st>>>(po, pl, ctx_lens, op, nq, (int)nsplit, hd,
                                                                     (int)per, window);
    r = cudaGetLastError();
    if (r != cudaSuccess) return fail(NVB_NOALLOC_ERR_CUDA, cudaGetErrorString(r));
  }
  return NVB_NOALLOC_OK;
}

}  // extern "C"
