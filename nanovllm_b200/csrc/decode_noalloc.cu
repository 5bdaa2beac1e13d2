// Allocation-free C entry point for paged decode attention; the interface, its callers and its contract are
// documented in decode_noalloc.h.  This entry point has no counterpart in the reference: the Java library has
// no GPU code and no C interface.
//
// Implementation notes:
//  * The scratch is ``g_noalloc_scratch`` (kNoallocScratchFloats fp32 values, 16 MiB).  In host code that name
//    is only a host-side stand-in for the device array; its device address comes from cudaGetSymbolAddress,
//    once per device with that device current (setup_device), and is passed to the kernels as a pointer.
//  * The kernels overwrite every partial they later read, so nothing in the scratch needs clearing; only the
//    error word is reset (cudaMemsetAsync on the caller's stream) at the start of every call.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "attention_kernels.cuh"
#include "decode_noalloc.h"

namespace {

constexpr long kNoallocScratchFloats = 4L * 1024 * 1024;  // 16 MiB of fp32 split partials
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_noalloc_scratch[kNoallocScratchFloats];
__device__ __align__(256) int g_noalloc_err[4];

float* g_scratch_dev[kMaxDevices] = {nullptr};
int* g_err_dev[kMaxDevices] = {nullptr};
int g_sms[kMaxDevices] = {0};
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
  // the kernels' dynamic shared-memory limit is a per-device function attribute: set it once here
  const cudaError_t a1 = cudaFuncSetAttribute(paged_decode_kernel<64, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)decode_smem<64, 4>());
  const cudaError_t a2 = cudaFuncSetAttribute(paged_decode_kernel<128, 3>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, (int)decode_smem<128, 3>());
  const cudaError_t a3 = cudaFuncSetAttribute(paged_decode_kernel<256, 2>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, (int)decode_smem<256, 2>());
  if (a1 != cudaSuccess || a2 != cudaSuccess || a3 != cudaSuccess)
    return fail(NVB_NOALLOC_ERR_CUDA, "cudaFuncSetAttribute failed for the decode kernels");
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return fail(NVB_NOALLOC_ERR_CUDA, "cannot read the SM count");
  g_sms[dev] = sms;
  g_scratch_dev[dev] = static_cast<float*>(s);
  g_err_dev[dev] = static_cast<int*>(e);
  return 0;
}

// Split rule shared with the framework op (ops.decode_partition): ~4 CTAs per SM, at most 16 tiles per split
// and at most 64 splits.  Returns (tiles per split, splits).
void split_rule(long B, long nkv, long max_len, int sms, long* per_out, long* nsplit_out) {
  const long tiles = (max_len + KT - 1) / KT;
  const long target = 4L * sms;
  long per = (B * nkv * tiles + target - 1) / target;
  if (per < 1) per = 1;
  if (per > 16) per = 16;
  const long per_min = (tiles + 63) / 64;
  if (per < per_min) per = per_min;
  *per_out = per;
  *nsplit_out = (tiles + per - 1) / per;
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
  const size_t sm = decode_smem<HD, STAGES>();  // attribute set once per device in setup_device
  kern<<<grid, 128, sm, st>>>(km, vm, q, bt, bt_stride, ctx, out, po, pl, nq, nkv, block_size, scale, softcap, window,
                              part_tiles, err, nullptr);  // split merge by the separate combine kernel below
  return cudaGetLastError();
}

}  // namespace

extern "C" {

long nvb_noalloc_scratch_capacity(void) { return kNoallocScratchFloats; }

const char* nvb_noalloc_last_error(void) { return g_last_error; }

int* nvb_noalloc_error_word(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  return g_err_dev[dev];
}

int nvb_noalloc_num_splits(int B, int nkv, int max_len) {
  int dev = 0;
  if (B <= 0 || nkv <= 0 || max_len <= 0) return 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  if (setup_device(dev) != 0) return 0;
  long per, nsplit;
  split_rule(B, nkv, max_len, g_sms[dev], &per, &nsplit);
  return (int)nsplit;
}

// Same kernels and split rule as the framework op; contract in decode_noalloc.h.
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
  if ((long)max_len > (long)bt_stride * block_size)
    return fail(NVB_NOALLOC_ERR_ARGS, "max_len exceeds what a block-table row (bt_stride * block_size) covers");
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
    return fail(NVB_NOALLOC_ERR_ARGS, "caches must be 16-byte aligned");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(NVB_NOALLOC_ERR_CUDA, "no current CUDA device");
  if (int rc = setup_device(dev)) return rc;

  long per, nsplit;
  split_rule(B, nkv, max_len, g_sms[dev], &per, &nsplit);
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
