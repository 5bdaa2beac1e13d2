// Paged attention for sm_100a: split-KV flash decoding and varlen (paged or contiguous) prefill.
//
// Reference semantics: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/Attention.java:245-396
// (online-softmax over paged slots; causal end kLen - qLen + qi + 1; optional sliding-window start
// absQ - W + 1; GQA head mapping kvh = h / (nq / nkv); score = dot(q, k) * scale) and
// BidirectionalAttention.java:71-145 (no mask).  Logit soft-capping cap * tanh(s / cap) is applied to the
// scaled score when ``softcap > 0``.
//
// Data movement: K/V tiles of 64 keys x head_dim are fetched by TMA (cp.async.bulk.tensor, no multicast) with
// the 128-byte swizzle into a multi-stage ring tracked by mbarriers; one thread issues the copies.  The
// cache layout is [num_blocks, nkv, block_size, hd], so a 64-key tile of one head is one contiguous
// 64 x hd box.  The contractions run on mma.sync m16n8k16 (bf16 in, fp32 accumulate): decode attention is
// bound by HBM bytes, not by the tensor pipe, and the register-resident online softmax keeps the whole tile
// in registers.
//
// Decode: one CTA per (kv-split, kv head, sequence); the G = nq / nkv query heads of the group are the
// 16-row M tile; the four warps split the 64 keys of each tile and merge their (max, sum, O) at the end.
// Splits write fp32 partials + log2-sum-exp to a scratch buffer that attn_combine merges.
// Prefill: one CTA per (64-row q tile, kv head, sequence); rows are (token, head-in-group) pairs so the K/V
// tile is shared by all G heads; each warp owns 16 rows.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "launch.h"
#include "tma_host.h"

#include "attention_kernels.cuh"
#include "attention_tc.cuh"

namespace {

int* err_ptr(c10::optional<torch::Tensor>& e) { return e.has_value() ? e->data_ptr<int>() : nullptr; }

void check_kv(const torch::Tensor& c, int64_t nkv, int64_t hd) {
  TORCH_CHECK(c.is_cuda() && c.scalar_type() == at::kBFloat16 && c.is_contiguous(), "cache must be contiguous bf16");
  TORCH_CHECK(c.dim() == 4 && c.size(1) == nkv && c.size(3) == hd, "cache must be [num_blocks, nkv, block, hd]");
  TORCH_CHECK(c.size(2) % KT == 0, "block size must be a multiple of 64");
}

}  // namespace

// q [B, nq, hd]; caches [num_blocks, nkv, block, hd]; out [B, nq, hd]; part_o [B, nq, nsplit, hd] fp32;
// part_lse [B, nq, nsplit] fp32 (unused when nsplit == 1).
void paged_decode_cuda(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                       torch::Tensor ctx_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_lse,
                       double scale, double softcap, int64_t window, int64_t part_tiles, int64_t nsplit,
                       c10::optional<torch::Tensor> err, c10::optional<torch::Tensor> combine_counters) {
  const int B = q.size(0), nq = q.size(1), hd = q.size(2);
  const int nkv = k_cache.size(1), block_size = k_cache.size(2);
  TORCH_CHECK(q.is_contiguous() && out.is_contiguous(), "q/out must be contiguous");
  TORCH_CHECK(nq % nkv == 0 && nq / nkv <= 16, "GQA group must be <= 16");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt, "int32 metadata");
  check_kv(k_cache, nkv, hd);
  check_kv(v_cache, nkv, hd);
  if (B == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (hd != 64 && hd != 128 && hd != 256) {
    // generic path: treat each sequence as a 1-token query
    auto cu_q = torch::arange(0, B + 1, ctx_lens.options());
    auto cu_k = torch::zeros({B + 1}, ctx_lens.options());
    cu_k.slice(0, 1).copy_(torch::cumsum(ctx_lens, 0));
    const int total = B * nq;
    C10_CUDA_CHECK(nvb::launch(attn_generic_kernel, dim3((total * 32 + 127) / 128), dim3(128), 0, stream, 
        reinterpret_cast<const bf16*>(q.data_ptr()), (long)nq * hd, reinterpret_cast<bf16*>(out.data_ptr()),
        (long)nq * hd, reinterpret_cast<const bf16*>(k_cache.data_ptr()),
        reinterpret_cast<const bf16*>(v_cache.data_ptr()), 0, cu_q.data_ptr<int>(), cu_k.data_ptr<int>(),
        block_tables.data_ptr<int>(), block_tables.size(1), 1, B, nq, nkv, hd, block_size, (float)scale,
        (float)softcap, (int)window, 1, B));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const uint64_t rows = (uint64_t)k_cache.size(0) * nkv * block_size;
  CUtensorMap km = nvb::make_tmap_2d_bf16(k_cache.data_ptr(), rows, hd, hd, KT);
  CUtensorMap vm = nvb::make_tmap_2d_bf16(v_cache.data_ptr(), rows, hd, hd, KT);
  dim3 grid((unsigned)nsplit, nkv, B);
  auto* qp = reinterpret_cast<const bf16*>(q.data_ptr());
  auto* op = reinterpret_cast<bf16*>(out.data_ptr());
  float* po = nsplit > 1 ? part_o.data_ptr<float>() : nullptr;
  float* pl = nsplit > 1 ? part_lse.data_ptr<float>() : nullptr;
  int* e = err_ptr(err);
#define LAUNCH_DEC(HD_, ST_)                                                                                     \
  {                                                                                                              \
    auto kern = paged_decode_kernel<HD_, ST_>;                                                                   \
    size_t sm = decode_smem<HD_, ST_>();                                                                         \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);                            \
    C10_CUDA_CHECK(nvb::launch(kern, dim3(grid), dim3(128), sm, stream, km, vm, qp, block_tables.data_ptr<int>(), block_tables.size(1),              \
                                    ctx_lens.data_ptr<int>(), op, po, pl, nq, nkv, block_size, (float)scale,     \
                                    (float)softcap, (int)window, (int)part_tiles, e, cnt));                       \
  }
  // the split merge runs inside the decode kernel (last split CTA per (sequence, kv head)) when the caller
  // provides a zeroed int32 counter array of at least B * nkv entries; otherwise as a separate kernel
  int* cnt = nullptr;
  if (nsplit > 1 && combine_counters.has_value()) {
    TORCH_CHECK(combine_counters->is_cuda() && combine_counters->scalar_type() == at::kInt &&
                    combine_counters->numel() >= (long)B * nkv,
                "combine counters must be int32 with at least B * nkv entries");
    cnt = combine_counters->data_ptr<int>();
  }
  if (hd == 64) LAUNCH_DEC(64, 4)
  else if (hd == 128) LAUNCH_DEC(128, 3)
  else LAUNCH_DEC(256, 2)
#undef LAUNCH_DEC
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (nsplit > 1 && cnt == nullptr) {
    C10_CUDA_CHECK(nvb::launch(attn_combine_kernel, dim3(dim3(nq, B)), dim3(hd < 128 ? hd : 128), 0, stream, 
        po, pl, ctx_lens.data_ptr<int>(), op, nq, (int)nsplit, hd, (int)part_tiles, (int)window));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// Varlen prefill.  paged: K/V from the caches through block_tables.  contiguous (paged == false): K/V are
// heads nq..nq+2nkv of the packed qkv tensor ``kv_src`` [T, (nq + 2 nkv) * hd] (BERT, no cache).
void prefill_attention_cuda(torch::Tensor q, torch::Tensor out, torch::Tensor cu_q, torch::Tensor cu_k,
                            int64_t max_q, c10::optional<torch::Tensor> k_cache, c10::optional<torch::Tensor> v_cache,
                            c10::optional<torch::Tensor> block_tables, c10::optional<torch::Tensor> kv_src,
                            int64_t nq, int64_t nkv, int64_t hd, double scale, double softcap, int64_t window,
                            bool causal, c10::optional<torch::Tensor> err) {
  const int nseq = cu_q.size(0) - 1;
  if (nseq <= 0 || max_q <= 0) return;
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1, "q/out inner dim must be contiguous");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && cu_k.scalar_type() == at::kInt, "cu_seqlens must be int32");
  const bool paged = k_cache.has_value();
  const long q_stride = q.dim() == 3 ? q.stride(0) : q.stride(0);
  const long o_stride = out.dim() == 3 ? out.stride(0) : out.stride(0);
  auto stream = at::cuda::getCurrentCUDAStream();
  int* e = err_ptr(err);
  const int G = nq / nkv;
  TORCH_CHECK(nq % nkv == 0 && 64 % G == 0, "GQA group must divide 64");
  int block_size = 1;
  const int* bt = nullptr;
  int bt_stride = 0;
  if (paged) {
    check_kv(*k_cache, nkv, hd);
    check_kv(*v_cache, nkv, hd);
    TORCH_CHECK(block_tables.has_value(), "block tables required for paged prefill");
    block_size = k_cache->size(2);
    bt = block_tables->data_ptr<int>();
    bt_stride = block_tables->size(1);
  } else {
    TORCH_CHECK(kv_src.has_value() && kv_src->stride(-1) == 1, "kv_src required for contiguous prefill");
  }
  if (hd == 32 && !paged && (128 % G == 0)) {
    // BERT-small head dim on the tcgen05 kernel in 64-wide tiles (attention_tc.cuh, HDR = 32)
    const uint64_t T = kv_src->size(0);
    const uint64_t row = (uint64_t)(nq + 2 * nkv) * hd;
    CUtensorMap tk = nvb::make_tmap_2d_bf16(kv_src->data_ptr(), T, row, kv_src->stride(0), 128);
    const int TPT = 128 / G;
    dim3 grid((unsigned)((max_q + TPT - 1) / TPT), nkv, nseq);
    auto kern = prefill_tc_kernel<64, 32>;
    const size_t sm = TcAttnCfg<64>::smem();
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    C10_CUDA_CHECK(nvb::launch(kern, grid, dim3(384), sm, stream, tk, tk, reinterpret_cast<const bf16*>(q.data_ptr()),
                               q_stride, reinterpret_cast<bf16*>(out.data_ptr()), o_stride, cu_q.data_ptr<int>(),
                               cu_k.data_ptr<int>(), bt, bt_stride, 0, (int)nq, (int)nkv, block_size, (float)scale,
                               (float)softcap, (int)window, causal ? 1 : 0, e));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  if (hd != 64 && hd != 128 && hd != 256) {
    const int total_q = q.size(0);
    const bf16* kc = paged ? reinterpret_cast<const bf16*>(k_cache->data_ptr())
                           : reinterpret_cast<const bf16*>(kv_src->data_ptr()) + nq * hd;
    const bf16* vc = paged ? reinterpret_cast<const bf16*>(v_cache->data_ptr())
                           : reinterpret_cast<const bf16*>(kv_src->data_ptr()) + (nq + nkv) * hd;
    const long kvs = paged ? 0 : kv_src->stride(0);
    C10_CUDA_CHECK(nvb::launch(attn_generic_kernel, dim3(((long)total_q * nq * 32 + 127) / 128), dim3(128), 0, stream, 
        reinterpret_cast<const bf16*>(q.data_ptr()), q_stride, reinterpret_cast<bf16*>(out.data_ptr()), o_stride, kc,
        vc, kvs, cu_q.data_ptr<int>(), cu_k.data_ptr<int>(), bt, bt_stride, paged ? 1 : 0, nseq, nq, nkv, hd,
        block_size, (float)scale, (float)softcap, (int)window, causal ? 1 : 0, total_q));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  // tcgen05 kernel (attention_tc.cuh) whenever its tiles fit: 128 query rows hold whole GQA groups and a paged
  // key tile never straddles a cache block; the mma.sync kernel below covers the rest (NVB_PREFILL_TC=0 forces it)
  const int tc_bn = hd == 256 ? 64 : 128;
  static const bool tc_on = [] {
    const char* v = getenv("NVB_PREFILL_TC");
    return v == nullptr || v[0] != '0';
  }();
  if (tc_on && 128 % G == 0 && (!paged || block_size % tc_bn == 0)) {
    CUtensorMap tk, tv;
    if (paged) {
      const uint64_t rows = (uint64_t)k_cache->size(0) * nkv * block_size;
      tk = nvb::make_tmap_2d_bf16(k_cache->data_ptr(), rows, hd, hd, tc_bn);
      tv = nvb::make_tmap_2d_bf16(v_cache->data_ptr(), rows, hd, hd, tc_bn);
    } else {
      const uint64_t T = kv_src->size(0);
      const uint64_t heads = nq + 2 * nkv;
      uint64_t dims[3] = {(uint64_t)hd, heads, T};
      uint64_t strides[2] = {(uint64_t)hd * 2, (uint64_t)kv_src->stride(0) * 2};
      uint32_t box[3] = {64, 1, (uint32_t)tc_bn};
      tk = nvb::make_tmap(kv_src->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box);
      tv = tk;
    }
    const int TPT = 128 / G;
    dim3 grid((unsigned)((max_q + TPT - 1) / TPT), nkv, nseq);
    auto* qp = reinterpret_cast<const bf16*>(q.data_ptr());
    auto* op = reinterpret_cast<bf16*>(out.data_ptr());
#define LAUNCH_TC(HD_)                                                                                           \
  {                                                                                                              \
    auto kern = prefill_tc_kernel<HD_>;                                                                          \
    const size_t sm = TcAttnCfg<HD_>::smem();                                                                    \
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));            \
    C10_CUDA_CHECK(nvb::launch(kern, grid, dim3(384), sm, stream, tk, tv, qp, q_stride, op, o_stride,            \
                               cu_q.data_ptr<int>(), cu_k.data_ptr<int>(), bt, bt_stride, paged ? 1 : 0, (int)nq, \
                               (int)nkv, block_size, (float)scale, (float)softcap, (int)window, causal ? 1 : 0, e)); \
  }
    if (hd == 64) LAUNCH_TC(64)
    else if (hd == 128) LAUNCH_TC(128)
    else LAUNCH_TC(256)
#undef LAUNCH_TC
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  CUtensorMap km, vm;
  if (paged) {
    const uint64_t rows = (uint64_t)k_cache->size(0) * nkv * block_size;
    km = nvb::make_tmap_2d_bf16(k_cache->data_ptr(), rows, hd, hd, KT);
    vm = nvb::make_tmap_2d_bf16(v_cache->data_ptr(), rows, hd, hd, KT);
  } else {
    const uint64_t T = kv_src->size(0);
    const uint64_t heads = nq + 2 * nkv;
    uint64_t dims[3] = {(uint64_t)hd, heads, T};
    uint64_t strides[2] = {(uint64_t)hd * 2, (uint64_t)kv_src->stride(0) * 2};
    uint32_t box[3] = {64, 1, KT};
    km = nvb::make_tmap(kv_src->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box);
    vm = km;
  }
  const int TPT = 64 / G;
  dim3 grid((unsigned)((max_q + TPT - 1) / TPT), nkv, nseq);
  auto* qp = reinterpret_cast<const bf16*>(q.data_ptr());
  auto* op = reinterpret_cast<bf16*>(out.data_ptr());
#define LAUNCH_PF(HD_, ST_)                                                                                      \
  {                                                                                                              \
    auto kern = prefill_attn_kernel<HD_, ST_>;                                                                   \
    size_t sm = prefill_smem<HD_, ST_>();                                                                        \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);                            \
    C10_CUDA_CHECK(nvb::launch(kern, dim3(grid), dim3(128), sm, stream, km, vm, qp, q_stride, op, o_stride, cu_q.data_ptr<int>(),                    \
                                    cu_k.data_ptr<int>(), bt, bt_stride, paged ? 1 : 0, nq, nkv, block_size,     \
                                    (float)scale, (float)softcap, (int)window, causal ? 1 : 0, e));               \
  }
  if (hd == 64) LAUNCH_PF(64, 4)
  else if (hd == 128) LAUNCH_PF(128, 2)
  else LAUNCH_PF(256, 2)
#undef LAUNCH_PF
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
