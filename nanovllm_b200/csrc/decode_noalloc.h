/* Allocation-free C entry point for paged decode attention (libnanovllm _C extension).
 *
 * This interface has no counterpart in the reference: the Java library has no GPU code and no C interface.
 *
 * Who it is for: callers that drive the GPU through a plain C ABI and cannot allocate device memory where they
 * run attention -- a JVM or native server calling through FFI has no access to the torch caching allocator of
 * this process, and a cudaMalloc/cudaFree pair per call would synchronise the device and stall a decode loop --
 * and serving loops whose policy forbids allocation after start-up.  The split-KV scratch lives in a fixed
 * file-scope device array (nvb_noalloc_scratch_capacity() fp32 values, resident on every GPU that loads the
 * library until the process exits); the caller passes only its inputs and the output buffer.
 *
 * Contract:
 *  - The first call on a device resolves the device addresses of the fixed arrays (cudaGetSymbolAddress, with
 *    that device current) and sets the kernels' shared-memory attribute; make that first call before any CUDA
 *    stream capture begins.
 *  - Every call shares the one scratch array, which keeps the previous call's contents.  Calls whose GPU work
 *    overlaps (unordered streams, several host threads) race on it: order them on one stream.
 *  - ctx_lens[b] must not exceed max_len, and max_len must not exceed bt_stride * block_size.  The host cannot
 *    read ctx_lens (it is device memory), so the kernel checks: a sequence with more keys than the split grid
 *    or its block-table row covers is skipped and NVB_NOALLOC_DEVICE_BAD_ARGUMENT is recorded in the error
 *    word; its output rows are then undefined.
 *  - A return value of NVB_NOALLOC_OK only means the work was queued.  Device-side failures (a bounded wait
 *    that gave up, a bad ctx_lens entry) are reported through the int at nvb_noalloc_error_word(): read it after
 *    synchronising the stream; each call resets it to 0 on its stream before launching.
 *  - No cudaMalloc, cudaFree or other allocating routine is called, and no torch API.
 */
#ifndef NANOVLLM_B200_DECODE_NOALLOC_H_
#define NANOVLLM_B200_DECODE_NOALLOC_H_

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes of nvb_paged_decode_noalloc. */
enum {
  NVB_NOALLOC_OK = 0,
  NVB_NOALLOC_ERR_ARGS = 1,      /* a null pointer or an unsupported size / alignment */
  NVB_NOALLOC_ERR_TOO_LARGE = 2, /* the split partials would not fit the fixed scratch; nothing launched */
  NVB_NOALLOC_ERR_CUDA = 3       /* a CUDA runtime / driver call failed (message in nvb_noalloc_last_error) */
};

/* Values the kernels write into the device error word (0 = none). */
enum {
  NVB_NOALLOC_DEVICE_OK = 0,
  NVB_NOALLOC_DEVICE_WAIT_TIMEOUT = 1, /* a bounded mbarrier wait gave up */
  NVB_NOALLOC_DEVICE_BAD_ARGUMENT = 3  /* a ctx_lens entry exceeded max_len or its block-table row */
};

/* Capacity of the shared scratch, in fp32 elements. */
long nvb_noalloc_scratch_capacity(void);

/* Message of the last failed call on this host thread ("" after a success). */
const char* nvb_noalloc_last_error(void);

/* Device address of the error word of the current device, or null before the first call on that device. */
int* nvb_noalloc_error_word(void);

/* Number of KV splits a call with these sizes launches on the current device (0 on a bad argument). */
int nvb_noalloc_num_splits(int B, int nkv, int max_len);

/* Paged decode attention, one query token per sequence.
 *   q               bf16 [B, nq, hd], contiguous
 *   k_cache/v_cache bf16 [num_blocks, nkv, block_size, hd], contiguous, 16-byte aligned
 *   block_tables    int32 [B, bt_stride] physical block ids
 *   ctx_lens        int32 [B] keys per sequence (<= max_len)
 *   out             bf16 [B, nq, hd]
 *   window          sliding window in keys (0 = none); softcap 0 = none
 *   stream          cudaStream_t (null = legacy default stream)
 * nq must be a multiple of nkv with nq / nkv <= 16; hd is 64, 128 or 256; block_size a multiple of 64. */
int nvb_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                             int bt_stride, const int* ctx_lens, void* out, int B, int nq, int nkv, int hd,
                             int num_blocks, int block_size, float scale, float softcap, int window, int max_len,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NANOVLLM_B200_DECODE_NOALLOC_H_ */
