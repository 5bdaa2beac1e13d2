"""The allocation-free C entry point ``nvb_paged_decode_noalloc`` (for callers that cannot allocate device memory,
e.g. a runtime driving the GPU through a plain C ABI) must give the same result as the framework's decode
attention op, call after call, while its split-KV scratch lives in a fixed file-scope device array.

It is called here through its exported C symbol with ctypes, on two consecutive calls with different inputs.
This file is named so that pytest collects it last."""
import ctypes

import pytest
import torch

from nanovllm_b200 import ops

pytestmark = pytest.mark.gpu


def _lib():
    lib = ctypes.CDLL(ops._cuda_ext().__file__)
    f = lib.nvb_paged_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.nvb_noalloc_last_error.restype = ctypes.c_char_p
    lib.nvb_noalloc_scratch_capacity.restype = ctypes.c_long
    lib.nvb_noalloc_error_word.restype = ctypes.c_void_p
    lib.nvb_noalloc_num_splits.restype = ctypes.c_int
    lib.nvb_noalloc_num_splits.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    return lib


def _device_error_word(lib) -> int:
    """The int at nvb_noalloc_error_word() (device memory), read after a synchronisation through a tensor view of
    that address (``__cuda_array_interface__``: no copy of the library's state, no allocation in the library)."""
    addr = lib.nvb_noalloc_error_word()
    assert addr, "the error word is resolved by the first call on the device"

    class _View:
        __cuda_array_interface__ = {"shape": (1,), "typestr": "<i4", "data": (addr, False), "version": 3}

    torch.cuda.synchronize()
    return int(torch.as_tensor(_View(), device="cuda").item())


def _case(seed, B=8, nq=32, nkv=8, hd=128, BS=256, max_len=4096):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, max_len + 1, (B,), generator=g)
    lens[0] = max_len
    nblk = (max_len + BS - 1) // BS
    NB = B * nblk + 2
    kc = torch.randn(NB, nkv, BS, hd, generator=g).bfloat16().cuda()
    vc = torch.randn(NB, nkv, BS, hd, generator=g).bfloat16().cuda()
    bt = torch.randperm(NB, generator=g)[:B * nblk].int().view(B, nblk).cuda()
    q = torch.randn(B, nq, hd, generator=g).bfloat16().cuda()
    return q, kc, vc, bt, lens.int().cuda()


def _call(lib, q, kc, vc, bt, lens, max_len, window=0):
    B, nq, hd = q.shape
    out = torch.empty_like(q)
    rc = lib.nvb_paged_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), bt.shape[1],
                                      lens.data_ptr(), out.data_ptr(), B, nq, kc.shape[1], hd, kc.shape[0],
                                      kc.shape[2], hd ** -0.5, 0.0, window, max_len,
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


def test_noalloc_decode_matches_framework_op_on_consecutive_calls():
    lib = _lib()
    max_len = 4096
    _, nsplit = ops.decode_partition(8, 8, max_len)
    # both sides take the SM count from the device: the C entry point plans the same split grid
    assert lib.nvb_noalloc_num_splits(8, 8, max_len) == nsplit
    assert nsplit > 1, "the case must exercise the split-KV scratch"
    for seed, window in ((1, 0), (2, 700)):
        q, kc, vc, bt, lens = _case(seed, max_len=max_len)
        rc, out = _call(lib, q, kc, vc, bt, lens, max_len, window)
        assert rc == 0, lib.nvb_noalloc_last_error()
        want = ops.paged_decode(q, kc, vc, bt, lens, q.shape[-1] ** -0.5, 0.0, window, max_len=max_len)
        torch.cuda.synchronize()
        assert (out.float() - want.float()).abs().max().item() <= 2e-2
        # a zero return code only says the work was queued: device-side failures land in the error word
        assert _device_error_word(lib) == 0
    torch.cuda.synchronize()


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch():
    lib = _lib()
    cap = lib.nvb_noalloc_scratch_capacity()
    assert cap > 0
    q, kc, vc, bt, lens = _case(3, B=2, max_len=512)
    big_b = 4096  # claims 4096 sequences: the partials would exceed the fixed array; nothing is launched
    # (a block-table row of 256 blocks covers max_len 65536; the size check rejects the call before any launch)
    rc = lib.nvb_paged_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), 256,
                                      lens.data_ptr(), q.data_ptr(), big_b, 32, 8, 128, kc.shape[0], 256,
                                      0.088, 0.0, 0, 65536, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 2
    assert b"fixed scratch" in lib.nvb_noalloc_last_error()


def test_noalloc_reports_context_longer_than_max_len_on_the_device():
    # ctx_lens lives in device memory, so the host cannot check it: the kernel skips such a sequence and records
    # NVB_NOALLOC_DEVICE_BAD_ARGUMENT (3) in the error word instead of silently dropping keys
    lib = _lib()
    max_len = 1024
    q, kc, vc, bt, lens = _case(4, B=4, max_len=max_len)
    lens[1] = max_len + 64
    rc, _ = _call(lib, q, kc, vc, bt, lens, max_len)
    assert rc == 0, lib.nvb_noalloc_last_error()
    assert _device_error_word(lib) == 3
    lens[1] = max_len
    rc, _ = _call(lib, q, kc, vc, bt, lens, max_len)  # each call resets the word
    assert rc == 0
    assert _device_error_word(lib) == 0
