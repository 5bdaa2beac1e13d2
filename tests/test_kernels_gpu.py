"""Numerics of every sm_100a kernel against the plain-PyTorch fp32 oracle (ops.reference_cpu)."""
import math

import pytest
import torch

from nanovllm_b200 import ops
from nanovllm_b200.exceptions import DeviceWaitTimeout
from nanovllm_b200.ops import reference_cpu as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(a, b, atol, rtol=0.02):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs()
    tol = atol + rtol * b.abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.4g}"


def test_extension_loaded():
    assert ops.extension_loaded(), "the CUDA extension must load on a GPU box"


@pytest.mark.parametrize("H", [640, 1024, 4096])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_rms_norm(H, mode):
    g = torch.Generator().manual_seed(H + mode)
    x = torch.randn(37, H, generator=g).bfloat16()
    r = torch.randn(37, H, generator=g).bfloat16()
    w = (torch.randn(H, generator=g) * 0.1 + 1).bfloat16()
    y_ref, _ = ref.rms_norm(x, w, 1e-6, mode)
    y, _ = ops.rms_norm(x.to(DEV), w.to(DEV), 1e-6, mode)
    close(y, y_ref, 2e-2)
    y_ref, r_ref = ref.rms_norm(x, w, 1e-6, mode, r)
    rd = r.to(DEV).clone()
    y, rd2 = ops.rms_norm(x.to(DEV), w.to(DEV), 1e-6, mode, rd)
    close(rd, r_ref, 1e-2)
    close(y, y_ref, 2e-2)


def test_layer_norm():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(19, 384, generator=g).bfloat16()
    r = torch.randn(19, 384, generator=g).bfloat16()
    w = torch.randn(384, generator=g).bfloat16()
    b = torch.randn(384, generator=g).bfloat16()
    close(ops.layer_norm(x.to(DEV), w.to(DEV), b.to(DEV), 1e-12, r.to(DEV)), ref.layer_norm(x, w, b, 1e-12, r), 3e-2)


@pytest.mark.parametrize("hd,nq,nkv,mode", [(128, 8, 2, 0), (64, 4, 4, -1), (256, 4, 1, 1), (128, 4, 1, 2)])
def test_qk_norm_rope_store(hd, nq, nkv, mode):
    g = torch.Generator().manual_seed(hd + nq)
    T, NB, BS = 21, 4, 256
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, generator=g).bfloat16()
    pos = torch.randint(0, 1000, (T,), generator=g)
    cs = ref.rope_cos_sin(hd, 1024, 10000.0, 0.5 if mode == 2 else 1.0)
    qw = (torch.randn(hd, generator=g) * 0.1 + 1).bfloat16()
    kw = (torch.randn(hd, generator=g) * 0.1 + 1).bfloat16()
    slots = torch.randperm(NB * BS, generator=g)[:T].int()
    slots[3] = -1
    kc = torch.zeros(NB, nkv, BS, hd).bfloat16()
    vc = torch.zeros_like(kc)
    q_ref, _, _ = ref.qk_norm_rope_store(qkv, pos, cs, qw, kw, mode, mode == 2, 1e-6, kc, vc, slots, nq, nkv, hd)
    kd, vd = torch.zeros_like(kc).to(DEV), torch.zeros_like(vc).to(DEV)
    q = ops.qk_norm_rope_store(qkv.to(DEV), pos.to(DEV), cs.to(DEV), qw.to(DEV), kw.to(DEV), mode, mode == 2, 1e-6,
                               kd, vd, slots.to(DEV), nq, nkv, hd)
    close(q, q_ref, 3e-2)
    close(kd, kc, 3e-2)
    close(vd, vc, 3e-2)


def _paged_setup(B, nq, nkv, hd, lens, BS=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    nblk = [(n + BS - 1) // BS for n in lens]
    NB = sum(nblk) + 3
    kc = (torch.randn(NB, nkv, BS, hd, generator=g)).bfloat16()
    vc = (torch.randn(NB, nkv, BS, hd, generator=g)).bfloat16()
    perm = torch.randperm(NB, generator=g).tolist()
    bt = torch.zeros(B, max(nblk), dtype=torch.int32)
    k = 0
    for b in range(B):
        for j in range(nblk[b]):
            bt[b, j] = perm[k]
            k += 1
    return kc, vc, bt


@pytest.mark.parametrize("hd,nq,nkv", [(128, 32, 8), (128, 16, 8), (64, 32, 8), (256, 4, 1), (128, 8, 8)])
@pytest.mark.parametrize("window,softcap", [(0, 0.0), (300, 0.0), (0, 30.0)])
def test_paged_decode(hd, nq, nkv, window, softcap):
    lens = [1, 63, 64, 65, 700, 2049, 5000]
    B = len(lens)
    kc, vc, bt = _paged_setup(B, nq, nkv, hd, lens, seed=hd + nq)
    q = torch.randn(B, nq, hd, generator=torch.Generator().manual_seed(1)).bfloat16()
    ctx = torch.tensor(lens, dtype=torch.int32)
    scale = hd ** -0.5
    o_ref = ref.paged_decode(q, kc, vc, bt, ctx, scale, softcap, window)
    o = ops.paged_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), ctx.to(DEV), scale, softcap, window,
                         max_len=8192)
    torch.cuda.synchronize()
    ops.check_device_errors()
    close(o, o_ref, 2e-2)
    # single split (grid.x == 1) path: contexts that fit max_len = 64
    ctx64 = ctx.clamp(max=64)
    o1_ref = ref.paged_decode(q, kc, vc, bt, ctx64, scale, softcap, window)
    o1 = ops.paged_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), ctx64.to(DEV), scale, softcap, window,
                          max_len=64)
    torch.cuda.synchronize()
    ops.check_device_errors()
    close(o1, o1_ref, 2e-2)


def test_paged_decode_reports_context_beyond_max_len():
    """A context longer than the split grid (max_len) is skipped and reported, never silently truncated."""
    lens = [10, 700]
    kc, vc, bt = _paged_setup(2, 8, 8, 128, lens, seed=3)
    q = torch.randn(2, 8, 128, generator=torch.Generator().manual_seed(1)).bfloat16()
    ops.error_word(torch.device(DEV)).zero_()
    ops.paged_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), torch.tensor(lens, dtype=torch.int32).to(DEV),
                     128 ** -0.5, max_len=64)
    torch.cuda.synchronize()
    with pytest.raises(DeviceWaitTimeout):
        ops.check_device_errors()


@pytest.mark.parametrize("hd,nq,nkv", [(128, 32, 8), (64, 8, 8), (256, 4, 1), (128, 16, 8)])
@pytest.mark.parametrize("window", [0, 100])
@pytest.mark.parametrize("amp", [1.0, 12.0])
def test_paged_prefill_with_prefix(hd, nq, nkv, window, amp):
    """amp 12: scores spread over tens of units, so the running max moves by more than 2^8 between key tiles and
    the kernel's lazy O / l rescale runs."""
    # three sequences: fresh prompt, prompt with cached prefix, single-token chunk
    qlens = [77, 130, 1]
    klens = [77, 530, 300]
    B = 3
    kc, vc, bt = _paged_setup(B, nq, nkv, hd, klens, seed=7 + hd)
    T = sum(qlens)
    q = (torch.randn(T, nq, hd, generator=torch.Generator().manual_seed(2)) * amp).bfloat16()
    cu_q = torch.tensor([0, 77, 207, 208], dtype=torch.int32)
    cu_k = torch.tensor([0, 77, 607, 907], dtype=torch.int32)
    scale = hd ** -0.5
    o_ref = ref.prefill_attention(q, cu_q, cu_k, nq, nkv, hd, scale, 0.0, window, True, kc, vc, bt)
    o = ops.prefill_attention(q.to(DEV), cu_q.to(DEV), cu_k.to(DEV), max(qlens), nq, nkv, hd, scale, 0.0, window, True,
                              kc.to(DEV), vc.to(DEV), bt.to(DEV))
    torch.cuda.synchronize()
    ops.check_device_errors()
    close(o, o_ref, 2e-2)


@pytest.mark.parametrize("hd,nh", [(32, 12), (64, 4)])
def test_bidirectional_contiguous(hd, nh):
    lens = [16, 100, 513]
    T = sum(lens)
    cu = torch.tensor([0, 16, 116, 629], dtype=torch.int32)
    qkv = torch.randn(T, 3 * nh * hd, generator=torch.Generator().manual_seed(hd)).bfloat16()
    q = qkv[:, :nh * hd]
    scale = hd ** -0.5
    o_ref = ref.prefill_attention(q.reshape(T, nh, hd), cu, cu, nh, nh, hd, scale, causal=False, kv_src=qkv)
    qd = qkv.to(DEV)  # head_dim 32 runs the tcgen05 kernel in 64-wide tiles
    o = ops.prefill_attention(qd[:, :nh * hd], cu.to(DEV), cu.to(DEV), max(lens), nh, nh, hd, scale, causal=False,
                              kv_src=qd)
    close(o, o_ref, 2e-2)


def test_bidirectional_generic_head_dim():
    hd, nh = 48, 8  # no tensor-core instantiation: the CUDA-core path
    lens = [16, 100]
    T = sum(lens)
    cu = torch.tensor([0, 16, 116], dtype=torch.int32)
    qkv = torch.randn(T, 3 * nh * hd, generator=torch.Generator().manual_seed(5)).bfloat16()
    scale = hd ** -0.5
    o_ref = ref.prefill_attention(qkv[:, :nh * hd].reshape(T, nh, hd), cu, cu, nh, nh, hd, scale, causal=False,
                                  kv_src=qkv)
    qd = qkv.to(DEV)
    o = ops.prefill_attention(qd[:, :nh * hd], cu.to(DEV), cu.to(DEV), max(lens), nh, nh, hd, scale, causal=False,
                              kv_src=qd)
    close(o, o_ref, 2e-2)


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (7, 6144, 4096), (128, 4096, 12288), (200, 1000, 1024),
                                   (256, 3072, 1024), (257, 2048, 1024), (1000, 6144, 4096), (4096, 1024, 3072),
                                   (300, 151936 // 16, 1024)])
def test_gemm(M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    x = (torch.randn(M, K, generator=g) * 0.5).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    y_ref = ref.linear(x, w)
    y = ops.linear(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    ops.check_device_errors()
    close(y, y_ref, 2e-3, 0.02)


@pytest.mark.parametrize("M", [3, 128, 512])
@pytest.mark.parametrize("act", [ops.ACT_SILU_MUL, ops.ACT_GELU_MUL])
def test_gemm_fused_gate_up(M, act):
    g = torch.Generator().manual_seed(M + act)
    K, I = 1024, 1536
    x = (torch.randn(M, K, generator=g) * 0.5).bfloat16()
    gate = (torch.randn(I, K, generator=g) * 0.05).bfloat16()
    up = (torch.randn(I, K, generator=g) * 0.05).bfloat16()
    w = ref.interleave_gate_up(torch.cat([gate, up]), 128).contiguous()
    yg, yu = ref.linear(x, gate).float(), ref.linear(x, up).float()
    y_ref = ((ref.silu(yg) if act == ops.ACT_SILU_MUL else ref.gelu_tanh(yg)) * yu).bfloat16()
    y = ops.linear(x.to(DEV), w.to(DEV), act)
    close(y, y_ref, 5e-3, 0.03)


@pytest.mark.parametrize("splits", [1, 2, 5])
def test_gemm_fused_gate_up_split_k(splits):
    """Decode-sized fused gate/up GEMM with the K range split over CTAs (activation after the split sum)."""
    g = torch.Generator().manual_seed(11 + splits)
    M, K, I = 96, 2048, 2048
    x = (torch.randn(M, K, generator=g) * 0.5).bfloat16()
    gate = (torch.randn(I, K, generator=g) * 0.05).bfloat16()
    up = (torch.randn(I, K, generator=g) * 0.05).bfloat16()
    w = ref.interleave_gate_up(torch.cat([gate, up]), 128).contiguous()
    yg, yu = ref.linear(x, gate).float(), ref.linear(x, up).float()
    y_ref = (ref.silu(yg) * yu).bfloat16()
    y = ops.linear(x.to(DEV), w.to(DEV), ops.ACT_SILU_MUL, force_splits=splits)
    torch.cuda.synchronize()
    ops.check_device_errors()
    close(y, y_ref, 5e-3, 0.03)


@pytest.mark.parametrize("M,N,K", [(5, 4096, 4096), (128, 6144, 4096), (200, 4096, 12288)])
def test_gemm_split_partials_fused_into_consumers(M, N, K):
    """Split-K partials summed by add+RMSNorm / RoPE match the materialised GEMM result."""
    g = torch.Generator().manual_seed(M * 7 + N)
    x = (torch.randn(M, K, generator=g) * 0.5).bfloat16().to(DEV)
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16().to(DEV)
    y = ops.linear(x, w, partial_ok=True)
    dense = ops.linear(x, w)
    if isinstance(y, ops.SplitK):
        close(ops.materialize(y), dense, 2e-3, 0.02)
        res = torch.randn(M, N, generator=g).bfloat16().to(DEV)
        wn = torch.ones(N).bfloat16().to(DEV)
        r1 = res.clone()
        a, _ = ops.rms_norm(y, wn, 1e-6, 0, r1)
        r2 = res.clone()
        b, _ = ops.rms_norm(dense, wn, 1e-6, 0, r2)
        close(a, b, 3e-2)
        close(r1, r2, 2e-2)
    close(ops.materialize(y), ref.linear(x.cpu(), w.cpu()), 2e-3, 0.02)


def test_rope_consumes_split_partials():
    g = torch.Generator().manual_seed(77)
    nq, nkv, hd, T, K = 8, 2, 128, 9, 4096
    x = (torch.randn(T, K, generator=g) * 0.5).bfloat16().to(DEV)
    w = (torch.randn((nq + 2 * nkv) * hd, K, generator=g) * 0.02).bfloat16().to(DEV)
    y = ops.linear(x, w, partial_ok=True, force_splits=4)
    assert isinstance(y, ops.SplitK)
    dense = ops.materialize(y)
    cs = ref.rope_cos_sin(hd, 64, 1e6).to(DEV)
    pos = torch.arange(T, device=DEV)
    nw = torch.ones(hd).bfloat16().to(DEV)
    kc = torch.zeros(2, nkv, 256, hd).bfloat16().to(DEV)
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    slots = torch.arange(T, device=DEV, dtype=torch.int32)
    q1 = ops.qk_norm_rope_store(y, pos, cs, nw, nw, 0, False, 1e-6, kc, vc, slots, nq, nkv, hd)
    q2 = ops.qk_norm_rope_store(dense, pos, cs, nw, nw, 0, False, 1e-6, kc2, vc2, slots, nq, nkv, hd)
    close(q1, q2, 3e-2)
    close(kc, kc2, 3e-2)
    close(vc, vc2, 3e-2)


def test_gemm_forced_splits_deterministic():
    g = torch.Generator().manual_seed(9)
    x = torch.randn(64, 4096, generator=g).bfloat16().to(DEV)
    w = (torch.randn(2048, 4096, generator=g) * 0.02).bfloat16().to(DEV)
    a = ops.linear(x, w, force_splits=8)
    b = ops.linear(x, w, force_splits=8)
    assert torch.equal(a, b)
    close(a, ops.linear(x, w, force_splits=1), 2e-3, 0.02)


def test_embedding_and_gather():
    g = torch.Generator().manual_seed(4)
    table = torch.randn(1000, 256, generator=g).bfloat16()
    ids = torch.randint(0, 1000, (33,), generator=g)
    close(ops.embedding(table[100:600].to(DEV), ids.to(DEV), 2.0, 100, 600), ref.embedding(table[100:600], ids, 2.0, 100, 600), 1e-2)
    idx = torch.tensor([3, 0, 32])
    src = torch.randn(40, 256, generator=g).bfloat16()
    assert torch.equal(ops.gather_rows(src.to(DEV), idx.to(DEV)).cpu(), src[idx])


def test_act_mul_bias_meanpool():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(17, 512, generator=g).bfloat16()
    close(ops.act_mul(x.to(DEV), ops.ACT_SILU_MUL), ref.act_mul(x, ops.ACT_SILU_MUL), 1e-2)
    b = torch.randn(512, generator=g).bfloat16()
    close(ops.bias_act_(x.to(DEV).clone(), b.to(DEV), ops.BIAS_ACT_GELU_ERF), ref.bias_act(x, b, ops.BIAS_ACT_GELU_ERF), 2e-2)
    cu = torch.tensor([0, 5, 17], dtype=torch.int32)
    close(ops.mean_pool_l2(x.to(DEV), cu.to(DEV)), ref.mean_pool_l2(x, cu), 1e-3)


@pytest.mark.parametrize("softcap", [0.0, 5.0])
def test_candidate_sampling_kernel_matches_full_rows(softcap):
    """Top-k rows sampled from a candidate row with an id map (the tensor-parallel exchange, here one rank) give
    the tokens of the sampler over the whole row: masses, cut-offs, ties and Philox draws keyed by vocabulary id."""
    from nanovllm_b200.layers.embedding import ParallelLMHead
    B, V = 16, 5003
    g = torch.Generator().manual_seed(4)
    full = (torch.randn(B, V, generator=g) * 3).bfloat16()
    full[3, 17] = full[3, 4000] = full[3, 18] = 11.0
    dev = torch.device(DEV)
    head = ParallelLMHead(torch.zeros(V, 8, dtype=torch.bfloat16, device=dev), V)
    temps = torch.full((B,), 0.9, device=dev)
    topk = torch.tensor([1, 2, 5, 20, 64, 7, 3, 40] * 2, dtype=torch.int32, device=dev)
    topp = torch.tensor([1.0, 0.9, 0.5, 0.95, 0.8, 1.0, 0.3, 0.99] * 2, device=dev)
    seeds = torch.arange(B, dtype=torch.int64, device=dev) + 11
    sids = torch.arange(B, dtype=torch.int64, device=dev)
    steps = torch.full((B,), 4, dtype=torch.int32, device=dev)
    x = full.to(dev)
    got = head.sample_candidates(x, temps, topk, topp, seeds, sids, steps, kmax=64, softcap=softcap)
    want = ops.sample(x, temps, topk, topp, seeds, sids, steps, softcap=softcap)
    torch.cuda.synchronize()
    assert got.tolist() == want.tolist()


def test_sampler_matches_oracle():
    g = torch.Generator().manual_seed(6)
    B, V = 6, 5000
    logits = (torch.randn(B, V, generator=g) * 3).float()
    temps = torch.tensor([1.0, 0.7, 1.3, 0.5, 1.0, 0.9])
    topk = torch.tensor([1, 0, 50, 0, 5, 20], dtype=torch.int32)
    topp = torch.tensor([1.0, 0.9, 0.95, 1.0, 1.0, 0.5])
    seeds = torch.tensor([1, 2, 3, 4, 5, 6], dtype=torch.int64)
    sids = torch.tensor([10, 11, 12, 13, 14, 15], dtype=torch.int64)
    steps = torch.tensor([5, 6, 7, 8, 9, 10], dtype=torch.int32)
    want = ref.sample(logits, temps, topk, topp, seeds, sids, steps)
    got = ops.sample(logits.to(DEV), temps.to(DEV), topk.to(DEV), topp.to(DEV), seeds.to(DEV), sids.to(DEV),
                     steps.to(DEV))
    assert got.cpu().tolist() == want.tolist()
    # bf16 logits, argmax rows agree with torch.argmax (first max)
    lb = logits.bfloat16()
    got = ops.sample(lb.to(DEV), temps.to(DEV), torch.ones(B, dtype=torch.int32, device=DEV), topp.to(DEV),
                     seeds.to(DEV), sids.to(DEV), steps.to(DEV))
    assert got.cpu().tolist() == torch.argmax(lb.float(), dim=1).tolist()


@pytest.mark.parametrize("V", [5000, 5003])
def test_sampler_bf16_paths_with_ties_match_oracle(V):
    """bf16 logits with many exact ties: the coalesced fast path (V % 8 == 0) and the generic path (V = 5003)
    keep the same "first k of equal values" ties as the oracle and draw the same tokens."""
    g = torch.Generator().manual_seed(7)
    B = 8
    lb = (torch.round(torch.randn(B, V, generator=g) * 2) / 2).bfloat16()  # coarse values: lots of ties
    temps = torch.tensor([1.0, 0.7, 1.3, 0.5, 1.0, 0.9, 0.8, 1.1])
    topk = torch.tensor([0, 0, 50, 3, 5, 20, 1, 7], dtype=torch.int32)
    topp = torch.tensor([0.9, 0.5, 0.95, 1.0, 1.0, 0.3, 1.0, 0.8])
    seeds = torch.arange(1, B + 1, dtype=torch.int64)
    sids = torch.arange(20, 20 + B, dtype=torch.int64)
    steps = torch.arange(3, 3 + B, dtype=torch.int32)
    want = ref.sample(lb.float(), temps, topk, topp, seeds, sids, steps)
    got = ops.sample(lb.to(DEV), temps.to(DEV), topk.to(DEV), topp.to(DEV), seeds.to(DEV), sids.to(DEV),
                     steps.to(DEV))
    assert got.cpu().tolist() == want.tolist()
