"""GGUF weights kept packed (ops/quant.py): sharding / concatenation / permutation of the block bytes match the
same operations on the dequantized tensor, the tile-major repack is a lossless byte permutation, and a model
built from packed projections matches the dense-dequantized one (CPU; the fused GEMM itself is in
test_quant_gpu.py)."""
import os

import numpy as np
import pytest
import torch

from nanovllm_b200.loaders import dequant as DQ
from nanovllm_b200.loaders.gguf import pack_random_blocks
from nanovllm_b200.ops.quant import FUSED_TYPES, GgufPacked, cat_rows, repack_tiles, shard_cols, shard_rows

TYPES = sorted(FUSED_TYPES)


def _packed(t, N=200, K=512, seed=0):
    raw = torch.from_numpy(np.frombuffer(pack_random_blocks(t, (N, K), seed), dtype=np.uint8).copy())
    return GgufPacked(raw, t, N, K)


@pytest.mark.parametrize("t", TYPES)
def test_packed_dequantize_matches_decoder(t):
    w = _packed(t)
    want = DQ.dequantize(w.raw.reshape(-1), t, w.N * w.K).reshape(w.N, w.K)
    got = w.dequantize(torch.float32)
    assert torch.equal(got, want)
    assert torch.isfinite(got).all() and 0.005 < float(got.std()) < 0.08  # random blocks with a sane spread


@pytest.mark.parametrize("t", TYPES)
def test_packed_shard_cat_permute_match_dense(t):
    w = _packed(t, N=256, K=1024, seed=3)
    d = w.dequantize(torch.float32)
    assert torch.equal(shard_rows(w, 1, 4).dequantize(torch.float32), shard_rows(d, 1, 4))
    assert torch.equal(shard_cols(w, 1, 2).dequantize(torch.float32), shard_cols(d, 1, 2))
    v = _packed(t, N=64, K=1024, seed=4)
    assert torch.equal(cat_rows([w, v]).dequantize(torch.float32), torch.cat([d, v.dequantize(torch.float32)], 0))
    perm = torch.randperm(256, generator=torch.Generator().manual_seed(0))
    assert torch.equal(w.permute_rows(perm).dequantize(torch.float32), d[perm])
    with pytest.raises(ValueError):
        w.cols(128, 640)  # K slices must fall on 256-element boundaries


@pytest.mark.parametrize("t", TYPES)
def test_repack_is_a_lossless_byte_permutation(t):
    N, K = 300, 768  # N not a multiple of the 128-row tile
    w = _packed(t, N=N, K=K, seed=5)
    tiles = repack_tiles(w.raw, t, N, K)
    bprs = FUSED_TYPES[t]
    assert tiles.numel() == 3 * (K // 256) * 128 * bprs
    # every raw 4-bit field survives with its multiplicity (FP4 codes are regrouped pair-adjacent; padding adds
    # zero bytes only)
    def nibbles(b):
        b = b.reshape(-1).long()
        return torch.bincount(torch.cat([b & 0xF, b >> 4]), minlength=16)
    pad = tiles.numel() - w.raw.numel()
    raw_h, tile_h = nibbles(w.raw), nibbles(tiles)
    assert torch.equal(tile_h[1:], raw_h[1:]) and int(tile_h[0] - raw_h[0]) == 2 * pad
    # row r, step s of the tile-major layout starts at ((r // 128) * S + s) * 128 + r % 128
    S = K // 256
    t4 = tiles.reshape(3, S, 128, bprs)
    row, step = 131, 2
    if t in (12, 13):  # K-quants keep their block bytes in order
        be, bb = DQ.block_info(t)
        assert torch.equal(t4[1, step, 3, :bb], w.raw[row, step * bb:(step + 1) * bb])


def test_packed_linear_cpu_matches_dense():
    w = _packed(12, N=256, K=512, seed=7)
    x = torch.randn(5, 512).bfloat16()
    y = w.linear(x).float()
    want = x.float() @ w.dequantize(torch.float32).bfloat16().float().t()
    assert torch.allclose(y, want, atol=1e-2, rtol=1e-2)


def test_gguf_model_with_packed_projections_matches_dequantized(tmp_path, monkeypatch):
    from nanovllm_b200.api.factory import LlmModelFactory
    from nanovllm_b200.config import EngineConfig, HfConfig
    from nanovllm_b200.engine.sequence import Sequence
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.models.writers import write_gguf_model
    from nanovllm_b200.sampling_params import SamplingParams

    hf = HfConfig(vocab_size=300, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=64, max_position_embeddings=2048, model_type="qwen3",
                  architectures=["Qwen3ForCausalLM"], tie_word_embeddings=False)
    p = write_gguf_model(str(tmp_path / "q.gguf"), hf, init_random_weights(hf, 0), "Q4_K", big_type="Q6_K",
                         random_packed=True)

    def logits(mode):
        monkeypatch.setenv("NVB_GGUF_PACKED", mode)
        m = LlmModelFactory.make(p, device="cpu")
        kinds = {type(v).__name__ for v in m.weights.values()}
        llm = LLM(m, EngineConfig(max_num_seqs=2, max_model_len=512, num_kvcache_blocks=4,
                                  max_num_batched_tokens=256, stop_on_degenerate=False), device="cpu")
        s = Sequence(list(range(3, 40)), SamplingParams(max_tokens=1), 256)
        bm = llm.scheduler.block_manager
        bm.allocate(s, 0)
        s.num_scheduled_tokens = len(s.token_ids)
        out = llm.runner.forward_logits([s], True)[0].float()
        bm.deallocate(s)
        return out, kinds

    a, ka = logits("force")
    b, kb = logits("0")
    assert "GgufPacked" in ka and "GgufPacked" not in kb
    assert torch.allclose(a, b, atol=2e-2, rtol=2e-2), (a - b).abs().max()


def _h(p, o):
    return float(np.frombuffer(bytes(p[o:o + 2]), dtype=np.float16)[0])


def _decode8_model(p, t, e0):
    """Host model of the fused kernel's decode8 for the low-bit families (csrc/qgemm.cu), read from one repacked
    row step ``p`` (bytes): the kernel's field offsets and index arithmetic, element by element."""
    out = []
    for j in range(8):
        e = e0 + j
        if t in (6, 7):
            m_off = 16 if t == 7 else 0
            b, i = e >> 5, e & 31
            qh = int.from_bytes(bytes(p[16 + m_off + 4 * b:20 + m_off + 4 * b]), "little")
            q = p[48 + m_off + b * 16 + (i & 15)]
            n = (q >> 4 if i >= 16 else q & 0xF) | (((qh >> i) & 1) << 4)
            out.append(_h(p, 2 * b) * (n - 16) if t == 6 else _h(p, 2 * b) * n + _h(p, 16 + 2 * b))
        elif t in (10, 11, 35):
            half, j2, l = e >> 7, (e >> 5) & 3, e & 31
            qs = {10: 16, 11: 32, 35: 0}[t]
            q = (p[qs + half * 32 + l] >> (2 * j2)) & 3
            if t == 10:
                sc = p[half * 8 + j2 * 2 + (l >> 4)]
                out.append(_h(p, 80) * (sc & 0xF) * q - _h(p, 82) * (sc >> 4))
            elif t == 11:
                si = half * 8 + j2 * 2 + (l >> 4)
                w, k = si >> 2, si & 3
                lo = p[96 + (4 if w & 1 else 0) + k] >> ((w >> 1) * 4)
                sc = ((lo & 0xF) | (((p[104 + k] >> (2 * w)) & 3) << 4)) - 32
                h = (p[l] >> (half * 4 + j2)) & 1
                out.append(_h(p, 108) * sc * (q - (0 if h else 4)))
            else:
                out.append(_h(p, 64) * (q - 1))
        else:  # TQ1_0
            if e < 160:
                x, k = p[e & 31], e >> 5
            elif e < 240:
                x, k = p[32 + ((e - 160) & 15)], (e - 160) >> 4
            else:
                x, k = p[48 + ((e - 240) & 3)], (e - 240) >> 2
            r = (x * 3 ** k) & 0xFF
            out.append(_h(p, 52) * (((r * 3) >> 8) - 1))
    return out


@pytest.mark.parametrize("t", [6, 7, 10, 11, 34, 35])
def test_low_bit_repacked_layout_decodes_like_the_reference_decoder(t):
    N, K = 128, 512
    w = _packed(t, N=N, K=K, seed=11)
    want = w.dequantize(torch.float32).numpy()
    tiles = repack_tiles(w.raw, t, N, K).reshape(1, K // 256, 128, FUSED_TYPES[t]).numpy()
    for r in (0, 77):
        for s in range(K // 256):
            p = tiles[0, s, r].tolist()
            got = [v for e0 in range(0, 256, 8) for v in _decode8_model(p, t, e0)]
            np.testing.assert_allclose(np.array(got, dtype=np.float32), want[r, s * 256:(s + 1) * 256], rtol=1e-6,
                                       atol=1e-7)
