"""Quantized KV cache (the reference's kv_bits path, src/mlx_dspark/target.py:166-185) on the GPU.

* dspark_kv_append_q quantizes each appended K/V row per group of 64 bit-exactly like the
  oracle's quantizer (codes, bf16 scales and biases), at each row's own length;
* trim is metadata only: the next append overwrites the rejected tail;
* dspark_verify_attn_q (dequantizing producers feeding the verify attention) matches the
  oracle's attention over the exactly dequantized K/V within the attention bar (1e-2 of max|ref|),
  4- and 8-bit, head_dim 64 and 128, GQA, several lengths, causal and not.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _np(t):
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("D", [64, 128])
def test_append_is_bit_exact_and_rollback_overwrites(cuda, oracle, bits, D):
    from mlx_dspark_b200.kvcache import QuantizedKVCache

    B, H, cap = 3, 4, 80
    c = QuantizedKVCache(B, H, cap, D, bits)
    g = torch.Generator(device=cuda).manual_seed(bits + D)
    c.lens.copy_(torch.tensor([0, 5, 17], dtype=torch.int32))
    k1 = torch.randn((B, H, 9, D), device=cuda, generator=g).to(torch.bfloat16)
    v1 = (3 * torch.randn((B, H, 9, D), device=cuda, generator=g)).to(torch.bfloat16)
    c.update(k1, v1)
    torch.cuda.synchronize()
    assert c.offset == [9, 14, 26]
    for b, L0 in enumerate([0, 5, 17]):
        for name, src in (("k", k1), ("v", v1)):
            wq, sc, bi = oracle.quantize_rows(src[b].float().cpu().numpy(), bits)
            got_q = _np(getattr(c, name + "q")[b, :, L0 : L0 + 9])
            got_s = _np(getattr(c, name + "s")[b, :, L0 : L0 + 9])
            got_b = _np(getattr(c, name + "b")[b, :, L0 : L0 + 9])
            assert np.array_equal(got_q, wq) and np.array_equal(got_s, sc)
            assert np.array_equal(got_b, bi)
    # reject 4 / 0 / 9: the next block lands right after the kept rows, overwriting the tail
    c.trim(torch.tensor([4, 0, 9], dtype=torch.int32, device=cuda))
    k2 = torch.randn((B, H, 2, D), device=cuda, generator=g).to(torch.bfloat16)
    c.update(k2, k2)
    torch.cuda.synchronize()
    assert c.offset == [7, 16, 19]
    wq, _, _ = oracle.quantize_rows(k2[0].float().cpu().numpy(), bits)
    assert np.array_equal(_np(c.kq[0, :, 5:7]), wq)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("B,Hq,Hk,qL,D,lens,causal", [
    (1, 32, 8, 16, 128, [2048], True),        # the BASELINE verify shape at 2k
    (2, 8, 2, 5, 64, [300, 129], True),
    (1, 16, 4, 12, 128, [777], False),
    (3, 32, 8, 16, 128, [1500, 64, 999], True),
])
def test_attention_over_quantized_cache(cuda, oracle, bits, B, Hq, Hk, qL, D, lens, causal):
    from mlx_dspark_b200.kvcache import QuantizedKVCache

    cap = max(lens) + 8
    c = QuantizedKVCache(B, Hk, cap, D, bits)
    g = torch.Generator(device=cuda).manual_seed(sum(lens) + bits)
    k = torch.randn((B, Hk, cap, D), device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn((B, Hk, cap, D), device=cuda, generator=g).to(torch.bfloat16)
    c.update(k, v)  # fill every position, then set the live lengths
    c.lens.copy_(torch.tensor(lens, dtype=torch.int32))
    q = torch.randn((B, Hq, qL, D), device=cuda, generator=g).to(torch.bfloat16)
    out = c.attention(q, scale=D ** -0.5, causal=causal)
    torch.cuda.synchronize()
    ref = oracle.sdpa_q(_np(q).reshape(B, Hq, qL, D), _np(c.kq), _np(c.ks), _np(c.kb),
                        _np(c.vq), _np(c.vs), _np(c.vb), bits, lens, D ** -0.5, causal)
    err = float(np.abs(out.float().cpu().numpy() - ref).max())
    assert err <= 1e-2 * float(np.abs(ref).max()), err
