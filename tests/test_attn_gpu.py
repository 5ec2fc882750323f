"""K2 parity on the GPU: dspark_verify_attn vs the CPU oracle (mirrors
tests/test_multirow_attn.py and the tree-mask cases of tests/test_tree.py:479-500).

Tolerances: rel-err max|out - ref| <= 1e-2 * max|ref| (the build's stated bound), and the
reference's own rule (tests/test_multirow_attn.py:80) with the ideal bf16 rounding of the
fp32 oracle standing in for MLX's error: err <= 2 * err(bf16(ref)) + 2e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL = 1e-2


def _mk(B, hq, hk, q_len, L, d, slack=0, seed=0, dev="cuda", dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn((B, hq, q_len, d), generator=g).to(dtype)
    k = torch.randn((B, hk, L + slack, d), generator=g).to(dtype)
    v = torch.randn((B, hk, L + slack, d), generator=g).to(dtype)
    q, k, v = q.to(dev), k.to(dev), v.to(dev)
    if slack:  # a cache-style view into a larger buffer
        k, v = k[:, :, :L], v[:, :, :L]
    return q, k, v


def _bits(t):
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _ref(oracle, q, k, v, scale, causal, anc=None):
    return oracle.sdpa(_bits(q), _bits(k), _bits(v), scale, causal, anc,
                       f16=q.dtype == torch.float16)


def _check(oracle, out, ref):
    o = out.float().cpu().numpy()
    mine = float(np.abs(o - ref).max())
    if out.dtype == torch.float16:
        ideal = float(np.abs(ref.astype(np.float16).astype(np.float32) - ref).max())
    else:
        ideal = float(np.abs(oracle.round_bf16(ref) - ref).max())
    assert mine <= REL * max(float(np.abs(ref).max()), 1e-6), (mine, float(np.abs(ref).max()))
    assert mine <= 2.0 * ideal + 2e-3, (mine, ideal)


CASES = [
    # B, hq, hk, q_len, L, d
    (1, 24, 4, 8, 1037, 256),     # Qwen3.8 geometry (head_dim 256), off-grid tail
    (1, 24, 4, 1, 300, 256),
    (1, 24, 4, 16, 33000, 256),   # head_dim 256 at a long context: split-and-merge plan
    (1, 32, 8, 15, 777, 128),     # drafter-block geometry, off-grid tail
    (1, 32, 8, 2, 64, 128),
    (1, 32, 2, 16, 500, 128),     # GQA 16 -> 256 rows: row groups
    (2, 8, 8, 5, 129, 64),        # MHA, batch 2
    (1, 16, 2, 7, 16, 128),       # KV exactly one 16-key tile
    (1, 4, 1, 3, 23, 64),         # MQA, short tail
    (1, 32, 8, 16, 1024, 128),    # BASELINE verify shape at 1k
    (3, 32, 8, 16, 2049, 128),    # batch 3, odd length
]


@pytest.mark.parametrize("B,hq,hk,q_len,L,d", CASES)
@pytest.mark.parametrize("causal", [True, False])
def test_matches_oracle(cuda, oracle, B, hq, hk, q_len, L, d, causal):
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    q, k, v = _mk(B, hq, hk, q_len, L, d, slack=37, seed=L + q_len)
    scale = d ** -0.5
    c = causal and q_len > 1
    out = multirow_sdpa(q, k, v, scale=scale, causal=c)
    assert out.shape == q.shape and out.dtype == q.dtype
    _check(oracle, out, _ref(oracle, q, k, v, scale, c))


@pytest.mark.parametrize("L", [1024, 4096, 16384, 32768])
def test_baseline_config(cuda, oracle, L):
    """GQA 32/8, head_dim 128, 16 causal rows, KV lengths 1k..32k."""
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    q, k, v = _mk(1, 32, 8, 16, L, 128, seed=L)
    out = multirow_sdpa(q, k, v, scale=128 ** -0.5, causal=True)
    _check(oracle, out, _ref(oracle, q, k, v, 128 ** -0.5, True))


@pytest.mark.parametrize("B,hq,hk,q_len,L,d", [(1, 24, 4, 8, 1037, 256), (1, 32, 8, 16, 2048, 128),
                                               (2, 8, 8, 5, 129, 64), (1, 32, 8, 16, 33000, 128),
                                               (3, 32, 8, 16, 2049, 128)])
def test_tensor_map_producer_matches_oracle(cuda, oracle, monkeypatch, B, hq, hk, q_len, L, d):
    """The optional tensor-map K/V producer (DSPARK_ATTN_TMA=1: 128-byte swizzled boxes,
    out-of-range keys zero-filled by the copy, keys past a split's end zeroed in the V
    fragments) gives the oracle's result, on cache views with slack rows too."""
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    monkeypatch.setenv("DSPARK_ATTN_TMA", "1")
    q, k, v = _mk(B, hq, hk, q_len, L, d, slack=37, seed=L + d)
    out = multirow_sdpa(q, k, v, scale=d ** -0.5, causal=True)
    _check(oracle, out, _ref(oracle, q, k, v, d ** -0.5, True))


@pytest.mark.parametrize("nrt", [1, 2, 4])
@pytest.mark.parametrize("L", [2048, 6000])
def test_row_tile_caps_agree(cuda, oracle, monkeypatch, nrt, L):
    """Every row-tile count the planner may pick (two up to 4k keys by default, four beyond;
    DSPARK_ATTN_NRT forces a cap) gives the oracle's result: fewer row tiles per CTA only
    re-partition the packed rows into more row groups."""
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    monkeypatch.setenv("DSPARK_ATTN_NRT", str(nrt))
    q, k, v = _mk(1, 32, 8, 16, L, 128, slack=11, seed=nrt * 7 + L)
    out = multirow_sdpa(q, k, v, scale=128 ** -0.5, causal=True)
    _check(oracle, out, _ref(oracle, q, k, v, 128 ** -0.5, True))


@pytest.mark.parametrize("B,hq,hk,q_len,L,d", [(1, 24, 4, 6, 900, 256), (1, 32, 8, 16, 2048, 128),
                                                (2, 8, 8, 5, 129, 64)])
def test_fp16_inputs(cuda, oracle, B, hq, hk, q_len, L, d):
    """fp16 q/k/v (tests/test_multirow_attn.py:83-87): fp16 output, the probabilities rounded
    to fp16 for P.V, against the oracle's fp16 restatement."""
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    q, k, v = _mk(B, hq, hk, q_len, L, d, slack=5, seed=d + L, dtype=torch.float16)
    out = multirow_sdpa(q, k, v, scale=d ** -0.5, causal=True)
    assert out.dtype == torch.float16 and out.shape == q.shape
    _check(oracle, out, _ref(oracle, q, k, v, d ** -0.5, True))


def test_head_dim_other_than_64_128_256_is_refused_loudly(cuda):
    from mlx_dspark_b200 import DSparkUnsupported
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    q, k, v = _mk(1, 24, 4, 8, 300, 96)
    with pytest.raises(DSparkUnsupported):
        multirow_sdpa(q, k, v, scale=96 ** -0.5, causal=True)


def test_causal_rows_see_only_their_prefix(cuda, oracle):
    """Masked keys made dominant: a mask leak would swamp the output
    (tests/test_multirow_attn.py:90-99)."""
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    q, k, v = _mk(1, 4, 4, 4, 64, 64)
    k = torch.cat([k[:, :, :-3], 50.0 * torch.ones_like(k[:, :, -3:])], dim=2)
    v = torch.cat([v[:, :, :-3], 1e3 * torch.ones_like(v[:, :, -3:])], dim=2)
    out = multirow_sdpa(q, k, v, scale=0.125, causal=True)
    ref = _ref(oracle, q, k, v, 0.125, True)
    assert float(np.abs(out.float().cpu().numpy() - ref).max()) < 50.0


def test_per_row_kv_lengths(cuda, oracle):
    """kv_len per batch row (ragged rows of the batch engine)."""
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    B, hq, hk, qL, L, d = 3, 32, 8, 12, 900, 128
    q, k, v = _mk(B, hq, hk, qL, L, d, seed=9)
    lens = [900, 413, 12]
    kv_len = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = multirow_sdpa(q, k, v, scale=d ** -0.5, causal=True, kv_len=kv_len)
    for b, Lb in enumerate(lens):
        ref = _ref(oracle, q[b : b + 1], k[b : b + 1, :, :Lb], v[b : b + 1, :, :Lb], d ** -0.5,
                   True)
        _check(oracle, out[b : b + 1], ref)


@pytest.mark.parametrize("tma", ["0", "1"])
def test_non_finite_cache_tail_is_never_read_into_the_result(cuda, oracle, monkeypatch, tma):
    """Cache rows past each request's kv_len may hold anything (here NaN): both K/V producers
    keep them out of the result (zero-filled copies, or zeroed V fragments behind a mask)."""
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    monkeypatch.setenv("DSPARK_ATTN_TMA", tma)
    B, hq, hk, qL, L, d = 2, 32, 8, 16, 1500, 128
    q, k, v = _mk(B, hq, hk, qL, L, d, seed=21)
    lens = [1500, 700]
    k[1, :, 700:] = float("nan")
    v[1, :, 700:] = float("nan")
    kv_len = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = multirow_sdpa(q, k, v, scale=d ** -0.5, causal=True, kv_len=kv_len)
    assert bool(torch.isfinite(out.float()).all())
    for b, Lb in enumerate(lens):
        ref = _ref(oracle, q[b : b + 1], k[b : b + 1, :, :Lb], v[b : b + 1, :, :Lb], d ** -0.5,
                   True)
        _check(oracle, out[b : b + 1], ref)


TREES = [
    [-1, 0, 0, 1, 1, 2, 3, 0],
    [-1, 0, 1, 2, 3, 0, 5, 1, 7, 2, 9, 0, 11, 12, 1, 14],
]


@pytest.mark.parametrize("parent", TREES)
@pytest.mark.parametrize("hq,hk,d", [(8, 2, 128), (32, 8, 128), (16, 4, 64)])
def test_tree_mask_variant(cuda, oracle, parent, hq, hk, d):
    from mlx_dspark_b200.multirow_attn import multirow_sdpa, tree_bits

    w = len(parent)
    q, k, v = _mk(1, hq, hk, w, 301 + w, d, seed=w)
    anc = np.array(tree_bits(parent), dtype=np.uint32)
    out = multirow_sdpa(q, k, v, scale=d ** -0.5, causal=False,
                        tree_anc=torch.from_numpy(anc.view(np.int32)).to(cuda))
    _check(oracle, out, _ref(oracle, q, k, v, d ** -0.5, False, anc))


def test_output_strides(cuda, oracle):
    """Output written straight into a [rows, heads*D] layout (the forward's o_proj input)."""
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    q, k, v = _mk(1, 32, 8, 16, 2048, 128, seed=4)
    buf = torch.zeros((16, 32 * 128), dtype=torch.bfloat16, device=cuda)
    view = buf.view(16, 32, 128).permute(1, 0, 2).unsqueeze(0)  # [1, 32, 16, 128]
    multirow_sdpa(q, k, v, scale=128 ** -0.5, causal=True, out=view)
    _check(oracle, view, _ref(oracle, q, k, v, 128 ** -0.5, True))
