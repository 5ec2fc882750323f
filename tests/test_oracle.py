"""The CPU oracle pinned before it is trusted (CPU only).

* Integer semantics against the reference's own goldens (tests/golden/reference_goldens.json,
  extracted from mlx-dspark's tests/test_batch_engine.py by extract_reference_goldens.py):
  BatchCache offsets / trims / moves / growth, build_batch_mask, _ctx_block_mask, and the
  argmax draft sampling.
* QMM and attention numerics against analytic known answers (MLX itself cannot be imported
  here, so numeric parity with MLX is unpinned; these cases pin the restatement instead):
  exact integer products through every nibble / byte position, one-hot inputs returning
  dequantized weights, float64 recomputation, attention with a single visible key, uniform
  scores (mean of V), the causal and tree visibility rules.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())


# ----------------------------------------------------------------------------- goldens

def _rows(lens, H=2, D=4, seed=0):
    rng = np.random.default_rng(seed)
    return [(rng.normal(size=(1, H, L, D)).astype(np.float32),
             rng.normal(size=(1, H, L, D)).astype(np.float32)) for L in lens]


@pytest.mark.parametrize("case", GOLD["batch_cache"], ids=lambda c: c["name"])
def test_batch_cache_goldens(case):
    c = oracle.BatchCacheRef.from_rows(_rows(case["lens"]))
    if "offset_view" in case:
        c.rows = 2
        assert c.offset == case["offset_view"]
    for op in case["ops"]:
        if op[0] == "update":
            B = len(case["lens"]) if c.rows is None else c.rows
            k = np.ones((B, 2, op[1], 4), np.float32)
            K, _ = c.update_and_fetch(k, k)
            if len(op) > 2:
                assert K.shape[2] == op[2]
        elif op[0] == "trim":
            c.trim(op[1])
        elif op[0] == "move":
            c.move_row(op[1], op[2])
        elif op[0] == "rows":
            c.rows = op[1]
        elif op[0] == "expect":
            assert c.offsets == op[1]


def test_batch_cache_writes_land_at_offsets():
    pairs = _rows([3, 1, 4])
    c = oracle.BatchCacheRef.from_rows(pairs)
    for b, (k, v) in enumerate(pairs):
        np.testing.assert_array_equal(c.keys[b, :, : k.shape[2]], k[0])
    new = np.full((3, 2, 1, 4), 7.0, np.float32)
    c.update_and_fetch(new, new)
    for b, L in enumerate([3, 1, 4]):
        np.testing.assert_array_equal(c.keys[b, :, L], new[b, :, 0])
    c.trim([0, 1, 2])
    new2 = np.full((3, 2, 1, 4), 9.0, np.float32)
    c.update_and_fetch(new2, new2)
    for b, off in enumerate([4, 1, 3]):  # next write overwrites the trimmed tail
        np.testing.assert_array_equal(c.keys[b, :, off], new2[b, :, 0])


def test_grow_keeps_step_multiple():
    c = oracle.BatchCacheRef.from_rows(_rows([oracle.STEP - 1, oracle.STEP - 1]))
    k = np.ones((2, 2, 3, 4), np.float32)
    c.update_and_fetch(k, k)
    assert c.keys.shape[2] % oracle.STEP == 0 and c.keys.shape[2] >= oracle.STEP + 2


@pytest.mark.parametrize("case", GOLD["batch_mask"], ids=lambda c: str(c["offsets"]))
def test_batch_mask_goldens(case):
    m = oracle.build_batch_mask(case["offsets"], case["T"])
    assert list(m.shape) == case["shape"]
    for (b, i), row in zip(case["index"], case["rows"]):
        assert m[b, 0, i].astype(int).tolist() == row


@pytest.mark.parametrize("case", GOLD["ctx_block_mask"], ids=lambda c: str(c["lens"]))
def test_ctx_block_mask_goldens(case):
    m = oracle.ctx_block_mask(case["lens"], case["k"])
    assert list(m.shape) == case["shape"]
    for (b, i), row in zip(case["index"], case["rows"]):
        assert m[b, 0, i].astype(int).tolist() == row


@pytest.mark.parametrize("case", GOLD["sample_block_argmax"])
def test_argmax_draft_goldens(case):
    base = np.zeros(case["shape"], np.float32)
    for r, c, v in case["hot"]:
        base[r, c, v] = 1.0
    assert oracle.argmax_first(base).tolist() == case["argmax"]


def test_argmax_first_index_on_ties():
    x = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, 5.0, 5.0, 5.0]], np.float32)
    assert oracle.argmax_first(x).tolist() == [1, 0]


@pytest.mark.parametrize("drafts,tt,n", [([5, 6, 7], [5, 6, 7, 8], 3), ([5, 6, 7], [5, 9, 7, 8], 1),
                                         ([5], [4, 1], 0), ([], [3], 0)])
def test_accept_rule(drafts, tt, n):
    got_n, committed, trim = oracle.accept(drafts, tt)
    assert got_n == n
    assert committed == drafts[:n] + [tt[n]]
    assert trim == len(drafts) - n


def test_rollback_clamps():
    assert oracle.rollback([5, 2, 0], [2, 5, 1]) == [3, 0, 0]


def test_pack_ragged_small():
    r = oracle.pack_ragged([2, 0, 3], [10, 4, 7], [0, 100, 200], [[1, 2, 0], [0, 0, 0], [5, 6, 7]])
    assert r["cu_rows"] == [0, 2, 2, 5]
    assert r["row_pos"] == [10, 11, 7, 8, 9]
    assert r["row_kv"] == [0, 0, 200, 200, 200]
    assert r["row_req"] == [0, 0, 2, 2, 2]
    assert r["ids"] == [1, 2, 5, 6, 7]
    assert r["kv_len_new"] == [12, 4, 10]


# ----------------------------------------------------------------------------- quantization

@pytest.mark.parametrize("bits", [4, 8])
def test_pack_unpack_roundtrip(bits):
    rng = np.random.default_rng(bits)
    q = rng.integers(0, 1 << bits, (16, 256), dtype=np.uint32)
    np.testing.assert_array_equal(oracle.unpack(oracle.pack(q, bits), bits), q)


def test_pack_is_lsb_first():
    q = np.arange(8, dtype=np.uint32)[None, :]  # k = 0..7 -> nibbles 0..7
    assert int(oracle.pack(q, 4)[0, 0]) == 0x76543210
    q8 = np.array([[1, 2, 3, 4]], dtype=np.uint32)
    assert int(oracle.pack(q8, 8)[0, 0]) == 0x04030201


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_error_bound(bits):
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (64, 512)).astype(np.float32)
    wq, sc, bi = oracle.quantize(w, bits)
    back = oracle.dequantize(wq, sc, bi, bits)
    step = oracle.from_bf16(sc).repeat(64, axis=1)
    # rounding to the grid (half a step) plus bf16 rounding of scale / bias
    assert np.all(np.abs(back - w) <= 0.5 * step + 2 ** -8 * (np.abs(w) + step * (1 << bits)))


# ----------------------------------------------------------------------------- qmm

@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_exact_integers(bits):
    rng = np.random.default_rng(1)
    N, K = 48, 512
    q = rng.integers(0, 1 << bits, (N, K), dtype=np.uint32)
    wq = oracle.pack(q, bits)
    ones = oracle.to_bf16(np.ones((N, K // 64), np.float32))
    zeros = oracle.to_bf16(np.zeros((N, K // 64), np.float32))
    x = rng.integers(-3, 4, (5, K)).astype(np.float32)
    y = oracle.qmm(oracle.to_bf16(x), wq, ones, zeros, bits)
    np.testing.assert_array_equal(y, x @ q.T.astype(np.float32))


@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_one_hot_reads_dequantized_columns(bits):
    rng = np.random.default_rng(2)
    N, K = 64, 1024
    wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), bits)
    ks = [0, 7, 63, 64, 511, 1023]
    x = np.zeros((len(ks), K), np.float32)
    x[np.arange(len(ks)), ks] = 1.0
    y = oracle.qmm(oracle.to_bf16(x), wq, sc, bi, bits)
    w = oracle.dequantize(wq, sc, bi, bits)
    np.testing.assert_allclose(y, w[:, ks].T, rtol=0, atol=1e-7)


@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_matches_float64(bits):
    rng = np.random.default_rng(3)
    N, K, M = 256, 2048, 16
    wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), bits)
    x = oracle.to_bf16(rng.normal(0, 1, (M, K)))
    y = oracle.qmm(x, wq, sc, bi, bits)
    ref = oracle.from_bf16(x).astype(np.float64) @ oracle.dequantize(wq, sc, bi, bits).T.astype(np.float64)
    assert np.abs(y - ref).max() <= 1e-5 * max(np.abs(ref).max(), 1.0)


# ----------------------------------------------------------------------------- attention

def _bf(a):
    return oracle.to_bf16(np.asarray(a, np.float32))


def _sdpa64(q, k, v, scale, mask):
    q, k, v = (oracle.from_bf16(t).astype(np.float64) for t in (q, k, v))
    B, Hq, qL, D = q.shape
    G = Hq // k.shape[1]
    k = np.repeat(k, G, axis=1)
    v = np.repeat(v, G, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    s = np.where(mask, s, -np.inf)
    p = np.exp(s - s.max(axis=-1, keepdims=True))
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


@pytest.mark.parametrize("B,Hq,Hk,qL,L,D", [(1, 8, 2, 5, 40, 64), (2, 4, 4, 3, 17, 32),
                                            (1, 32, 8, 16, 300, 128)])
def test_sdpa_causal_matches_float64(B, Hq, Hk, qL, L, D):
    rng = np.random.default_rng(L)
    q, k, v = _bf(rng.normal(size=(B, Hq, qL, D))), _bf(rng.normal(size=(B, Hk, L, D))), \
        _bf(rng.normal(size=(B, Hk, L, D)))
    i = np.arange(qL)[:, None]
    j = np.arange(L)[None, :]
    ref = _sdpa64(q, k, v, D ** -0.5, j <= L - qL + i)
    got = oracle.sdpa(q, k, v, D ** -0.5, True)
    assert np.abs(got - ref).max() < 1e-5


def test_sdpa_single_visible_key_returns_its_value():
    rng = np.random.default_rng(0)
    q = _bf(rng.normal(size=(1, 2, 1, 16)))
    k = _bf(rng.normal(size=(1, 1, 1, 16)))
    v = _bf(rng.normal(size=(1, 1, 1, 16)))
    got = oracle.sdpa(q, k, v, 0.25, True)
    np.testing.assert_array_equal(got[0, :, 0], np.repeat(oracle.from_bf16(v)[0, :, 0], 2, 0))


def test_sdpa_uniform_scores_average_values():
    q = _bf(np.zeros((1, 1, 1, 8)))
    v = np.arange(10 * 8, dtype=np.float32).reshape(1, 1, 10, 8)
    got = oracle.sdpa(q, _bf(np.ones((1, 1, 10, 8))), _bf(v), 1.0, False)
    np.testing.assert_allclose(got[0, 0, 0], v[0, 0].mean(axis=0), rtol=1e-6)


def test_sdpa_causal_rule_hides_future_keys():
    # row i of a 3-row block over 8 keys sees keys <= 5 + i: a dominant masked key must not leak
    q = _bf(np.ones((1, 1, 3, 8)))
    k = np.zeros((1, 1, 8, 8), np.float32)
    k[0, 0, 7] = 50.0
    v = np.zeros((1, 1, 8, 8), np.float32)
    v[0, 0, 7] = 1000.0
    got = oracle.sdpa(q, _bf(k), _bf(v), 1.0, True)
    assert np.abs(got[0, 0, :2]).max() == 0.0 and got[0, 0, 2].max() > 900.0


def test_sdpa_tree_rule():
    # tree over the last 3 keys: row 1 sees key L-3 (its parent) and itself, not row 2's key
    rng = np.random.default_rng(1)
    q, k, v = _bf(rng.normal(size=(1, 2, 3, 16))), _bf(rng.normal(size=(1, 1, 9, 16))), \
        _bf(rng.normal(size=(1, 1, 9, 16)))
    anc = np.array([0b001, 0b011, 0b101], np.uint32)
    L = 9
    mask = np.ones((3, L), bool)
    for i in range(3):
        for j in range(3):
            mask[i, L - 3 + j] = bool((anc[i] >> j) & 1)
    ref = _sdpa64(q, k, v, 0.25, mask)
    got = oracle.sdpa(q, k, v, 0.25, False, anc)
    assert np.abs(got - ref).max() < 1e-5


# ----------------------------------------------------------------------------- forward pieces

def test_rmsnorm_rope_silu_definitions():
    x = np.array([[3.0, 4.0]], np.float32)
    np.testing.assert_allclose(oracle.rmsnorm(x, np.ones(2), 0.0), x / np.sqrt(12.5), rtol=4e-3)
    # rope at position 0 is the identity; at pi/2 rotates the (i, i+D/2) pairs
    v = oracle.round_bf16(np.arange(8, dtype=np.float32)[None, None, :])
    np.testing.assert_array_equal(oracle.rope(v, [0], 1e6), v)
    r = oracle.rope(np.array([[[1.0, 0, 0, 0, 0, 0, 0, 0]]], np.float32), [np.pi / 2], 1e6)
    assert abs(r[0, 0, 4] - 1.0) < 1e-2 and abs(r[0, 0, 0]) < 1e-2
    assert abs(float(oracle.silu_mul(np.float32(1.0), np.float32(2.0))) - 2 / (1 + np.exp(-1))) < 1e-2


def test_partition_requests_balances_kv():
    """Data-parallel placement: every request lands on exactly one rank and the ranks' summed
    KV lengths stay within one request of each other (longest-first greedy)."""
    import mlx_dspark_b200  # noqa: F401  (ctypes load only; no GPU call)
    from mlx_dspark_b200.batch_engine import partition_requests

    rng = np.random.default_rng(0)
    lengths = [int(x) for x in np.exp(rng.uniform(np.log(256), np.log(16384), 256))]
    for world in (1, 2, 4, 8):
        parts = partition_requests(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(256))
        loads = [sum(lengths[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lengths)
