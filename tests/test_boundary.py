"""The C-ABI boundary and the host-side operator surface (CPU only: no kernel launches).

* libdspark.so loads and exports every entry point include/dspark.h declares, with the
  ctypes signatures the shim binds;
* argument validation fails loudly with a status (no launch, no fallback);
* the reference-shaped dispatch surface: eligibility gates, shape keys, allowlists, the
  scoped patches (restore on exit / on exception / nesting), multirow windows and gates —
  mirroring tests/test_small_m_qmm.py and tests/test_multirow_attn.py of the reference;
* CPU tensors are refused (there is no CPU path).
"""

from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest
import torch

import mlx_dspark_b200  # noqa: F401
from mlx_dspark_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = (ROOT / "include" / "dspark.h").read_text()


def _declared() -> list[str]:
    return sorted(set(re.findall(r"^\s*(?:int|size_t|long long|const char\*)\s+(dspark_\w+)\(",
                                 HEADER, re.M)))


def test_header_declares_the_boundary():
    names = _declared()
    for must in ("dspark_qmm", "dspark_verify_attn", "dspark_kv_append", "dspark_kv_rollback",
                 "dspark_pack_ragged", "dspark_accept", "dspark_verify_forward"):
        assert must in names


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (dspark_\w+)$", out, re.M))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing


def test_shim_binds_every_declared_symbol():
    assert set(_declared()) == set(_lib.EXPORTED)


def test_version_and_error_string():
    assert _lib.lib.dspark_version() >= 100
    assert isinstance(_lib.last_error(), str)


def test_qmm_argument_checks_fail_loudly():
    buf = (C.c_uint8 * 64)()
    p = C.cast(buf, C.c_void_p)
    assert _lib.lib.dspark_qmm(p, 4, 512, p, p, p, 64, 3, 64, p, None) == _lib.ERR_UNSUPPORTED
    assert "bits" in _lib.last_error()
    assert _lib.lib.dspark_qmm(p, 4, 512, p, p, p, 64, 4, 32, p, None) == _lib.ERR_UNSUPPORTED
    assert _lib.lib.dspark_qmm(p, 4, 500, p, p, p, 64, 4, 64, p, None) == _lib.ERR_UNSUPPORTED
    assert _lib.lib.dspark_qmm(p, 40, 512, p, p, p, 64, 4, 64, p, None) == _lib.ERR_UNSUPPORTED
    assert _lib.lib.dspark_qmm(None, 4, 512, p, p, p, 64, 4, 64, p, None) == _lib.ERR_ARG


def test_attention_argument_checks_fail_loudly():
    buf = (C.c_uint8 * 64)()
    p = C.cast(buf, C.c_void_p)
    s = _lib.i64_array([0, 0, 0])
    rc = _lib.lib.dspark_verify_attn(p, s, p, s, p, s, 1, 6, 4, 2, 128, 64, None, 0.1, 1, None, p,
                                     s, None, 0, None)
    assert rc == _lib.ERR_ARG  # Hq not a multiple of Hk
    rc = _lib.lib.dspark_verify_attn(p, s, p, s, p, s, 1, 8, 2, 2, 96, 64, None, 0.1, 1, None, p,
                                     s, None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED and "head_dim" in _lib.last_error()
    rc = _lib.lib.dspark_verify_attn_dt(7, p, s, p, s, p, s, 1, 8, 2, 2, 128, 64, None, 0.1, 1,
                                        None, p, s, None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED and "dtype" in _lib.last_error()


def test_status_needs_init():
    code = C.c_int(0)
    assert _lib.lib.dspark_device_status(63, C.byref(code), 0) == _lib.ERR_NOT_INIT


def test_cpu_tensors_are_refused():
    from mlx_dspark_b200 import DSparkUnsupported, skinny_qmm

    with pytest.raises(DSparkUnsupported):
        skinny_qmm.qmm(torch.zeros(2, 512, dtype=torch.bfloat16), torch.zeros(64, 64, dtype=torch.int32),
                       torch.zeros(64, 8, dtype=torch.bfloat16), torch.zeros(64, 8, dtype=torch.bfloat16), 4)


# ----------------------------------------------------------------- small-M dispatch surface

K, N = 512, 4096


def _qlinear(out_features=N, in_features=K, bits=4, group_size=64, bias=False):
    from mlx_dspark_b200.small_m_qmm import QuantizedLinear

    lin = torch.nn.Linear(in_features, out_features, bias=bias)
    return QuantizedLinear.from_linear(lin, group_size=group_size, bits=bits)


class _Tiny(torch.nn.Module):
    def __init__(self, **kw):
        super().__init__()
        self.proj = _qlinear(**kw)


def test_eligibility_gates():
    from mlx_dspark_b200.small_m_qmm import eligible

    assert eligible(_qlinear())
    assert eligible(_qlinear(bits=8))
    assert not eligible(_qlinear(bits=2))
    assert not eligible(_qlinear(group_size=32))
    assert eligible(_qlinear(out_features=1024))
    assert eligible(_qlinear(in_features=K + 128))
    assert eligible(_qlinear(bits=8, out_features=1024, in_features=K + 64))
    assert not eligible(_qlinear(out_features=1020))
    assert not eligible(torch.nn.Linear(K, N))


def test_shape_key_and_allowlist():
    from mlx_dspark_b200.small_m_qmm import ids_for_shapes, shape_key

    assert shape_key(_qlinear()) != shape_key(_qlinear(bits=8))
    model = _Tiny()
    assert ids_for_shapes([shape_key(model.proj)], model) == frozenset({id(model.proj)})
    assert ids_for_shapes(["1x1b4"], model) == frozenset()


def test_patch_scope_restores():
    from mlx_dspark_b200.small_m_qmm import QuantizedLinear, _orig_call, active, small_m_matmul

    with small_m_matmul(None):
        assert not active()
    with small_m_matmul(frozenset()):
        assert not active()
    with small_m_matmul(frozenset({1})):
        assert active()
        with small_m_matmul(frozenset({2})):  # nested: no-op, stays active
            assert active()
        assert active()
    assert not active() and QuantizedLinear.__call__ is _orig_call
    with pytest.raises(RuntimeError), small_m_matmul(frozenset({1})):
        raise RuntimeError("boom")
    assert not active()


def test_windows_cover_the_verify_widths():
    from mlx_dspark_b200 import skinny_qmm

    for bits in (4, 8):
        lo, hi = skinny_qmm.WINDOW[bits]
        assert lo <= 5 and hi >= 16  # the reference's windows (5-16 / 6-16) are inside


# ----------------------------------------------------------------- multirow attention surface

def _qkv(B, hq, hk, q_len, L, d, dtype=torch.bfloat16):
    return (torch.zeros(B, hq, q_len, d, dtype=dtype), torch.zeros(B, hk, L, d, dtype=dtype),
            torch.zeros(B, hk, L, d, dtype=dtype))


def test_multirow_eligible_gate():
    from mlx_dspark_b200.multirow_attn import MultirowConfig, Window, eligible

    cfg = MultirowConfig((Window(8, 2, 64, min_q=2, max_q=16, min_kv=64),))
    q, k, v = _qkv(1, 8, 2, 4, 128, 64)
    assert eligible(q, k, v, "causal", None, cfg)
    assert eligible(q, k, v, None, None, cfg)
    assert not eligible(q, k, v, torch.ones(1, 1, 4, 128, dtype=torch.bool), None, cfg)
    assert not eligible(q, k, v, "causal", torch.zeros(8), cfg)
    assert not eligible(*_qkv(1, 8, 2, 1, 128, 64), "causal", None, cfg)     # q_len below window
    assert not eligible(*_qkv(1, 8, 2, 17, 128, 64), "causal", None, cfg)    # prefill-wide q
    assert not eligible(*_qkv(1, 8, 2, 4, 32, 64), "causal", None, cfg)      # short KV
    assert not eligible(*_qkv(1, 16, 2, 4, 128, 64), "causal", None, cfg)    # unconfigured shape
    assert not eligible(*_qkv(1, 8, 2, 4, 128, 64, torch.float32), "causal", None, cfg)
    assert eligible(*_qkv(1, 8, 2, 4, 128, 64, torch.float16), "causal", None, cfg)  # fp16 served
    cfg256 = MultirowConfig((Window(24, 4, 256, min_q=1, max_q=16, min_kv=16),))
    assert eligible(*_qkv(1, 24, 4, 8, 1037, 256), "causal", None, cfg256)  # head_dim 256
    assert cfg.window(8, 2, 64) is not None and cfg.window(8, 2, 128) is None


def test_multirow_patch_scope_and_passthrough():
    from mlx_dspark_b200 import multirow_attn as mra

    orig = mra.scaled_dot_product_attention
    cfg = mra.MultirowConfig((mra.Window(8, 2, 64, min_kv=64),))
    g = torch.Generator().manual_seed(0)
    qo = torch.randn(1, 16, 4, 64, generator=g).to(torch.bfloat16)  # unconfigured -> passes
    ko = torch.randn(1, 2, 128, 64, generator=g).to(torch.bfloat16)
    stock = orig(qo, ko, ko, scale=0.125, mask="causal")
    with mra.multirow_attention(cfg):
        assert mra.active()
        passed = mra.sdpa(qo, ko, ko, scale=0.125, mask="causal")
        with mra.multirow_attention(cfg):  # nested no-op
            assert mra.active()
    assert mra.scaled_dot_product_attention is orig and not mra.active()
    assert torch.equal(passed, stock)
    with mra.multirow_attention(None):
        assert not mra.active()


def test_tree_bits():
    from mlx_dspark_b200.multirow_attn import tree_bits

    assert tree_bits([-1, 0, 0, 1]) == [0b1, 0b11, 0b101, 0b1011]


_MIRRORS = {"QWeight": "dspark_qweight", "Layer": "dspark_layer", "Model": "dspark_model",
            "FwdBuffers": "dspark_fwd_buffers", "P2PGatherArgs": "dspark_p2p_gather_args",
            "QmmArgs": "dspark_qmm_args", "QKV": "dspark_qkv"}


def test_ctypes_mirrors_match_the_header_layout(tmp_path):
    """Every struct the shim passes by pointer has, field by field, the offsets and the size the
    C compiler gives include/dspark.h (a drifted mirror would hand the kernels shifted fields)."""
    import shutil

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "dspark.h"', "int main(void) {"]
    want = {}
    for py, c in _MIRRORS.items():
        cls = getattr(_lib, py)
        lines.append(f'  printf("{py} %zu\\n", sizeof({c}));')
        want[py] = C.sizeof(cls)
        for name, _ in cls._fields_:
            lines.append(f'  printf("{py}.{name} %zu\\n", offsetof({c}, {name}));')
            want[f"{py}.{name}"] = getattr(cls, name).offset
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-std=c11", "-I", str(ROOT / "include"), str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                       text=True).stdout.splitlines())
    assert {k: int(v) for k, v in got.items()} == want


def test_fp16_and_fp32_scales_do_not_fit_the_kernel():
    """The reference's fits() accepts bf16/fp16/fp32 scales (src/mlx_dspark/skinny_qmm.py:
    174-181); the kernels read bf16 scales only, so other scale types are refused by fits()
    and by qmm() (no silent misread), and such layers stay on the stock path."""
    from mlx_dspark_b200 import DSparkUnsupported, quant, skinny_qmm, small_m_qmm

    qw = quant.QWeight(torch.zeros(64, 64, dtype=torch.int32),
                       torch.ones(64, 8, dtype=torch.bfloat16),
                       torch.zeros(64, 8, dtype=torch.bfloat16), 4)
    assert skinny_qmm.fits(small_m_qmm.QuantizedLinear(qw))
    for dt in (torch.float16, torch.float32):
        q2 = quant.QWeight(qw.wq, qw.scales.to(dt), qw.biases.to(dt), 4)
        mod = small_m_qmm.QuantizedLinear(q2)
        assert not skinny_qmm.fits(mod) and not small_m_qmm.eligible(mod)
        with pytest.raises(DSparkUnsupported, match="scales"):
            skinny_qmm.qmm(torch.zeros(2, 512, dtype=torch.bfloat16), q2.wq, q2.scales,
                           q2.biases, 4)


# ----------------------------------------------------------------- wide-M surface (wide_gemm)

def test_wide_matmul_patch_scope_restore_and_nesting():
    """Mirrors tests/test_wide_gemm.py: disabled is a no-op, the patch applies and restores
    (also on an exception), nesting is a no-op, the row floor is kept."""
    from mlx_dspark_b200 import wide_gemm as wg

    orig = wg.QuantizedLinear.__call__
    with wg.wide_matmul(None):
        assert not wg.active()
    with wg.wide_matmul(0):
        assert not wg.active()
    with wg.wide_matmul(8):
        assert wg.active() and wg._min_rows == wg.SAFE_MIN_ROWS
        with wg.wide_matmul(512):
            assert wg._min_rows == wg.SAFE_MIN_ROWS  # nested: the outer setting stands
    assert wg.QuantizedLinear.__call__ is orig and not wg.active()
    with pytest.raises(RuntimeError), wg.wide_matmul(64):
        raise RuntimeError("boom")
    assert not wg.active() and wg.QuantizedLinear.__call__ is orig
    with pytest.raises(Exception, match="cpu_split"), wg.wide_matmul(64, cpu_split={"fracs": {1: 0.3}}):
        pass


def test_wide_eligibility():
    from mlx_dspark_b200 import quant, small_m_qmm, wide_gemm as wg

    def mod(k, bits=4, sdt=torch.bfloat16):
        qw = quant.QWeight(torch.zeros(128, k * bits // 32, dtype=torch.int32),
                           torch.ones(128, k // 64, dtype=sdt), torch.zeros(128, k // 64, dtype=sdt),
                           bits)
        return small_m_qmm.QuantizedLinear(qw)

    assert wg._eligible(mod(4096)) and wg._eligible(mod(1536, 8))
    assert not wg._eligible(mod(576))                     # K % 512 != 0
    assert not wg._eligible(mod(4096, sdt=torch.float16))  # bf16 scales only
    assert wg.shape_key(mod(4096)) == "4096x128x4"
    assert wg.widest_quantized_linear([mod(1024), mod(4096)])["weight"].shape[1] == 512
