"""ctypes binding of libdspark.so (the C ABI in include/dspark.h).

The library is loaded from this package directory; when it is missing or fails to load the
import raises — there is no fallback path. Every C entry point returns a status code; a
non-zero status raises :class:`DSparkError` carrying ``dspark_last_error()``.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("DSPARK_LIB", HERE / "libdspark.so"))

OK, ERR_ARG, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_NOT_INIT = range(6)
_NAMES = {1: "invalid argument", 2: "unsupported", 3: "CUDA error", 4: "timeout",
          5: "not initialised"}


class DSparkError(RuntimeError):
    """A dspark C-ABI call returned a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"dspark: {_NAMES.get(code, code)}: {msg}")
        self.code = code


class DSparkUnsupported(DSparkError, ValueError):
    """Shape / format the kernels do not serve (status DSPARK_ERR_UNSUPPORTED)."""


vp, i32, i64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t
P_i64 = C.POINTER(C.c_int64)
P_i32 = C.POINTER(C.c_int32)
P_int = C.POINTER(C.c_int)


class QWeight(C.Structure):
    _fields_ = [("wq", vp), ("scales", vp), ("biases", vp), ("N", i32), ("K", i32), ("bits", i32)]


class Layer(C.Structure):
    _fields_ = [("qkv", QWeight), ("o", QWeight), ("gate_up", QWeight), ("down", QWeight),
                ("in_norm", vp), ("post_norm", vp), ("q_norm", vp), ("k_norm", vp),
                ("k_cache", vp), ("v_cache", vp)]


class Model(C.Structure):
    _fields_ = [("n_layers", i32), ("hidden", i32), ("n_heads", i32), ("n_kv_heads", i32),
                ("head_dim", i32), ("intermediate", i32), ("vocab", i32),
                ("rms_eps", f32), ("rope_theta", f32),
                ("embed", QWeight), ("lm_head", QWeight), ("final_norm", vp),
                ("layers", C.POINTER(Layer)),
                ("k_sh", i64), ("k_ss", i64), ("v_sh", i64), ("v_ss", i64), ("kv_cap", i32)]


class FwdBuffers(C.Structure):
    _fields_ = [("h", vp), ("xq", vp), ("attn", vp), ("act", vp), ("ssq_a", vp), ("ssq_b", vp),
                ("inv_freq", vp), ("row_pos", vp), ("row_kv", vp), ("kv_len", vp),
                ("row_start", vp), ("q_len", vp), ("kv_off", vp), ("attn_ws", vp),
                ("attn_ws_bytes", sz), ("rows_cap", i32), ("wide_ws", vp), ("wide_ws_bytes", sz)]


IPC_HANDLE_BYTES = 64


class P2PGatherArgs(C.Structure):
    """``dspark_p2p_gather_args`` (include/dspark.h)."""
    _fields_ = [("arenas", C.POINTER(vp)), ("src", vp), ("seg_bytes", sz), ("flags_off", sz),
                ("count_off", sz), ("dst_off", sz), ("rank", i32), ("world", i32), ("buf", i32)]


class QmmArgs(C.Structure):
    _fields_ = [("x", vp), ("ldx", i64), ("x_seg", i64), ("x_seg_stride", i64),
                ("M", i32), ("K", i32), ("N", i32), ("bits", i32),
                ("wq", vp), ("scales", vp), ("biases", vp), ("out", vp), ("ldo", i64),
                ("epilogue", i32), ("bias", vp), ("norm_w", vp), ("ssq_in", vp),
                ("ssq_n", i32), ("ssq_stride", i32), ("eps", f32),
                ("resid", vp), ("ldr", i64), ("ssq_out", vp), ("n_act", i32),
                ("hq", i32), ("hk", i32), ("q_norm", vp), ("k_norm", vp), ("inv_freq", vp),
                ("q_out", vp), ("ldq", i64), ("k_cache", vp), ("v_cache", vp),
                ("k_sh", i64), ("k_ss", i64), ("v_sh", i64), ("v_ss", i64), ("kv_cap", i32),
                ("row_pos", vp), ("row_kv", vp), ("ssq_seg", i32), ("ssq_seg_stride", i64),
                ("peer_world", i32), ("peer_delta", i64 * 8), ("peer_flag", vp),
                ("wait_flag", vp), ("wait_world", i32), ("wait_elems", C.c_uint32),
                ("wait_state", vp)]


class QKV(C.Structure):
    """``dspark_qkv`` (include/dspark.h): a quantized K/V cache."""
    _fields_ = [("kq", vp), ("ks", vp), ("kb", vp), ("vq", vp), ("vs", vp), ("vb", vp),
                ("q_strides", i64 * 3), ("s_strides", i64 * 3), ("bits", i32)]


EPI_PLAIN, EPI_RESID, EPI_SWIGLU, EPI_QKROPE = range(4)

_SIGS = {
    "dspark_qmm_fused": (i32, [C.POINTER(QmmArgs), vp]),
    "dspark_ipc_alloc": (i32, [sz, C.POINTER(vp), vp]),
    "dspark_ipc_open": (i32, [vp, C.POINTER(vp)]),
    "dspark_ipc_close": (i32, [vp]),
    "dspark_ipc_free": (i32, [vp]),
    "dspark_p2p_allgather": (i32, [C.POINTER(P2PGatherArgs), vp]),
    "dspark_rope_inv_freq": (i32, [vp, i32, f32, vp]),
    "dspark_qmm_wide": (i32, [vp, i64, i32, i32, vp, vp, vp, i32, i32, vp, i64, vp]),
    "dspark_qmm_wide_workspace": (sz, [i32, i32, i32, i32, i32]),
    "dspark_version": (i32, []),
    "dspark_last_error": (C.c_char_p, []),
    "dspark_init": (i32, [i32]),
    "dspark_device_status": (i32, [i32, P_int, i32]),
    "dspark_set_wait_limit_ns": (i32, [i32, C.c_uint64]),
    "dspark_sm_count": (i32, [i32]),
    "dspark_launch_count": (C.c_longlong, []),
    "dspark_qmm": (i32, [vp, i32, i32, vp, vp, vp, i32, i32, i32, vp, vp]),
    "dspark_qmm_ex": (i32, [vp, i64, i32, i32, vp, vp, vp, vp, i32, i32, i32, vp, i64, vp]),
    "dspark_qmm_plan": (i32, [i32, i32, i32, P_int, P_int, P_int, P_int]),
    "dspark_qmm_plan_rows": (i32, [i32, i32, i32, i32, P_int]),
    "dspark_verify_attn": (i32, [vp, P_i64, vp, P_i64, vp, P_i64, i32, i32, i32, i32, i32, i32,
                                 vp, f32, i32, vp, vp, P_i64, vp, sz, vp]),
    "dspark_verify_attn_dt": (i32, [i32, vp, P_i64, vp, P_i64, vp, P_i64, i32, i32, i32, i32,
                                    i32, i32, vp, f32, i32, vp, vp, P_i64, vp, sz, vp]),
    "dspark_verify_attn_noalloc": (i32, [vp, P_i64, vp, P_i64, vp, P_i64, i32, i32, i32, i32, i32,
                                         i32, vp, f32, i32, vp, vp, P_i64, vp]),
    "dspark_verify_attn_workspace": (sz, [i32, i32, i32, i32, i32, i32]),
    "dspark_verify_attn_plan": (i32, [i32, i32, i32, i32, i32, i32, P_int]),
    "dspark_verify_attn_ragged": (i32, [vp, i64, i64, vp, i64, i64, vp, i64, i64, vp, vp, vp, vp,
                                        i32, i32, i32, i32, i32, i32, f32, vp, i64, i64, vp, sz,
                                        vp]),
    "dspark_kv_append": (i32, [vp, P_i64, vp, P_i64, vp, P_i64, vp, P_i64, vp, i32, i32, i32, i32,
                               i32, i32, vp]),
    "dspark_kv_rollback": (i32, [vp, vp, i32, vp]),
    "dspark_kv_append_q": (i32, [vp, P_i64, vp, P_i64, C.POINTER(QKV), vp, i32, i32, i32, i32,
                                 i32, vp]),
    "dspark_verify_attn_q": (i32, [vp, P_i64, C.POINTER(QKV), i32, i32, i32, i32, i32, i32, vp,
                                   f32, i32, vp, P_i64, vp, sz, vp]),
    "dspark_kv_move_row": (i32, [vp, P_i64, vp, P_i64, vp, i32, i32, i32, i32, i32, i32, vp]),
    "dspark_argmax": (i32, [vp, i64, i32, i32, vp, vp]),
    "dspark_accept": (i32, [vp, vp, vp, i32, vp, vp, vp, vp]),
    "dspark_pack_ragged": (i32, [vp, vp, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]),
    "dspark_batch_mask": (i32, [vp, i32, i32, i32, vp, vp]),
    "dspark_embed": (i32, [vp, i32, vp, vp, vp, i32, i32, i32, vp, vp, vp]),
    "dspark_rmsnorm": (i32, [vp, i64, i32, i32, vp, f32, vp, i64, vp]),
    "dspark_verify_forward": (i32, [C.POINTER(Model), C.POINTER(FwdBuffers), vp, i32, i32, i32,
                                    i32, vp, i64, vp]),
    "dspark_verify_prepare": (i32, [vp, i32, C.POINTER(FwdBuffers), vp]),
}

EXPORTED = tuple(_SIGS)


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"dspark: {LIB_PATH} is missing — build it with `python mlx-dspark_b200/build.py` "
            "(there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    return (lib.dspark_last_error() or b"").decode(errors="replace")


def check(rc: int) -> None:
    if rc != OK:
        msg = last_error()
        if rc == ERR_UNSUPPORTED:
            raise DSparkUnsupported(rc, msg)
        raise DSparkError(rc, msg)


def i64_array(vals) -> C.Array:
    return (C.c_int64 * len(vals))(*[int(v) for v in vals])


_inited: set[int] = set()


def ensure_init(device: int) -> None:
    """dspark_init once per device (allocates the device status word)."""
    if device not in _inited:
        check(lib.dspark_init(device))
        _inited.add(device)


def set_wait_limit_ns(device: int, ns: int) -> None:
    """Bound of every kernel wait on ``device`` (0 restores the built-in 2 s)."""
    check(lib.dspark_set_wait_limit_ns(device, int(ns)))


def device_status(device: int = 0, clear: bool = True) -> int:
    code = C.c_int(0)
    check(lib.dspark_device_status(device, C.byref(code), int(clear)))
    return code.value
