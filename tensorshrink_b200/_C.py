"""ctypes binding of `libtensorshrink_b200.so` (the C ABI in
`include/tensorshrink_b200.h`).

The library is built in-tree by `tensorshrink_b200.build`. Loading fails
loudly when it is missing: there is no CPU or Python fallback for the hot
path.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtensorshrink_b200.so"

TS_F16, TS_BF16, TS_F32 = 0, 1, 2
TS_QMODE_UNIFORM, TS_QMODE_CODEBOOK, TS_QMODE_LLOYD = 0, 1, 2

_STATUS = {
    -1: ValueError,          # TS_ERR_INVALID
    -2: NotImplementedError,  # TS_ERR_UNSUPPORTED
    -3: RuntimeError,        # TS_ERR_CUDA
    -4: RuntimeError,        # TS_ERR_WORKSPACE
    -5: RuntimeError,        # TS_ERR_TIMEOUT
}
TS_ERR_TIMEOUT = -5

_vp = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int32


class TsQWeight(C.Structure):
    """struct ts_qweight."""
    _fields_ = [
        ("rows", _i64), ("cols", _i64), ("padded_cols", _i64), ("n_groups", _i64),
        ("packed_row_bytes", _i64), ("bits", _i32), ("group_size", _i32),
        ("packed", _vp), ("scale", _vp), ("gmin", _vp),
        ("dq_scale_codes", _vp), ("dq_scale_meta", _vp), ("dq_gmin_codes", _vp), ("dq_gmin_meta", _vp),
        ("dq_group_size", _i32), ("reserved0", _i32),
        ("codebook", _vp),
        ("n_outliers", _i64), ("outlier_row_ptr", _vp), ("outlier_row", _vp), ("outlier_col", _vp),
        ("outlier_delta", _vp),
    ]


class TsQuantParams(C.Structure):
    """struct ts_quant_params."""
    _fields_ = [
        ("rows", _i64), ("cols", _i64), ("bits", _i32), ("group_size", _i32),
        ("k_outliers", _i64), ("double_quant", _i32), ("dq_group_size", _i32),
        ("mode", _i32), ("lloyd_iters", _i32), ("codebook", _vp),
        ("lloyd_sample", _vp), ("lloyd_n_sample", _i64),
    ]


class TsQuantOutputs(C.Structure):
    """struct ts_quant_outputs."""
    _fields_ = [
        ("packed", _vp), ("scale", _vp), ("gmin", _vp),
        ("dq_scale_codes", _vp), ("dq_scale_meta", _vp), ("dq_gmin_codes", _vp), ("dq_gmin_meta", _vp),
        ("codebook_out", _vp), ("codebook_f16", _vp),
        ("outlier_idx", _vp), ("outlier_val", _vp), ("outlier_row", _vp), ("outlier_col", _vp),
        ("outlier_delta", _vp), ("outlier_row_ptr", _vp), ("threshold", _vp),
    ]


class TsQlinearOp(C.Structure):
    """struct ts_qlinear_op (one layer of ts_qlinear_ex / ts_qlinear_chain)."""
    _fields_ = [
        ("w", C.POINTER(TsQWeight)), ("x", _vp), ("x_row_stride", _i64), ("x_dtype", _i32), ("flags", _i32),
        ("bias", _vp), ("bias_dtype", _i32), ("out_dtype", _i32), ("out", _vp), ("out_row_stride", _i64),
        ("norm_weight", _vp), ("norm_eps", C.c_float), ("act_dtype", _i32),
        ("residual", _vp), ("residual_row_stride", _i64),
    ]


OP_GATED = 1
OP_RMSNORM = 2

# (name, restype, argtypes)
_SIGNATURES = [
    ("ts_qlinear_workspace_size", C.c_size_t, [C.POINTER(TsQWeight), _i64]),
    ("ts_qlinear", C.c_int, [C.POINTER(TsQWeight), _vp, C.c_int, _i64, _i64, _vp, C.c_int, _vp,
                             C.c_int, _i64, _vp, C.c_size_t, _vp]),
    ("ts_qlinear_gated", C.c_int, [C.POINTER(TsQWeight), _vp, C.c_int, _i64, _i64, _vp, C.c_int, _vp,
                                   C.c_int, _i64, _vp, C.c_size_t, _vp]),
    ("ts_qlinear_ex", C.c_int, [C.POINTER(TsQlinearOp), _i64, _vp, C.c_size_t, _vp]),
    ("ts_qlinear_chain", C.c_int, [C.POINTER(TsQlinearOp), C.c_int, _i64, C.c_int, _vp, C.c_size_t, _vp]),
    ("ts_qlinear_chain_max", C.c_int, []),
    ("ts_qlinear_noalloc_max_scratch", C.c_size_t, []),
    ("ts_qlinear_noalloc", C.c_int, [C.POINTER(TsQWeight), _vp, C.c_int, _i64, _i64, _vp, C.c_int,
                                     _vp, C.c_int, _i64, _vp]),
    ("ts_qlinear_status", C.c_int, [_vp, C.c_size_t, C.c_int, _vp]),
    ("ts_test_inject_stall", C.c_int, [C.c_uint64]),
    ("ts_apply_outlier_correction", C.c_int, [_vp, _i64, _i64, _i64, _vp, C.c_int, _i64, _vp, _vp,
                                              _vp, _i64, _vp]),
    ("ts_outlier_tables_from_stream", C.c_int, [C.POINTER(TsQWeight), _vp, _vp, C.c_int, _vp, _i64, _vp, _vp,
                                                _vp, _vp, _vp, _vp]),
    ("ts_peer_buffer_bytes", C.c_size_t, [C.c_int, _i64]),
    ("ts_peer_alloc", C.c_int, [C.c_int, _i64, C.POINTER(_vp)]),
    ("ts_peer_free", C.c_int, [_vp]),
    ("ts_ipc_get_handle", C.c_int, [_vp, _vp]),
    ("ts_ipc_open", C.c_int, [_vp, C.POINTER(_vp)]),
    ("ts_ipc_close", C.c_int, [_vp]),
    ("ts_allreduce_oneshot", C.c_int, [C.POINTER(C.c_void_p), C.c_int, C.c_int, _i64, _vp, _vp, _vp, _i64, _vp, _vp]),
    ("ts_decode_attention", C.c_int, [_vp, _i64, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp,
                                      _i64, _i64, C.c_int, C.c_int, _vp, _i64, _vp]),
    ("ts_dequantize_weight", C.c_int, [C.POINTER(TsQWeight), _vp, C.c_int, _i64, C.c_int, _vp]),
    ("ts_quantize_workspace_size", C.c_size_t, [C.POINTER(TsQuantParams)]),
    ("ts_quantize_pack", C.c_int, [_vp, C.c_int, C.POINTER(TsQuantParams), C.POINTER(TsQuantOutputs),
                                   _vp, C.c_size_t, _vp]),
    ("ts_lloyd_fit_workspace_size", C.c_size_t, [_i64, C.c_int]),
    ("ts_lloyd_fit", C.c_int, [_vp, _i64, C.c_int, C.c_int, _vp, _vp, C.c_size_t, _vp]),
    ("ts_last_error", C.c_char_p, []),
    ("ts_version", C.c_char_p, []),
    ("ts_launch_count", _i64, [C.c_int]),
]

EXPORTED_SYMBOLS = tuple(name for name, _, _ in _SIGNATURES)

_lib = None
_lock = threading.Lock()


def lib_path() -> Path:
    return _LIB_PATH


def load() -> C.CDLL:
    """Load (once) and return the shared library; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise ImportError(
                    f"{_LIB_PATH} is missing: build it with `python -m tensorshrink_b200.build` "
                    "(tensorshrink_b200 has no CPU fallback for its CUDA kernels)")
            lib = C.CDLL(str(_LIB_PATH))
            for name, res, args in _SIGNATURES:
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Raise the Python exception matching a ts_status code."""
    if rc != 0:
        msg = load().ts_last_error().decode(errors="replace")
        raise _STATUS.get(rc, RuntimeError)(f"{what}: {msg}")


_TORCH_LIB_PATH = _LIB_PATH.parent / "libtensorshrink_torch.so"
_ops = None


def torch_ops():
    """The `torch.ops.tensorshrink` namespace (operators over this library,
    built beside it), loaded once; None when that library was not built."""
    global _ops
    if _ops is None:
        load()
        if not _TORCH_LIB_PATH.exists():
            _ops = False
        else:
            import torch
            torch.ops.load_library(str(_TORCH_LIB_PATH))
            _ops = torch.ops.tensorshrink
    return _ops or None


def launch_count(reset: bool = False) -> int:
    return int(load().ts_launch_count(1 if reset else 0))
