"""ctypes binding of libdcinfer.so (the C ABI declared in include/dcinfer.h).

The shared library is built in-tree by ``make -C daisychain-infer_b200/csrc``.
There is no CPU fallback: if the library is missing, importing the package's
device entry points raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdcinfer.so")

DC_OK, DC_E_ACCBOUND, DC_E_NONFINITE, DC_E_INVAL, DC_E_NOMEM, DC_E_CUDA, DC_E_TIMEOUT, DC_E_LUT, DC_E_GATE = range(9)
DC_RELU, DC_ACC, DC_REQUANT = 1, 2, 4
MAX_INT32_K = 131071

_lib = None


class NonFiniteError(ValueError):
    """A non-finite value reached a quantiser (verified_core.js:16-27)."""


class AccumulatorBoundError(ValueError):
    """A contraction longer than 131071 could wrap int32 (verified_core.js:41-49)."""


class DeviceError(RuntimeError):
    """Any other library failure (CUDA error, gate or LUT failure, timeout)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def raise_for(code: int, msg: str) -> None:
    if code == DC_OK:
        return
    if code == DC_E_NONFINITE:
        raise NonFiniteError(msg)
    if code == DC_E_ACCBOUND:
        raise AccumulatorBoundError(msg)
    raise DeviceError(code, msg)


# (name, restype, argtypes) of every exported entry point.
_p, _i, _u, _f, _d = C.c_void_p, C.c_int, C.c_uint, C.c_float, C.c_double
_i64, _u32, _u64 = C.c_int64, C.c_uint32, C.c_uint64
SIGNATURES = [
    ("dc_init", _i, [_i, C.POINTER(_p)]),
    ("dc_destroy", None, [_p]),
    ("dc_backend_label", C.c_char_p, [_p]),
    ("dc_last_error", C.c_char_p, [_p]),
    ("dc_init_error", C.c_char_p, []),
    ("dc_stream", _p, [_p]),
    ("dc_set_stream", _i, [_p, _p]),
    ("dc_tc_enabled", _i, [_p]),
    ("dc_launch_count", C.c_ulonglong, []),
    ("dc_timing", _i, [_p, _i]),
    ("dc_timing_read", _i, [_p, _i, C.POINTER(_d), C.POINTER(C.c_longlong), C.POINTER(_d), C.POINTER(_d)]),
    ("dc_luts", _i, [_p, _p, _p, _p]),
    ("dc_sync", _i, [_p]),
    ("dc_bgemm", _i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _u, _p]),
    ("dc_bgemm_dev", _i, [_p, _p, _i, _p, _i, _p, _p, _i, _i, _i, _i, _u, _p]),
    ("dc_bgemm_dev_kind", _i, [_p, _p, _i, _p, _i, _p, _p, _i, _i, _i, _i, _u, _p, _i]),
    ("dc_bgemm_dev_noalloc", _i, [_p, _p, _i, _p, _i, _p, _p, _i, _i, _i, _i, _u, _p]),
    ("dc_bgemm_lut_dev", _i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _u, _p]),
    ("dc_quantize_rows", _i, [_p, _p, _i, _i, _p, _i, _p]),
    ("dc_quantize_cols_t", _i, [_p, _p, _i, _i, _p, _i, _p]),
    ("dc_weight_register", _i, [_p, _p, _i, _i, C.POINTER(_p)]),
    ("dc_weight_free", None, [_p]),
    ("dc_weight_info", _i, [_p, C.POINTER(_p), C.POINTER(_i), C.POINTER(_p), C.POINTER(_i), C.POINTER(_i)]),
    ("dc_vgemm", _i, [_p, _p, _i, _p, _u, _p]),
    ("dc_ordered_sum_dev", _i, [_p, _p, _i, _i, _p]),
    ("dc_exp_dev", _i, [_p, _p, _i, _p, _i]),
    ("dc_rmsnorm_dev", _i, [_p, _p, _i, _i, _p, _d, _p, _i]),
    ("dc_l2_prefetch", _i, [_p, _p, C.c_size_t]),
    ("dc_kernel_probe", _i, [_p, C.POINTER(_u32)]),
    ("dc_fnv1a", _u32, [_p, C.c_size_t]),
    ("dc_stage_create", _i, [_p, _p, _i, _i, _i, _i, _i, C.POINTER(_p)]),
    ("dc_stage_free", None, [_p]),
    ("dc_stage_set_layer", _i, [_p, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    ("dc_stage_set_head", _i, [_p, _p, _p, _p]),
    ("dc_stage_synth", _i, [_p, _u64, _d]),
    ("dc_stage_embed", _i, [_p, _p, _i, _p]),
    ("dc_stage_forward", _i, [_p, _p, _i, _i, _i]),
    ("dc_stage_forward_chunks", _i, [_p, _p, _i, _i, _p, _i]),
    ("dc_stage_set_row_graph", _i, [_p, _i]),
    ("dc_stage_handoff", _i, [_p, _p, _p, _p, _i]),
    ("dc_stage_set_timeline", _i, [_p, _p, _i, _i]),
    ("dc_stage_timeline_info", _i, [_p, _p, _p, _i]),
    ("dc_stage_set_row_fusion", _i, [_p, _i]),
    ("dc_stage_set_pass_attention", _i, [_p, _i]),
    ("dc_stage_logits", _i, [_p, _p, _i, _p, _i, _p, _p]),
    ("dc_decode_run", _i, [C.POINTER(_p), _i, _p, _i, _p, _i]),
    ("dc_stage_kv_reset", _i, [_p]),
    ("dc_stage_kv_len", _i, [_p]),
    ("dc_stage_kv_read", _i, [_p, _i, _p, _p, _p]),
]


class DcSpec(C.Structure):
    """dc_spec of include/dcinfer.h."""
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("vocab", C.c_int), ("norm_eps", C.c_double),
                ("rope_theta", C.c_double), ("tie", C.c_int)]


def load(path: str | None = None):
    """Load libdcinfer.so and declare every entry point.  Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is not built: run `make -C daisychain-infer_b200/csrc` "
                           "(the CUDA library is the only implementation; there is no CPU fallback)")
    L = C.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L
