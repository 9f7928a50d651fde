"""ctypes binding of the C ABI in ``include/treeattn_b200.h``.

The library is loaded from ``treeattn_b200/lib/libtreeattn_b200.so`` (built in-tree by
``treeattn_b200.build``). There is no fallback: if the library is missing or fails to load,
every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

TA_OK = 0
TA_ERR_INVALID = 1
TA_ERR_UNSUPPORTED = 2
TA_ERR_CUDA = 3
TA_ERR_WORKSPACE = 4

TA_F32 = 0
TA_F16 = 1
TA_BF16 = 2
TA_LAYOUT_REFERENCE = 0
TA_LAYOUT_TREE = 1


class Layout(ctypes.Structure):
    _fields_ = [("seq", ctypes.c_int64), ("batch", ctypes.c_int64), ("head", ctypes.c_int64)]


class Shard(ctypes.Structure):
    _fields_ = [("row_total", ctypes.c_int64), ("row0", ctypes.c_int64), ("row_count", ctypes.c_int64),
                ("batch_total", ctypes.c_int64), ("batch0", ctypes.c_int64),
                ("batch_count", ctypes.c_int64), ("head_total", ctypes.c_int64),
                ("head0", ctypes.c_int64), ("head_count", ctypes.c_int64)]


class Blocked(ctypes.Structure):
    _fields_ = [("fanout", ctypes.c_int32), ("leaf_block", ctypes.c_int32),
                ("causal", ctypes.c_int32), ("softmax_scale", ctypes.c_float),
                ("row0", ctypes.c_int64), ("row_total", ctypes.c_int64),
                ("batch0", ctypes.c_int64), ("batch_total", ctypes.c_int64),
                ("head0", ctypes.c_int64), ("head_total", ctypes.c_int64)]


class Shape(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64),
        ("num_queries", ctypes.c_int64),
        ("num_leaves", ctypes.c_int64),
        ("num_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("num_samples", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
        ("max_logit", ctypes.c_float),
    ]


class Rng(ctypes.Structure):
    _fields_ = [
        ("seed", ctypes.c_uint64),
        ("offset", ctypes.c_uint64),
        ("offset_step", ctypes.c_uint64),
        ("draw_stride", ctypes.c_int64),
    ]


class TreeAttnError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


# every symbol the header declares: (name, restype, argtypes)
_P = ctypes.c_void_p
_L = Layout
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t
SIGNATURES = {
    "ta_last_error": (ctypes.c_char_p, []),
    "ta_abi_version": (_I32, []),
    "ta_device_rng_geometry": (ctypes.c_int, [_I32, ctypes.POINTER(_I32), ctypes.POINTER(_I32)]),
    "ta_profile_enable": (ctypes.c_int, [_I32]),
    "ta_profile_collect": (_I64, [ctypes.c_char_p, _SZ]),
    "ta_philox_plan": (ctypes.c_int, [_I64, _I32, _I32, ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(_I64)]),
    "ta_gumbel_fill": (ctypes.c_int, [_P, _I64, ctypes.POINTER(Rng), _I32, _I32, _P]),
    "ta_branch_prob_stride": (_I32, [_I64]),
    "ta_gumbel_fill_shard": (ctypes.c_int, [_P, ctypes.POINTER(Rng), ctypes.POINTER(Shard), _I64,
                                            _I32, _I32, _P]),
    "ta_blocked_summary_rows": (ctypes.c_int64, [_I64, _I32, _I32]),
    "ta_blocked_build": (ctypes.c_int, [ctypes.POINTER(Shape), ctypes.POINTER(Blocked), _P, _L, _P, _P]),
    "ta_blocked_gumbel_fill": (ctypes.c_int, [ctypes.POINTER(Shape), ctypes.POINTER(Blocked),
                                              ctypes.POINTER(Rng), _P, _P]),
    "ta_blocked_set_tcgen05": (_I32, [_I32]),
    "ta_blocked_set_tcgen05_backward": (_I32, [_I32]),
    "ta_blocked_status": (_I32, [_I32]),
    "ta_blocked_set_tc_wait_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "ta_backward_set_node_range": (_I32, [_I32]),
    "ta_forward_set_tensor_dots": (_I32, [_I32]),
    "ta_blocked_uses_tensor_cores": (_I32, [ctypes.POINTER(Shape), ctypes.POINTER(Blocked), _I32]),
    "ta_blocked_forward_workspace_size": (_SZ, [ctypes.POINTER(Shape), ctypes.POINTER(Blocked)]),
    "ta_blocked_forward": (ctypes.c_int, [ctypes.POINTER(Shape), ctypes.POINTER(Blocked), _P, _L, _P, _L,
                                          _P, _L, _P, _P, _L, ctypes.POINTER(Rng), _P, _P, _P, _P, _P,
                                          _SZ, _P]),
    "ta_blocked_backward_workspace_size": (_SZ, [ctypes.POINTER(Shape), ctypes.POINTER(Blocked)]),
    "ta_blocked_backward": (ctypes.c_int, [ctypes.POINTER(Shape), ctypes.POINTER(Blocked), _P, _L, _P, _L,
                                           _P, _L, _P, _P, _L, _P, _P, _P, _P, _L, _P, _L, _P, _L,
                                           _P, _SZ, _P]),
    "ta_tree_build_workspace_size": (_SZ, [_I64, _I64, _I64, _I64, _I32]),
    "ta_tree_build": (ctypes.c_int, [_I32, _I64, _I64, _I64, _I64, _P, _L, _P, _L, _P, _SZ, _P]),
    "ta_tree_build_noalloc": (ctypes.c_int, [_I32, _I64, _I64, _I64, _I64, _P, _L, _P, _L, _P]),
    "ta_tree_build_ex": (ctypes.c_int, [_I32, _I64, _I64, _I64, _I64, _P, _L, _P, _L, _I32, _P, _SZ, _P]),
    "ta_tree_build_backward_ex": (ctypes.c_int, [_I32, _I64, _I64, _I64, _I64, _P, _L, _P, _L, _I32,
                                                 _P, _SZ, _P]),
    "ta_tree_build_backward_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "ta_tree_build_backward": (ctypes.c_int, [_I32, _I64, _I64, _I64, _I64, _P, _L, _P, _L, _P,
                                              _SZ, _P]),
    "ta_forward": (ctypes.c_int, [ctypes.POINTER(Shape), _P, _L, _P, _L, _P, _L, _P, _L,
                                  ctypes.POINTER(Rng), _P, _P, _P, _P, _P, _P]),
    "ta_backward_workspace_size": (_SZ, [ctypes.POINTER(Shape)]),
    "ta_backward": (ctypes.c_int, [ctypes.POINTER(Shape), _P, _L, _P, _L, _P, _L, _P, _L, _P, _P,
                                   _P, _P, _L, _P, _L, _I32, _P, _L, _I32, _P, _SZ, _P]),
    "ta_backward_coef": (ctypes.c_int, [ctypes.POINTER(Shape), _P, _L, _P, _L, _P, _L, _P, _P, _P,
                                        _P, _P, _L, _P, _L, _I32, _P, _L, _I32, _P, _SZ, _P]),
    "ta_causal_forward": (ctypes.c_int, [ctypes.POINTER(Shape), _I64, _P, _L, _P, _L, _P, _L, _P,
                                         _L, ctypes.POINTER(Rng), _P, _P, _P, _P, _P, _P, _P]),
    "ta_causal_coefficients": (ctypes.c_int, [ctypes.POINTER(Shape), _I64, _P, _L, _P, _L, _P, _L,
                                              _P, _L, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "ta_exact_workspace_size": (_SZ, [ctypes.POINTER(Shape)]),
    "ta_exact_forward": (ctypes.c_int, [ctypes.POINTER(Shape), _I32, _I64, _P, _L, _P, _L, _P, _L,
                                        _P, _L, _P, _P, _SZ, _P]),
    "ta_exact_backward": (ctypes.c_int, [ctypes.POINTER(Shape), _I32, _I64, _P, _L, _P, _L, _P, _L,
                                         _P, _L, _P, _L, _P, _L, _P, _L, _I32, _P, _SZ, _P]),
    "ta_sample_paths": (ctypes.c_int, [ctypes.POINTER(Shape), _P, _L, _P, _L,
                                       ctypes.POINTER(Rng), _P, _P, _P, _P, _P]),
    "ta_replay_paths": (ctypes.c_int, [ctypes.POINTER(Shape), _P, _L, _P, _L, _P, _I32, _P, _P,
                                       _P]),
    "ta_weighted_value_sum": (ctypes.c_int, [ctypes.POINTER(Shape), _P, _L, _P, _P, _P, _L, _P]),
}

_lock = threading.Lock()
_lib = None


def library_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if absent and ``build_if_missing``) and return the library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = os.environ.get("TREEATTN_B200_LIB") or _build.LIB
        if os.environ.get("TREEATTN_B200_LIB"):
            build_if_missing = False  # an explicitly chosen library is used as is
        if build_if_missing:
            _build.build()  # no-op when the library matches the sources
        elif not os.path.exists(path):
            raise OSError(f"treeattn_b200 CUDA library not built: {path}")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.ta_abi_version() != 1:
            raise OSError("treeattn_b200: ABI version mismatch")
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise TreeAttnError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != TA_OK:
        msg = lib.ta_last_error().decode(errors="replace")
        if rc == TA_ERR_INVALID:
            raise ValueError(f"{name}: {msg}")
        raise TreeAttnError(name, rc, msg)
