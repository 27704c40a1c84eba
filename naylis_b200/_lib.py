"""ctypes binding of ``libnaylis_mom.so`` (the C ABI in include/naylis_mom.h).

The library is built in-tree by ``naylis_b200.build``; this module never falls
back to anything when it is missing — every op raises with the reason.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnaylis_mom.so")

# status codes (mom_status)
OK = 0
STATUS_NAMES = {
    0: "MOM_OK", 1: "MOM_ERR_INVALID_ARGUMENT", 2: "MOM_ERR_UNSUPPORTED", 3: "MOM_ERR_ARCH",
    4: "MOM_ERR_WORKSPACE", 5: "MOM_ERR_LAUNCH", 6: "MOM_ERR_DEVICE_TIMEOUT", 7: "MOM_ERR_DEVICE_INDEX",
}
# dtypes (mom_dtype) and scan modes (mom_scan_mode)
F32, BF16, I32, I64 = 0, 1, 2, 3
SCAN_MODES = {"fp64": 0, "fp32": 1}

_c = ctypes
_vp, _i64, _int, _sz, _fp = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_size_t, _c.c_void_p

# name -> (restype, argtypes); must match include/naylis_mom.h
SIGNATURES = {
    "mom_version": (_int, []),
    "mom_kernel_launches": (_c.c_uint64, []),
    "mom_last_error_string": (_c.c_char_p, []),
    "mom_device_check": (_int, [_int]),
    "mom_prefix_mean": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _int, _int, _vp]),
    "mom_route_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _int]),
    "mom_route_fwd": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _int, _i64, _i64, _i64, _fp,
                             _int, _fp, _vp, _int, _fp, _fp, _vp, _vp, _sz, _vp]),
    "mom_route_shard_stats": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp]),
    "mom_route_shard_carry": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
    "mom_route_fwd_shard": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _int, _i64, _i64, _i64, _fp,
                                   _int, _i64, _vp, _vp, _fp, _vp, _int, _fp, _fp, _vp, _vp, _sz, _vp]),
    "mom_route_bwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "mom_route_bwd": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _int, _i64, _i64, _i64, _fp,
                             _vp, _int, _fp, _vp, _fp, _fp, _fp, _vp, _int, _int, _fp, _fp, _vp,
                             _sz, _vp]),
    "mom_plan_size": (_sz, [_i64, _i64, _i64]),
    "mom_bucket": (_int, [_vp, _int, _fp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "mom_plan_check": (_int, [_vp, _i64, _i64, _i64, _vp]),
    "mom_scale_fwd": (_int, [_vp, _int, _i64, _fp, _fp, _vp]),
    "mom_scale_bwd": (_int, [_vp, _int, _vp, _int, _i64, _fp, _vp, _fp, _vp]),
    "mom_gumbel": (_int, [_fp, _i64, _c.c_float, _fp, _vp]),
    "mom_kv_pack_bf16": (_int, [_fp, _fp, _i64, _i64, _vp, _vp]),
    "mom_read_fwd": (_int, [_vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                            _vp, _fp, _vp, _vp]),
    "mom_read_bwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "mom_read_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _fp, _int, _i64, _i64, _i64, _i64, _i64,
                            _i64, _i64, _vp, _vp, _vp, _fp, _fp, _fp, _vp, _sz, _vp]),
    "mom_plan_split_size": (_sz, [_i64, _i64, _i64]),
    "mom_bucket_split": (_int, [_vp, _int, _fp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "mom_read_split_fwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "mom_read_split_fwd": (_int, [_vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                                  _int, _vp, _vp, _fp, _fp, _vp, _vp, _sz, _vp]),
    "mom_read_split_bwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "mom_read_split_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _fp, _fp, _int, _i64, _i64, _i64, _i64, _i64,
                                  _i64, _i64, _vp, _int, _vp, _vp, _vp, _fp, _fp, _fp, _vp, _sz, _vp]),
    "mom_read_f32_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "mom_read_f32_fwd": (_int, [_fp, _fp, _fp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _int, _vp, _fp,
                                _fp, _vp, _sz, _vp]),
    "mom_read_f32_bwd": (_int, [_fp, _fp, _fp, _fp, _fp, _fp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                                _int, _vp, _fp, _fp, _fp, _fp, _vp, _sz, _vp]),
    "mom_rope_qkv_fwd": (_int, [_vp, _fp, _fp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "mom_rope_qkv_bwd": (_int, [_vp, _vp, _vp, _fp, _fp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "mom_swiglu_fwd": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "mom_swiglu_bwd": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "mom_add_rmsnorm_fwd": (_int, [_fp, _vp, _int, _fp, _fp, _i64, _i64, _c.c_double, _fp, _vp, _fp, _fp, _vp]),
    "mom_add_rmsnorm_bwd": (_int, [_fp, _fp, _fp, _vp, _int, _fp, _vp, _fp, _fp, _i64, _i64, _fp, _vp, _fp, _fp,
                                   _vp]),
    "mom_router_aux_workspace_size": (_sz, [_i64, _i64]),
    "mom_router_aux": (_int, [_fp, _vp, _int, _i64, _i64, _i64, _vp, _sz, _fp, _vp]),
    "mom_adamw_step": (_int, [_vp, _i64, _vp, _i64, _c.c_double, _c.c_double, _c.c_double, _c.c_double, _c.c_double,
                              _i64, _vp]),
    "mom_xent_fwd": (_int, [_vp, _vp, _i64, _i64, _i64, _fp, _fp, _vp]),
    "mom_xent_bwd": (_int, [_vp, _vp, _fp, _fp, _i64, _i64, _i64, _vp, _vp]),
    "mom_read_bwd_noalloc_max_bytes": (_sz, []),
    "mom_read_bwd_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _fp, _int, _i64, _i64, _i64, _i64, _i64,
                                    _i64, _i64, _vp, _vp, _vp, _fp, _fp, _fp, _vp]),
}

_lock = threading.Lock()
_lib = None


class MomError(RuntimeError):
    """A C-ABI call returned a non-zero mom_status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        super().__init__(f"{func} -> {STATUS_NAMES.get(status, status)}: {message}")


def load(path: str = LIB_PATH):
    """Load (once) and return the ctypes handle of libnaylis_mom.so."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"naylis_b200: {path} is not built. Run `python -m naylis_b200.build` "
                "(nvcc, sm_100a) — the MoM kernels have no fallback.")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return load().mom_last_error_string().decode(errors="replace")


def check(status: int, func: str) -> None:
    if status != OK:
        raise MomError(status, func, last_error())


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise MomError on failure."""
    check(getattr(load(), name)(*args), name)
