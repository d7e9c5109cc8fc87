"""ctypes binding of ``libsilogic_b200.so`` (the C ABI in ``include/silogic_b200.h``).

The shared library is built in-tree by :mod:`silogic_b200.build`.  There is no
CPU implementation behind these calls: every op requires CUDA tensors and raises
if the library or a GPU is missing.
"""
import ctypes
import os

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
# SILOGIC_B200_LIB points at another build of the same library (e.g. a tuning variant)
LIB_PATH = os.environ.get("SILOGIC_B200_LIB") or os.path.join(_PKG, "libsilogic_b200.so")

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_p = ctypes.c_void_p
_f32 = ctypes.c_float

# name -> argtypes (all return int status)
_SIGS = {
    "slg_version": [],
    "slg_check_index_range": [_p, _i64, _i64, _p, _p],
    "slg_tuning_set": [_i32, _i64],
    "slg_pack_u8": [_p, _i64, _i64, _p, _i64, _p],
    "slg_pack_f32": [_p, _i64, _i64, _p, _i64, _p],
    "slg_unpack_u8": [_p, _i64, _i64, _i64, _p, _p],
    "slg_thermo_pack": [_p, _i64, _i64, _i64, _p, _i64, _i32, _p, _i64, _p],
    "slg_thermo_pack_u8": [_p, _i64, _i64, _i64, _p, _i64, _i32, _p, _i64, _p],
    "slg_fc_hard": [_p, _i64, _i64, _p, _p, _i32, _i64, _i64, _p, _p],
    "slg_conv_hard": [_p, _i64, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _i64, _i64,
                      _i32, _p, _p],
    "slg_groupsum": [_p, _i64, _i64, _i64, _i32, _p, _p],
    "slg_packed_linear": [_p, _i64, _i64, _i64, _p, _p, _i32, _p, _p],
    "slg_fc_chain_encode": [_p, _p, _i64, _i64, _p, _p],
    "slg_fc_chain_plan": [_i64, _i32, _p, _p, _p, _p, _i32, _i32, _p, _i64, _p, _p],
    "slg_fc_chain_counts": [_p, _i64, _i64, _i64, _p, _p, _i32, _i32, _p, _p, _p],
    "slg_fc_soft_fwd": [_p, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _p, _i32, _f32, _i64,
                        _i64, _p, _p],
    "slg_fc_soft_bwd": [_p, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _p, _i32, _f32, _i64,
                        _i64, _p, _p, _p, _p, _p, _i64, _p],
    "slg_conv_soft_bwd_det": [_p, _i64, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _i32, _p,
                              _i32, _f32, _i32, _i32, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p,
                              _i64, _p],
    "slg_to_feature_major": [_p, _i64, _i64, _p, _i64, _p],
    "slg_from_feature_major": [_p, _i64, _i64, _i64, _p, _p],
    "slg_groupsum_soft_fwd": [_p, _i64, _i64, _i64, _i32, _f32, _i32, _p, _p],
    "slg_groupsum_soft_bwd": [_p, _i64, _i64, _i64, _i32, _f32, _p, _p],
    "slg_or_pool_fwd": [_p, _i64, _i64, _i64, _i32, _p, _p],
    "slg_or_pool_bwd": [_p, _p, _i64, _i64, _i64, _i32, _p, _p],
    "slg_thermo_soft_fwd": [_p, _p, _i64, _i64, _i32, _p, _p],
    "slg_thermo_soft_bwd": [_p, _p, _p, _i64, _i64, _i32, _f32, _p, _p, _p],
    "slg_conv_soft_fwd": [_p, _i64, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _i32, _p,
                          _i32, _f32, _i32, _i32, _i64, _i64, _i32, _p, _p, _p],
    "slg_conv_soft_bwd": [_p, _i64, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _i32, _p,
                          _i32, _f32, _i32, _i32, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _i64,
                          _p],
}
# entry points that do not return a status
_RESTYPES = {
    "slg_fc_chain_smem_bytes": ([_i64, _p, _i32], ctypes.c_int64),
    "slg_fc_soft_workspace_bytes": ([_i64, _i32, _i32, _i32, _i64], ctypes.c_int64),
    "slg_conv_soft_workspace_bytes": ([_i64, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                       _i64], ctypes.c_int64),
}

_lib = None


class SilogicError(RuntimeError):
    """A non-zero status returned by the native library."""


def lib():
    """Load (once) and return the native library; raise if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SilogicError(
                f"{LIB_PATH} is missing: build it with `python -m silogic_b200.build` "
                "(silogic_b200 has no CPU implementation)")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        for name, (args, res) in _RESTYPES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        L.slg_last_error.restype = ctypes.c_char_p
        L.slg_last_error.argtypes = []
        _apply_env_tuning(L)
        _lib = L
    return _lib


def _apply_env_tuning(L):
    """SLG_TUNING="key=value,..." sets ``slg_tuning_set`` knobs when the library loads
    (kernel variants; results are identical for every setting)."""
    spec = os.environ.get("SLG_TUNING", "").strip()
    for item in filter(None, (t.strip() for t in spec.split(","))):
        try:
            key, val = (int(v) for v in item.split("="))
        except ValueError:
            raise SilogicError(f"SLG_TUNING: bad item {item!r} (want key=value)") from None
        if L.slg_tuning_set(key, val) != 0:
            raise SilogicError(f"SLG_TUNING: {L.slg_last_error().decode()}")


def declare(name, argtypes):
    """Register the argtypes of an entry point added by another module."""
    _SIGS[name] = argtypes
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int


def call(name, *args):
    """Invoke ``name`` and raise :class:`SilogicError` on a non-zero status."""
    L = lib()
    st = getattr(L, name)(*args)
    if st != 0:
        msg = L.slg_last_error().decode(errors="replace")
        raise SilogicError(f"{name} failed with status {st}: {msg}")


def stream_ptr(device=None):
    """Raw handle of torch's current CUDA stream on ``device``."""
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "silogic_b200 runs only on CUDA tensors (sm_100a kernels, no CPU path); "
                f"got a tensor on {t.device}")
