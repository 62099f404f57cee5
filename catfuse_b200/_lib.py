"""ctypes binding of ``libcatfuse_sm100.so`` (the C ABI in include/catfuse_b200.h).

The library is loaded lazily on first use.  There is no fallback: if the
shared object is missing or no sm_100 device is current, every kernel call
raises :class:`CatfuseNativeError`.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libcatfuse_sm100.so"

CF_OK = 0
CF_ERR_INVALID_ARG = -1
CF_ERR_UNSUPPORTED = -2
CF_ERR_CUDA = -3
CF_ERR_NO_DEVICE = -4
CF_ERR_DEVICE_TIMEOUT = -5

FMT_F32, FMT_F16, FMT_U8, FMT_BITS = 0, 1, 2, 3
RES_NONE, RES_ADD_POST, RES_AND_POST, RES_IAND_POST, RES_ADD_PRE, RES_Z_ONLY = 0, 1, 2, 3, 4, 5

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float
_INT = ctypes.c_int

# name -> (restype, argtypes); must match include/catfuse_b200.h exactly.
SIGNATURES = {
    "cf_version": (ctypes.c_char_p, []),
    "cf_get_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "cf_device_supported": (_INT, []),
    "cf_check_device_error": (_INT, [_P, ctypes.POINTER(_I32)]),
    "cf_lif_fwd": (_INT, [_P, _INT, _P, _P, _INT, _P, _I64, _I64, _F, _F, _F, _INT, _INT, _P]),
    "cf_bn_lif": (_INT, [_P, _INT, _P, _P, _P, _INT, _P, _P, _INT, _P, _I64, _I64, _I64, _I64,
                         _F, _F, _F, _INT, _INT, _P]),
    "cf_add_lif": (_INT, [_P, _P, _P, _P, _INT, _P, _I64, _I64, _F, _F, _F, _INT, _INT, _P]),
    "cf_avgpool_lif": (_INT, [_P, _P, _P, _INT, _P, _I64, _I64, _I64, _I64, _I64, _INT, _F, _F,
                              _F, _INT, _INT, _P]),
    "cf_pack_tbchw": (_INT, [_P, _INT, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "cf_pack_im2col": (_INT, [_P, _INT, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "cf_unpack_bhwtc": (_INT, [_P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _P]),
    "cf_v_layout": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _INT, _P]),
    "cf_pack_conv_weight": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "cf_ssa_lif": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _F, _F, _F,
                          _INT, _INT, _P]),
    "cf_conv_geometry": (_INT, [_I64, _I64, _I64, _I64, _I64, ctypes.POINTER(_I32)]),
    "cf_conv_geometry_ex": (_INT, [_I64, _I64, _I64, _I64, _I64, _I64, _I64, _INT,
                                   ctypes.POINTER(_I32)]),
    "cf_conv_bn_lif": (_INT, [_P, _P, _P, _P, _P, _INT, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                              _I64, _I64, _I64, _I64, _I64, _I64, _F, _F, _F, _INT, _INT, _P]),
    "cf_linear_bn_lif": (_INT, [_P, _P, _P, _P, _P, _INT, _P, _P, _P, _I64, _I64, _I64, _I64,
                                _I64, _F, _F, _F, _INT, _INT, _P]),
    "cf_prescan": (_INT, [_P, _INT, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                          _I64, _I64, _I64, _I64, _F, _P]),
    "cf_prescan_conv_tiles": (_INT, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                     _I64, _I64, _I64, _P]),
    "cf_conv_chunk": (_INT, [_I64, _INT]),
    "cf_maxpool_bhwtc": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "cf_conv_bn_lif_split": (_INT, [_P, _P, _P, _P, _P, _INT, _P, _P, _P, _P, _I64, _I64, _I64,
                                    _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F, _F, _F, _INT,
                                    _INT, _P]),
    "cf_pack_conv_weight_split": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P]),
    "cf_pack_im2col_split": (_INT, [_P, _INT, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                    _I64, _P]),
    "cf_conv_bn_lif_dual": (_INT, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                   _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F, _F, _F, _INT,
                                   _INT, _P]),
    "cf_conv_bn_lif_egd": (_INT, [_P, _P, _P, _P, _P, _INT, _P, _P, _P, _P, _I64, _I64, _I64,
                                  _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F, _F, _F, _INT,
                                  _INT, _F, _P]),
    "cf_conv_bn_lif_egd_noalloc": (_INT, [_P, _P, _P, _P, _P, _INT, _P, _P, _P, _I64, _I64,
                                          _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F,
                                          _F, _F, _INT, _INT, _F, _P]),
    "cf_conv_bn_lif_planes": (_INT, [_P, _P, _P, _P, _P, _INT, _P, _P, _P, _I64, _I64, _I64,
                                     _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F, _F, _F, _INT,
                                     _INT, _P]),
    "cf_pack_conv_weight_planes": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P]),
    "cf_token_mean_lif_fc": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _F,
                                    _F, _INT, _INT, _P]),
    "cf_set_wait_limit": (_INT, [ctypes.c_uint32]),
    "cf_test_arm_stalled_load": (_INT, [_INT]),
    "cf_avgpool_fc": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
}


class CatfuseNativeError(RuntimeError):
    """Raised when the sm_100a library is missing or a kernel call fails."""

    def __init__(self, msg: str, code: int = CF_ERR_CUDA):
        super().__init__(msg)
        self.code = code


_lib = None
_lock = threading.Lock()


def load(path: Path | None = None):
    """Load (once) and return the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise CatfuseNativeError(
                f"{p.name} not found at {p}; build it with `python -m catfuse_b200.build` "
                "(there is no CPU fallback)", CF_ERR_NO_DEVICE)
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return _lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.cf_get_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != CF_OK:
        raise CatfuseNativeError(f"{what}: {last_error()} (code {rc})", rc)


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise on failure."""
    fn = getattr(load(), name)
    check(fn(*args), name)
