"""The C-ABI library loads and exports every symbol include/*.h declares;
the Python binding declares exactly those symbols.  No compute calls."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"CF_API\s+[\w\s\*]+?\b(cf_\w+)\s*\(", h.read_text()))
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert {"cf_conv_bn_lif", "cf_lif_fwd", "cf_prescan", "cf_bn_lif"} <= names
    assert len(names) >= 19


def test_library_exports_every_declared_symbol():
    from catfuse_b200 import _lib
    from catfuse_b200.build import build
    build()
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(_declared()) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_lib.SIGNATURES) == _declared()
    handle = _lib.load()
    assert b"sm_100a" in handle.cf_version()


def test_error_path_without_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("host without GPU only")
    from catfuse_b200 import _lib, ops
    lib = _lib.load()
    assert lib.cf_device_supported() == 0
    # a kernel call without a device reports CF_ERR_NO_DEVICE, never computes
    rc = lib.cf_lif_fwd(1, 0, None, 1, 0, None, 1, 4, 2.0, 1.0, 0.0, 1, 1, None)
    assert rc == _lib.CF_ERR_NO_DEVICE
    assert "device" in _lib.last_error().lower()
    # argument validation happens before any device access
    rc = lib.cf_conv_bn_lif(None, None, None, None, None, 0, None, None, None, None,
                            4, 1, 8, 8, 16, 32, 3, 3, 1, 1, 2.0, 1.0, 0.0, 1, 1, None)
    assert rc == _lib.CF_ERR_INVALID_ARG
    with pytest.raises(_lib.CatfuseNativeError):
        ops.lif_fwd(torch.zeros(2, 8))
