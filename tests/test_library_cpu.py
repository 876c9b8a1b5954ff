"""CPU-side checks of the native library: it builds, loads, exports every entry point the C header declares, and
rejects bad arguments with FB_ERR_ARG before touching a GPU."""
import os
import re

import pytest

from flashb import _native, build, kernels, backbone

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'include', 'flashb.h')


def declared():
    src = open(HEADER).read()
    src = re.sub(r'/\*.*?\*/', '', src, flags=re.S)
    return sorted(set(re.findall(r'\b(flashb_\w+)\s*\(', src)))


def test_library_builds_and_exports_every_declared_symbol():
    build.build()
    import ctypes
    h = ctypes.CDLL(build.LIB)
    missing = [n for n in declared() if not hasattr(h, n)]
    assert not missing, missing
    assert set(declared()) <= set(_native._PROTOS), 'every declared symbol has a ctypes prototype'


def test_argument_errors_need_no_gpu():
    L = _native.lib()
    rc = L.flashb_gemv_seg(None, 8, 2, 2048, None, 1e-6, None, 0, None, 0, None, 0, None, 8, None)
    assert rc == _native.FB_ERR_ARG
    assert 'null' in _native.last_error()
    rc = L.flashb_gemv_seg(16, 8, (1 << 20) + 1, 2048, None, 1e-6, 16, 8, None, 0, None, 0, 16, 8, None)
    assert rc == _native.FB_ERR_ARG and f'M={(1 << 20) + 1}' in _native.last_error()
    rc = L.flashb_attn_decode(16, 0, 0, 16, 16, 0, 0, 2, 16, 4, 64, 64, 16, 1, 0, 1.0, 16, 1 << 20, 16, 16, None)
    assert rc == _native.FB_ERR_UNSUPPORTED and 'head_dim' in _native.last_error()
    with pytest.raises(_native.FlashbError):
        _native.check(rc)


def test_reference_call_surface_present():
    for n in ('load', 'load_all', 'attn', 'fused', 'depth', 'info', 'SPECS'):
        assert hasattr(kernels, n)
    assert set(kernels.SPECS) == {'flash_bb_attn', 'flash_bb_fused', 'flash_dd_full', 'flash_dd_kv'}
    for n in ('install', 'fused_decode_step', 'GEMV_CFG', 'ORIG'):
        assert hasattr(backbone, n)
    a, f = kernels.attn(), kernels.fused()
    for n in ('attn_decode', 'attn_decode_fused'):
        assert callable(getattr(a, n))
    for n in ('gemv_seg', 'gemv_resid', 'gemv_gateup', 'rmsnorm'):
        assert callable(getattr(f, n))
