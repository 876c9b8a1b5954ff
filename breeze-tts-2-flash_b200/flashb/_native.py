"""ctypes binding of ``libflashb.so`` (declarations in ``include/flashb.h``).

The library is the only compute path: if it is missing or fails to load, every call raises ``FlashbError``; there is
no CPU or torch fallback.  ``check(rc)`` turns a non-zero FB_ERR_* return code into ``FlashbError`` carrying the
library's message, as ``TORCH_CHECK`` raises ``RuntimeError`` in the reference's pybind functions.
"""
import ctypes
import os
import threading

from . import build as _build

_LOCK = threading.Lock()
_LIB = None

FB_OK, FB_ERR_ARG, FB_ERR_CUDA, FB_ERR_UNSUPPORTED, FB_ERR_STATE, FB_ERR_TIMEOUT, FB_ERR_DEVICE, FB_ERR_ABORTED = range(8)
_NAMES = {1: 'invalid argument', 2: 'CUDA error', 3: 'unsupported', 4: 'bad state', 5: 'device wait timed out',
          6: 'device error', 7: 'aborted'}


class FlashbError(RuntimeError):
    def __init__(self, rc, msg):
        super().__init__(f'flashb: {_NAMES.get(rc, rc)}: {msg}')
        self.rc = rc


P = ctypes.c_void_p
I = ctypes.c_int
L = ctypes.c_int64
F = ctypes.c_float

_PROTOS = {
    'flashb_last_error': (ctypes.c_char_p, []),
    'flashb_version': (ctypes.c_char_p, []),
    'flashb_device_error': (I, [I]),
    'flashb_set_pdl': (None, [I]),
    'flashb_set_sm_budget': (None, [I]),
    'flashb_sm_budget': (I, []),
    'flashb_gemv_last_path': (I, []),
    'flashb_gemv_last_split': (I, []),
    'flashb_attn_last_path': (I, []),
    'flashb_set_gemv_split': (None, [I]),
    'flashb_set_gemv_group_rows': (I, [I]),
    'flashb_set_gemv_trace': (None, [P]),
    'flashb_set_gemv_rows_path': (None, [I]),
    'flashb_attn_ws_floats': (L, [I, I, I, I, I]),
    'flashb_attn_decode': (I, [P, L, L, P, P, L, L, I, I, I, I, I, P, I, L, F, P, L, P, P, P]),
    'flashb_attn_decode_fused': (I, [P, L, P, P, F, P, P, L, P, P, L, L, I, I, I, I, I, P, I, L, P, F, P, L, P, P,
                                     P]),
    'flashb_gemv_seg': (I, [P, L, I, I, P, F, P, I, P, I, P, I, P, L, P]),
    'flashb_gemv_resid': (I, [P, L, I, I, P, I, P, L, P, L, P]),
    'flashb_gemv_gateup': (I, [P, L, I, I, P, F, P, P, I, P, L, P]),
    'flashb_rmsnorm': (I, [P, L, I, I, P, F, P, L, P]),
    'flashb_embed_rope': (I, [P, I, I, I, P, I, P, P, P, I, I, P, P, P, P]),
    'flashb_lm_head_cfg': (I, [P, I, I, P, F, P, I, P, P, P, P, P]),
    'flashb_lm_head_cfg_blocks': (I, [P, I, I, P, F, P, I, P, I, P, P, P, P]),
    'flashb_step_advance': (I, [P, P, I, P, I, L, I, P]),
    'flashb_cb0_greedy': (I, [P, L, I, I, I, P, P]),
    'flashb_cb0_sample': (I, [P, L, I, I, P, L, F, P, I, P, P, P, P, P, L, P, I, P, I, P]),
    'flashb_frame_ids': (I, [P, P, I, I, I, P, P]),
    'flashb_prefill_attn': (I, [P, L, L, L, P, L, L, L, P, L, L, L, P, I, L, L, I, I, I, I, I, I, F, I, I, I, P, L, L,
                                L, P]),
    'flashb_prefill_attn_tiles': (I, [P, L, L, L, P, L, L, L, P, L, L, L, P, I, L, L, I, I, I, I, I, I, F, I, I, I,
                                      I, I, P, L, L, L, P]),
    'flashb_prefill_qkv': (I, [P, L, I, I, I, I, P, P, F, P, P, I, P, P, P, P, L, L, I, P]),
    'flashb_ln12_decode': (I, [P, P, P, ctypes.c_uint32, ctypes.c_uint32, I, I, P, L, P]),
    'flashb_lm_head_rows': (I, [P, L, I, I, P, I, P, P]),
    'flashb_dd_scratch_bytes': (L, [P]),
    'flashb_dd_tab_build': (I, [P, P, P, P, P]),
    'flashb_dd_layer_bytes': (L, []),
    'flashb_dd_barrier_offset': (L, [P]),
    'flashb_dd_frame': (I, [P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P]),
    'flashb_dd_frame_noalloc': (I, [P, P, P, P, P, P, P, P, P, P, P, P, P, P, P]),
}


class FbDDLayer(ctypes.Structure):
    """fb_dd_layer of include/flashb.h."""
    _fields_ = [(n, ctypes.c_void_p) for n in ('ln1', 'wq', 'wk', 'wv', 'wo', 'ln2', 'wg', 'wu', 'wd')]


class FbDDConfig(ctypes.Structure):
    """fb_dd_config of include/flashb.h."""
    _fields_ = [('layers', I), ('batch', I), ('hidden', I), ('embed_dim', I), ('heads', I), ('kv_heads', I),
                ('head_dim', I), ('ffn', I), ('vocab', I), ('codebook_size', I), ('n_decode', I), ('eps', F),
                ('scaling', F), ('embed', P), ('proj', P), ('normf', P), ('head_t', P), ('cos_tab', P),
                ('sin_tab', P), ('trace', P), ('grid', I), ('layers_host', P), ('wait_ns', L), ('ptab', P),
                ('ttab', P), ('ln12', P)]


class FbLn12Mat(ctypes.Structure):
    """fb_ln12_mat of include/flashb.h."""
    _fields_ = [('data', P), ('meta', P), ('ovf', P), ('n_ovf', L), ('lut_lo', ctypes.c_uint32),
                ('lut_hi', ctypes.c_uint32)]


def lib_path():
    return _build.LIB


def lib():
    """Load (and on first use in a fresh checkout, build) libflashb.so."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = lib_path()
        if not os.path.exists(path):
            try:
                _build.build()
            except Exception as e:  # no silent fallback: the library is the product
                raise FlashbError(FB_ERR_STATE, f'libflashb.so missing at {path} and the build failed: {e}') from e
        try:
            h = ctypes.CDLL(path)
        except OSError as e:
            raise FlashbError(FB_ERR_STATE, f'cannot load {path}: {e}') from e
        for name, (res, args) in _PROTOS.items():
            fn = getattr(h, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _LIB = h
        return _LIB


def exported_symbols():
    """Names from include/flashb.h that the loaded library exports."""
    h = lib()
    return [n for n in _PROTOS if getattr(h, n, None) is not None]


def check(rc):
    if rc != FB_OK:
        msg = lib().flashb_last_error()
        raise FlashbError(rc, msg.decode() if msg else '')


def last_error():
    m = lib().flashb_last_error()
    return m.decode() if m else ''


def device_error(clear=True):
    """The device error word (0 = no bounded wait expired).  Synchronises the device."""
    return int(lib().flashb_device_error(1 if clear else 0))


def check_device(clear=True):
    """Raise FlashbError when a kernel reported a device-side failure (an expired bounded wait, an abort); the
    error word is cleared (unless clear=False).  Synchronises the device."""
    rc = device_error(clear)
    if rc:
        raise FlashbError(rc, last_error())
