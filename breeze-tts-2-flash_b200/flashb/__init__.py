"""flashb: B200-native (sm_100a) kernels for the Breeze-TTS-2 streaming-decode hot path.

Drop-in modules with the call surface of the reference's hook package (AsherHou/Breeze-TTS-2-flash ``flash/``):

  flashb.kernels       load / load_all / attn / fused / depth / info / SPECS       (flash/kernels.py)
  flashb.backbone      install / fused_decode_step / GEMV_CFG / ORIG               (flash/backbone.py)
  flashb.depth         install / attach / DepthMegakernel / manifest / BUILDS / GRIDS (flash/depth.py)
  flashb.prefill_attn  install / bz_prefill_attention                              (flash/prefill_attn.py)
  flashb.prefill       install / prefill_forward: the whole BackbonePrefillGraphCache._forward on flashb kernels
                       (no reference module: the reference runs the eager layers with its attention hook)

``install(api)`` installs the hot-path hooks on the official runtime, as ``flash.install`` does for them
(``flash/__init__.py:37-70``; the reference's other hooks -- weight packing, codec, streaming loop, reference cache --
are outside this library).  ``FLASHB_DISABLE=1`` installs nothing.

All compute runs in ``libflashb.so`` (C ABI in ``include/flashb.h``); without it every call raises.
"""
import os

__version__ = '0.1.0'
_STATE = dict(enabled=None, reason=None, installed=[])


def install(api=None):
    """Install the prefill, backbone and depth hooks.  Idempotent.  Returns True when active; False (the official
    code path) when disabled or when the library cannot be loaded on a GPU."""
    if _STATE['enabled'] is not None:
        return _STATE['enabled']
    if os.environ.get('FLASHB_DISABLE') == '1':
        _STATE.update(enabled=False, reason='FLASHB_DISABLE=1')
        return False
    from . import kernels
    try:
        kernels.load_all()
    except Exception as ex:  # noqa: BLE001 - the official path stays available
        _STATE.update(enabled=False, reason=f'{type(ex).__name__}: {ex}')
        print(f'[flashb] acceleration OFF, official code path: {_STATE["reason"]}', flush=True)
        return False
    from . import backbone, depth, prefill, prefill_attn
    prefill_attn.install(api)
    prefill.install(api)
    backbone.install(api)
    depth.install(api)
    _STATE.update(enabled=True, installed=['prefill_attn', 'prefill', 'backbone', 'depth'])
    print(f'[flashb] acceleration ON ({", ".join(_STATE["installed"])})', flush=True)
    return True


def info():
    return dict(version=__version__, **_STATE)
