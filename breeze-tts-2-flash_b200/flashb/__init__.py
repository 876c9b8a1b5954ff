"""flashb: B200-native (sm_100a) kernels for the Breeze-TTS-2 streaming-decode hot path.

Drop-in modules with the call surface of the reference's hook package (AsherHou/Breeze-TTS-2-flash ``flash/``):

  flashb.kernels       load / load_all / attn / fused / depth / info / SPECS       (flash/kernels.py)
  flashb.backbone      install / fused_decode_step / GEMV_CFG / ORIG               (flash/backbone.py)
  flashb.depth         install / attach / DepthMegakernel / manifest / BUILDS / GRIDS (flash/depth.py)
  flashb.prefill_attn  install / bz_prefill_attention                              (flash/prefill_attn.py)

All compute runs in ``libflashb.so`` (C ABI in ``include/flashb.h``); without it every call raises.
"""
__version__ = '0.1.0'
