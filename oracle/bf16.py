"""bf16 emulation on float32 numpy arrays (test infrastructure; see ``oracle/__init__.py``).

PyTorch stores bf16 as the upper 16 bits of an IEEE float32 and rounds float32 -> bf16 to nearest, ties to even
(c10/util/BFloat16.h round_to_nearest_even).  Every eager bf16 op in the reference computes in float32 and rounds
once with that rule, so ``round_bf16`` after each float32 op reproduces an eager bf16 op.
"""
import numpy as np


def round_bf16(x):
    """float32 -> nearest bf16 value (ties to even), returned as float32.  NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32).reshape(x.shape)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, np.float32(np.nan), out)
    return out


def bits_to_f32(u16):
    """bf16 bit patterns (uint16) -> float32 values."""
    return (np.asarray(u16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bits(x):
    """float32 -> bf16 bit patterns (uint16), rounding to nearest even."""
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_torch(t):
    """A torch tensor (bf16 or float) -> float32 numpy array holding exactly the same values."""
    import torch
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return bits_to_f32(t.contiguous().view(torch.int16).numpy().view(np.uint16))
    return t.float().numpy()
