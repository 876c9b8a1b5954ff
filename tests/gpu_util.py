"""Helpers for the GPU parity tests: seeded bf16 tensors on the device, their exact float32 copies for the oracle,
and the tolerance used throughout (the BASELINE bf16 bar: max |gpu - ref| <= 1e-2 * max |ref|)."""
import numpy as np
import torch

from oracle.bf16 import from_torch

TOL = 1e-2


def randn(shape, seed, std=1.0, mean=0.0, dtype=torch.bfloat16, device='cuda'):
    g = torch.Generator(device='cpu').manual_seed(seed)
    t = torch.randn(shape, generator=g) * std + mean
    return t.to(dtype).to(device)


def np32(t):
    return from_torch(t)


def rel_err(got, ref):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    return float(np.max(np.abs(got - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


def assert_close(got, ref, tol=TOL, what=''):
    e = rel_err(got, ref)
    assert e <= tol, f'{what}: max rel err {e:.3e} > {tol}'
    return e


def bf16_min():
    return torch.finfo(torch.bfloat16).min


def assert_argmax_agree(got, ref, min_frac=0.999, what=''):
    """Argmax agreement over the last axis, the north-star bar (>= 99.9%), counted on rows whose decision is not a
    near tie: a row where the GPU picks another index counts as a near tie when that index's reference value is
    within 2 x the measured max |got - ref| of the reference maximum (the two values are closer than the rounding
    error of the comparison itself).  Every disagreement must be such a near tie."""
    got = np.asarray(got, np.float32).reshape(-1, np.shape(got)[-1])
    ref = np.asarray(ref, np.float32).reshape(-1, np.shape(ref)[-1])
    err = float(np.max(np.abs(got - ref)))
    ga, ra = np.argmax(got, -1), np.argmax(ref, -1)
    rows = np.arange(ref.shape[0])
    tie = ref[rows, ga] >= ref[rows, ra] - 2 * err
    differ = ga != ra
    assert not np.any(differ & ~tie), f'{what}: argmax disagreement that is not a near tie (err {err:.3e})'
    decided = ~(differ & tie)
    frac = float(np.mean(ga[decided] == ra[decided])) if decided.any() else 1.0
    assert frac >= min_frac, f'{what}: argmax agreement {frac:.4f} < {min_frac}'
    return float(np.mean(~differ))
