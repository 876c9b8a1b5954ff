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
