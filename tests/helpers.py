"""Shared assertions for the parity tests.

Tolerances are the contract's: bit-exact where the operation is exactly
specified (ReLU, the upsampling index/weight maths, and every op whose
accumulation order matches the reference's), otherwise, against the oracle,
max |got - want| / max |want| <= 1e-4 and ||got - want||_2 / ||want||_2 <= 1e-5.
"""
from __future__ import annotations

import numpy as np

MAX_REL = 1e-4
L2_REL = 1e-5


def rel_errs(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    if want.size == 0:
        return 0.0, 0.0
    d = got - want
    scale = np.abs(want).max()
    nrm = np.linalg.norm(want.ravel())
    mx = float(np.abs(d).max() / scale) if scale > 0 else float(np.abs(d).max())
    l2 = float(np.linalg.norm(d.ravel()) / nrm) if nrm > 0 else float(np.linalg.norm(d.ravel()))
    return mx, l2


def assert_close(got, want, max_rel=MAX_REL, l2_rel=L2_REL, what=""):
    mx, l2 = rel_errs(got, want)
    assert mx <= max_rel and l2 <= l2_rel, f"{what}: max_rel={mx:.3e} (<= {max_rel}), l2_rel={l2:.3e} (<= {l2_rel})"


def assert_bitexact(got, want, what=""):
    got = np.ascontiguousarray(got, np.float32)
    want = np.ascontiguousarray(want, np.float32)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    eq = got.view(np.uint32) == want.view(np.uint32)
    if not eq.all():
        idx = np.argwhere(~eq)[:5]
        raise AssertionError(f"{what}: {int((~eq).sum())} of {eq.size} elements differ in bits, e.g. at "
                             f"{idx.tolist()}: got {got[tuple(idx[0])]!r} want {want[tuple(idx[0])]!r}")


def to_np(t):
    return t.detach().cpu().numpy()
