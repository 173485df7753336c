"""Shared test helpers: seeded inputs and the parity error metric."""
from __future__ import annotations

import numpy as np


def randn(rng: np.random.Generator, *shape) -> np.ndarray:
    return rng.standard_normal(shape).astype(np.float32)


def max_rel_err(x: np.ndarray, r: np.ndarray) -> float:
    """max_i |x_i - r_i| / max(|r_i|, 1e-3 * max_j |r_j|): elementwise relative error with a
    floor, so that entries near zero do not dominate."""
    x = np.asarray(x, np.float64)
    r = np.asarray(r, np.float64)
    floor = 1e-3 * max(float(np.max(np.abs(r))), 1e-30)
    return float(np.max(np.abs(x - r) / np.maximum(np.abs(r), floor)))


def normwise_err(x: np.ndarray, r: np.ndarray) -> float:
    x = np.asarray(x, np.float64)
    r = np.asarray(r, np.float64)
    return float(np.max(np.abs(x - r)) / max(float(np.max(np.abs(r))), 1e-30))


# Tolerances stated by the target: fp32-KV path and bf16-KV path.
TOL_F32 = 1e-3
TOL_BF16 = 2e-2


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 -> float32 (the cache's storage rounding)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def parity(got: np.ndarray, oracle_out: np.ndarray, exact: np.ndarray | None, tol: float) -> tuple[float, float]:
    """Return (error vs the oracle, allowed).  The allowance is `tol`, plus -- when the float64
    ground truth `exact` is given -- the oracle's own distance from it: the oracle sums in
    float32 in sequential order, so over thousands of positions its own rounding is of the
    order of the bound, and a kernel that sums in a different order is judged against the
    oracle up to that amount."""
    err = max_rel_err(got, oracle_out)
    allowed = tol + (max_rel_err(oracle_out, exact) if exact is not None else 0.0)
    return err, allowed


def rope_agrees(y: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    """RoPE on the device uses the reference's float32 angle and rounding-exact products; only
    the last bit of cos/sin may differ between glibc and the device.  A rotated value that
    cancels to near zero (x0*c - x1*s) turns that into many ulps of itself, so the difference
    is measured in ulps of the largest value.  Returns (fraction of bit-identical elements,
    max |difference| in ulps of max |ref|)."""
    y = np.asarray(y, np.float32)
    ref = np.asarray(ref, np.float32)
    same = float(np.mean(y == ref))
    ulp = float(np.spacing(np.float32(np.max(np.abs(ref)))))
    return same, float(np.max(np.abs(y.astype(np.float64) - ref)) / ulp)


def check_rope(y: np.ndarray, ref: np.ndarray) -> None:
    same, ulps = rope_agrees(y, ref)
    assert ulps <= 2 and same >= 0.98, (same, ulps)
