"""Comparison helpers shared by the parity tests.

Tolerances (from the project's parity contract):
  fp32 activations / gradients / loss: relative error <= 1e-4, measured per
  tensor as ||a - b|| / ||b|| and elementwise as |a - b| <= 1e-4 * max|b|
  (the reference itself sums with atomics, so per-element relative error
  near zero is not meaningful);
  top-k indices: bit-exact as index sets per token, excluding tokens whose
  selection margin (k-th vs (k+1)-th score, or ties within the k) is < 1e-6.
"""
from __future__ import annotations

import numpy as np

FP32_TOL = 1e-4


def rel_err(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (nb if nb > 0 else 1.0))


def max_err_vs_scale(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    s = np.abs(b).max()
    return float(np.abs(a - b).max() / (s if s > 0 else 1.0))


def assert_close(a, b, tol=FP32_TOL, what=""):
    r = rel_err(a, b)
    m = max_err_vs_scale(a, b)
    assert r <= tol and m <= tol, f"{what}: norm-rel {r:.3e}, max/scale {m:.3e} (tol {tol:g})"


def per_tensor_report(cfg, a, b, layout_fn):
    out, off = [], 0
    for name, n in layout_fn(cfg):
        out.append((name, rel_err(a[off:off + n], b[off:off + n]),
                    max_err_vs_scale(a[off:off + n], b[off:off + n])))
        off += n
    return out


def assert_grads_close(cfg, a, b, layout_fn, tol=FP32_TOL, what="grads"):
    bad = [(n, r, m) for n, r, m in per_tensor_report(cfg, a, b, layout_fn) if r > tol or m > tol]
    assert not bad, f"{what}: tensors over tolerance {tol:g}: " + ", ".join(
        f"{n} (rel {r:.2e}, max {m:.2e})" for n, r, m in bad[:12])


def topk_sets_match(idx_a, idx_b, scores_margin=None, margin=1e-6):
    """Fraction of tokens whose top-k index SETS agree; tokens with a selection
    margin below `margin` (when margins are given) are excluded."""
    a = np.sort(np.asarray(idx_a).reshape(-1, idx_a.shape[-1]), axis=1)
    b = np.sort(np.asarray(idx_b).reshape(-1, idx_b.shape[-1]), axis=1)
    ok = np.all(a == b, axis=1)
    if scores_margin is not None:
        keep = np.asarray(scores_margin).reshape(-1) >= margin
        ok = ok | ~keep
    return ok


def update_rel_err(p0, pa, pb) -> float:
    """Norm-relative difference of two SGD updates (pa - p0 vs pb - p0),
    ignoring elements where the two updated fp32 parameters are within one
    ulp of each other: both sides round p - lr*g to fp32, so an update that
    differs by 1e-6 relative can still land one ulp apart, which is a
    rounding of the parameter, not a difference of the update."""
    p0 = np.asarray(p0, np.float32)
    pa = np.asarray(pa, np.float32)
    pb = np.asarray(pb, np.float32)
    ulp = np.spacing(np.maximum(np.abs(pa), np.abs(pb)))
    diff = (pa.astype(np.float64) - pb.astype(np.float64))
    diff[np.abs(diff) <= ulp] = 0.0
    db = pb.astype(np.float64) - p0.astype(np.float64)
    n = np.linalg.norm(db)
    return float(np.linalg.norm(diff) / (n if n > 0 else 1.0))
