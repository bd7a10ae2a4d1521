"""Shared comparison metrics for the parity tests (tolerances are written in each test)."""
import numpy as np


def max_rel_err_per_head(got, ref):
    """max over heads of max|got-ref| / max|ref| within the head (the decode tolerance metric: relative error
    per head, so near-zero elements do not make it ill-conditioned). Arrays [..., H, D]."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    h = ref.shape[-2]
    g = np.moveaxis(got, -2, 0).reshape(h, -1)
    r = np.moveaxis(ref, -2, 0).reshape(h, -1)
    denom = np.maximum(np.abs(r).max(1), 1e-30)
    return float((np.abs(g - r).max(1) / denom).max())


def min_cosine_per_head(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    h = ref.shape[-2]
    g = np.moveaxis(got, -2, 0).reshape(h, -1)
    r = np.moveaxis(ref, -2, 0).reshape(h, -1)
    num = (g * r).sum(1)
    den = np.linalg.norm(g, axis=1) * np.linalg.norm(r, axis=1)
    return float((num / np.maximum(den, 1e-300)).min())
