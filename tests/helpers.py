"""Shared test helpers: golden fixtures and comparison rules."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["s1", "s2", "s3", "s4_b0", "s4_b512"]

# Scores: |delta| <= SCORE_RTOL * max|reference score| of the row (fp32 summation order differs).
SCORE_RTOL = 1e-3
# Top-k: scores within TIE_EPS * max|score| of the k-th selected score count as ties.
TIE_EPS = 1e-5


def load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def load_config0():
    with open(os.path.join(GOLDEN, "config0.json")) as f:
        meta = json.load(f)
    topk = np.load(os.path.join(GOLDEN, "config0_topk.npz"))["topk"].astype(np.int64)
    return meta, topk


def score_rel_err(got, ref):
    """max over rows of max|got - ref| / max|ref| (rows = all leading dims)."""
    got = np.asarray(got, np.float64).reshape(-1, got.shape[-1])
    ref = np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    den = np.maximum(np.abs(ref).max(-1), 1e-30)
    return float((np.abs(got - ref).max(-1) / den).max())


def topk_sets_agree(scores, idx_a, idx_b, kk, eps=TIE_EPS):
    """True if two selections of the kk largest of `scores` rows agree up to ties.

    Every token whose score is clearly above the kk-th largest (by more than eps * max|row|)
    must be in both selections; every token clearly below must be in neither; both
    selections must have kk distinct entries."""
    s = np.asarray(scores, np.float64).reshape(-1, scores.shape[-1])
    a = np.asarray(idx_a).reshape(s.shape[0], -1)[:, :kk]
    b = np.asarray(idx_b).reshape(s.shape[0], -1)[:, :kk]
    for r in range(s.shape[0]):
        row = s[r]
        if len(set(a[r].tolist())) != kk or len(set(b[r].tolist())) != kk:
            return False
        thr = np.sort(row)[::-1][kk - 1]
        tol = eps * max(np.abs(row[np.isfinite(row)]).max(initial=0.0), 1e-30)
        sure_in = set(np.nonzero(row > thr + tol)[0].tolist())
        sure_out = set(np.nonzero(row < thr - tol)[0].tolist())
        for sel in (set(a[r].tolist()), set(b[r].tolist())):
            if not sure_in <= sel or sel & sure_out:
                return False
    return True
