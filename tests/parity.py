"""Comparison metrics used by the parity tests (the reference's own test
metrics: max-abs, mean-abs, cosine; tests/test_utils.h:107-147)."""
import numpy as np


def compare(out, ref):
    out = np.asarray(out, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    d = np.abs(out - ref)
    cos = float(np.dot(out, ref) / (np.linalg.norm(out) * np.linalg.norm(ref) + 1e-30))
    return {"max_abs": float(d.max()), "mean_abs": float(d.mean()), "cos": cos,
            "ref_max": float(np.abs(ref).max()), "ref_mean": float(np.abs(ref).mean())}


def assert_close(out, ref, cos_min, mean_rel_max, max_rel_max, what=""):
    m = compare(out, ref)
    msg = f"{what}: {m}"
    assert m["cos"] >= cos_min, msg
    assert m["mean_abs"] <= mean_rel_max * max(m["ref_mean"], 1e-12), msg
    assert m["max_abs"] <= max_rel_max * max(m["ref_max"], 1e-12), msg
    return m
