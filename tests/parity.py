"""Tolerance helpers shared by the parity tests.

Output tolerance of the path (fp32 accumulation): cos >= 0.99999 and
max relative error <= 1e-3, where the relative error of element i is
|a_i - b_i| / max(|b_i|, floor) and floor = 1e-2 * rms(b): matvec outputs are
sums of mixed-sign products, so elements that cancel to ~0 are judged against
the vector's scale instead of their own magnitude.
"""
import numpy as np

COS_MIN = 0.99999
REL_MAX = 1e-3


def cos_sim(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def max_rel_err(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    floor = 1e-2 * np.sqrt(np.mean(b * b)) + 1e-30
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), floor)))


def assert_close(a, b, what="", cos_min=COS_MIN, rel_max=REL_MAX):
    assert np.all(np.isfinite(np.asarray(a))), f"{what}: non-finite values"
    c, r = cos_sim(a, b), max_rel_err(a, b)
    assert c >= cos_min and r <= rel_max, f"{what}: cos={c:.8f} max_rel={r:.3e}"
    return c, r
