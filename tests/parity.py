"""Tolerance helpers shared by the parity tests.

Output tolerance of the path (fp32 accumulation): cos >= 0.99999 and
max relative error <= 1e-3, where the relative error of element i is
|a_i - b_i| / max(|b_i|, rms(b)): matvec outputs are sums of mixed-sign
products, so elements that cancel to below the vector's rms are judged against
the rms instead of their own magnitude (stricter than the usual
max|a-b| / max|b|).  TIGHT_REL is the bound the kernels are additionally held
to against a floor of 1% of the rms -- it documents the accuracy actually
delivered (tensor-core fp32 accumulation truncates, so ~1e-5 of the rms).
"""
import numpy as np

COS_MIN = 0.99999
REL_MAX = 1e-3
TIGHT_REL = 5e-3


def cos_sim(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def max_rel_err(a, b, floor_frac=1.0):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    floor = floor_frac * np.sqrt(np.mean(b * b)) + 1e-30
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), floor)))


def assert_close(a, b, what="", cos_min=COS_MIN, rel_max=REL_MAX, tight_rel=TIGHT_REL):
    """tight_rel=None skips the extra bound: the bf16 path rounds SiLU(gate)*up to bf16, and a last-bit
    difference in an accumulator can move that rounding by one bf16 step (0.4 % of one term), which
    is far below REL_MAX of the rms but not below 0.5 % of an element that cancels to 1 % of the rms."""
    assert np.all(np.isfinite(np.asarray(a))), f"{what}: non-finite values"
    c, r = cos_sim(a, b), max_rel_err(a, b)
    assert c >= cos_min and r <= rel_max, f"{what}: cos={c:.8f} max_rel={r:.3e}"
    if tight_rel is not None:
        tight = max_rel_err(a, b, 1e-2)
        assert tight <= tight_rel, f"{what}: error against 1% of rms = {tight:.3e}"
    return c, r


def oracle_layer(blocks_by_expert, ids, w, valid, x, cfg, shared=None, score=None, h_mid=None, accum=None):
    """The MoE layer of T tokens on the CPU oracle (fp64 accumulation unless told otherwise): experts that are
    masked or missing from blocks_by_expert are skipped, as the library skips them."""
    from oracle import oracle as orc
    accum = orc.ACC_F64 if accum is None else accum
    T = ids.shape[0]
    out = np.empty((T, cfg["hidden"]), np.float32)
    for t in range(T):
        v = None if valid is None else valid[t]
        blocks = [blocks_by_expert.get(int(e)) if (v is None or v[k]) else None for k, e in enumerate(ids[t])]
        vv = np.array([1 if (b is not None and (v is None or v[k])) else 0 for k, b in enumerate(blocks)], np.uint8)
        out[t] = orc.moe_layer(blocks, w[t], vv, x[t], bits=3, scale_dtype=cfg["sd"], hidden=cfg["hidden"],
                               inter=cfg["inter"], h_mid=None if h_mid is None else h_mid[t], shared=shared,
                               shared_gate_score=0.0 if score is None else float(score[t]), accum=accum)
    return out
