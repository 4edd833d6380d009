"""The restated CPU oracle against the reference's own compiled C.

`make -C oracle ref` compiles the pure-C region of the reference's engine source
(finchmoe/infer.m:690-702, 1575-1868) from a reference checkout into
oracle/_ref/libfinch_ref.so; the build travels with the tree, so these tests also
run where the checkout is absent, and skip only when there is neither.  In its
sequential-fp32 mode the restatement must equal the reference bit for bit.
"""
import ctypes as C

import numpy as np
import pytest

from finchmoe_b200 import synth
from oracle import oracle as orc

REF = orc.ref_lib()
pytestmark = pytest.mark.skipif(REF is None, reason="no reference checkout and no earlier build of oracle/_ref")

F32P, U16P, I32P = C.POINTER(C.c_float), C.POINTER(C.c_uint16), C.POINTER(C.c_int)


def _f(a):
    return a.ctypes.data_as(F32P)


def _ref_matvec(t, x, bits):
    out = np.empty(t["out_dim"], np.float32)
    W = np.ascontiguousarray(t["W"])
    S = np.ascontiguousarray(t["S"]) if t.get("S") is not None else None
    B = np.ascontiguousarray(t["B"]) if t.get("B") is not None else None
    REF.ref_cpu_dequant_matvec(W.ctypes.data, S.ctypes.data if S is not None else None, B.ctypes.data if B is not None else None,
                               _f(x), _f(out), t["out_dim"], t["in_dim"], 64, bits)
    return out


def test_widening_all_65536_inputs():
    for h in range(0, 65536, 1):
        a = np.float32(REF.ref_fp16_to_f32(h))
        b = np.float32(orc.lib().fo_fp16_to_f32(h))
        assert a.view(np.uint32) == b.view(np.uint32) or (np.isnan(a) and np.isnan(b)), h
        assert np.float32(REF.ref_bf16_to_f32(h)).view(np.uint32) == np.float32(orc.lib().fo_bf16_to_f32(h)).view(np.uint32)


@pytest.mark.parametrize("bits,o,i", [(3, 48, 2048), (3, 2048, 512), (4, 64, 2048), (4, 40, 4096), (8, 33, 512), (8, 16, 2048)])
def test_affine_matvec_bit_for_bit(bits, o, i):
    rng = synth.rng_for(9, bits, o)
    t = synth.affine_tensor(rng, o, i, bits, orc.SCALE_BF16)   # the reference's files carry bf16 scales
    x = (synth.activations(rng, i) + rng.normal(0, 1e-3, size=i)).astype(np.float32)
    want = _ref_matvec(t, x, bits)
    got = orc.matvec(t["W"], t["S"], t["B"], orc.SCALE_BF16, x, o, i, 64, bits, orc.ACC_F32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # and the fp64 yardstick agrees with it to fp32 accumulation noise
    y64 = orc.matvec(t["W"], t["S"], t["B"], orc.SCALE_BF16, x, o, i, 64, bits, orc.ACC_F64)
    assert np.abs(y64 - want).max() <= 1e-4 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("ty,bits", [(12, 10), (14, 11)])
def test_gguf_rows_and_matvec_bit_for_bit(ty, bits):
    rng = synth.rng_for(9, ty)
    t = synth.gguf_tensor(rng, 24, 2048, ty)
    W = np.ascontiguousarray(t["W"])
    rb = W.size // 24
    want = np.empty((24, 2048), np.float32)
    for r in range(24):
        REF.ref_gguf_dequant_row(W.ctypes.data + r * rb, _f(want[r]), 2048, ty)
    got = orc.dequant_gguf(t["W"], 24, 2048, ty)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    x = synth.activations(rng, 2048)
    y = _ref_matvec(dict(W=W, S=None, B=None, out_dim=24, in_dim=2048), x, bits)
    mine = orc.matvec(t["W"], None, None, orc.SCALE_BF16, x, 24, 2048, 256, bits, orc.ACC_F32)
    assert np.array_equal(mine.view(np.uint32), y.view(np.uint32))


def test_bf16_rows_bit_for_bit():
    rng = synth.rng_for(9, 0)
    wf = synth.activations(rng, 12, 512)
    W = synth.f32_to_bf16_rne(wf)
    x = synth.activations(rng, 512)
    y = _ref_matvec(dict(W=W, S=None, B=None, out_dim=12, in_dim=512), x, 0)
    mine = orc.matvec(W, None, None, orc.SCALE_BF16, x, 12, 512, 64, 0, orc.ACC_F32)
    assert np.array_equal(mine.view(np.uint32), y.view(np.uint32))


def test_swiglu_softmax_topk_normalise_madd_norm():
    rng = synth.rng_for(9, 77)
    g, u = synth.activations(rng, 512) * 3, synth.activations(rng, 512)
    want = np.empty(512, np.float32)
    REF.ref_cpu_swiglu(_f(g), _f(u), _f(want), 512)
    assert np.array_equal(orc.swiglu(g, u).view(np.uint32), want.view(np.uint32))
    for trial in range(20):
        logits = rng.normal(0, 1, 256).astype(np.float32)
        if trial % 4 == 0:   # ties: the earlier index must win, in both
            logits[rng.integers(0, 256, 40)] = logits[3]
        p = logits.copy()
        REF.ref_cpu_softmax(_f(p), 256)
        idx, val = np.empty(8, np.int32), np.empty(8, np.float32)
        REF.ref_cpu_topk(_f(p), 256, 8, idx.ctypes.data_as(I32P), _f(val))
        REF.ref_cpu_normalize_weights(_f(val), 8)
        ids, w = orc.route(logits, 8)
        assert np.array_equal(ids, idx) and np.array_equal(w.view(np.uint32), val.view(np.uint32))
    # combine = h_mid + sum_k w_k out_k + sigmoid(score) shared: the reference's fallback chains cpu_vec_madd
    # (finchmoe/infer.m:10190-10258)
    outs = synth.activations(rng, 8, 2048)
    w = np.abs(rng.normal(0, 1, 8)).astype(np.float32)
    w /= w.sum()
    h_mid, shared = synth.activations(rng, 2048), synth.activations(rng, 2048)
    score = np.float32(0.3)
    moe = np.zeros(2048, np.float32)
    for k in range(8):
        REF.ref_cpu_vec_madd(_f(moe), _f(outs[k]), C.c_float(w[k]), 2048)
    hidden = h_mid + moe
    REF.ref_cpu_vec_madd(_f(hidden), _f(shared), C.c_float(REF.ref_cpu_sigmoid(C.c_float(score))), 2048)
    mine = orc.combine(h_mid, outs, w, np.ones(8, np.uint8), shared, float(score))
    assert np.abs(mine - hidden).max() <= 2e-6 * np.abs(hidden).max()   # fma(w, out, acc) vs mul + add: one rounding apart
    # RMS norm
    x = synth.activations(rng, 2048)
    nw = synth.f32_to_bf16_rne(np.abs(synth.activations(rng, 2048)) + 0.5)
    want = np.empty(2048, np.float32)
    REF.ref_cpu_rms_norm(_f(x), nw.ctypes.data_as(U16P), _f(want), 2048, C.c_float(1e-6))
    _, h_post = orc.residual_norm(x, None, nw, 1e-6)
    assert np.abs(h_post - want).max() <= 2e-6 * np.abs(want).max()
