"""CPU oracle pinned against the golden vectors (reference Python packers /
dequantizers, gguf-py block decoders) and against itself (C vs numpy)."""
import os

import numpy as np
import pytest

from finchmoe_b200 import synth
from oracle import oracle as orc
from parity import assert_close


@pytest.fixture(scope="module")
def aff(golden_dir):
    return np.load(os.path.join(golden_dir, "affine_reference.npz"))


@pytest.fixture(scope="module")
def gg(golden_dir):
    return np.load(os.path.join(golden_dir, "gguf_reference.npz"))


def test_pack3_matches_reference_packer(aff):
    q = aff["pack3_codes"]
    assert np.array_equal(synth.pack_codes(q[None, :], 3)[0], aff["pack3_bytes"])
    assert np.array_equal(orc.unpack_codes(aff["pack3_bytes"], 1, q.size, 3)[0], q)
    assert np.array_equal(orc.np_unpack_codes(aff["pack3_bytes"], 1, q.size, 3)[0], q)


@pytest.mark.parametrize("tag,bits", [("rp3", 3), ("rp4", 4), ("qn4", 4), ("qn8", 8)])
def test_affine_dequant_bit_exact_vs_reference(aff, tag, bits):
    pk, s, b = aff[tag + "_packed"], aff[tag + "_scales"], aff[tag + "_biases"]
    o = pk.shape[0]
    i = pk.shape[1] * 8 // bits
    want = aff[tag + "_dequant"]
    got_c = orc.dequant_affine(pk, s, b, orc.SCALE_BF16, o, i, 64, bits)
    got_np = orc.np_dequant_affine(pk, s, b, orc.SCALE_BF16, o, i, 64, bits)
    assert np.array_equal(got_c.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(got_np.view(np.uint32), want.view(np.uint32))
    if tag == "rp4":
        assert np.array_equal(got_c.view(np.uint32), aff["rp4_dequant_inplace"].view(np.uint32))


@pytest.mark.parametrize("tag,bits", [("rp3", 3), ("rp4", 4)])
def test_codes_requantize_to_reference_bytes(aff, tag, bits):
    """Re-derive the codes from the float weights with the quantizer's
    published rule and check our packer reproduces the reference's bytes."""
    w, s = aff[tag + "_w"], aff[tag + "_scales"]
    o, i = w.shape
    g = w.reshape(o, i // 64, 64)
    mn, mx = g.min(axis=2), g.max(axis=2)
    sc = np.maximum((mx - mn) / ((1 << bits) - 1), 1e-8)
    q = np.clip(np.round((g - mn[:, :, None]) / sc[:, :, None]), 0, (1 << bits) - 1).astype(np.uint8)
    assert np.array_equal(synth.pack_codes(q.reshape(o, i), bits), aff[tag + "_packed"])
    assert np.array_equal(synth.f32_to_bf16_trunc(sc.astype(np.float32)), s)


@pytest.mark.parametrize("bits", [4, 8])
def test_matvec_vs_reference_python(aff, bits):
    t = f"qn{bits}"
    pk, s, b, x = aff[t + "_packed"], aff[t + "_scales"], aff[t + "_biases"], aff[t + "_x"]
    o, i = pk.shape[0], pk.shape[1] * 8 // bits
    y64 = orc.matvec(pk, s, b, orc.SCALE_BF16, x, o, i, 64, bits, orc.ACC_F64)
    y32 = orc.matvec(pk, s, b, orc.SCALE_BF16, x, o, i, 64, bits, orc.ACC_F32)
    np.testing.assert_allclose(y64, aff[t + "_matvec_f64"], rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(y32, aff[t + "_matvec_f64"], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("name,ty", [("q4k", 12), ("q6k", 14)])
def test_gguf_dequant_vs_gguf_py(gg, name, ty):
    raw, want = gg[name + "_raw"], gg[name + "_dequant"]
    got = orc.dequant_gguf(raw, raw.shape[0], want.shape[1], ty)
    # gguf-py evaluates d*sc*q in numpy fp32 with the same association for
    # Q4_K; Q6_K multiplies (d*sc) first too -- both bit-exact here.
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.abs(got - want).max()


def test_fp16_widening_exhaustive():
    L = orc.lib()
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([L.fo_fp16_to_f32(int(v)) for v in h], np.float32)
    magic = np.array([L.fo_fp16_to_f32_magic(int(v)) for v in h], np.float32)
    fin = np.isfinite(want)
    assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))
    assert np.array_equal(magic[fin].view(np.uint32), want[fin].view(np.uint32))
    assert np.all(np.isnan(got[~fin]) == np.isnan(want[~fin]))


def test_expert_layout_matches_reference_constants():
    # finchmoe/infer.m:223-234
    L = orc.expert_layout(2048, 512, 64, 3)
    assert (L["gate_w"], L["gate_s"], L["gate_b"]) == (0, 393216, 425984)
    assert (L["up_w"], L["up_s"], L["up_b"]) == (458752, 851968, 884736)
    assert (L["down_w"], L["down_s"], L["down_b"]) == (917504, 1310720, 1343488)
    assert L["size"] == 1376256
    # finchmoe/infer.m:175-184 (4-bit) and 187-196 (8-bit)
    assert orc.expert_layout(2048, 512, 64, 4)["size"] == 1769472
    assert orc.expert_layout(2048, 512, 64, 8)["size"] == 3342336
    assert synth.expert_layout() == L


def test_c_matches_numpy_on_synthetic():
    rng = synth.rng_for(9, 0)
    for bits in (3, 4, 8):
        for sd in (synth.SCALE_BF16, synth.SCALE_FP16):
            t = synth.affine_tensor(rng, 20, 192, bits, sd)
            assert np.array_equal(orc.unpack_codes(t["W"], 20, 192, bits), t["codes"])
            a = orc.dequant_affine(t["W"], t["S"], t["B"], sd, 20, 192, 64, bits)
            b = orc.np_dequant_affine(t["W"], t["S"], t["B"], sd, 20, 192, 64, bits)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
            x = synth.activations(rng, 192)
            y = orc.matvec(t["W"], t["S"], t["B"], sd, x, 20, 192, 64, bits, orc.ACC_F64)
            np.testing.assert_allclose(y, (a.astype(np.float64) @ x.astype(np.float64)), rtol=1e-6, atol=1e-6)


def test_topk_reference_semantics():
    # ties keep the earlier index; output is in slot order, not sorted
    s = np.zeros(16, np.float32)
    s[[3, 5, 7, 9]] = [0.5, 0.5, 0.9, 0.5]
    L = orc.lib()
    idx = np.zeros(3, np.int32)
    val = np.zeros(3, np.float32)
    L.fo_topk(s.ctypes.data_as(orc.C.c_void_p), 16, 3, idx.ctypes.data_as(orc.C.c_void_p),
              val.ctypes.data_as(orc.C.c_void_p))
    assert sorted(idx.tolist()) == [3, 5, 7]
    lg = synth.router_logits(synth.rng_for(9, 1), 5)
    ids, w = orc.route(lg, 8)
    p = np.exp(lg - lg.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    for t in range(5):
        want = set(np.argsort(-p[t], kind="stable")[:8].tolist())
        assert set(ids[t].tolist()) == want
        np.testing.assert_allclose(w[t].sum(), 1.0, rtol=1e-6)
        np.testing.assert_allclose(w[t], p[t][ids[t]] / p[t][ids[t]].sum(), rtol=1e-5)


def test_combine_forms():
    rng = synth.rng_for(9, 2)
    eo = rng.normal(size=(8, 64)).astype(np.float32)
    w = np.full(8, 0.125, np.float32)
    hm = rng.normal(size=64).astype(np.float32)
    so = rng.normal(size=64).astype(np.float32)
    valid = np.ones(8, np.uint8)
    valid[2] = 0
    eo[2] = np.nan  # an unselected / failed expert must be skipped, not multiplied
    out = orc.combine(hm, eo, w, valid, so, 0.3)
    want = hm + sum(w[k] * eo[k] for k in range(8) if k != 2) + so / (1 + np.exp(-0.3))
    np.testing.assert_allclose(out, want, rtol=1e-5, atol=1e-6)
    # guard form: drops the non-finite expert and renormalises by kept weight
    out_g = orc.combine(hm, eo, w, None, so, 0.3, guard=1)
    want_g = hm + sum(w[k] * eo[k] for k in range(8) if k != 2) / 0.875 + so / (1 + np.exp(-0.3))
    np.testing.assert_allclose(out_g, want_g, rtol=1e-5, atol=1e-6)


def test_moe_layer_f32_order_vs_f64_spread():
    """The reference's sequential-fp32 CPU order and the fp64 yardstick agree
    to well inside the output tolerance (documents the reference's own spread)."""
    rng = synth.rng_for(1, 0)
    hid, inter = 256, 128
    blocks = [synth.expert_block(rng, hid, inter, 64, 3, synth.SCALE_BF16) for _ in range(8)]
    x = synth.activations(rng, hid)
    _, w = orc.route(synth.router_logits(rng, 1), 8)
    a = orc.moe_layer(blocks, w[0], None, x, scale_dtype=0, hidden=hid, inter=inter, accum=orc.ACC_F32)
    b = orc.moe_layer(blocks, w[0], None, x, scale_dtype=0, hidden=hid, inter=inter, accum=orc.ACC_F64)
    c = orc.moe_layer(blocks, w[0], None, x, scale_dtype=0, hidden=hid, inter=inter, accum=orc.ACC_F64, nthreads=8)
    assert np.array_equal(b, c)
    assert_close(a, b, "f32-order vs f64")


def test_residual_norm_restatement_against_numpy():
    """fo_residual_norm follows residual_norm_fused / cpu_rms_norm; pinned here against a float64 numpy form."""
    rng = np.random.default_rng(5)
    resid, oproj = rng.normal(0, 1, 2048).astype(np.float32), rng.normal(0, 1, 2048).astype(np.float32)
    w = synth.f32_to_bf16_rne(rng.normal(1, 0.1, 2048).astype(np.float32))
    h_mid, h_post = orc.residual_norm(resid, oproj, w, 1e-6)
    h = resid.astype(np.float64) + oproj
    want = h / np.sqrt((h * h).mean() + 1e-6) * synth.bf16_to_f32(w)
    assert np.array_equal(h_mid, resid + oproj)
    assert np.allclose(h_post, want, rtol=2e-6, atol=1e-7)
    _, plain = orc.residual_norm(resid, None, w, 1e-6)
    r = resid.astype(np.float64)
    assert np.allclose(plain, r / np.sqrt((r * r).mean() + 1e-6) * synth.bf16_to_f32(w), rtol=2e-6, atol=1e-7)
