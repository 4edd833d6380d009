"""Tensor-core (tcgen05) dequant-GEMM: the dense 4-bit projection and the grouped 3-bit expert GEMMs of
chunked prefill, against a numpy oracle that rounds where the kernels round: weights = RNE-to-bf16 of the
exact dequantised value fl32(fl32(q*s)+b) (the oracle's dequant_affine, pinned to the reference packers),
activations bf16, fp32 accumulation (float64 here), SiLU(gate)*up kept as two bf16 planes (value and
remainder) in front of both down GEMMs."""
import numpy as np
import pytest

from finchmoe_b200 import lib as L
from finchmoe_b200 import synth
from oracle import oracle
from parity import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    from finchmoe_b200 import api as _api
    return _api


def _bf16(x):
    return synth.bf16_to_f32(synth.f32_to_bf16_rne(np.ascontiguousarray(x, np.float32)))


def _wb(t):
    """bf16-rounded dequantised weights of an affine tensor dict, as float64."""
    w = oracle.dequant_affine(t["W"], t["S"], t["B"], t["scale_dtype"], t["out_dim"], t["in_dim"], 64, t["bits"])
    return _bf16(w).astype(np.float64)


def _swiglu_bf16(g64, u64, planes=2):
    """SiLU(g)*u in fp32, kept as bf16(value) [+ bf16(value - that)] like the kernels keep it."""
    g, u = g64.astype(np.float32), u64.astype(np.float32)
    act = (g / (np.float32(1.0) + np.exp(-g))) * u
    hi = _bf16(act)
    if planes == 1:
        return hi.astype(np.float64)
    return hi.astype(np.float64) + _bf16(act - hi).astype(np.float64)


@pytest.mark.parametrize("shape", [(256, 2048), (2048, 512), (8192, 2048), (2048, 4096)])
@pytest.mark.parametrize("M", [16, 37, 300])
def test_dense_4bit_gemm_vs_oracle(api, shape, M):
    if shape[0] * shape[1] > 8 * 2 ** 20 and M != 37:
        pytest.skip("large shapes once")
    out_dim, in_dim = shape
    ctx = api.Context(hidden=256, n_experts=8, top_k=8, moe_inter=128, shared_inter=128, n_layers=1, max_tokens=1)
    try:
        rng = synth.rng_for(5, out_dim + M)
        for sd in (L.FP16, L.BF16):
            t = synth.affine_tensor(rng, out_dim, in_dim, 4, sd)
            w = ctx.upload_tensor(t)
            xb = synth.f32_to_bf16_rne(rng.normal(0, 1, size=(M, in_dim)).astype(np.float32))
            got = ctx.dense_gemm(w, xb)
            want = synth.bf16_to_f32(xb).astype(np.float64) @ _wb(t).T
            assert_close(got, want.astype(np.float32), f"dense 4-bit {shape} M={M}")
            # the only difference from the oracle is the order of the fp32 additions
            err = np.abs(got - want).max() / np.sqrt((want ** 2).mean())
            assert err < 1e-4, err   # tensor-core fp32 accumulation truncates
        assert ctx.device_status() == 0
    finally:
        ctx.destroy()


def _oracle_prefill(blocks, ids, w, valid, xb, cfg, shared=None, score=None, h_mid=None):
    """xb: fp32 values already on the bf16 grid.  Returns fp32 [T, hidden]."""
    T, K = ids.shape
    H, I, sd = cfg["hidden"], cfg["inter"], cfg["sd"]
    wts = {}
    for e, blk in blocks.items():
        wts[e] = tuple(_wb(dict(synth.block_tensor(blk, n, H, I, 64, 3, sd), scale_dtype=sd, bits=3))
                       for n in ("gate", "up", "down"))
    out = np.zeros((T, H), np.float64) if h_mid is None else h_mid.astype(np.float64).copy()
    x64 = xb.astype(np.float64)
    for t in range(T):
        moe = np.zeros(H, np.float32)
        for k in range(K):
            e = int(ids[t, k])
            if (valid is not None and not valid[t, k]) or e not in wts:
                continue
            g, u, d = wts[e]
            act = _swiglu_bf16(x64[t] @ g.T, x64[t] @ u.T)
            moe = (np.float32(w[t, k]) * (act @ d.T).astype(np.float32) + moe).astype(np.float32)
        out[t] += moe
    if shared is not None:
        g, u, d = (_wb(s) for s in shared)
        act = _swiglu_bf16(x64 @ g.T, x64 @ u.T)
        so = act @ d.T
        out += (1.0 / (1.0 + np.exp(-score.astype(np.float64))))[:, None] * so
    return out.astype(np.float32)


@pytest.mark.parametrize("T,act_dtype", [(16, L.F32), (23, L.BF16), (64, L.F32), (200, L.BF16)])
def test_prefill_tensor_core_small_vs_oracle(api, T, act_dtype):
    cfg = dict(hidden=256, inter=128, sd=L.BF16)
    ctx = api.Context(hidden=256, n_experts=16, top_k=8, moe_inter=128, shared_inter=128, n_layers=1,
                      scale_dtype=L.BF16, act_dtype=act_dtype, max_tokens=256)
    pool = ctx.pool()
    try:
        rng = synth.rng_for(6, T)
        blocks = {e: synth.expert_block(rng, 256, 128, 64, 3, L.BF16) for e in range(15)}   # expert 15 is absent
        for e, blk in blocks.items():
            pool.put(0, e, blk)
        x = synth.activations(rng, T, 256)          # on the bf16 grid, so both act dtypes see the same values
        ids, w = synth.zipf_routing(rng, T, 16, 8)
        valid = (rng.random((T, 8)) > 0.1).astype(np.uint8)
        sh = synth.shared_expert(rng, 256, 128, 64, 4, L.BF16)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh])
        score = rng.normal(0, 1, size=T).astype(np.float32)
        h_mid = rng.normal(0, 1, size=(T, 256)).astype(np.float32)
        ctx.set_prefill_mode(2)
        out = ctx.moe_forward_host(pool, 0, x, ids, w, valid=valid, shared=shd, gate_score=score, h_mid=h_mid)
        want = _oracle_prefill(blocks, ids, w, valid, x, cfg, shared=sh, score=score, h_mid=h_mid)
        assert_close(out, want, f"tensor-core prefill T={T}", tight_rel=None)
        out2 = ctx.moe_forward_host(pool, 0, x, ids, w)
        want2 = _oracle_prefill(blocks, ids, w, None, x, cfg)
        assert_close(out2, want2, f"tensor-core prefill, routed only T={T}", tight_rel=None)
        # and close to the exact (fp32-activation, unrounded-weight) path: bf16 rounding only
        ctx.set_prefill_mode(1)
        exact = ctx.moe_forward_host(pool, 0, x, ids, w, valid=valid, shared=shd, gate_score=score, h_mid=h_mid)
        rel = np.abs(out - exact).max() / np.sqrt((exact.astype(np.float64) ** 2).mean())
        assert rel < 3e-2, rel
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


def test_prefill_tensor_core_full_size_vs_oracle(api):
    """BASELINE shapes (hidden 2048, inter 512, 256 experts, top-8, Zipf routing), a 64-token chunk."""
    T = 64
    ctx = api.Context(max_tokens=64, n_layers=1, scale_dtype=L.FP16, act_dtype=L.BF16)
    ctx.set_prefill_mode(2)
    pool = ctx.pool(n_layers=1)
    try:
        rng = synth.rng_for(7, T)
        ids, w = synth.zipf_routing(rng, T, 256, 8)
        blocks = {}
        for e in sorted(set(ids.ravel().tolist())):
            blocks[e] = synth.expert_block(rng, scale_dtype=L.FP16)
            pool.put(0, e, blocks[e])
        x = synth.activations(rng, T, 2048)
        sh = synth.shared_expert(rng, scale_dtype=L.FP16)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh])
        score = rng.normal(0, 1, size=T).astype(np.float32)
        h_mid = synth.activations(rng, T, 2048)
        out = ctx.moe_forward_host(pool, 0, x, ids, w, shared=shd, gate_score=score, h_mid=h_mid)
        want = _oracle_prefill(blocks, ids, w, None, x, dict(hidden=2048, inter=512, sd=L.FP16), shared=sh, score=score, h_mid=h_mid)
        assert_close(out, want, "tensor-core prefill, full size", tight_rel=None)
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


def test_prefill_512_tokens_full_size_sampled_oracle_and_exact_path(api):
    """BASELINE's largest chunk (512 tokens, hidden 2048, 256 experts, Zipf top-8) through the tensor-core path: every
    row finite, 24 sampled rows against the oracle, and all rows close to the exact sub-batch path (bf16 rounding only)."""
    T = 512
    ctx = api.Context(max_tokens=T, n_layers=1, scale_dtype=L.FP16, act_dtype=L.BF16)
    pool = ctx.pool(n_layers=1)
    try:
        pool.fill_synthetic(0, 1, 77)
        rng = synth.rng_for(8, T)
        ids, w = synth.zipf_routing(rng, T, 256, 8)
        x = synth.activations(rng, T, 2048)
        sh = synth.shared_expert(rng, scale_dtype=L.FP16)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh])
        score = rng.normal(0, 1, size=T).astype(np.float32)
        h_mid = synth.activations(rng, T, 2048)
        ctx.set_prefill_mode(2)
        out = ctx.moe_forward_host(pool, 0, x, ids, w, shared=shd, gate_score=score, h_mid=h_mid)
        assert np.all(np.isfinite(out))
        sample = rng.choice(T, size=24, replace=False)
        blocks = {int(e): pool.get(0, int(e)) for e in set(ids[sample].ravel().tolist())}
        want = _oracle_prefill(blocks, ids[sample], w[sample], None, x[sample], dict(hidden=2048, inter=512, sd=L.FP16), shared=sh,
                               score=score[sample], h_mid=h_mid[sample])
        assert_close(out[sample], want, "512-token chunk, sampled rows", tight_rel=None)
        ctx.set_prefill_mode(1)
        exact = ctx.moe_forward_host(pool, 0, x, ids, w, shared=shd, gate_score=score, h_mid=h_mid)
        rel = np.abs(out - exact).max() / np.sqrt((exact.astype(np.float64) ** 2).mean())
        assert rel < 3e-2, rel
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()
