"""Tensor-core (tcgen05) dequant-GEMM: the dense 4-bit projection and the grouped 3-bit expert GEMMs of
chunked prefill, against the CPU oracle's exact arithmetic (exact fp32 dequantised weights, fp32 activations,
fp64 accumulation -- the yardstick of finchmoe/test_engine_path.m:28-44, 126-149) under the same bar as the
decode path: cos >= 0.99999 and max relative error <= 1e-3 (parity.assert_close).  The kernels carry the
weights and SiLU(gate)*up as a bf16 value plus a bf16 remainder, so nothing is rounded to 8 bits."""
import numpy as np
import pytest

from finchmoe_b200 import lib as L
from finchmoe_b200 import synth
from oracle import oracle
from parity import assert_close, cos_sim, max_rel_err, oracle_layer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    from finchmoe_b200 import api as _api
    return _api


def _report(tag, got, want):
    print(f"[parity] {tag}: cos={cos_sim(got, want):.9f} max_rel={max_rel_err(got, want):.3e}")


@pytest.mark.parametrize("shape", [(256, 2048), (2048, 512), (8192, 2048), (2048, 4096)])
@pytest.mark.parametrize("M", [16, 37, 64, 300, 512])
def test_dense_4bit_gemm_vs_oracle(api, shape, M):
    """The 4-bit g64 projections (2048 -> 8192, 4096 -> 2048 among them) at the benchmarked token counts; the
    oracle computes a sample of the tokens."""
    out_dim, in_dim = shape
    if out_dim * in_dim < 2 ** 21 and M in (64, 512):
        pytest.skip("small shapes at three token counts")
    ctx = api.Context(hidden=256, n_experts=8, top_k=8, moe_inter=128, shared_inter=128, n_layers=1, max_tokens=1)
    try:
        rng = synth.rng_for(5, out_dim + M)
        for sd in (L.FP16, L.BF16):
            t = synth.affine_tensor(rng, out_dim, in_dim, 4, sd)
            w = ctx.upload_tensor(t)
            xb = synth.f32_to_bf16_rne(rng.normal(0, 1, size=(M, in_dim)).astype(np.float32))
            got = ctx.dense_gemm(w, xb)
            assert np.all(np.isfinite(got))
            rows = np.arange(M) if out_dim * in_dim * M <= 2 ** 28 else np.sort(rng.choice(M, size=max(4, 2 ** 28 // (out_dim * in_dim)), replace=False))
            want = oracle.matvec(t["W"], t["S"], t["B"], sd, synth.bf16_to_f32(xb[rows]), out_dim, in_dim, 64, 4, oracle.ACC_F64)
            _report(f"dense 4-bit {shape} M={M}", got[rows], want)
            assert_close(got[rows], want, f"dense 4-bit {shape} M={M}")
        assert ctx.device_status() == 0
    finally:
        ctx.destroy()


@pytest.mark.parametrize("T,act_dtype", [(16, L.F32), (23, L.BF16), (64, L.F32), (200, L.BF16)])
@pytest.mark.parametrize("mode", [2, 3, 4])
def test_prefill_tensor_core_small_vs_oracle(api, T, act_dtype, mode):
    cfg = dict(hidden=256, inter=128, sd=L.BF16)
    ctx = api.Context(hidden=256, n_experts=16, top_k=8, moe_inter=128, shared_inter=128, n_layers=1,
                      scale_dtype=L.BF16, act_dtype=act_dtype, max_tokens=256)
    pool = ctx.pool()
    try:
        rng = synth.rng_for(6, T)
        blocks = {e: synth.expert_block(rng, 256, 128, 64, 3, L.BF16) for e in range(15)}   # expert 15 is absent
        for e, blk in blocks.items():
            pool.put(0, e, blk)
        x = synth.activations(rng, T, 256)
        if act_dtype == L.F32:   # full-precision activations (not bf16-representable)
            x = (x + rng.normal(0, 1e-3, size=x.shape)).astype(np.float32)
        ids, w = synth.zipf_routing(rng, T, 16, 8)
        valid = (rng.random((T, 8)) > 0.1).astype(np.uint8)
        sh = synth.shared_expert(rng, 256, 128, 64, 4, L.BF16)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh])
        score = rng.normal(0, 1, size=T).astype(np.float32)
        h_mid = rng.normal(0, 1, size=(T, 256)).astype(np.float32)
        ctx.set_prefill_mode(mode)
        out = ctx.moe_forward_host(pool, 0, x, ids, w, valid=valid, shared=shd, gate_score=score, h_mid=h_mid)
        want = oracle_layer(blocks, ids, w, valid, x, cfg, shared=sh, score=score, h_mid=h_mid)
        _report(f"prefill mode {mode} T={T}", out, want)
        assert_close(out, want, f"tensor-core prefill T={T}")
        out2 = ctx.moe_forward_host(pool, 0, x, ids, w)
        want2 = oracle_layer(blocks, ids, w, None, x, cfg)
        assert_close(out2, want2, f"tensor-core prefill, routed only T={T}")
        # and the same as the sub-batch path (the decode kernels) to the accuracy of both
        ctx.set_prefill_mode(1)
        exact = ctx.moe_forward_host(pool, 0, x, ids, w, valid=valid, shared=shd, gate_score=score, h_mid=h_mid)
        assert_close(out, exact, "tensor-core path against the sub-batch path")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


@pytest.mark.parametrize("mode", [2, 3, 4])
def test_prefill_tensor_core_full_size_vs_oracle(api, mode):
    """Hidden 2048, inter 512, 256 experts, top-8, Zipf routing, fp16 scales, bf16 activations: a 64-token chunk."""
    T = 64
    ctx = api.Context(max_tokens=64, n_layers=1, scale_dtype=L.FP16, act_dtype=L.BF16)
    ctx.set_prefill_mode(mode)
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
        cfg = dict(hidden=2048, inter=512, sd=L.FP16)
        want = oracle_layer(blocks, ids, w, None, x, cfg, shared=sh, score=score, h_mid=h_mid)
        _report("tensor-core prefill, full size, T=64", out, want)
        assert_close(out, want, "tensor-core prefill, full size")
        out2 = ctx.moe_forward_host(pool, 0, x, ids, w)
        want2 = oracle_layer(blocks, ids, w, None, x, cfg)
        _report("tensor-core prefill, full size, routed only, T=64", out2, want2)
        assert_close(out2, want2, "tensor-core prefill, full size, routed only")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


@pytest.mark.parametrize("mode", [2, 3, 4])
def test_prefill_512_tokens_full_size_sampled_oracle_and_exact_path(api, mode):
    """The largest chunk (512 tokens, hidden 2048, 256 experts, Zipf top-8) through the tensor-core path: every row
    finite, 24 sampled rows against the oracle's exact arithmetic, and all rows against the sub-batch path."""
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
        ctx.set_prefill_mode(mode)
        out = ctx.moe_forward_host(pool, 0, x, ids, w, shared=shd, gate_score=score, h_mid=h_mid)
        assert np.all(np.isfinite(out))
        sample = rng.choice(T, size=24, replace=False)
        blocks = {int(e): pool.get(0, int(e)) for e in set(ids[sample].ravel().tolist())}
        want = oracle_layer(blocks, ids[sample], w[sample], None, x[sample], dict(hidden=2048, inter=512, sd=L.FP16), shared=sh,
                            score=score[sample], h_mid=h_mid[sample])
        _report("tensor-core prefill, full size, T=512 (24 rows)", out[sample], want)
        assert_close(out[sample], want, "512-token chunk, sampled rows")
        ctx.set_prefill_mode(1)
        exact = ctx.moe_forward_host(pool, 0, x, ids, w, shared=shd, gate_score=score, h_mid=h_mid)
        assert_close(out, exact, "512-token chunk against the sub-batch path")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()
