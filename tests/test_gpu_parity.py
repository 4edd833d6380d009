"""GPU parity: the CUDA path, called through the C ABI, against the CPU oracle
and the committed golden vectors.

Bit-exact: unpacked codes, fp32 dequantized weights, their 16-bit images.
Tolerance (fp32 accumulation): cos >= 0.99999, max rel err <= 1e-3 (parity.py).
"""
import os

import numpy as np
import pytest

from finchmoe_b200 import lib as L
from finchmoe_b200 import synth
from oracle import oracle as orc
from parity import assert_close, oracle_layer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    from finchmoe_b200 import api as A
    return A


@pytest.fixture(scope="module")
def ctx_small(api):
    c = api.Context(hidden=256, n_experts=16, top_k=8, moe_inter=128, shared_inter=128, n_layers=2,
                    scale_dtype=L.BF16, act_dtype=L.F32, max_tokens=8)
    yield c
    c.destroy()


def _rne16(w32, dt):
    if dt == L.FP16:
        return w32.astype(np.float16).view(np.uint16)
    return synth.f32_to_bf16_rne(w32)


# ------------------------------------------------------------------ dequant
@pytest.mark.parametrize("bits", [3, 4, 8])
@pytest.mark.parametrize("sd", [L.BF16, L.FP16])
def test_dequant_affine_bit_exact(ctx_small, bits, sd):
    t = synth.affine_tensor(synth.rng_for(2, bits, sd), 40, 512, bits, sd)
    w = ctx_small.upload_tensor(t)
    codes, w32, w16 = ctx_small.debug_dequant(w, L.BF16)
    assert np.array_equal(codes, t["codes"])
    want = orc.dequant_affine(t["W"], t["S"], t["B"], sd, 40, 512, 64, bits)
    assert np.array_equal(w32.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(w16, _rne16(want, L.BF16))
    _, _, h16 = ctx_small.debug_dequant(w, L.FP16)
    assert np.array_equal(h16, _rne16(want, L.FP16))


def test_dequant_matches_reference_golden(ctx_small, golden_dir):
    aff = np.load(os.path.join(golden_dir, "affine_reference.npz"))
    for tag, bits in (("rp3", 3), ("rp4", 4), ("qn4", 4), ("qn8", 8)):
        pk = aff[tag + "_packed"]
        o, i = pk.shape[0], pk.shape[1] * 8 // bits
        t = dict(W=pk, S=aff[tag + "_scales"], B=aff[tag + "_biases"], out_dim=o, in_dim=i, bits=bits, scale_dtype=L.BF16)
        _, w32, _ = ctx_small.debug_dequant(ctx_small.upload_tensor(t))
        assert np.array_equal(w32.view(np.uint32), aff[tag + "_dequant"].view(np.uint32)), tag


@pytest.mark.parametrize("ty,bits", [(12, 10), (14, 11)])
def test_dequant_gguf_bit_exact(ctx_small, golden_dir, ty, bits):
    gg = np.load(os.path.join(golden_dir, "gguf_reference.npz"))
    name = "q4k" if ty == 12 else "q6k"
    raw, want = gg[name + "_raw"], gg[name + "_dequant"]
    t = dict(W=raw, S=None, B=None, out_dim=raw.shape[0], in_dim=want.shape[1], bits=bits, group=256)
    codes, w32, _ = ctx_small.debug_dequant(ctx_small.upload_tensor(t))
    assert np.array_equal(w32.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(codes, orc.gguf_unpack_codes(raw, raw.shape[0], want.shape[1], ty))
    t2 = synth.gguf_tensor(synth.rng_for(4, ty), 24, 1024, ty)
    _, w32b, _ = ctx_small.debug_dequant(ctx_small.upload_tensor(t2))
    assert np.array_equal(w32b.view(np.uint32), orc.dequant_gguf(t2["W"], 24, 1024, ty).view(np.uint32))


# ------------------------------------------------------------------- matvec
@pytest.mark.parametrize("bits,o,i", [(3, 96, 2048), (4, 64, 4096), (8, 40, 512), (10, 72, 2048), (11, 72, 512), (11, 33, 2048),
                                      (3, 33, 512), (4, 45, 1536), (10, 41, 512), (4, 2048, 4096), (8, 1000, 2048)])
@pytest.mark.parametrize("M", [1, 3, 9])
def test_matvec_vs_oracle(ctx_small, bits, o, i, M):
    rng = synth.rng_for(4, bits, M)
    if bits in (10, 11):
        t = synth.gguf_tensor(rng, o, i, 12 if bits == 10 else 14)
    else:
        t = synth.affine_tensor(rng, o, i, bits, L.FP16)
    x = synth.activations(rng, M, i)
    y = ctx_small.fast_dequant_matvec(ctx_small.upload_tensor(t), x)
    want = orc.matvec(t["W"], t["S"], t["B"], L.FP16, x, o, i, t["group"], bits, orc.ACC_F64)
    assert_close(y, want, f"matvec bits={bits} M={M}")


@pytest.mark.parametrize("ty,bits", [(12, 10), (14, 11)])
@pytest.mark.parametrize("o,i", [(512, 2048), (2048, 512), (8192, 2048)])
@pytest.mark.parametrize("T", [1, 8, 90])
def test_gguf_matvec_benchmark_shapes_vs_oracle(ctx_small, ty, bits, o, i, T):
    """Q4_K / Q6_K at the shapes and token counts of the GGUF benchmark rows ([512 x 2048], [2048 x 512], [8192 x 2048]
    at 1, 8 and 90 positions; 90 positions run as several passes of the streaming kernel).  The oracle takes a sample
    of the positions of the large cases."""
    rng = synth.rng_for(4, ty, o + T)
    t = synth.gguf_tensor(rng, o, i, ty)
    x = synth.activations(rng, T, i)
    y = ctx_small.fast_dequant_matvec(ctx_small.upload_tensor(t), x)
    assert y.shape == (T, o) and np.all(np.isfinite(y))
    rows = np.arange(T) if o * i * T <= 2 ** 27 else np.sort(rng.choice(T, size=8, replace=False))
    want = orc.matvec(t["W"], None, None, L.FP16, x[rows], o, i, 256, bits, orc.ACC_F64)
    assert_close(y[rows], want, f"GGUF type {ty} [{o} x {i}] T={T}")


@pytest.mark.parametrize("bits,o,i", [(8, 4100, 2048), (4, 8192, 2048), (4, 4099, 4096), (8, 5000, 512), (4, 33001, 512), (8, 32800, 1024)])
@pytest.mark.parametrize("M", [1, 3, 9])
@pytest.mark.parametrize("xdt", [L.F32, L.BF16])
def test_large_affine_matvec_streaming_kernel_vs_oracle(ctx_small, bits, o, i, M, xdt):
    """Large row-major 4- / 8-bit tensors: from 32,768 rows the tensor-core streaming kernel, below that the row-pair
    kernel, both straight from the reference tensor layout; row counts that are not multiples of 16, fp32 and bf16
    activations, several passes."""
    import torch
    rng = synth.rng_for(4, bits, o + M)
    t = synth.affine_tensor(rng, o, i, bits, L.FP16 if (o + M) % 2 else L.BF16)
    x = synth.activations(rng, M, i)
    if xdt == L.F32:
        x = (x + rng.normal(0, 1e-3, size=x.shape)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
    else:
        xd = torch.from_numpy(synth.f32_to_bf16_rne(x)).cuda().view(torch.bfloat16)
    out = torch.empty((M, o), dtype=torch.float32, device="cuda")
    ctx_small.fast_batch_matvec(xd, xdt, [ctx_small.upload_tensor(t)], [out], M=M)
    ctx_small.sync()
    want = orc.matvec(t["W"], t["S"], t["B"], t["scale_dtype"], x, o, i, 64, bits, orc.ACC_F64)
    assert_close(out.cpu().numpy(), want, f"streaming matvec bits={bits} [{o} x {i}] M={M}")


@pytest.mark.parametrize("ty,bits", [(12, 10), (14, 11)])
@pytest.mark.parametrize("o,i", [(72, 512), (1001, 2048), (8192, 2048)])
@pytest.mark.parametrize("M", [9, 33, 64, 65, 90, 128, 130])
@pytest.mark.parametrize("xdt", [L.F32, L.BF16])
def test_gguf_many_positions_one_pass_vs_oracle(ctx_small, ty, bits, o, i, M, xdt):
    """Q4_K / Q6_K at 9 and more positions: one pass over the weights on the tensor cores (codes as fp16 subnormals,
    activations as fp16 planes scaled per position).  Row counts that are not multiples of 16, position counts around
    the tile and pass boundaries (64 per pass with fp32 activations, 128 with bf16), two tensors sharing the
    activations, and positions whose magnitudes differ by five orders."""
    import torch
    if o == 8192 and M not in (9, 90, 130):
        pytest.skip("the large shape at three position counts")
    rng = synth.rng_for(4, ty, o + M)
    t = synth.gguf_tensor(rng, o, i, ty)
    t2 = synth.gguf_tensor(rng, 40, i, ty)
    x = synth.activations(rng, M, i)
    x[1] *= 300.0
    x[2] *= 1.0e-3
    if xdt == L.F32:
        x = (x * (1.0 + rng.normal(0, 1e-3, size=x.shape))).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
    else:
        x = synth.bf16_to_f32(synth.f32_to_bf16_rne(x))
        xd = torch.from_numpy(synth.f32_to_bf16_rne(x)).cuda().view(torch.bfloat16)
    out = torch.empty((M, o), dtype=torch.float32, device="cuda")
    out2 = torch.empty((M, 40), dtype=torch.float32, device="cuda")
    ctx_small.fast_batch_matvec(xd, xdt, [ctx_small.upload_tensor(t), ctx_small.upload_tensor(t2)], [out, out2], M=M)
    ctx_small.sync()
    rows = np.arange(M) if o * i * M <= 2 ** 27 else np.sort(rng.choice(M, size=8, replace=False))
    rows = np.union1d(rows, [1, 2])
    want = orc.matvec(t["W"], None, None, L.FP16, x[rows], o, i, 256, bits, orc.ACC_F64)
    got = out.cpu().numpy()
    assert np.all(np.isfinite(got))
    for j, r in enumerate(rows):      # row by row: the positions have very different scales
        assert_close(got[r], want[j], f"GGUF type {ty} [{o} x {i}] M={M} position {r}")
    want2 = orc.matvec(t2["W"], None, None, L.FP16, x[rows], 40, i, 256, bits, orc.ACC_F64)
    assert_close(out2.cpu().numpy()[rows], want2, f"second tensor, GGUF type {ty} M={M}", tight_rel=None)
    assert ctx_small.device_status() == 0


@pytest.mark.parametrize("ty,bits", [(14, 11), (12, 10)])
@pytest.mark.parametrize("o,i,xdt", [(248320, 2048, L.BF16), (33001, 512, L.F32), (40000, 1280, L.BF16), (33003, 1024, L.F32)])
def test_gguf_output_projection_tier_row_slices_vs_oracle(ctx_small, ty, bits, o, i, xdt):
    """The lm_head tier of a GGUF model (finchmoe/infer.m:5728-5815): a Q6_K / Q4_K tensor with tens of thousands of
    rows at one position takes the K-quant streaming kernel (odd row counts, an odd number of blocks per row, fp32 and
    bf16 activations); slices of rows against the oracle."""
    import torch
    rng = synth.rng_for(4, ty, o + i)
    base = synth.gguf_tensor(rng, 4096, i, ty)
    reps = o // 4096 + 1
    perm = rng.permutation(4096)
    W = np.ascontiguousarray(np.concatenate([base["W"][np.roll(perm, r)] for r in range(reps)])[:o])
    t = dict(base, W=W, out_dim=o)
    x = synth.activations(rng, 1, i)
    xd = torch.from_numpy(synth.f32_to_bf16_rne(x)).cuda().view(torch.bfloat16) if xdt == L.BF16 else torch.from_numpy(x).cuda()
    out = torch.empty((1, o), dtype=torch.float32, device="cuda")
    w = ctx_small.upload_tensor(t)
    ctx_small.fast_batch_matvec(xd, xdt, [w], [out], M=1)
    ctx_small.sync()
    got = out.cpu().numpy()[0]
    assert np.all(np.isfinite(got))
    for r0 in (0, o // 2 + 17, o - 600):
        sl = slice(r0, r0 + 600)
        want = orc.matvec(W[sl], None, None, L.FP16, x[0], 600, i, 256, bits, orc.ACC_F64)
        assert_close(got[sl], want, f"GGUF type {ty} output projection rows {r0}..")
    assert ctx_small.device_status() == 0


def test_lm_head_tier_row_slices_vs_oracle(ctx_small):
    """The lm_head / embedding tier (finchmoe/infer.m:5728-5815): 8-bit g64 [248,320 x 2048] at one position;
    three slices of rows against the oracle."""
    import torch
    OUT, K = 248320, 2048
    rng = synth.rng_for(4, 8, 248320)
    base = synth.affine_tensor(rng, 8192, K, 8, L.FP16)
    reps = OUT // 8192 + 1
    perm = rng.permutation(8192)
    t = dict(base, out_dim=OUT)
    for k in ("W", "S", "B"):   # rows of the small tensor, repeated in a shuffled order
        t[k] = np.ascontiguousarray(np.concatenate([base[k][np.roll(perm, r)] for r in range(reps)])[:OUT])
    x = synth.activations(rng, 1, K)
    xd = torch.from_numpy(synth.f32_to_bf16_rne(x)).cuda().view(torch.bfloat16)
    out = torch.empty((1, OUT), dtype=torch.float32, device="cuda")
    w = ctx_small.upload_tensor(t)
    ctx_small.fast_batch_matvec(xd, L.BF16, [w], [out], M=1)
    ctx_small.sync()
    got = out.cpu().numpy()[0]
    assert np.all(np.isfinite(got))
    for r0 in (0, 123456, OUT - 700):
        sl = slice(r0, r0 + 700)
        want = orc.matvec(t["W"][sl], t["S"][sl], t["B"][sl], L.FP16, x[0], 700, K, 64, 8, orc.ACC_F64)
        assert_close(got[sl], want, f"lm_head rows {r0}..")


def test_matvec_bf16_weights_and_bad_args(ctx_small):
    rng = synth.rng_for(4, 99)
    wf = synth.activations(rng, 24, 256)
    t = dict(W=synth.f32_to_bf16_rne(wf), S=None, B=None, out_dim=24, in_dim=256, bits=0)
    x = synth.activations(rng, 256)
    y = ctx_small.fast_dequant_matvec(ctx_small.upload_tensor(t), x)
    assert_close(y, wf.astype(np.float64) @ x.astype(np.float64), "bf16 matvec")
    w = ctx_small.upload_tensor(t)
    w.bits = 5
    with pytest.raises(L.FinchError) as e:
        ctx_small.fast_dequant_matvec(w, x)
    assert e.value.status == L.E_UNSUPPORTED
    w.bits = 4  # affine without scales
    with pytest.raises(L.FinchError) as e:
        ctx_small.fast_dequant_matvec(w, x)
    assert e.value.status == L.E_ARG


def test_batch_matvec_mixed_bits_device_pointers(ctx_small):
    import torch
    rng = synth.rng_for(4, 7)
    ts = [synth.affine_tensor(rng, 256, 2048, 8, L.BF16), synth.affine_tensor(rng, 512, 2048, 4, L.BF16),
          synth.affine_tensor(rng, 512, 2048, 4, L.BF16), synth.affine_tensor(rng, 1, 2048, 8, L.BF16)]
    specs = [ctx_small.upload_tensor(t) for t in ts]
    for M, xdt in ((1, L.F32), (4, L.BF16)):
        x = synth.activations(rng, M, 2048)
        xd = torch.from_numpy(x).cuda() if xdt == L.F32 else torch.from_numpy(x).cuda().to(torch.bfloat16)
        outs = [torch.full((M, t["out_dim"]), float("nan"), device="cuda") for t in ts]
        ctx_small.fast_batch_matvec(xd, xdt, specs, outs, M, stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        for t, o in zip(ts, outs):
            want = orc.matvec(t["W"], t["S"], t["B"], L.BF16, x, t["out_dim"], 2048, 64, t["bits"], orc.ACC_F64)
            assert_close(o.cpu().numpy(), want, f"batch bits={t['bits']} M={M}")


# -------------------------------------------------------------------- router
def test_route_topk_vs_oracle(ctx_small):
    import torch
    rng = synth.rng_for(1, 5)
    lg = synth.router_logits(rng, 37, 256)
    lg[3, 10] = lg[3, 200] = lg[3].max() + 1.0  # exact tie at the top: lower index must rank first
    lg[4, :] = 0.25                             # all equal: experts 0..7
    ids_o, w_o = orc.route(lg, 8)
    d = torch.from_numpy(lg).cuda()
    ids = torch.empty((37, 8), dtype=torch.int32, device="cuda")
    w = torch.empty((37, 8), dtype=torch.float32, device="cuda")
    ctx_small.route_topk(d, 256, 8, ids, w, 37, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    for t in range(37):
        assert set(ids[t].tolist()) == set(ids_o[t].tolist()), t
        mine = dict(zip(ids[t].tolist(), w[t].tolist()))
        for e, wo in zip(ids_o[t].tolist(), w_o[t].tolist()):
            assert abs(mine[e] - wo) <= 2e-6 * max(1.0, abs(wo))
        assert np.all(np.diff(w[t]) <= 1e-7)  # emitted by descending probability
    assert ids[3, 0] == 10 and ids[3, 1] == 200
    assert ids[4].tolist() == list(range(8))


# ----------------------------------------------------------------- MoE layer
_oracle_layer = oracle_layer


def _mk_small(api, sd, ad, n_experts=16, max_tokens=8, seed=0):
    cfg = dict(hidden=256, inter=128, sd=sd)
    ctx = api.Context(hidden=256, n_experts=n_experts, top_k=8, moe_inter=128, shared_inter=128, n_layers=2,
                      scale_dtype=sd, act_dtype=ad, max_tokens=max_tokens)
    rng = synth.rng_for(1, seed)
    pool = ctx.pool()
    blocks = {}
    for e in range(n_experts):
        blocks[e] = synth.expert_block(rng, 256, 128, 64, 3, sd)
        pool.put(1, e, blocks[e])
    return ctx, pool, blocks, cfg, rng


@pytest.mark.parametrize("sd", [L.BF16, L.FP16])
@pytest.mark.parametrize("ad", [L.F32, L.BF16])
@pytest.mark.parametrize("B", [1, 2, 3, 8])
def test_moe_decode_small_vs_oracle(api, sd, ad, B):
    ctx, pool, blocks, cfg, rng = _mk_small(api, sd, ad, seed=B)
    try:
        x = synth.activations(rng, B, 256)
        if ad == L.F32:  # full-precision activations (not bf16-representable)
            x = (x + rng.normal(0, 1e-3, size=x.shape)).astype(np.float32)
        ids, w = synth.zipf_routing(rng, B, 16, 8)
        out = ctx.moe_forward_host(pool, 1, x, ids, w)
        want = _oracle_layer(blocks, ids, w, None, x, cfg)
        assert_close(out, want, f"moe B={B}")
        again = ctx.moe_forward_host(pool, 1, x, ids, w)
        assert np.array_equal(out.view(np.uint32), again.view(np.uint32)), "not deterministic"
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


@pytest.mark.parametrize("B", [1, 2, 5, 8])
def test_moe_decode_is_deterministic_run_to_run(api, B):
    """No atomics on floats and fixed summation orders: repeated calls give bit-identical outputs, and they match the oracle."""
    ctx, pool, blocks, cfg, rng = _mk_small(api, L.FP16, L.BF16, seed=40 + B)
    try:
        x = synth.activations(rng, B, 256)
        ids, w = synth.zipf_routing(rng, B, 16, 8)
        sh = synth.shared_expert(rng, 256, 128, 64, 4, L.FP16)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh])
        score = rng.normal(0, 1, size=B).astype(np.float32)
        outs = [ctx.moe_forward_host(pool, 1, x, ids, w, shared=shd, gate_score=score) for _ in range(3)]
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
        assert np.array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32))
        want = _oracle_layer(blocks, ids, w, None, x, cfg, shared=sh, score=score)
        assert_close(outs[0], want, f"repeat B={B}")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


def test_moe_decode_shared_residual_valid_masks(api):
    ctx, pool, blocks, cfg, rng = _mk_small(api, L.BF16, L.F32, seed=11)
    try:
        B = 5
        x = rng.normal(0, 1, size=(B, 256)).astype(np.float32)
        ids, w = synth.zipf_routing(rng, B, 16, 8)
        valid = np.ones((B, 8), np.uint8)
        valid[0, 2] = valid[3, 7] = 0
        valid[4, :] = 0                  # a token with no usable expert at all
        ids[1, 5] = 999                  # out-of-range id: skipped
        h_mid = rng.normal(0, 1, size=(B, 256)).astype(np.float32)
        sh = synth.shared_expert(rng, 256, 128, 64, 4, L.BF16)
        score = rng.normal(0, 1, size=B).astype(np.float32)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh])
        out = ctx.moe_forward_host(pool, 1, x, ids, w, valid=valid, shared=shd, gate_score=score, h_mid=h_mid)
        v2 = valid.copy()
        v2[1, 5] = 0
        ids2 = ids.copy()
        ids2[1, 5] = 0
        want = _oracle_layer(blocks, ids2, w, v2, x, cfg, shared=sh, score=score, h_mid=h_mid)
        assert_close(out, want, "moe shared+residual+valid")
        # shared expert alone (every routed expert invalid) == residual + gated shared MLP
        allz = np.zeros((B, 8), np.uint8)
        out0 = ctx.moe_forward_host(pool, 1, x, ids, w, valid=allz, shared=shd, gate_score=score, h_mid=h_mid)
        want0 = _oracle_layer(blocks, ids2, w, allz, x, cfg, shared=sh, score=score, h_mid=h_mid)
        assert_close(out0, want0, "shared only")
        # nothing at all: output is the residual, bit for bit
        out1 = ctx.moe_forward_host(pool, 1, x, ids, w, valid=allz, h_mid=h_mid)
        assert np.array_equal(out1, h_mid)
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


def test_moe_skips_non_resident_and_poisoned_experts(api):
    """An expert that is not in the pool behaves as valid = 0; a resident expert
    whose block decodes to NaN is skipped (never multiplied by 0) when masked."""
    ctx, pool, blocks, cfg, rng = _mk_small(api, L.BF16, L.F32, n_experts=16, seed=12)
    try:
        x = rng.normal(0, 1, size=(1, 256)).astype(np.float32)
        ids = np.arange(8, dtype=np.int32)[None, :]
        w = np.full((1, 8), 0.125, np.float32)
        bad = blocks[3].copy()
        Lo = synth.expert_layout(256, 128, 64, 3)
        bad[Lo["gate_s"]:Lo["gate_s"] + 2] = np.array([0xC0, 0x7F], np.uint8)  # bf16 NaN scale
        pool.put(1, 3, bad)
        valid = np.ones((1, 8), np.uint8)
        valid[0, 3] = 0
        out = ctx.moe_forward_host(pool, 1, x, ids, w, valid=valid)
        assert np.all(np.isfinite(out))
        want = _oracle_layer(blocks, ids, w, valid, x, cfg)
        assert_close(out, want, "masked NaN expert")
        # layer 0 holds nothing: every expert is non-resident there
        out_empty = ctx.moe_forward_host(pool, 0, x, ids, w)
        assert np.array_equal(out_empty, np.zeros_like(out_empty))
    finally:
        pool.destroy()
        ctx.destroy()


@pytest.mark.parametrize("B", [1, 3, 5, 8])
def test_moe_decode_full_size_vs_oracle(api, B):
    """The model's shapes: hidden 2048, inter 512, 256 experts, top-8, fp16 scales, bf16 activations."""
    ctx = api.Context(max_tokens=8, n_layers=1)
    pool = ctx.pool(n_layers=1)
    try:
        rng = synth.rng_for(2, B)
        ids, w = synth.zipf_routing(rng, B, 256, 8)
        blocks = {}
        for e in sorted(set(ids.ravel().tolist())):
            blocks[e] = synth.expert_block(rng, scale_dtype=L.FP16)
            pool.put(0, e, blocks[e])
        x = synth.activations(rng, B, 2048)
        sh = synth.shared_expert(rng, scale_dtype=L.FP16)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh])
        score = rng.normal(0, 1, size=B).astype(np.float32)
        h_mid = synth.activations(rng, B, 2048)
        out = ctx.moe_forward_host(pool, 0, x, ids, w, shared=shd, gate_score=score, h_mid=h_mid)
        cfg = dict(hidden=2048, inter=512, sd=L.FP16)
        want = _oracle_layer(blocks, ids, w, None, x, cfg, shared=sh, score=score, h_mid=h_mid)
        assert_close(out, want, f"full-size B={B}")
        # without residual/shared: the pure sum_k w_k * expert_k(x) of a single MoE layer
        out2 = ctx.moe_forward_host(pool, 0, x, ids, w)
        want2 = _oracle_layer(blocks, ids, w, None, x, cfg)
        assert_close(out2, want2, f"full-size routed only B={B}")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


@pytest.mark.parametrize("T", [9, 23, 64])
def test_moe_prefill_chunk_vs_oracle_and_per_token(api, T):
    """A prefill chunk must equal the oracle within tolerance and equal, bit for bit, the rows the
    decode entry point gives token by token (the reference's chunked == per-token claim, README.md:25)."""
    cfg = dict(hidden=256, inter=128, sd=L.BF16)
    ctx = api.Context(hidden=256, n_experts=16, top_k=8, moe_inter=128, shared_inter=128, n_layers=1,
                      scale_dtype=L.BF16, act_dtype=L.F32, max_tokens=64)
    ctx.set_prefill_mode(1)   # the sub-batch path: exact weights, fp32 activations, bit-identical to decode
    pool = ctx.pool()
    try:
        rng = synth.rng_for(3, T)
        blocks = {e: synth.expert_block(rng, 256, 128, 64, 3, L.BF16) for e in range(16)}
        for e, blk in blocks.items():
            pool.put(0, e, blk)
        x = rng.normal(0, 1, size=(T, 256)).astype(np.float32)
        ids, w = synth.zipf_routing(rng, T, 16, 8)
        sh = synth.shared_expert(rng, 256, 128, 64, 4, L.BF16)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh])
        score = rng.normal(0, 1, size=T).astype(np.float32)
        h_mid = rng.normal(0, 1, size=(T, 256)).astype(np.float32)
        out = ctx.moe_forward_host(pool, 0, x, ids, w, shared=shd, gate_score=score, h_mid=h_mid)
        want = _oracle_layer(blocks, ids, w, None, x, cfg, shared=sh, score=score, h_mid=h_mid)
        assert_close(out, want, f"prefill T={T}")
        for t in (0, T // 2, T - 1):
            one = ctx.moe_forward_host(pool, 0, x[t:t + 1], ids[t:t + 1], w[t:t + 1], shared=shd,
                                       gate_score=score[t:t + 1], h_mid=h_mid[t:t + 1])
            assert np.array_equal(one[0].view(np.uint32), out[t].view(np.uint32)), f"token {t} differs from per-token decode"
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


# ---------------------------------------------------------------------- pool
def test_pool_lru_and_roundtrip(api):
    ctx = api.Context(hidden=256, n_experts=8, top_k=8, moe_inter=128, shared_inter=128, n_layers=2, max_tokens=1)
    pool = ctx.pool(max_slots=3)
    try:
        rng = synth.rng_for(3, 0)
        blks = [synth.expert_block(rng, 256, 128, 64, 3, L.FP16) for _ in range(5)]
        for e in range(3):
            pool.put(0, e, blks[e])
        assert pool.lookup(0, 0) is not None      # touch 0: now 1 is the least recently used
        pool.put(0, 3, blks[3])                   # evicts expert 1
        assert pool.lookup(0, 1) is None
        assert pool.lookup(0, 0) is not None and pool.lookup(0, 3) is not None
        assert np.array_equal(pool.get(0, 3), blks[3])
        st = pool.stats()
        assert st["evictions"] == 1 and st["slots"] == 3 and st["used"] == 3 and st["misses"] == 1
        with pytest.raises(L.FinchError):
            pool.put(5, 0, blks[0])
    finally:
        pool.destroy()
        ctx.destroy()


def test_synthetic_fill_distribution_and_property_parity(api):
    """Device-generated pool: sample experts are read back and pushed through
    the oracle; every scale is finite, positive and small, bias == -4*scale."""
    ctx = api.Context(hidden=2048, n_experts=16, top_k=8, moe_inter=512, n_layers=2, max_tokens=2)
    pool = ctx.pool()
    try:
        pool.fill_synthetic(0, 2, 1234)
        Lo = synth.expert_layout()
        blk = pool.get(1, 5)
        s = blk[Lo["gate_s"]:Lo["gate_b"]].view(np.float16).astype(np.float32)
        b = blk[Lo["gate_b"]:Lo["up_w"]].view(np.float16).astype(np.float32)
        assert np.all(np.isfinite(s)) and np.all(s >= 0) and 0.004 < s.mean() < 0.012
        assert np.array_equal(b, (-4 * s).astype(np.float16).astype(np.float32))
        codes = orc.unpack_codes(blk[Lo["down_w"]:Lo["down_s"]], 2048, 512, 3)
        hist = np.bincount(codes.ravel(), minlength=8) / codes.size
        assert np.all(np.abs(hist - 0.125) < 0.01)
        assert not np.array_equal(blk, pool.get(1, 6)) and not np.array_equal(blk, pool.get(0, 5))
        rng = synth.rng_for(2, 77)
        x = synth.activations(rng, 2, 2048)
        ids, w = synth.zipf_routing(rng, 2, 16, 8)
        out = ctx.moe_forward_host(pool, 1, x, ids, w)
        blocks = {int(e): pool.get(1, int(e)) for e in set(ids.ravel().tolist())}
        want = _oracle_layer(blocks, ids, w, None, x, dict(hidden=2048, inter=512, sd=L.FP16))
        assert_close(out, want, "synthetic pool")
    finally:
        pool.destroy()
        ctx.destroy()


def test_event_wait_and_launch_count(api):
    import ctypes as C
    ctx = api.Context(hidden=256, n_experts=8, top_k=8, moe_inter=128, shared_inter=128, n_layers=1, max_tokens=1)
    try:
        ev = C.c_void_p()
        ctx.check(ctx.lib.finch_event_create(ctx.h, C.byref(ev)))
        ctx.check(ctx.lib.finch_event_record(ev, None))
        ctx.check(ctx.lib.finch_event_wait(ev, 2000))
        ctx.lib.finch_event_destroy(ev)
        n0 = ctx.launch_count()
        t = synth.affine_tensor(synth.rng_for(3, 3), 8, 64, 4, L.BF16)
        ctx.fast_dequant_matvec(ctx.upload_tensor(t), np.ones(64, np.float32))
        assert ctx.launch_count() == n0 + 1
    finally:
        ctx.destroy()


@pytest.mark.parametrize("T", [1, 8, 20])
def test_router_front_end_vs_oracle(api, T):
    """gate (BF16 rows, the default quantizer's choice) x h_post -> softmax / top-8 / renormalise, plus the shared
    expert's gate score, all on the device (finch_encode_router) against the oracle's matvec + route."""
    import torch
    ctx = api.Context(hidden=512, n_experts=64, top_k=8, moe_inter=128, shared_inter=128, n_layers=1, act_dtype=L.BF16, max_tokens=32)
    try:
        rng = synth.rng_for(16, T)
        gate = synth.f32_to_bf16_rne(rng.normal(0, 0.2, size=(64, 512)).astype(np.float32))
        sgate = synth.f32_to_bf16_rne(rng.normal(0, 0.2, size=(1, 512)).astype(np.float32))
        wg = ctx.upload_tensor(dict(W=gate, S=None, B=None, out_dim=64, in_dim=512, bits=0, scale_dtype=L.BF16))
        ws = ctx.upload_tensor(dict(W=sgate, S=None, B=None, out_dim=1, in_dim=512, bits=0, scale_dtype=L.BF16))
        x = synth.activations(rng, T, 512)
        xd = torch.from_numpy(x).cuda().to(torch.bfloat16)
        ids = torch.empty((T, 8), dtype=torch.int32, device="cuda")
        w = torch.empty((T, 8), dtype=torch.float32, device="cuda")
        score = torch.empty(T, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        import ctypes as C
        ctx.check(ctx.lib.finch_encode_router(ctx.h, None, C.byref(wg), C.byref(ws), xd.data_ptr(), ids.data_ptr(), w.data_ptr(),
                                              score.data_ptr(), T))
        ctx.sync()
        g64 = synth.bf16_to_f32(gate).astype(np.float64)
        for t in range(T):
            logits = (g64 @ x[t].astype(np.float64)).astype(np.float32)
            want_ids, want_w = orc.route(logits, 8)
            got_ids, got_w = ids[t].cpu().numpy(), w[t].cpu().numpy()
            assert sorted(got_ids.tolist()) == sorted(want_ids.tolist()), f"token {t}"
            order = {int(e): i for i, e in enumerate(want_ids)}
            assert np.allclose(got_w, want_w[[order[int(e)] for e in got_ids]], rtol=1e-4, atol=1e-6)
        want_s = synth.bf16_to_f32(sgate).astype(np.float64)[0] @ x.astype(np.float64).T
        assert np.allclose(score.cpu().numpy(), want_s, rtol=1e-4, atol=1e-5)
    finally:
        ctx.destroy()


@pytest.mark.parametrize("ad", [L.F32, L.BF16])
def test_residual_norm_vs_oracle(api, ad):
    import ctypes as C

    import torch
    ctx = api.Context(hidden=2048, n_layers=1, act_dtype=ad, max_tokens=4)
    try:
        rng = synth.rng_for(17, ad)
        T = 3
        resid, oproj = rng.normal(0, 1, (T, 2048)).astype(np.float32), rng.normal(0, 1, (T, 2048)).astype(np.float32)
        w = synth.f32_to_bf16_rne(rng.normal(1, 0.1, 2048).astype(np.float32))
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        rd, od, wd = d(resid), d(oproj), d(w.view(np.int16))
        h_mid = torch.empty((T, 2048), dtype=torch.float32, device="cuda")
        h_post = torch.empty((T, 2048), dtype=torch.float32 if ad == L.F32 else torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        for op in (od, None):
            ctx.check(ctx.lib.finch_encode_residual_norm(ctx.h, None, rd.data_ptr(), op.data_ptr() if op is not None else None, wd.data_ptr(),
                                                         C.c_float(1e-6), h_mid.data_ptr(), h_post.data_ptr(), T))
            ctx.sync()
            for t in range(T):
                want_mid, want_post = orc.residual_norm(resid[t], oproj[t] if op is not None else None, w, 1e-6)
                assert np.array_equal(h_mid[t].cpu().numpy(), want_mid)
                got = h_post[t].float().cpu().numpy()
                tol = 2e-6 if ad == L.F32 else 2 ** -8
                assert np.allclose(got, want_post, rtol=tol, atol=1e-6)
    finally:
        ctx.destroy()


@pytest.mark.parametrize("shape", ["all_same", "all_distinct", "one_hot_expert"])
def test_moe_decode_extreme_routings_full_size(api, shape):
    """Group sizes at their extremes, the model's shapes, batch 8: every token picks the same eight experts (eight groups of
    eight pairs), all 64 pairs distinct (64 groups of one), and one expert shared by all tokens next to distinct ones."""
    B = 8
    ctx = api.Context(max_tokens=8, n_layers=1)
    pool = ctx.pool(n_layers=1)
    try:
        rng = synth.rng_for(18, len(shape))
        if shape == "all_same":
            ids = np.tile(rng.permutation(256)[:8].astype(np.int32), (B, 1))
        elif shape == "all_distinct":
            ids = rng.permutation(256)[:64].astype(np.int32).reshape(B, 8)
        else:
            ids = rng.permutation(256)[:64].astype(np.int32).reshape(B, 8)
            ids[:, 3] = ids[0, 3]
        lg = rng.normal(0, 1, size=(B, 8))
        w = np.exp(lg - lg.max(axis=1, keepdims=True))
        w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
        blocks = {}
        for e in sorted(set(ids.ravel().tolist())):
            blocks[e] = synth.expert_block(rng, scale_dtype=L.FP16)
            pool.put(0, e, blocks[e])
        x = synth.activations(rng, B, 2048)
        out = ctx.moe_forward_host(pool, 0, x, ids, w)
        want = _oracle_layer(blocks, ids, w, None, x, dict(hidden=2048, inter=512, sd=L.FP16))
        assert_close(out, want, f"routing {shape}")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


def test_bounded_wait_runs_out_and_reports_timeout(api):
    """A warp of the gate/up kernel withholds its weight fetch (finch_debug_fault): the warps that wait for it give up
    after their (shortened) limit, the device status word reads FINCH_E_TIMEOUT, the host entry point returns that
    code, nothing hangs or faults, and after clearing the status the same context computes correct results again."""
    ctx, pool, blocks, cfg, rng = _mk_small(api, L.FP16, L.BF16, seed=77)
    try:
        x = synth.activations(rng, 4, 256)
        ids, w = synth.zipf_routing(rng, 4, 16, 8)
        good = ctx.moe_forward_host(pool, 1, x, ids, w)
        ctx.debug_fault(1)
        with pytest.raises(L.FinchError) as e:
            ctx.moe_forward_host(pool, 1, x, ids, w)
        assert e.value.status == L.E_TIMEOUT
        assert ctx.device_status() == L.E_TIMEOUT
        ctx.debug_fault(0)
        ctx.device_status_clear()
        assert ctx.device_status() == 0
        again = ctx.moe_forward_host(pool, 1, x, ids, w)
        assert np.array_equal(good.view(np.uint32), again.view(np.uint32))
        assert_close(again, _oracle_layer(blocks, ids, w, None, x, cfg), "after a timeout")
    finally:
        pool.destroy()
        ctx.destroy()


def test_host_path_top_k_4_more_than_8_tokens(api):
    """T = 12 with top_k = 4 is 48 pairs (fewer than 64) but more tokens than the decode entry takes: the host
    entry point must route it through the chunked path."""
    ctx = api.Context(hidden=256, n_experts=16, top_k=4, moe_inter=128, shared_inter=128, n_layers=1,
                      scale_dtype=L.FP16, act_dtype=L.BF16, max_tokens=16)
    rng = synth.rng_for(1, 512)
    pool = ctx.pool()
    try:
        blocks = {}
        for e in range(16):
            blocks[e] = synth.expert_block(rng, 256, 128, 64, 3, L.FP16)
            pool.put(0, e, blocks[e])
        x = synth.activations(rng, 12, 256)
        ids, w = synth.zipf_routing(rng, 12, 16, 4)
        out = ctx.moe_forward_host(pool, 0, x, ids, w)
        want = _oracle_layer(blocks, ids, w, None, x, dict(hidden=256, inter=128, sd=L.FP16))
        assert_close(out, want, "top_k=4, T=12")
    finally:
        pool.destroy()
        ctx.destroy()


def test_pool_put_between_decode_calls_with_fewer_slots_than_experts(api):
    """LRU mode (fewer slots than experts): puts that evict are interleaved with decode calls without any host
    synchronisation by the caller; every call must see the experts it was given."""
    import torch
    ctx = api.Context(hidden=256, n_experts=16, top_k=4, moe_inter=128, shared_inter=128, n_layers=1, scale_dtype=L.FP16,
                      act_dtype=L.BF16, max_tokens=2)
    pool = ctx.pool(max_slots=10)   # a call needs up to eight experts at once
    try:
        rng = synth.rng_for(1, 4242)
        blocks = {e: synth.expert_block(rng, 256, 128, 64, 3, L.FP16) for e in range(16)}
        cfg = dict(hidden=256, inter=128, sd=L.FP16)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        outs, wants = [], []
        for step in range(6):
            ids = np.stack([rng.permutation(16)[:4] for _ in range(2)]).astype(np.int32)
            w = rng.random((2, 4)).astype(np.float32)
            x = synth.activations(rng, 2, 256)
            for e in sorted(set(ids.ravel().tolist())):
                if pool.lookup(0, int(e)) is None:
                    pool.put(0, int(e), blocks[int(e)])     # evicts once the ten slots are taken
            out = torch.empty((2, 256), dtype=torch.float32, device="cuda")
            xd = d(synth.f32_to_bf16_rne(x)).view(torch.bfloat16)
            ctx.encode_moe_decode(pool, 0, xd, d(ids), d(w), None, None, None, out, 2)   # enqueued only
            outs.append((out, xd))
            resident = {e: blocks[e] for e in range(16)}
            wants.append(oracle_layer(resident, ids, w, None, x, cfg))
        ctx.sync()
        for step, ((out, _), want) in enumerate(zip(outs, wants)):
            assert_close(out.cpu().numpy(), want, f"step {step}")
        assert ctx.device_status() == 0 and pool.stats()["evictions"] > 0
    finally:
        pool.destroy()
        ctx.destroy()


@pytest.mark.parametrize("n_batches,B,own", [(2, 8, 1), (8, 8, 3), (4, 5, 0), (16, 2, 15)])
def test_moe_decode_multi_equals_the_batches_one_by_one(api, n_batches, B, own):
    """finch_encode_moe_decode_multi at full size (hidden 2048, inter 512, 256 experts, top-8): the pool holds the
    experts of one expert-parallel rank (every n_batches-th block of them), so most pairs of every row are skipped.
    Every batch must equal, bit for bit, what finch_encode_moe_decode gives for it alone (the own batch with h_mid
    and the shared expert, the others routed sums only); the own batch is also held against the oracle."""
    import torch
    ctx = api.Context(max_tokens=n_batches * B, n_layers=1)
    per = 256 // n_batches
    pool = ctx.pool(n_layers=1, max_slots=per)
    try:
        rng = synth.rng_for(31, n_batches * 100 + B)
        blocks = {}
        for e in range(own * per, (own + 1) * per):        # this rank's contiguous block of experts
            blocks[e] = synth.expert_block(rng, scale_dtype=L.FP16)
            pool.put(0, e, blocks[e])
        R = n_batches * B
        perm = synth.zipf_popularity(rng, 256)
        ids, w = synth.zipf_routing_shared(rng, R, perm, 8)
        valid = (rng.random((R, 8)) > 0.05).astype(np.uint8)
        x = synth.activations(rng, R, 2048)
        sh = synth.shared_expert(rng, scale_dtype=L.FP16)
        score = rng.normal(0, 1, size=B).astype(np.float32)
        h_mid = synth.activations(rng, B, 2048)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        xd = d(x).to(torch.bfloat16)
        idd, wd, vd, hd, sd = d(ids), d(w), d(valid), d(h_mid), d(score)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh], gate_score=sd)
        out = torch.zeros((B, 2048), dtype=torch.float32, device="cuda")
        rows = torch.full((R, 2048), 7.0, dtype=torch.float32, device="cuda")
        import ctypes as C
        ctx.check(ctx.lib.finch_encode_moe_decode_multi(ctx.h, None, pool.h, 0, n_batches, B, xd.data_ptr(), idd.data_ptr(), wd.data_ptr(), vd.data_ptr(),
                                                        own, C.byref(shd), hd.data_ptr(), out.data_ptr(), rows.data_ptr()))
        ctx.sync()
        torch.cuda.synchronize()
        one = torch.empty((B, 2048), dtype=torch.float32, device="cuda")
        for c in range(n_batches):
            sl = slice(c * B, (c + 1) * B)
            if c == own:
                ctx.encode_moe_decode(pool, 0, xd[sl], idd[sl], wd[sl], vd[sl], shd, hd, one, B)
            else:
                ctx.encode_moe_decode(pool, 0, xd[sl], idd[sl], wd[sl], vd[sl], None, None, one, B)
            ctx.sync()
            got = out if c == own else rows[sl]
            assert torch.equal(got, one), f"batch {c} differs from the single call"
        assert torch.all(rows[own * B:(own + 1) * B] == 7.0)           # the own block of rows_out is left alone
        sl = slice(own * B, (own + 1) * B)
        want = _oracle_layer(blocks, ids[sl], w[sl], valid[sl], x[sl], dict(hidden=2048, inter=512, sd=L.FP16), shared=sh, score=score, h_mid=h_mid)
        assert_close(out.cpu().numpy(), want, f"own batch of {n_batches} x {B}")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()
