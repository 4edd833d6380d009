"""GGUF expert MLP for decode (finch_encode_moe_gguf) against the oracle: Q4_K gate / up, Q6_K down (the Q4_K_M
mix), stacked slabs, the reference's guarded combine (finite-energy test and renormalisation)."""
import numpy as np
import pytest

from finchmoe_b200 import lib as L
from finchmoe_b200 import synth
from oracle import oracle
from parity import assert_close

pytestmark = pytest.mark.gpu


def _expert_out(gate, up, down, x):
    g = oracle.matvec(gate["W"], None, None, 1, x, gate["out_dim"], gate["in_dim"], 256, gate["bits"])
    u = oracle.matvec(up["W"], None, None, 1, x, up["out_dim"], up["in_dim"], 256, up["bits"])
    act = oracle.swiglu(g, u)
    return oracle.matvec(down["W"], None, None, 1, act, down["out_dim"], down["in_dim"], 256, down["bits"])


@pytest.mark.parametrize("types", [(12, 12, 14), (12, 14, 12), (14, 14, 14)])
@pytest.mark.parametrize("B", [1, 3])
def test_gguf_expert_moe_vs_oracle(types, B):
    import torch
    from finchmoe_b200 import api
    H, I, NE, K = 512, 256, 6, 4
    ctx = api.Context(hidden=H, n_experts=NE, top_k=K, moe_inter=I, shared_inter=256, n_layers=1, act_dtype=L.F32, max_tokens=4)
    try:
        rng = synth.rng_for(14, B, types[1])
        ex = [(synth.gguf_tensor(rng, I, H, types[0]), synth.gguf_tensor(rng, I, H, types[1]), synth.gguf_tensor(rng, H, I, types[2]))
              for _ in range(NE)]
        slabs = [np.stack([e[i]["W"] for e in ex]) for i in range(3)]          # [NE, rows, row_bytes]
        dev = [torch.from_numpy(s).cuda() for s in slabs]
        ge = L.GgufExperts(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), slabs[0][0].nbytes, slabs[1][0].nbytes, slabs[2][0].nbytes,
                           ex[0][0]["bits"], ex[0][1]["bits"], ex[0][2]["bits"])
        x = rng.normal(0, 1, size=(B, H)).astype(np.float32)
        ids = np.stack([rng.permutation(NE)[:K] for _ in range(B)]).astype(np.int32)
        w = rng.random((B, K)).astype(np.float32)
        w /= w.sum(axis=1, keepdims=True)
        valid = np.ones((B, K), np.uint8)
        valid[0, 1] = 0                       # a masked expert: the accepted weight drops below 0.99 -> renormalised
        if B > 1:
            ids[1, 2] = -1                    # an absent expert
        h_mid = rng.normal(0, 1, size=(B, H)).astype(np.float32)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        out = torch.empty((B, H), dtype=torch.float32, device="cuda")
        xd, idd, wd, vd, hd = d(x), d(ids), d(w), d(valid), d(h_mid)
        torch.cuda.synchronize()
        for rep in range(2):
            ctx.encode_moe_gguf(ge, xd, idd, wd, vd, hd, out, B)
        ctx.sync()
        got = out.cpu().numpy()
        for b in range(B):
            outs = np.zeros((K, H), np.float32)
            ok = np.zeros(K, np.uint8)
            for k in range(K):
                e = int(ids[b, k])
                if valid[b, k] and 0 <= e < NE:
                    outs[k] = _expert_out(*ex[e], x[b])
                    ok[k] = 1
            want = oracle.combine(h_mid[b], outs, w[b], ok, np.zeros(H, np.float32), 0.0, guard=1)
            assert_close(got[b], want, f"GGUF MoE types={types} token {b}")
        assert ctx.device_status() == 0
    finally:
        ctx.destroy()


def test_gguf_expert_moe_full_size_vs_oracle():
    """The model's own dimensions: hidden 2048, expert intermediate 512, 256 experts, top-8; Q4_K gate / up and Q6_K
    down slabs.  Only the experts that are routed to carry data (the other slabs stay zero)."""
    import torch
    from finchmoe_b200 import api
    H, I, NE, K, B = 2048, 512, 256, 8, 2
    ctx = api.Context(hidden=H, n_experts=NE, top_k=K, moe_inter=I, shared_inter=512, n_layers=1, act_dtype=L.F32, max_tokens=4)
    try:
        rng = synth.rng_for(14, 2048)
        ids, w = synth.zipf_routing(rng, B, NE, K)
        used = sorted(set(ids.ravel().tolist()))
        ex = {e: (synth.gguf_tensor(rng, I, H, 12), synth.gguf_tensor(rng, I, H, 12), synth.gguf_tensor(rng, H, I, 14)) for e in used}
        proto = ex[used[0]]
        slabs = [np.zeros((NE,) + proto[i]["W"].shape, np.uint8) for i in range(3)]
        for e in used:
            for i in range(3):
                slabs[i][e] = ex[e][i]["W"]
        dev = [torch.from_numpy(s).cuda() for s in slabs]
        ge = L.GgufExperts(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), slabs[0][0].nbytes, slabs[1][0].nbytes, slabs[2][0].nbytes,
                           proto[0]["bits"], proto[1]["bits"], proto[2]["bits"])
        x = (synth.activations(rng, B, H) + rng.normal(0, 1e-3, size=(B, H))).astype(np.float32)
        h_mid = synth.activations(rng, B, H)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        out = torch.empty((B, H), dtype=torch.float32, device="cuda")
        xd, idd, wd, hd = d(x), d(ids), d(w), d(h_mid)
        torch.cuda.synchronize()
        ctx.encode_moe_gguf(ge, xd, idd, wd, None, hd, out, B)
        ctx.sync()
        got = out.cpu().numpy()
        for b in range(B):
            outs = np.stack([_expert_out(*ex[int(e)], x[b]) for e in ids[b]])
            want = oracle.combine(h_mid[b], outs, w[b], np.ones(K, np.uint8), np.zeros(H, np.float32), 0.0, guard=1)
            assert_close(got[b], want, f"GGUF MoE at model size, token {b}")
        assert ctx.device_status() == 0
    finally:
        ctx.destroy()


@pytest.mark.parametrize("types", [(12, 12, 14), (12, 14, 12), (14, 14, 14)])
@pytest.mark.parametrize("B,act_dtype", [(9, L.F32), (40, L.BF16), (90, L.F32)])
def test_gguf_expert_prefill_chunk_grouped_by_expert_vs_oracle_and_per_token(types, B, act_dtype):
    """A chunk of 9 and more tokens: the pairs are sorted by expert and every selected expert's rows are read once for
    all its tokens (de-duplication).  Few experts, so that several get more than 32 and more than 64 pairs (both item
    lists, chunks of one expert); masked pairs, absent experts, a token with every pair masked.  Against the oracle,
    and against the token-by-token path of the same entry point."""
    import torch
    from finchmoe_b200 import api
    H, I, NE, K = 512, 256, 6, 4
    ctx = api.Context(hidden=H, n_experts=NE, top_k=K, moe_inter=I, shared_inter=256, n_layers=1, act_dtype=act_dtype, max_tokens=128)
    try:
        rng = synth.rng_for(16, B, types[1])
        ex = [(synth.gguf_tensor(rng, I, H, types[0]), synth.gguf_tensor(rng, I, H, types[1]), synth.gguf_tensor(rng, H, I, types[2]))
              for _ in range(NE)]
        slabs = [np.stack([e[i]["W"] for e in ex]) for i in range(3)]
        dev = [torch.from_numpy(s).cuda() for s in slabs]
        ge = L.GgufExperts(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), slabs[0][0].nbytes, slabs[1][0].nbytes, slabs[2][0].nbytes,
                           ex[0][0]["bits"], ex[0][1]["bits"], ex[0][2]["bits"])
        x = synth.activations(rng, B, H)
        if act_dtype == L.F32:
            x = (x * (1.0 + rng.normal(0, 1e-3, size=x.shape))).astype(np.float32)
        # expert 0 is in almost every token's set, expert 5 in few
        pop = np.array([0.45, 0.2, 0.15, 0.1, 0.07, 0.03])
        ids = np.stack([rng.choice(NE, size=K, replace=False, p=pop) for _ in range(B)]).astype(np.int32)
        w = rng.random((B, K)).astype(np.float32)
        w /= w.sum(axis=1, keepdims=True)
        valid = (rng.random((B, K)) > 0.1).astype(np.uint8)
        valid[3] = 0                          # nothing selected: the row is h_mid
        ids[5, 2] = -1                        # an absent expert
        ids[6, 0] = NE                        # an id out of range
        h_mid = rng.normal(0, 1, size=(B, H)).astype(np.float32)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        xd = d(x) if act_dtype == L.F32 else d(synth.f32_to_bf16_rne(x)).view(torch.bfloat16)
        idd, wd, vd, hd = d(ids), d(w), d(valid), d(h_mid)
        out = torch.empty((B, H), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        for rep in range(2):
            ctx.encode_moe_gguf(ge, xd, idd, wd, vd, hd, out, B)
        ctx.sync()
        got = out.cpu().numpy()
        assert np.all(np.isfinite(got))
        # token by token through the same entry point (calls of at most 8 tokens take the per-token path)
        one = torch.empty((B, H), dtype=torch.float32, device="cuda")
        for b0 in range(0, B, 8):
            n = min(8, B - b0)
            ctx.encode_moe_gguf(ge, xd[b0:b0 + n], idd[b0:b0 + n], wd[b0:b0 + n], vd[b0:b0 + n], hd[b0:b0 + n], one[b0:b0 + n], n)
        ctx.sync()
        assert_close(got, one.cpu().numpy(), f"grouped chunk against the per-token path, B={B}")
        for b in list(range(8)) + [B - 1]:
            outs = np.zeros((K, H), np.float32)
            ok = np.zeros(K, np.uint8)
            for k in range(K):
                e = int(ids[b, k])
                if valid[b, k] and 0 <= e < NE:
                    outs[k] = _expert_out(*ex[e], x[b])
                    ok[k] = 1
            want = oracle.combine(h_mid[b], outs, w[b], ok, np.zeros(H, np.float32), 0.0, guard=1)
            assert_close(got[b], want, f"grouped GGUF MoE types={types} B={B} token {b}")
        assert ctx.device_status() == 0
    finally:
        ctx.destroy()
