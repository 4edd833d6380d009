"""Expert-parallel layer on GPUs: the device plan against its host mirror, the single-rank protocol
against the plain layer, and (with two GPUs) two NCCL ranks against the oracle."""
import os
import subprocess
import sys

import numpy as np
import pytest

from finchmoe_b200 import ep, synth
from finchmoe_b200 import lib as L
from parity import assert_close

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _ctx(api, **kw):
    return api.Context(hidden=256, n_experts=16, top_k=8, moe_inter=128, shared_inter=128, n_layers=1, scale_dtype=L.BF16,
                       act_dtype=L.F32, **kw)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_device_plan_matches_host_mirror(world):
    import torch
    from finchmoe_b200 import api
    ctx = _ctx(api, max_tokens=8)
    try:
        rng = synth.rng_for(11, world)
        for T in (1, 33, 1500):
            ids = rng.integers(-1, 17, size=(T, 8)).astype(np.int32)       # includes out-of-range ids
            valid = (rng.random((T, 8)) > 0.3).astype(np.uint8)
            be = ep.GpuBackend(ctx, ctx.pool(max_slots=1), 8)
            for v in (valid, None):
                p = be.plan(torch.from_numpy(ids).cuda(), None if v is None else torch.from_numpy(v).cuda(), world)
                torch.cuda.synchronize()
                counts, offs, send_tok, slot_of = ep.plan_numpy(ids, v, 16, world)
                assert p.counts.cpu().numpy().tolist() == counts.tolist()
                assert p.offs.cpu().numpy().tolist() == offs.tolist()
                assert p.send_tok.cpu().numpy()[:offs[-1]].tolist() == send_tok.tolist()
                assert np.array_equal(p.slot_of.cpu().numpy(), slot_of)
            # nothing goes to the rank that is left out (the home rank, when it works on its own tokens in place)
            skip = world - 1
            p = be.plan(torch.from_numpy(ids).cuda(), torch.from_numpy(valid).cuda(), world, skip)
            torch.cuda.synchronize()
            counts, offs, send_tok, slot_of = ep.plan_numpy(ids, valid, 16, world, skip)
            assert counts[skip] == 0 and np.all(slot_of[:, skip] == -1)
            assert p.counts.cpu().numpy().tolist() == counts.tolist()
            assert p.offs.cpu().numpy().tolist() == offs.tolist()
            assert p.send_tok.cpu().numpy()[:offs[-1]].tolist() == send_tok.tolist()
            assert np.array_equal(p.slot_of.cpu().numpy(), slot_of)
            be.pool.destroy()
    finally:
        ctx.destroy()


@pytest.mark.parametrize("T", [5, 40, 200])
@pytest.mark.parametrize("static", [False, True])
@pytest.mark.parametrize("direct", [False, True])
def test_single_rank_protocol_matches_plain_layer(T, static, direct):
    import torch
    from finchmoe_b200 import api
    ctx = _ctx(api, max_tokens=256)
    pool = ctx.pool()
    try:
        rng = synth.rng_for(12, T)
        for e in range(15):                                                  # expert 15 stays absent
            pool.put(0, e, synth.expert_block(rng, 256, 128, 64, 3, L.BF16))
        x = synth.activations(rng, T, 256)
        ids, w = synth.zipf_routing(rng, T, 16, 8)
        valid = (rng.random((T, 8)) > 0.1).astype(np.uint8)
        sh = synth.shared_expert(rng, 256, 128, 64, 4, L.BF16)
        score = rng.normal(0, 1, size=T).astype(np.float32)
        h_mid = rng.normal(0, 1, size=(T, 256)).astype(np.float32)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        score_d = d(score)
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh], gate_score=score_d)
        want = ctx.moe_forward_host(pool, 0, x, ids, w, valid=valid, shared=shd, gate_score=score, h_mid=h_mid)
        be = ep.GpuBackend(ctx, pool, T)
        be.home_direct = direct      # False: the rank's own rows also go through pack / unpack / combine
        out = torch.empty((T, 256), dtype=torch.float32, device="cuda")
        (ep.ep_layer_static if static else ep.ep_layer)(be, None, None, 0, d(x), d(ids), d(w), d(valid), shd, d(h_mid), out)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), want, f"single-rank protocol T={T} static={static} direct={direct}")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


def test_single_rank_protocol_with_nothing_to_send():
    """Every pair masked: the plan sends no row anywhere, pack and unpack see zero rows (and NULL-sized buffers), and
    the layer is h_mid + the gated shared expert."""
    import torch
    from finchmoe_b200 import api
    T = 6
    ctx = _ctx(api, max_tokens=8)
    pool = ctx.pool()
    try:
        rng = synth.rng_for(12, 999)
        for e in range(16):
            pool.put(0, e, synth.expert_block(rng, 256, 128, 64, 3, L.BF16))
        x = synth.activations(rng, T, 256)
        ids, w = synth.zipf_routing(rng, T, 16, 8)
        valid = np.zeros((T, 8), np.uint8)
        sh = synth.shared_expert(rng, 256, 128, 64, 4, L.BF16)
        score = rng.normal(0, 1, size=T).astype(np.float32)
        h_mid = rng.normal(0, 1, size=(T, 256)).astype(np.float32)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh], gate_score=d(score))
        want = ctx.moe_forward_host(pool, 0, x, ids, w, valid=valid, shared=shd, gate_score=score, h_mid=h_mid)
        be = ep.GpuBackend(ctx, pool, T)
        out = torch.empty((T, 256), dtype=torch.float32, device="cuda")
        ep.ep_layer(be, None, None, 0, d(x), d(ids), d(w), d(valid), shd, d(h_mid), out)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), want, "nothing to send")
        assert ctx.device_status() == 0
    finally:
        pool.destroy()
        ctx.destroy()


WORKER = r'''
import os, sys
sys.path.insert(0, sys.argv[3]); sys.path.insert(0, os.path.dirname(sys.argv[3]))
import numpy as np, torch, torch.distributed as dist
rank, world = int(sys.argv[1]), int(sys.argv[4])
torch.cuda.set_device(rank)
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
dist.init_process_group("nccl", init_method="tcp://127.0.0.1:" + sys.argv[2], rank=rank, world_size=world, device_id=torch.device("cuda", rank))
from finchmoe_b200 import api, ep, synth, lib as L
from oracle import oracle
from parity import assert_close
NE, K, H, I = 16, 8, 256, 128
ctx = api.Context(device=rank, hidden=H, n_experts=NE, top_k=K, moe_inter=I, shared_inter=I, n_layers=1, scale_dtype=L.BF16, act_dtype=L.F32, max_tokens=64)
per = NE // world
pool = ctx.pool(max_slots=per)
rng = synth.rng_for(13, 1)
blocks = {e: synth.expert_block(rng, H, I, 64, 3, L.BF16) for e in range(NE)}
sh = synth.shared_expert(rng, H, I, 64, 4, L.BF16)
for e in range(rank * per, (rank + 1) * per):
    pool.put(0, e, blocks[e])
T = 37 + 11 * rank
r2 = synth.rng_for(13, 2, rank)
x = synth.activations(r2, T, H)
ids, w = synth.zipf_routing(r2, T, NE, K)
valid = (r2.random((T, K)) > 0.1).astype(np.uint8)
score = r2.normal(0, 1, size=T).astype(np.float32)
h_mid = r2.normal(0, 1, size=(T, H)).astype(np.float32)
d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
score_d = d(score)
shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh], gate_score=score_d)
be = ep.GpuBackend(ctx, pool, 64 * world)
out = torch.empty((T, H), dtype=torch.float32, device="cuda")
for rep in range(2):
    ep.ep_layer(be, dist, None, 0, d(x), d(ids), d(w), d(valid), shd, d(h_mid), out)
torch.cuda.synchronize()
want = np.stack([oracle.moe_layer([blocks[int(e)] if valid[t, k] else None for k, e in enumerate(ids[t])], w[t], valid[t], x[t], bits=3,
                                  scale_dtype=oracle.SCALE_BF16, hidden=H, inter=I, h_mid=h_mid[t], shared=sh,
                                  shared_gate_score=float(score[t])) for t in range(T)])
assert_close(out.cpu().numpy(), want, f"rank {rank}")
# fixed-capacity exchange (same token count on every rank), launched from the host and replayed from a CUDA graph
Ts = 32
args = (d(x[:Ts]), d(ids[:Ts]), d(w[:Ts]), d(valid[:Ts]), shd, d(h_mid[:Ts]), torch.zeros((Ts, H), dtype=torch.float32, device="cuda"))
ep.ep_layer_static(be, dist, None, 0, *args)
torch.cuda.synchronize()
assert_close(args[-1].cpu().numpy(), want[:Ts], f"rank {rank} fixed capacity")
args[-1].zero_()
torch.cuda.synchronize()
dist.barrier()
g = torch.cuda.CUDAGraph()
with torch.cuda.graph(g, stream=be.stream, capture_error_mode="thread_local"):
    ep.ep_layer_static(be, dist, None, 0, *args, in_scope=True)
for rep in range(2):
    g.replay()
torch.cuda.synchronize()
assert_close(args[-1].cpu().numpy(), want[:Ts], f"rank {rank} fixed capacity, graph replay")
assert ctx.device_status() == 0
del g                                   # the graph holds the recorded all-to-alls: it goes before the communicator
torch.cuda.synchronize()
dist.barrier()
print("rank", rank, "ok", flush=True)
os._exit(0)                             # leave without tearing NCCL down after a capture
'''


@pytest.mark.parametrize("world", [2])
def test_two_nccl_ranks_match_oracle(tmp_path, world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    script = tmp_path / "ep_worker.py"
    script.write_text(WORKER)
    port = str(29900 + os.getpid() % 90)
    procs = [subprocess.Popen([sys.executable, str(script), str(r), port, HERE, str(world)], stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                              text=True) for r in range(world)]
    outs = [p.communicate(timeout=600)[0] for p in procs]
    for r, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {r} failed:\n{o[-3000:]}"
