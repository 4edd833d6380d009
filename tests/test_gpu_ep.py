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
        be.home_direct = be.planned_direct = direct      # False: the rank's own rows also go through pack / unpack / combine
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


def _two_ranks_one_process(api, T=8):
    """Two ranks' contexts, sharded pools and connected peer areas on one GPU, plus a full pool for the yardstick."""
    NE, H, I = 16, 256, 128
    rng = synth.rng_for(14, 1)
    blocks = {e: synth.expert_block(rng, H, I, 64, 3, L.BF16) for e in range(NE - 1)}      # expert 15 is nowhere
    sh = synth.shared_expert(rng, H, I, 64, 4, L.BF16)
    ranks = []
    for r in range(2):
        ctx = _ctx(api, max_tokens=2 * T)
        pool = ctx.pool(max_slots=8)
        for e in range(r * 8, r * 8 + 8):
            if e in blocks:
                pool.put(0, e, blocks[e])
        be = ep.GpuBackend(ctx, pool, 2 * T)
        be.peer = ep.PeerExchange(ctx, r, 2, T)
        ranks.append((ctx, pool, be))
    ranks[0][2].peer.attach(1, ranks[1][2].peer.area())
    ranks[1][2].peer.attach(0, ranks[0][2].peer.area())
    return blocks, sh, ranks


@pytest.mark.parametrize("multi", [False, True, "fused"])
def test_peer_exchange_two_ranks_in_one_process_match_oracle(multi):
    """The exchange through peer memory (dispatch / receive / return / combine with one flag per slot), its two
    ranks run from one process on one GPU: each step of both ranks is launched before the step that waits for it, so
    no kernel ever waits for one that has not run.  Twice, so that the cleared flags are exercised."""
    import torch
    from finchmoe_b200 import api
    from oracle import oracle
    T, H, I, K = 8, 256, 128, 8
    blocks, sh, ranks = _two_ranks_one_process(api, T)
    try:
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        for rep in range(2):
            inputs, outs = [], []
            for r in range(2):
                r2 = synth.rng_for(14, 2 + rep, r)
                x = synth.activations(r2, T, H)
                ids, w = synth.zipf_routing(r2, T, 16, K)
                valid = (r2.random((T, K)) > 0.1).astype(np.uint8)
                score = r2.normal(0, 1, size=T).astype(np.float32)
                h_mid = r2.normal(0, 1, size=(T, H)).astype(np.float32)
                ctx = ranks[r][0]
                score_d = d(score)
                shd = ctx.make_shared(*[ctx.upload_tensor(t) for t in sh], gate_score=score_d)
                inputs.append((x, ids, w, valid, score, h_mid, d(x), d(ids), d(w), d(valid), shd, d(h_mid), score_d))
                outs.append(torch.zeros((T, H), dtype=torch.float32, device="cuda"))
            for r, (ctx, pool, be) in enumerate(ranks):
                with be.stream_scope():
                    be.peer_dispatch(*inputs[r][6:10])
            torch.cuda.synchronize()
            for r, (ctx, pool, be) in enumerate(ranks):
                with be.stream_scope():
                    if multi == "fused":   # ... whose last kernel also stores the other rank's rows into its area
                        assert be.can_multi(T, 2)
                        be.peer_decode(0, inputs[r][10], inputs[r][11], outs[r])
                        continue
                    if multi:       # every rank's batch, the rank's own among them, in one launch sequence
                        assert be.can_multi(T, 2)
                        part = be.peer_local_multi(0, T, 2, r, inputs[r][10], inputs[r][11], outs[r])
                    else:
                        be.home(0, *inputs[r][6:10], inputs[r][10], inputs[r][11], outs[r])
                        part = be.peer_local_moe(0, 2 * T, (r * T, T))
                    be.peer_return(part)
            torch.cuda.synchronize()
            for r, (ctx, pool, be) in enumerate(ranks):
                with be.stream_scope():
                    be.peer_combine(outs[r])
            torch.cuda.synchronize()
            for r, (ctx, pool, be) in enumerate(ranks):
                x, ids, w, valid, score, h_mid = inputs[r][:6]
                want = np.stack([oracle.moe_layer([blocks.get(int(e)) if valid[t, k] else None for k, e in enumerate(ids[t])], w[t],
                                                  np.array([1 if (valid[t, k] and int(e) in blocks) else 0 for k, e in enumerate(ids[t])], np.uint8),
                                                  x[t], bits=3, scale_dtype=oracle.SCALE_BF16, hidden=H, inter=I, h_mid=h_mid[t], shared=sh,
                                                  shared_gate_score=float(score[t])) for t in range(T)])
                assert_close(outs[r].cpu().numpy(), want, f"peer exchange, rank {r}, pass {rep}, multi={multi}")
                assert ctx.device_status() == 0
    finally:
        for ctx, pool, be in ranks:
            be.peer.destroy()
            pool.destroy()
            ctx.destroy()


def test_peer_receive_wait_runs_out_and_reports_timeout():
    """Nobody dispatches: the receive kernel's bounded wait gives up after a fraction of a millisecond, records
    FINCH_E_TIMEOUT in the device status word, masks the rows it did not get and returns; the context stays usable
    (the same exchange then works after a reset)."""
    import torch
    from finchmoe_b200 import api
    T = 8
    blocks, sh, ranks = _two_ranks_one_process(api, T)
    try:
        ctx, pool, be = ranks[0]
        be.peer.set_wait_limit(2000)
        be.rv.fill_(1)
        with be.stream_scope():
            be.peer_receive(True)
        torch.cuda.synchronize()
        assert ctx.device_status() == L.E_TIMEOUT
        assert int(be.rv[:2 * T].sum().item()) == 0            # nothing arrived: every row is masked
        out = torch.zeros((T, 256), dtype=torch.float32, device="cuda")
        with be.stream_scope():
            be.peer_combine(out)                               # the status word is set: this wait does not spin
        torch.cuda.synchronize()
        assert float(out.abs().sum().item()) == 0.0
        ctx.device_status_clear()
        be.peer.reset()
        assert ctx.device_status() == 0
    finally:
        for ctx, pool, be in ranks:
            be.peer.destroy()
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
# decode-sized batches (8 rows per rank): both ranks' batches in one launch sequence, over the all-to-alls
a8 = (d(x[:8]), d(ids[:8]), d(w[:8]), d(valid[:8]), shd, d(h_mid[:8]), torch.zeros((8, H), dtype=torch.float32, device="cuda"))
assert be.can_multi(8, world)
ep.ep_layer_static(be, dist, None, 0, *a8)
torch.cuda.synchronize()
assert_close(a8[-1].cpu().numpy(), want[:8], f"rank {rank} multi-batch decode over NCCL")
# ... and through peer memory
px8 = ep.PeerExchange.connect(ctx, dist, None, 8)
assert px8 is not None, "the ranks could not map each other's receive areas"
be.peer = px8
for rep in range(2):
    a8[-1].zero_()
    ep.ep_layer_static(be, dist, None, 0, *a8)
torch.cuda.synchronize()
assert_close(a8[-1].cpu().numpy(), want[:8], f"rank {rank} multi-batch decode over peer memory")
assert ctx.device_status() == 0
dist.barrier()
# the same layer with the exchange through peer memory instead of the all-to-alls: from the host, then from a graph
be.peer = ep.PeerExchange.connect(ctx, dist, None, Ts)
assert be.peer is not None, "the ranks could not map each other's receive areas"
args[-1].zero_()
ep.ep_layer_static(be, dist, None, 0, *args)
torch.cuda.synchronize()
assert_close(args[-1].cpu().numpy(), want[:Ts], f"rank {rank} peer exchange")
dist.barrier()
g2 = torch.cuda.CUDAGraph()
with torch.cuda.graph(g2, stream=be.stream, capture_error_mode="thread_local"):
    ep.ep_layer_static(be, dist, None, 0, *args, in_scope=True)
for rep in range(3):
    args[-1].zero_()
    g2.replay()
torch.cuda.synchronize()
assert_close(args[-1].cpu().numpy(), want[:Ts], f"rank {rank} peer exchange, graph replay")
assert ctx.device_status() == 0
dist.barrier()
del g2
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
