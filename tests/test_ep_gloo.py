"""The expert-parallel protocol (finchmoe_b200/ep.py) on CPU: two gloo ranks, numpy backend, oracle
arithmetic.  Checks the plan (one record per token and destination), the variable-size all-to-alls and the
fixed-order combine against a single-process oracle run over all experts."""
import os
import subprocess
import sys

import numpy as np

from finchmoe_b200 import ep, synth

HERE = os.path.dirname(os.path.abspath(__file__))


def test_plan_sends_a_token_once_per_rank_and_skips_unusable_pairs():
    ids = np.array([[0, 1, 4, 7], [5, 6, 7, 4], [2, 3, 0, 1], [9, -1, 3, 3]], np.int32)   # 8 experts, 2 ranks: 0-3 | 4-7
    valid = np.ones_like(ids, dtype=np.uint8)
    valid[0, 2] = 0                                  # token 0's expert 4 is masked; expert 7 still sends it to rank 1
    counts, offs, send_tok, slot_of = ep.plan_numpy(ids, valid, 8, 2)
    assert counts.tolist() == [3, 2]                 # rank 0: tokens 0, 2, 3; rank 1: tokens 0, 1
    assert offs.tolist() == [0, 3, 5]
    assert send_tok.tolist() == [0, 2, 3, 0, 1]
    assert slot_of.tolist() == [[0, 0], [-1, 1], [1, -1], [2, -1]]
    # a token whose pairs are all unusable goes nowhere
    c2, _, _, s2 = ep.plan_numpy(np.array([[8, -5]], np.int32), None, 8, 2)
    assert c2.tolist() == [0, 0] and s2.tolist() == [[-1, -1]]


def test_plan_leaves_out_the_home_rank_when_asked():
    rng = synth.rng_for(21, 3)
    ids = rng.integers(0, 16, size=(50, 8)).astype(np.int32)
    full = ep.plan_numpy(ids, None, 16, 4)
    cut = ep.plan_numpy(ids, None, 16, 4, skip=2)
    assert cut[0][2] == 0 and np.all(cut[3][:, 2] == -1)
    for d in (0, 1, 3):                                   # the other destinations keep their lists
        assert cut[0][d] == full[0][d]
        assert np.array_equal(cut[3][:, d], full[3][:, d])
        assert cut[2][cut[1][d]:cut[1][d + 1]].tolist() == full[2][full[1][d]:full[1][d + 1]].tolist()
    assert cut[1][-1] == full[1][-1] - full[0][2]


def test_static_plan_sends_every_token_to_every_rank():
    counts, offs, send_tok, slot_of = ep.static_plan_numpy(3, 4)
    assert counts.tolist() == [3, 3, 3, 3] and offs.tolist() == [0, 3, 6, 9, 12]
    assert send_tok.tolist() == [0, 1, 2] * 4
    assert slot_of.tolist() == [[0] * 4, [1] * 4, [2] * 4]
    # the home rank's column is left out of the combine step when it adds its own share directly
    assert ep.static_plan_numpy(3, 4, skip=2)[3].tolist() == [[0, 0, -1, 0], [1, 1, -1, 1], [2, 2, -1, 2]]


WORKER = r'''
import os, sys
sys.path.insert(0, sys.argv[3]); sys.path.insert(0, os.path.dirname(sys.argv[3]))
import numpy as np, torch, torch.distributed as dist
from finchmoe_b200 import ep, synth
from oracle import oracle
from ep_cpu_backend import NumpyBackend
rank, world = int(sys.argv[1]), int(sys.argv[5])
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:" + sys.argv[2], rank=rank, world_size=world)
cfg = dict(hidden=256, inter=128, n_experts=8, K=4, sd=oracle.SCALE_BF16)
rng = synth.rng_for(9, 1)                          # both ranks draw the same model
blocks = {e: synth.expert_block(rng, 256, 128, 64, 3, cfg["sd"]) for e in range(8)}
shared = synth.shared_expert(rng, 256, 128, 64, 4, cfg["sd"])
T = (5, 7, 3, 6)[rank]                             # ragged: the ranks own different numbers of tokens
if sys.argv[4] == "static":
    T = 6                                          # the fixed-capacity exchange wants the same count everywhere
r2 = synth.rng_for(9, 2, rank)
x = r2.normal(0, 1, size=(T, 256)).astype(np.float32)
ids, w = synth.zipf_routing(r2, T, 8, 4)
if sys.argv[4] == "one_sided":                     # every token picks rank 0's experts only: rank 1 receives nothing
    ids = np.stack([r2.permutation(4) for _ in range(T)]).astype(np.int32)
valid = (r2.random((T, 4)) > 0.2).astype(np.uint8)
if rank == 1:
    valid[0] = 0                                   # a token with no usable expert at all
score = r2.normal(0, 1, size=T).astype(np.float32)
h_mid = r2.normal(0, 1, size=(T, 256)).astype(np.float32)
per = 8 // world
backend = NumpyBackend(cfg, {e: b for e, b in blocks.items() if e // per == rank}, shared)
out = torch.empty((T, 256), dtype=torch.float32)
layer_fn = ep.ep_layer_static if sys.argv[4] == "static" else ep.ep_layer
layer_fn(backend, dist, None, 0, torch.from_numpy(x), torch.from_numpy(ids), torch.from_numpy(w), torch.from_numpy(valid),
         score, torch.from_numpy(h_mid), out)
want = np.stack([oracle.moe_layer([blocks[int(e)] if valid[t, k] else None for k, e in enumerate(ids[t])], w[t], valid[t], x[t], bits=3,
                                  scale_dtype=cfg["sd"], hidden=256, inter=128, h_mid=h_mid[t], shared=shared,
                                  shared_gate_score=float(score[t])) for t in range(T)])
err = np.abs(out.numpy() - want).max() / np.sqrt((want.astype(np.float64) ** 2).mean())
assert err < 1e-5, err                             # same arithmetic, only the order of the fp32 additions differs
dist.barrier()
dist.destroy_process_group()
print("rank", rank, "ok", err)
'''


import pytest


@pytest.mark.parametrize("mode,world", [("mixed", 2), ("one_sided", 2), ("static", 2), ("mixed", 4), ("static", 4)])
def test_ranks_match_single_process_oracle(tmp_path, mode, world):
    script = tmp_path / "ep_worker.py"
    script.write_text(WORKER)
    port = str(29600 + (os.getpid() + {"mixed": 7, "one_sided": 13, "static": 19}[mode] + 31 * world) % 300)
    procs = [subprocess.Popen([sys.executable, str(script), str(r), port, HERE, mode, str(world)], stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                              text=True) for r in range(world)]
    outs = [p.communicate(timeout=240)[0] for p in procs]
    for r, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {r} failed:\n{o[-3000:]}"
        assert f"rank {r} ok" in o
