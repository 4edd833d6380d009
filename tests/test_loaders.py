"""Loaders for the reference's on-disk formats: the parsing runs on CPU against files written the way the
reference writes them (repack_experts.py:137-151, 540-551; quantize_non_experts.py:366-445); the GPU tests load
such files into a pool / device buffer and check the bytes and a matvec."""
import json
import os

import numpy as np
import pytest

from finchmoe_b200 import loaders, synth
from finchmoe_b200 import lib as L


def _write_expert_dir(d, blocks_by_layer, hidden, inter):
    size = blocks_by_layer[0][0].size
    comps, off = [], 0
    for name, (o, i) in (("gate_proj", (inter, hidden)), ("up_proj", (inter, hidden)), ("down_proj", (hidden, inter))):
        for suffix, sz, dt, shape in ((".weight", o * i * 3 // 8, "U8", [o, i * 3 // 8]), (".scales", o * (i // 64) * 2, "BF16", [o, i // 64]),
                                      (".biases", o * (i // 64) * 2, "BF16", [o, i // 64])):
            comps.append({"name": name + suffix, "offset": off, "size": sz, "dtype": dt, "shape": shape})
            off += sz
    assert off == size
    with open(os.path.join(d, "layout.json"), "w") as f:
        json.dump({"expert_size": size, "num_layers": len(blocks_by_layer), "num_experts": len(blocks_by_layer[0]), "components": comps}, f)
    for l, blocks in enumerate(blocks_by_layer):
        with open(os.path.join(d, f"layer_{l:02d}.bin"), "wb") as f:
            for b in blocks:
                f.write(b.tobytes())


def _write_weight_dir(d, tensors):
    """tensors: name -> affine dict (synth.affine_tensor with BF16 scales) or bf16 array; 64-byte alignment like the reference."""
    manifest, blob, off = {"tensors": {}}, bytearray(), 0

    def put(name, data, shape, dtype, **extra):
        nonlocal off
        pad = (-off) % 64
        blob.extend(b"\0" * pad)
        off += pad
        manifest["tensors"][name] = dict(offset=off, size=len(data), shape=shape, dtype=dtype, **extra)
        blob.extend(data)
        off += len(data)
    for name, t in tensors.items():
        if isinstance(t, dict):
            words = t["W"].view(np.uint32).reshape(t["out_dim"], -1)
            put(name + ".weight", words.tobytes(), list(words.shape), "U32", bits=t["bits"], group_size=64)
            put(name + ".scales", t["S"].tobytes(), list(t["S"].shape), "BF16", bits=t["bits"], group_size=64)
            put(name + ".biases", t["B"].tobytes(), list(t["B"].shape), "BF16", bits=t["bits"], group_size=64)
        else:
            put(name, t.tobytes(), list(t.shape), "U16")
    manifest["num_tensors"] = len(manifest["tensors"])
    with open(os.path.join(d, "model_weights_quant.json"), "w") as f:
        json.dump(manifest, f)
    with open(os.path.join(d, "model_weights_quant.bin"), "wb") as f:
        f.write(bytes(blob))


def test_layout_check_and_manifest_parsing(tmp_path):
    rng = synth.rng_for(15, 1)
    blocks = [[synth.expert_block(rng, 256, 128, 64, 3, L.BF16) for _ in range(3)]]
    _write_expert_dir(tmp_path, blocks, 256, 128)
    lay = loaders.read_expert_layout(str(tmp_path))
    loaders.check_expert_layout(lay, 256, 128)
    with pytest.raises(ValueError):
        loaders.check_expert_layout(lay, 512, 128)          # another model's block does not pass
    t4 = synth.affine_tensor(rng, 64, 256, 4, L.BF16)
    gate = synth.f32_to_bf16_rne(rng.normal(0, 1, size=(8, 256)).astype(np.float32))
    _write_weight_dir(tmp_path, {"model.layers.0.mlp.shared_expert.gate_proj": t4, "model.layers.0.mlp.gate.weight": gate})
    with open(tmp_path / "model_weights_quant.json") as f:
        entries = loaders.parse_weight_manifest(json.load(f))
    e = entries["model.layers.0.mlp.shared_expert.gate_proj.weight"]
    assert (e["kind"], e["out_dim"], e["in_dim"], e["bits"]) == ("affine", 64, 256, 4)
    assert e["offset"] % 64 == 0 and e["scales_offset"] % 64 == 0
    g = entries["model.layers.0.mlp.gate.weight"]
    assert (g["kind"], g["out_dim"], g["in_dim"]) == ("bf16", 8, 256)
    bad = {"tensors": {"x.weight": {"offset": 0, "size": 4, "shape": [1, 1], "dtype": "U32", "bits": 4}}}
    with pytest.raises(ValueError):
        loaders.parse_weight_manifest(bad)                  # quantized tensor without scales


@pytest.mark.gpu
def test_files_load_into_pool_and_device_buffer(tmp_path):
    from finchmoe_b200 import api
    from oracle import oracle
    from parity import assert_close
    rng = synth.rng_for(15, 2)
    blocks = [[synth.expert_block(rng, 256, 128, 64, 3, L.BF16) for _ in range(4)] for _ in range(2)]
    _write_expert_dir(tmp_path, blocks, 256, 128)
    t4 = synth.affine_tensor(rng, 64, 256, 4, L.BF16)
    gate = synth.f32_to_bf16_rne(rng.normal(0, 1, size=(8, 256)).astype(np.float32))
    _write_weight_dir(tmp_path, {"shared.gate_proj": t4, "mlp.gate.weight": gate})
    ctx = api.Context(hidden=256, n_experts=4, top_k=4, moe_inter=128, shared_inter=128, n_layers=2, scale_dtype=L.BF16, act_dtype=L.F32,
                      max_tokens=1)
    pool = ctx.pool()
    try:
        assert loaders.load_packed_experts(pool, str(tmp_path)) == 8
        for l in range(2):
            for e in range(4):
                assert np.array_equal(pool.get(l, e), blocks[l][e])      # the reference's byte order comes back out
        assert loaders.load_packed_experts(pool, str(tmp_path), layers=[1], experts=[2, 3]) == 2
        wf = loaders.WeightFile(ctx, str(tmp_path))
        x = rng.normal(0, 1, size=256).astype(np.float32)
        got = ctx.fast_dequant_matvec(wf.wdesc("shared.gate_proj.weight"), x)
        want = oracle.matvec(t4["W"], t4["S"], t4["B"], L.BF16, x, 64, 256, 64, 4)
        assert_close(got, want, "4-bit tensor from the weight file")
        got = ctx.fast_dequant_matvec(wf.wdesc("mlp.gate.weight"), x)
        want = synth.bf16_to_f32(gate).astype(np.float64) @ x.astype(np.float64)
        assert_close(got, want.astype(np.float32), "BF16 router gate from the weight file")
    finally:
        pool.destroy()
        ctx.destroy()
