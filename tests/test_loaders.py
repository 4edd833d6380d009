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


# ------------------------------------------------------------------ GGUF container
def _write_gguf(path, layers, NE, H, I, alignment=None, rng=None):
    """A GGUF v3 file written by gguf-py's own writer (an independent implementation of the format): metadata of
    every value kind the reader has to skip, the stacked expert tensors of `layers`, one dense Q6_K matrix and an
    F32 vector between them.  Returns what was written."""
    import gguf
    rng = rng or synth.rng_for(15, 1)
    w = gguf.GGUFWriter(path, "finchtest")
    w.add_block_count(len(layers))
    w.add_string("general.name", "synthetic")
    w.add_float32("finchtest.rope_base", 1.0e6)
    w.add_bool("finchtest.flag", True)
    w.add_uint64("finchtest.big", 1 << 40)
    w.add_array("tokenizer.ggml.tokens", ["a", "bc", "def", ""])
    w.add_array("finchtest.ints", [1, 2, 3, 4, 5])
    if alignment:
        w.add_custom_alignment(alignment)
    written = {}
    Q = {12: gguf.GGMLQuantizationType.Q4_K, 14: gguf.GGMLQuantizationType.Q6_K}
    norm = rng.normal(0, 1, size=H).astype(np.float32)
    for l, types in layers.items():
        w.add_tensor(f"blk.{l}.attn_norm.weight", norm)
        for which, ty, (o, i) in (("gate", types[0], (I, H)), ("up", types[1], (I, H)), ("down", types[2], (H, I))):
            ex = [synth.gguf_tensor(rng, o, i, ty) for _ in range(NE)]
            slab = np.stack([e["W"] for e in ex])                      # [NE, out, row_bytes]
            w.add_tensor(f"blk.{l}.ffn_{which}_exps.weight", slab, raw_dtype=Q[ty])
            written[(l, which)] = ex
    dense = synth.gguf_tensor(rng, 96, H, 14)
    w.add_tensor("output.weight", dense["W"], raw_dtype=Q[14])
    written["output.weight"] = dense
    written["norm"] = norm
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return written


@pytest.mark.parametrize("alignment", [None, 64])
def test_gguf_container_reader_finds_every_tensor_where_the_writer_put_it(tmp_path, alignment):
    import gguf
    path = str(tmp_path / "m.gguf")
    NE, H, I = 5, 512, 256
    written = _write_gguf(path, {0: (12, 12, 14), 3: (14, 12, 12)}, NE, H, I, alignment)
    g = loaders.GgufFile(path)
    assert g.version == 3 and g.alignment == (alignment or 32) and g.data_offset % g.alignment == 0
    assert sorted(g.experts) == [0, 3]
    # the same offsets as gguf-py's reader reports
    rd = gguf.GGUFReader(path)
    by_name = {t.name: t for t in rd.tensors}
    for l in (0, 3):
        for which, (o, i) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            e = g.experts[l][which]
            t = by_name[f"blk.{l}.ffn_{which}_exps.weight"]
            assert e["offset"] == t.data_offset and e["n_experts"] == NE and e["in_dim"] == i and e["out_dim"] == o
            assert e["type"] == int(t.tensor_type)
            for x in range(NE):
                assert np.array_equal(g.expert_slab(l, which, x), written[(l, which)][x]["W"].reshape(-1)), (l, which, x)
    # ordinary tensors: listed under their GGUF names with the writer's bytes
    assert np.array_equal(g.tensor_bytes("output.weight"), written["output.weight"]["W"].reshape(-1))
    assert g.tensors["output.weight"]["dims"] == [H, 96] and g.tensors["output.weight"]["type"] == 14
    assert np.array_equal(g.tensor_bytes("blk.3.attn_norm.weight").view(np.float32), written["norm"])
    assert not any("_exps" in n for n in g.tensors)


def test_gguf_container_reader_rejects_damaged_files(tmp_path):
    path = str(tmp_path / "m.gguf")
    _write_gguf(path, {0: (12, 12, 14)}, 2, 256, 256)
    raw = open(path, "rb").read()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + raw[4:])
    with pytest.raises(ValueError, match="not a GGUF"):
        loaders.GgufFile(str(bad))
    bad.write_bytes(raw[:4] + (9).to_bytes(4, "little") + raw[8:])
    with pytest.raises(ValueError, match="version"):
        loaders.GgufFile(str(bad))
    bad.write_bytes(raw[:len(raw) // 2])                    # tensor data cut off
    with pytest.raises(ValueError, match="ends at byte|truncated|overruns"):
        loaders.GgufFile(str(bad))
    bad.write_bytes(raw[:40])                               # cut inside the key/value block
    with pytest.raises(ValueError, match="truncated|overruns"):
        loaders.GgufFile(str(bad))


@pytest.mark.gpu
def test_gguf_file_experts_on_the_device_vs_oracle(tmp_path):
    """A GGUF file's stacked expert tensors loaded by the container reader and run through finch_encode_moe_gguf,
    and its dense Q6_K matrix through the matvec seam, against the oracle."""
    import torch
    from finchmoe_b200 import api
    from oracle import oracle
    from parity import assert_close
    path = str(tmp_path / "m.gguf")
    NE, H, I, K, B = 6, 512, 256, 4, 3
    written = _write_gguf(path, {1: (12, 12, 14)}, NE, H, I)
    g = loaders.GgufFile(path)
    ctx = api.Context(hidden=H, n_experts=NE, top_k=K, moe_inter=I, shared_inter=256, n_layers=2, act_dtype=L.F32, max_tokens=4)
    try:
        ge = g.upload_experts(ctx, 1)
        rng = synth.rng_for(15, 2)
        x = rng.normal(0, 1, size=(B, H)).astype(np.float32)
        ids = np.stack([rng.permutation(NE)[:K] for _ in range(B)]).astype(np.int32)
        w = rng.random((B, K)).astype(np.float32)
        w /= w.sum(axis=1, keepdims=True)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        out = torch.empty((B, H), dtype=torch.float32, device="cuda")
        ctx.encode_moe_gguf(ge, d(x), d(ids), d(w), None, None, out, B)
        ctx.sync()

        def mv(t, v):
            return oracle.matvec(t["W"], None, None, 1, v, t["out_dim"], t["in_dim"], 256, t["bits"])
        want = np.zeros((B, H), np.float32)
        for b in range(B):
            for k in range(K):
                e = int(ids[b, k])
                act = oracle.swiglu(mv(written[(1, "gate")][e], x[b]), mv(written[(1, "up")][e], x[b]))
                want[b] += w[b, k] * mv(written[(1, "down")][e], act)
        assert_close(out.cpu().numpy(), want, "experts of a GGUF file")
        wd = g.wdesc(ctx, "output.weight")
        got = ctx.fast_dequant_matvec(wd, x)
        assert_close(got, mv(written["output.weight"], x), "dense Q6_K matrix of a GGUF file")
        assert ctx.device_status() == 0
    finally:
        ctx.destroy()
