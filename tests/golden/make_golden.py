"""Generates the golden vectors under tests/golden/ (run once, where the
reference checkout is available; the fixtures are committed, this script is
kept so they can be regenerated).

Sources of truth executed here:
  * the reference's own Python packers / dequantizers, imported unmodified:
      finchmoe/repack_experts.py      pack_3bit, quantize_affine_pack,
                                      _dequant_packed_weights
      finchmoe/quantize_non_experts.py quantize_affine
      finchmoe/finchTool/tools/quant_audit.py   dequant_block (bits 3/4/8)
      finchmoe/finchTool/tools/debug_compare.py cpu_dequant_matvec_py (4/8-bit)
  * gguf-py (the ``gguf`` package of llama.cpp, version recorded in the file)
    for the Q4_K / Q6_K block decoders: gguf.quants.dequantize.

Usage: python tests/golden/make_golden.py /path/to/reference/checkout
"""
import os
import sys

import numpy as np

if len(sys.argv) < 2:
    sys.exit(__doc__)
REF = sys.argv[1]
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REF, "finchmoe"))
sys.path.insert(0, os.path.join(REF, "finchmoe", "finchTool", "tools"))

import repack_experts as rp  # noqa: E402
import quantize_non_experts as qn  # noqa: E402
import quant_audit as qa  # noqa: E402
import debug_compare as dc  # noqa: E402


def affine():
    rng = np.random.Generator(np.random.PCG64(20240601))
    out = {}
    # 3-bit and 4-bit through the expert repacker
    for bits, (o, i) in ((3, (24, 256)), (4, (16, 192))):
        w = (rng.normal(0, 0.02, size=(o, i)) * rng.uniform(0.2, 3.0, size=(o, 1))).astype(np.float32)
        pk, s, b = rp.quantize_affine_pack(w, bits)
        deq = qa.dequant_block(bits, np.ascontiguousarray(pk).tobytes(), s.tobytes(), b.tobytes(), o, i // 64)
        out[f"rp{bits}_w"] = w
        out[f"rp{bits}_packed"] = np.ascontiguousarray(pk).view(np.uint8).reshape(o, -1)
        out[f"rp{bits}_scales"] = s
        out[f"rp{bits}_biases"] = b
        out[f"rp{bits}_dequant"] = deq.astype(np.float32)
        if bits == 4:
            out["rp4_dequant_inplace"] = rp._dequant_packed_weights(pk, s, b, i, 4)
    # pack_3bit alone on every code value in every slot
    q = np.arange(8 * 64, dtype=np.uint8) % 8
    q = np.concatenate([q, rng.integers(0, 8, size=512, dtype=np.uint8)])
    out["pack3_codes"] = q
    out["pack3_bytes"] = rp.pack_3bit(q)
    # 4-bit and 8-bit through the non-expert quantizer + the pure-Python matvec
    for bits, (o, i) in ((4, (12, 128)), (8, (10, 128))):
        w = rng.normal(0, 0.05, size=(o, i)).astype(np.float32)
        pk, s, b = qn.quantize_affine(w, bits)
        x = rng.uniform(-0.5, 0.5, size=i).astype(np.float32)
        y = dc.cpu_dequant_matvec_py(pk, s, b, x, o, i, 64, bits)
        deq = qa.dequant_block(bits, pk.tobytes(), s.tobytes(), b.tobytes(), o, i // 64)
        out[f"qn{bits}_packed"] = pk.view(np.uint8).reshape(o, -1)
        out[f"qn{bits}_scales"] = s
        out[f"qn{bits}_biases"] = b
        out[f"qn{bits}_x"] = x
        out[f"qn{bits}_matvec_f64"] = y
        out[f"qn{bits}_dequant"] = deq.astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "affine_reference.npz"), **out)
    print("affine_reference.npz", {k: v.shape for k, v in out.items()})


def gguf_blocks():
    import gguf
    from gguf import quants
    import importlib.metadata as md

    rng = np.random.Generator(np.random.PCG64(20240602))
    out = {"gguf_py_version": np.array(md.version("gguf"))}
    for name, qt, bs in (("q4k", gguf.GGMLQuantizationType.Q4_K, 144), ("q6k", gguf.GGMLQuantizationType.Q6_K, 210)):
        rows, nb = 6, 3
        raw = rng.integers(0, 256, size=(rows, nb * bs), dtype=np.uint8)
        blk = raw.reshape(rows, nb, bs)
        d = np.abs(rng.normal(0, 0.01, size=(rows, nb, 2))).astype(np.float16)
        d[0, 0, :] = np.float16(3e-6)      # fp16 subnormal super-scale
        d[1, 0, :] = np.float16(0.0)
        if name == "q4k":
            blk[:, :, 0:4] = d.view(np.uint8).reshape(rows, nb, 4)
        else:
            blk[:, :, 208:210] = d[:, :, :1].copy().view(np.uint8).reshape(rows, nb, 2)
        raw = blk.reshape(rows, nb * bs)
        out[name + "_raw"] = raw
        out[name + "_dequant"] = quants.dequantize(raw, qt).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "gguf_reference.npz"), **out)
    print("gguf_reference.npz", {k: v.shape for k, v in out.items()})


def hot_sets():
    # The one data fixture the reference ships for this path: int32[40][64]
    # expert ids per layer in descending routing frequency
    # (finchmoe/build_hot_sets.py:5-9).  Stored as statistics only.
    hs = np.fromfile(os.path.join(REF, "finchmoe", "hot_sets.bin"), dtype=np.int32).reshape(40, 64)
    np.savez_compressed(os.path.join(HERE, "hot_sets_shape.npz"), shape=np.array(hs.shape),
                        min=hs.min(), max=hs.max(),
                        distinct_per_layer=np.array([len(set(r)) for r in hs]))
    print("hot_sets", hs.shape, hs.min(), hs.max())


if __name__ == "__main__":
    affine()
    gguf_blocks()
    hot_sets()
