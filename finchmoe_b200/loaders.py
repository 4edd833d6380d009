"""Loaders for the reference's on-disk formats, so that real model files drop into the library.

* packed routed experts: `<dir>/layer_LL.bin` (expert e at byte e * expert_size) + `<dir>/layout.json`
  as written by finchmoe/repack_experts.py:137-151, 349, 540-551 -> `finch_pool_put`
* flat non-expert weights: `model_weights_quant.bin` + `model_weights_quant.json` as written by
  finchmoe/quantize_non_experts.py:258-456 (read by finchmoe/infer.m:727-923) -> one device buffer and a
  `finch_wdesc` per tensor, pointers = buffer + offset exactly like `wf_buf + offset`
  (finchmoe/infer.m:2892-2894)
"""
from __future__ import annotations

import json
import os

import numpy as np

from . import lib as L


def read_expert_layout(directory: str) -> dict:
    """layout.json of a packed-expert directory: expert_size, num_layers, num_experts, components."""
    with open(os.path.join(directory, "layout.json")) as f:
        lay = json.load(f)
    for key in ("expert_size", "num_layers", "num_experts", "components"):
        if key not in lay:
            raise ValueError(f"layout.json: missing {key!r}")
    return lay


def check_expert_layout(lay: dict, hidden: int, inter: int, group: int = 64, bits: int = 3):
    """The component table must be the block layout the kernels assume (finchmoe/infer.m:223-234)."""
    rows = {"gate_proj": (inter, hidden), "up_proj": (inter, hidden), "down_proj": (hidden, inter)}
    off = 0
    want = []
    for name in ("gate_proj", "up_proj", "down_proj"):
        o, i = rows[name]
        wb, sb = o * i * bits // 8, o * (i // group) * 2
        for suffix, size in ((".weight", wb), (".scales", sb), (".biases", sb)):
            want.append((name + suffix, off, size))
            off += size
    got = [(c["name"], int(c["offset"]), int(c["size"])) for c in lay["components"]]
    if got != want or int(lay["expert_size"]) != off:
        raise ValueError(f"layout.json does not describe the {bits}-bit g{group} block of hidden {hidden} / inter {inter}")


def load_packed_experts(pool, directory: str, layers=None, experts=None) -> int:
    """Puts the experts of `<directory>/layer_LL.bin` into the pool.  layers / experts: iterables restricting
    what is loaded (an expert-parallel rank passes its block of experts).  Returns the number of experts put."""
    ctx = pool.ctx
    lay = read_expert_layout(directory)
    check_expert_layout(lay, ctx.cfg.hidden, ctx.cfg.moe_inter, ctx.cfg.group_size, ctx.cfg.expert_bits)
    size = int(lay["expert_size"])
    n = 0
    for layer in (range(int(lay["num_layers"])) if layers is None else layers):
        path = os.path.join(directory, f"layer_{layer:02d}.bin")
        data = np.memmap(path, dtype=np.uint8, mode="r")
        n_file = data.size // size
        for e in (range(n_file) if experts is None else experts):
            if e >= n_file:
                raise ValueError(f"{path}: holds {n_file} experts, expert {e} requested")
            pool.put(layer, e, np.ascontiguousarray(data[e * size:(e + 1) * size]))
            n += 1
    return n


_DTYPE_BYTES = {"U32": 4, "BF16": 2, "U16": 2, "F32": 4, "U8": 1}


def parse_weight_manifest(manifest: dict) -> dict:
    """name -> dict(kind, offset, out_dim, in_dim, bits, group, scales_offset, biases_offset, ...) from the
    manifest's "tensors" table.  kind: "affine" (U32 words + BF16 scales/biases), "bf16" (U16 rows), "f32"."""
    out = {}
    tensors = manifest["tensors"]
    for name, t in tensors.items():
        if name.endswith(".scales") or name.endswith(".biases"):
            continue
        dtype, shape = t["dtype"], [int(x) for x in t["shape"]]
        if dtype == "U32" and "bits" in t:
            bits, gs = int(t["bits"]), int(t.get("group_size", 64))
            base = name[:-len(".weight")] if name.endswith(".weight") else name
            s, b = tensors.get(base + ".scales"), tensors.get(base + ".biases")
            if s is None or b is None:
                raise ValueError(f"{name}: quantized tensor without .scales / .biases entries")
            out[name] = dict(kind="affine", offset=int(t["offset"]), out_dim=shape[0], in_dim=shape[1] * 32 // bits, bits=bits, group=gs,
                             scales_offset=int(s["offset"]), biases_offset=int(b["offset"]), scale_dtype=L.BF16)
        elif dtype == "U16":
            rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
            out[name] = dict(kind="bf16", offset=int(t["offset"]), out_dim=rows, in_dim=shape[-1], shape=shape)
        elif dtype == "F32":
            out[name] = dict(kind="f32", offset=int(t["offset"]), shape=shape)
        else:
            raise ValueError(f"{name}: unsupported dtype {dtype!r}")
        if int(t["offset"]) + int(t["size"]) > manifest.get("_file_size", 1 << 62):
            raise ValueError(f"{name}: runs past the end of the weight file")
    return out


class WeightFile:
    """model_weights_quant.{bin,json} resident on the device (metal_set_weights, finchmoe/infer.m:2813)."""

    def __init__(self, ctx, directory: str):
        with open(os.path.join(directory, "model_weights_quant.json")) as f:
            self.manifest = json.load(f)
        path = os.path.join(directory, "model_weights_quant.bin")
        self.manifest["_file_size"] = os.path.getsize(path)
        self.entries = parse_weight_manifest(self.manifest)
        self.buf = ctx.upload(np.memmap(path, dtype=np.uint8, mode="r"))
        self.ctx = ctx

    def wdesc(self, name: str) -> L.WDesc:
        """Descriptor of a quantized or BF16 tensor for finch_matvec / finch_encode_batch_matvec."""
        e = self.entries[name]
        base = self.buf.ptr
        if e["kind"] == "affine":
            return L.WDesc(base + e["offset"], base + e["scales_offset"], base + e["biases_offset"], e["out_dim"], e["in_dim"], e["group"],
                           e["bits"], e["scale_dtype"])
        if e["kind"] == "bf16":
            return L.WDesc(base + e["offset"], None, None, e["out_dim"], e["in_dim"], 64, L.BITS_BF16, L.BF16)
        raise KeyError(f"{name} is a raw fp32 tensor: use ptr()")

    def ptr(self, name: str) -> int:
        return self.buf.ptr + self.entries[name]["offset"]
