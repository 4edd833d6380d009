"""Loaders for the reference's on-disk formats, so that real model files drop into the library.

* packed routed experts: `<dir>/layer_LL.bin` (expert e at byte e * expert_size) + `<dir>/layout.json`
  as written by finchmoe/repack_experts.py:137-151, 349, 540-551 -> `finch_pool_put`
* flat non-expert weights: `model_weights_quant.bin` + `model_weights_quant.json` as written by
  finchmoe/quantize_non_experts.py:258-456 (read by finchmoe/infer.m:727-923) -> one device buffer and a
  `finch_wdesc` per tensor, pointers = buffer + offset exactly like `wf_buf + offset`
  (finchmoe/infer.m:2892-2894)
* GGUF v3 containers (finchmoe/infer.m:1025-1247): `GgufFile` -> the stacked expert tensors as a
  `finch_gguf_experts` per layer, Q4_K / Q6_K / BF16 matrices as `finch_wdesc`
"""
from __future__ import annotations

import json
import os
import re
import struct

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


# ------------------------------------------------------------------ GGUF v3
# ggml type -> (elements per block, bytes per block)
GGML_BLOCK = {0: (1, 4), 1: (1, 2), 30: (1, 2), 12: (256, 144), 14: (256, 210), 8: (32, 34), 2: (32, 18), 13: (256, 176)}
_KV_FIXED = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}   # u8 i8 u16 i16 u32 i32 f32 bool u64 i64 f64
_EXPERT_RE = re.compile(r"^blk\.(\d+)\.ffn_(gate|up|down)_exps\.weight$")


class GgufFile:
    """A GGUF v3 container read the way open_gguf does (finchmoe/infer.m:1025-1247): header, the key/value block
    skipped by value type (only `general.alignment` is kept, default 32), the tensor infos, and the data section
    that starts at the next multiple of the alignment after them; tensor offsets are relative to that start.
    The stacked expert tensors `blk.L.ffn_{gate,up,down}_exps.weight` (dims [in, out, n_experts]) become one
    (offset, bytes per expert, ggml type) entry per layer and projection, the reference's GgufExpertInfo
    (infer.m:1017-1021); every other tensor is listed by its GGUF name with dims, type, offset and size."""

    MAGIC = 0x46554747

    def __init__(self, path: str):
        self.path = path
        self.data = np.memmap(path, dtype=np.uint8, mode="r")
        buf = memoryview(self.data)
        size = len(buf)
        pos = 0

        def rd(fmt):
            nonlocal pos
            n = struct.calcsize(fmt)
            if pos + n > size:
                raise ValueError(f"{path}: truncated at byte {pos}")
            v = struct.unpack_from("<" + fmt, buf, pos)[0]
            pos += n
            return v

        def rstr():
            nonlocal pos
            n = rd("Q")
            if pos + n > size:
                raise ValueError(f"{path}: string of {n} bytes overruns the file")
            s = bytes(buf[pos:pos + n])
            pos += n
            return s

        if rd("I") != self.MAGIC:
            raise ValueError(f"{path} is not a GGUF file")
        self.version = rd("I")
        if self.version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {self.version} is not supported")
        n_tensors, n_kv = rd("Q"), rd("Q")
        self.alignment = 32
        self.kv_count = n_kv
        for _ in range(n_kv):
            key = rstr()
            vt = rd("I")
            if vt in _KV_FIXED:
                if key == b"general.alignment" and vt == 4:
                    self.alignment = rd("I")
                else:
                    pos += _KV_FIXED[vt]
            elif vt == 8:
                rstr()
            elif vt == 9:
                at, n = rd("I"), rd("Q")
                if at == 8:
                    for _ in range(n):
                        rstr()
                elif at in _KV_FIXED:
                    pos += n * _KV_FIXED[at]
                else:
                    raise ValueError(f"{path}: array of value type {at} in key {key!r}")
            else:
                raise ValueError(f"{path}: value type {vt} in key {key!r}")
        if self.alignment < 1 or self.alignment & (self.alignment - 1):
            raise ValueError(f"{path}: alignment {self.alignment} is not a power of two")
        infos = []
        for _ in range(n_tensors):
            name = rstr().decode("utf-8")
            nd = rd("I")
            dims = [rd("Q") for _ in range(nd)]
            gtype, toff = rd("I"), rd("Q")
            infos.append((name, dims, gtype, toff))
        self.data_offset = (pos + self.alignment - 1) & ~(self.alignment - 1)
        self.tensors = {}
        self.experts = {}          # layer -> {"gate" | "up" | "down": dict(offset, slab, type, in_dim, out_dim, n_experts)}
        for name, dims, gtype, toff in infos:
            be, bs = GGML_BLOCK.get(gtype, (0, 0))
            nelem = int(np.prod(dims, dtype=np.uint64)) if dims else 1
            tsize = (nelem + be - 1) // be * bs if be else 0
            off = self.data_offset + toff
            if be and off + tsize > size:
                raise ValueError(f"{path}: tensor {name} ends at byte {off + tsize}, the file has {size}")
            m = _EXPERT_RE.match(name)
            if m and len(dims) == 3 and be:
                row_bytes = dims[0] // be * bs                       # dims[0] = in_dim
                self.experts.setdefault(int(m.group(1)), {})[m.group(2)] = dict(
                    offset=off, slab=dims[1] * row_bytes, type=gtype, in_dim=dims[0], out_dim=dims[1], n_experts=dims[2])
                continue
            self.tensors[name] = dict(dims=dims, type=gtype, offset=off, size=tsize)

    def tensor_bytes(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        if t["type"] not in GGML_BLOCK:
            raise KeyError(f"{name}: ggml type {t['type']} is not handled")
        return self.data[t["offset"]:t["offset"] + t["size"]]

    def expert_slab(self, layer: int, which: str, expert: int) -> np.ndarray:
        """The rows of one expert's projection, as the reference's pool preads them (infer.m:2633-2700)."""
        e = self.experts[layer][which]
        o = e["offset"] + expert * e["slab"]
        return self.data[o:o + e["slab"]]

    def wdesc(self, ctx, name: str) -> L.WDesc:
        """Uploads a Q4_K / Q6_K / BF16 matrix [in, out] and returns its descriptor for the matvec seam."""
        t = self.tensors[name]
        bits = {12: 10, 14: 11, 30: L.BITS_BF16}.get(t["type"])
        if bits is None or len(t["dims"]) != 2:
            raise KeyError(f"{name}: ggml type {t['type']} with dims {t['dims']} has no matvec tier")
        buf = ctx.upload(self.tensor_bytes(name))
        ctx._keep.append(buf)
        return L.WDesc(buf.ptr, None, None, t["dims"][1], t["dims"][0], 256 if bits != L.BITS_BF16 else 64, bits, L.FP16 if bits != L.BITS_BF16 else L.BF16)

    def upload_experts(self, ctx, layer: int) -> L.GgufExperts:
        """The layer's three stacked expert tensors on the device -> the finch_gguf_experts of finch_encode_moe_gguf
        (the reference keeps them on disk and preads the selected slabs; here they are resident)."""
        e = self.experts[layer]
        missing = [w for w in ("gate", "up", "down") if w not in e]
        if missing:
            raise KeyError(f"layer {layer}: no ffn_{missing[0]}_exps tensor")
        ptr, slab, ty = [], [], []
        for w in ("gate", "up", "down"):
            if e[w]["type"] not in (12, 14):
                raise KeyError(f"layer {layer} {w}: ggml type {e[w]['type']} is not Q4_K / Q6_K")
            buf = ctx.upload(self.data[e[w]["offset"]:e[w]["offset"] + e[w]["slab"] * e[w]["n_experts"]])
            ctx._keep.append(buf)
            ptr.append(buf.ptr)
            slab.append(e[w]["slab"])
            ty.append(10 if e[w]["type"] == 12 else 11)
        return L.GgufExperts(ptr[0], ptr[1], ptr[2], slab[0], slab[1], slab[2], ty[0], ty[1], ty[2])
