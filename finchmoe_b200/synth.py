"""Seeded synthetic tensors with the shapes and value distributions of the
quantized-expert path (numpy, host side).

Packed layouts are produced from their bitstream definition: a packed row of
the 3-, 4- or 8-bit affine tiers is one little-endian bitstream with code ``i``
at bits ``[bits*i, bits*i+bits)`` -- for 3-bit that is the 24-bit-triplet form
of finchmoe/repack_experts.py:242-257, for 4/8-bit the u32 form of
finchmoe/quantize_non_experts.py:57-65.

Value distributions: codes uniform over their range; scale = |N(0, 0.01)| and
bias = -4*scale, both stored as 16-bit floats (fp16 or bf16); activations
~N(0,1) rounded to bf16; router logits ~N(0,1); expert popularity per layer
Zipf(s=1.1) over a seeded permutation of the experts.
"""
from __future__ import annotations

import numpy as np

SCALE_BF16, SCALE_FP16 = 0, 1
Q4K_BLOCK, Q6K_BLOCK = 144, 210
GGML_Q4_K, GGML_Q6_K = 12, 14


def rng_for(config: int, layer: int = 0, extra: int = 0) -> np.random.Generator:
    """seed = 1000*config + layer (+ a stream id), PCG64."""
    return np.random.Generator(np.random.PCG64([1000 * config + layer, extra]))


# ------------------------------------------------------------ 16-bit floats
def f32_to_bf16_trunc(a) -> np.ndarray:
    """fp32 -> bf16 by truncation, as the reference's quantizers store scales
    (finchmoe/repack_experts.py:232-234)."""
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def f32_to_bf16_rne(a) -> np.ndarray:
    u = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def bf16_to_f32(u16) -> np.ndarray:
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_16(a, scale_dtype) -> np.ndarray:
    if scale_dtype == SCALE_FP16:
        return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)
    return f32_to_bf16_rne(a)


def w16_to_f32(u16, scale_dtype) -> np.ndarray:
    if scale_dtype == SCALE_FP16:
        return np.asarray(u16, np.uint16).view(np.float16).astype(np.float32)
    return bf16_to_f32(u16)


# ------------------------------------------------------------------ packers
def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """codes uint8 [rows, n] -> packed bytes uint8 [rows, n*bits/8]."""
    codes = np.ascontiguousarray(codes, np.uint8)
    rows, n = codes.shape
    assert (n * bits) % 8 == 0
    b = np.unpackbits(codes[:, :, None], axis=2, bitorder="little")[:, :, :bits]
    return np.packbits(b.reshape(rows, n * bits), axis=1, bitorder="little")


def affine_tensor(rng, out_dim, in_dim, bits, scale_dtype=SCALE_FP16, group=64):
    """Random affine-quantized tensor: dict(W uint8 [out, in*bits/8], S, B
    uint16 [out, in/group], ...)."""
    codes = rng.integers(0, 1 << bits, size=(out_dim, in_dim), dtype=np.uint8)
    s = np.abs(rng.normal(0.0, 0.01, size=(out_dim, in_dim // group))).astype(np.float32)
    S = f32_to_16(s, scale_dtype)
    # bias from the stored scale so that bias == -4*scale holds exactly
    half = float((1 << bits) - 1) / 2.0 if bits != 3 else 4.0
    Bv = f32_to_16(-half * w16_to_f32(S, scale_dtype), scale_dtype)
    return dict(W=pack_codes(codes, bits), S=S, B=Bv, out_dim=out_dim, in_dim=in_dim, group=group,
                bits=bits, scale_dtype=scale_dtype, codes=codes)


def expert_layout(hidden=2048, inter=512, group=64, bits=3) -> dict:
    """Byte offsets of [gate W|S|B|up W|S|B|down W|S|B] inside one packed
    expert block (finchmoe/infer.m:223-234 for 3-bit at 2048/512/64)."""
    gw, gs = inter * hidden * bits // 8, inter * (hidden // group) * 2
    dw, ds = hidden * inter * bits // 8, hidden * (inter // group) * 2
    o = dict(gate_w=0, gate_s=gw, gate_b=gw + gs, up_w=gw + 2 * gs)
    o["up_s"] = o["up_w"] + gw
    o["up_b"] = o["up_s"] + gs
    o["down_w"] = o["up_b"] + gs
    o["down_s"] = o["down_w"] + dw
    o["down_b"] = o["down_s"] + ds
    o["size"] = o["down_b"] + ds
    return o


def expert_block(rng, hidden=2048, inter=512, group=64, bits=3, scale_dtype=SCALE_FP16) -> np.ndarray:
    """One packed routed-expert block (uint8[size])."""
    L = expert_layout(hidden, inter, group, bits)
    blk = np.empty(L["size"], np.uint8)
    for name, (o, i) in (("gate", (inter, hidden)), ("up", (inter, hidden)), ("down", (hidden, inter))):
        t = affine_tensor(rng, o, i, bits, scale_dtype, group)
        blk[L[name + "_w"]:L[name + "_w"] + t["W"].size] = t["W"].reshape(-1)
        blk[L[name + "_s"]:L[name + "_s"] + t["S"].size * 2] = t["S"].reshape(-1).view(np.uint8)
        blk[L[name + "_b"]:L[name + "_b"] + t["B"].size * 2] = t["B"].reshape(-1).view(np.uint8)
    return blk


def block_tensor(blk: np.ndarray, which: str, hidden=2048, inter=512, group=64, bits=3,
                 scale_dtype=SCALE_FP16) -> dict:
    """View one of gate/up/down of a packed block as an affine tensor dict."""
    L = expert_layout(hidden, inter, group, bits)
    o, i = (hidden, inter) if which == "down" else (inter, hidden)
    wb, sb = o * i * bits // 8, o * (i // group) * 2
    return dict(W=blk[L[which + "_w"]:L[which + "_w"] + wb].reshape(o, -1),
                S=blk[L[which + "_s"]:L[which + "_s"] + sb].view(np.uint16).reshape(o, -1),
                B=blk[L[which + "_b"]:L[which + "_b"] + sb].view(np.uint16).reshape(o, -1),
                out_dim=o, in_dim=i, group=group, bits=bits, scale_dtype=scale_dtype)


def shared_expert(rng, hidden=2048, inter=512, group=64, bits=4, scale_dtype=SCALE_FP16):
    """(gate, up, down) affine tensors of the shared SwiGLU expert."""
    return (affine_tensor(rng, inter, hidden, bits, scale_dtype, group),
            affine_tensor(rng, inter, hidden, bits, scale_dtype, group),
            affine_tensor(rng, hidden, inter, bits, scale_dtype, group))


def gguf_tensor(rng, out_dim, in_dim, ggml_type) -> dict:
    """Random Q4_K / Q6_K rows: quant bytes and packed sub-scales uniform,
    d / dmin = |N(0, 0.01)| as fp16 (subnormal draws are kept)."""
    nb = in_dim // 256
    bs = Q4K_BLOCK if ggml_type == GGML_Q4_K else Q6K_BLOCK
    W = rng.integers(0, 256, size=(out_dim, nb, bs), dtype=np.uint8)
    d = np.abs(rng.normal(0.0, 0.01, size=(out_dim, nb, 2))).astype(np.float16)
    if ggml_type == GGML_Q4_K:
        W[:, :, 0:4] = d.view(np.uint8).reshape(out_dim, nb, 4)
    else:
        W[:, :, 208:210] = d[:, :, :1].copy().view(np.uint8).reshape(out_dim, nb, 2)
    return dict(W=W.reshape(out_dim, nb * bs), S=None, B=None, out_dim=out_dim, in_dim=in_dim,
                group=256, bits=10 if ggml_type == GGML_Q4_K else 11, scale_dtype=SCALE_FP16,
                ggml_type=ggml_type)


# --------------------------------------------------------------- activations
def activations(rng, *shape) -> np.ndarray:
    """~N(0,1) values exactly representable in bf16, returned as fp32."""
    return bf16_to_f32(f32_to_bf16_rne(rng.normal(0.0, 1.0, size=shape).astype(np.float32)))


# ------------------------------------------------------------------- routing
def zipf_routing(rng, T, n_experts=256, K=8, s=1.1):
    """Per token: K distinct experts drawn without replacement from a
    Zipf(s) popularity over a seeded permutation; weights = softmax of K
    N(0,1) logits.  Returns ids int32 [T,K], weights fp32 [T,K]."""
    p = 1.0 / np.arange(1, n_experts + 1, dtype=np.float64) ** s
    p /= p.sum()
    perm = rng.permutation(n_experts)
    ids = np.empty((T, K), np.int32)
    for t in range(T):
        ids[t] = perm[rng.choice(n_experts, size=K, replace=False, p=p)]
    lg = rng.normal(0.0, 1.0, size=(T, K))
    w = np.exp(lg - lg.max(axis=1, keepdims=True))
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids, w


def zipf_popularity(rng, n_experts=256):
    """A seeded order of popularity: expert perm[i] has Zipf rank i + 1."""
    return rng.permutation(n_experts)


def zipf_routing_shared(rng, T, perm, K=8, s=1.1):
    """zipf_routing for tokens that share one order of popularity `perm` (a layer's, whichever rank owns the
    token).  K distinct experts per token, drawn without replacement from the Zipf(s) popularity: the K largest
    of log p + Gumbel noise, which is the same distribution as drawing them one after another."""
    n = perm.shape[0]
    logp = -s * np.log(np.arange(1, n + 1, dtype=np.float64))
    keys = logp[None, :] + rng.gumbel(size=(T, n))
    top = np.argsort(-keys, axis=1)[:, :K]
    ids = perm[top].astype(np.int32)
    lg = rng.normal(0.0, 1.0, size=(T, K))
    w = np.exp(lg - lg.max(axis=1, keepdims=True))
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids, w


def router_logits(rng, T, n_experts=256) -> np.ndarray:
    return rng.normal(0.0, 1.0, size=(T, n_experts)).astype(np.float32)
