"""ctypes + numpy front end of the CPU oracle (``finch_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, by ``__graft_entry__.smoke``
and by ``bench.py``'s CPU-baseline / reference legs as the checker and the
timed CPU arm.  The product package never imports it.

Two independent restatements live here so they can be checked against each
other: the C library (sequential fp32 order of the reference's CPU path, plus
an fp64-accumulating yardstick) and small vectorised numpy decoders written
from the bit-layout definitions (finchmoe/repack_experts.py:242-257,
finchmoe/quantize_non_experts.py:57-65, finchmoe/infer.m:1595-1657).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libfinch_oracle.so")

SCALE_BF16, SCALE_FP16 = 0, 1
ACC_F32, ACC_F64 = 0, 1


def build(force: bool = False) -> str:
    """Compile the C oracle next to its source (gcc, a second or two)."""
    src = os.path.join(_HERE, "finch_oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.check_call(["make", "-C", _HERE, "-s", "-B", "libfinch_oracle.so"])
    return _SO


_REF_SO = os.path.join(_HERE, "_ref", "libfinch_ref.so")
_ref_lib = None


def build_ref(ref_root: str | None = None) -> str | None:
    """Compile the reference's own CPU math (``make ref``: its pure-C region, from a reference checkout)
    into ``oracle/_ref/``.  Returns the library's path, the path of an earlier build when the checkout is
    absent (the build travels with the tree), or None."""
    # default: a checkout beside this repository (or wherever FINCH_REFERENCE points)
    ref_root = ref_root or os.environ.get("FINCH_REFERENCE", os.path.normpath(os.path.join(_HERE, "..", "..", "reference")))
    src = os.path.join(ref_root, "finchmoe", "infer.m")
    if os.path.exists(src):
        subprocess.check_call(["make", "-C", _HERE, "-s", "ref", f"REF={ref_root}"])
    return _REF_SO if os.path.exists(_REF_SO) else None


def ref_lib():
    """ctypes handle of oracle/_ref/libfinch_ref.so (the reference's CPU functions), or None if it cannot be had."""
    global _ref_lib
    if _ref_lib is None:
        so = build_ref()
        if so is None:
            return None
        R = C.CDLL(so)
        f32p, u16p, i32p = C.POINTER(C.c_float), C.POINTER(C.c_uint16), C.POINTER(C.c_int)
        R.ref_bf16_to_f32.restype = C.c_float
        R.ref_bf16_to_f32.argtypes = [C.c_uint16]
        R.ref_f32_to_bf16.restype = C.c_uint16
        R.ref_f32_to_bf16.argtypes = [C.c_float]
        R.ref_fp16_to_f32.restype = C.c_float
        R.ref_fp16_to_f32.argtypes = [C.c_uint16]
        R.ref_cpu_sigmoid.restype = C.c_float
        R.ref_cpu_sigmoid.argtypes = [C.c_float]
        R.ref_gguf_dequant_row.argtypes = [C.c_void_p, f32p, C.c_int, C.c_int]
        R.ref_cpu_dequant_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int]
        R.ref_cpu_rms_norm.argtypes = [f32p, u16p, f32p, C.c_int, C.c_float]
        R.ref_cpu_swiglu.argtypes = [f32p, f32p, f32p, C.c_int]
        R.ref_cpu_softmax.argtypes = [f32p, C.c_int]
        R.ref_cpu_topk.argtypes = [f32p, C.c_int, C.c_int, i32p, f32p]
        R.ref_cpu_normalize_weights.argtypes = [f32p, C.c_int]
        R.ref_cpu_vec_madd.argtypes = [f32p, f32p, C.c_float, C.c_int]
        for n in ("ref_gguf_dequant_row", "ref_cpu_dequant_matvec", "ref_cpu_rms_norm", "ref_cpu_swiglu", "ref_cpu_softmax",
                  "ref_cpu_topk", "ref_cpu_normalize_weights", "ref_cpu_vec_madd"):
            getattr(R, n).restype = None
        _ref_lib = R
    return _ref_lib


class _WDesc(C.Structure):
    _fields_ = [("W", C.c_void_p), ("S", C.c_void_p), ("B", C.c_void_p), ("out_dim", C.c_int),
                ("in_dim", C.c_int), ("group", C.c_int), ("bits", C.c_int), ("scale_dtype", C.c_int)]


class _Layout(C.Structure):
    _fields_ = [(n, C.c_size_t) for n in ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b",
                                          "down_w", "down_s", "down_b", "size")]


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_SO)
        L.fo_bf16_to_f32.restype = C.c_float
        L.fo_bf16_to_f32.argtypes = [C.c_uint16]
        L.fo_fp16_to_f32.restype = C.c_float
        L.fo_fp16_to_f32.argtypes = [C.c_uint16]
        L.fo_fp16_to_f32_magic.restype = C.c_float
        L.fo_fp16_to_f32_magic.argtypes = [C.c_uint16]
        L.fo_gguf_row_bytes.restype = C.c_size_t
        L.fo_gguf_row_bytes.argtypes = [C.c_int, C.c_int]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype=None):
    if a is None:
        return None
    return np.ascontiguousarray(a, dtype=dtype)


# ----------------------------------------------------------------- scalars
def bf16_to_f32(u16):
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def fp16_to_f32(u16):
    return np.asarray(u16, dtype=np.uint16).view(np.float16).astype(np.float32)


def widen16(u16, scale_dtype):
    return fp16_to_f32(u16) if scale_dtype == SCALE_FP16 else bf16_to_f32(u16)


# ------------------------------------------------------- numpy bit decoders
def np_unpack_codes(W, out_dim, in_dim, bits):
    """Codes from the packed rows, written from the bitstream definition: for
    3-, 4- and 8-bit alike a row is one little-endian bitstream with code i at
    bits [bits*i, bits*i+bits)."""
    raw = np.ascontiguousarray(W).view(np.uint8).reshape(out_dim, in_dim * bits // 8)
    b = np.unpackbits(raw, axis=1, bitorder="little").reshape(out_dim, in_dim, bits)
    return (b * (1 << np.arange(bits, dtype=np.uint8))).sum(axis=2).astype(np.uint8)


def np_dequant_affine(W, S, B, scale_dtype, out_dim, in_dim, group, bits):
    q = np_unpack_codes(W, out_dim, in_dim, bits).astype(np.float32)
    s = np.repeat(widen16(S, scale_dtype).reshape(out_dim, -1), group, axis=1)
    b = np.repeat(widen16(B, scale_dtype).reshape(out_dim, -1), group, axis=1)
    return (q * s).astype(np.float32) + b


# ---------------------------------------------------------------- C wrappers
def unpack_codes(W, out_dim, in_dim, bits):
    W = _c(W)
    out = np.empty((out_dim, in_dim), np.uint8)
    rc = lib().fo_unpack_codes(_p(W), out_dim, in_dim, bits, _p(out))
    assert rc == 0
    return out


def dequant_affine(W, S, B, scale_dtype, out_dim, in_dim, group, bits):
    W, S, B = _c(W), _c(S, np.uint16), _c(B, np.uint16)
    out = np.empty((out_dim, in_dim), np.float32)
    rc = lib().fo_dequant_affine(_p(W), _p(S), _p(B), scale_dtype, out_dim, in_dim, group, bits, _p(out))
    assert rc == 0
    return out


def dequant_gguf(W, out_dim, in_dim, ggml_type):
    W = _c(W)
    out = np.empty((out_dim, in_dim), np.float32)
    rc = lib().fo_dequant_gguf(_p(W), out_dim, in_dim, ggml_type, _p(out))
    assert rc == 0
    return out


def gguf_unpack_codes(W, out_dim, in_dim, ggml_type):
    W = _c(W)
    out = np.empty((out_dim, in_dim), np.uint8)
    rc = lib().fo_gguf_unpack_codes(_p(W), out_dim, in_dim, ggml_type, _p(out))
    assert rc == 0
    return out


def matvec(W, S, B, scale_dtype, x, out_dim, in_dim, group, bits, accum=ACC_F64):
    """x: [in] or [M, in] fp32 -> [out] or [M, out]."""
    W, S, B = _c(W), _c(S, np.uint16), _c(B, np.uint16)
    x = _c(x, np.float32)
    xs = x.reshape(-1, in_dim)
    out = np.empty((xs.shape[0], out_dim), np.float32)
    for m in range(xs.shape[0]):
        rc = lib().fo_matvec(_p(W), _p(S), _p(B), scale_dtype, _p(xs[m]), _p(out[m]), out_dim, in_dim,
                             group, bits, accum)
        assert rc == 0
    return out.reshape(x.shape[:-1] + (out_dim,))


def swiglu(g, u):
    g, u = _c(g, np.float32), _c(u, np.float32)
    out = np.empty_like(g)
    lib().fo_swiglu(_p(g), _p(u), _p(out), g.size)
    return out


def residual_norm(resid, oproj, norm_w_bf16, eps):
    """(h_mid, h_post) of residual_norm_fused; oproj may be None."""
    resid, oproj, w = _c(resid, np.float32), _c(oproj, np.float32), _c(norm_w_bf16, np.uint16)
    h_mid, h_post = np.empty_like(resid), np.empty_like(resid)
    lib().fo_residual_norm(_p(resid), _p(oproj), _p(w), resid.size, C.c_float(eps), _p(h_mid), _p(h_post))
    return h_mid, h_post


def route(logits, K):
    """softmax -> top-K (reference tie rule, slot order) -> renormalise."""
    logits = _c(logits, np.float32)
    ls = logits.reshape(-1, logits.shape[-1])
    ids = np.empty((ls.shape[0], K), np.int32)
    w = np.empty((ls.shape[0], K), np.float32)
    for t in range(ls.shape[0]):
        lib().fo_route(_p(ls[t]), ls.shape[1], K, _p(ids[t]), _p(w[t]))
    return ids.reshape(logits.shape[:-1] + (K,)), w.reshape(logits.shape[:-1] + (K,))


def combine(h_mid, expert_out, w, valid, shared_out, shared_gate_score, guard=0):
    expert_out = _c(expert_out, np.float32)
    K, dim = expert_out.shape
    h_mid, shared_out = _c(h_mid, np.float32), _c(shared_out, np.float32)
    w, valid = _c(w, np.float32), _c(valid, np.uint8)
    out = np.empty(dim, np.float32)
    lib().fo_combine(_p(h_mid), _p(expert_out), _p(w), _p(valid), _p(shared_out),
                     C.c_float(shared_gate_score), dim, K, guard, _p(out))
    return out


def expert_layout(hidden, inter, group, bits):
    L = _Layout()
    lib().fo_expert_layout(hidden, inter, group, bits, C.byref(L))
    return {n: getattr(L, n) for n, _ in _Layout._fields_}


def expert_forward(block, bits, scale_dtype, hidden, inter, group, x, accum=ACC_F64):
    block, x = _c(block, np.uint8), _c(x, np.float32)
    out = np.empty(hidden, np.float32)
    lib().fo_expert_forward(_p(block), bits, scale_dtype, hidden, inter, group, _p(x), _p(out), accum)
    return out


def _wdesc(t):
    """t = dict(W,S,B,out_dim,in_dim,group,bits,scale_dtype) of numpy arrays."""
    keep = [_c(t["W"]), _c(t.get("S"), np.uint16), _c(t.get("B"), np.uint16)]
    d = _WDesc(_p(keep[0]), _p(keep[1]), _p(keep[2]), t["out_dim"], t["in_dim"], t.get("group", 64),
               t["bits"], t.get("scale_dtype", SCALE_BF16))
    return d, keep


def shared_forward(gate, up, down, x, accum=ACC_F64):
    dg, k0 = _wdesc(gate)
    du, k1 = _wdesc(up)
    dd, k2 = _wdesc(down)
    x = _c(x, np.float32)
    out = np.empty(down["out_dim"], np.float32)
    lib().fo_shared_forward(C.byref(dg), C.byref(du), C.byref(dd), _p(x), _p(out), accum)
    del k0, k1, k2
    return out


def moe_layer(blocks, w, valid, x, *, bits=3, scale_dtype=SCALE_BF16, hidden=2048, inter=512,
              group=64, h_mid=None, shared=None, shared_gate_score=0.0, guard=0, accum=ACC_F64,
              nthreads=1):
    """One token through one layer.  blocks: list of K uint8 arrays (or None
    where valid == 0); shared: None or (gate, up, down) dicts as in _wdesc."""
    K = len(blocks)
    keep = [None if b is None else _c(b, np.uint8) for b in blocks]
    ptrs = (C.c_void_p * K)(*[None if b is None else b.ctypes.data for b in keep])
    w, valid = _c(w, np.float32), _c(valid, np.uint8)
    x, h_mid = _c(x, np.float32), _c(h_mid, np.float32)
    descs = [None, None, None]
    kk = []
    if shared is not None:
        for i, t in enumerate(shared):
            d, k = _wdesc(t)
            descs[i] = d
            kk.append(k)
    out = np.empty(hidden, np.float32)
    lib().fo_moe_layer(ptrs, _p(w), _p(valid), K, bits, scale_dtype, hidden, inter, group, _p(x),
                       _p(h_mid), *[C.byref(d) if d is not None else None for d in descs],
                       C.c_float(shared_gate_score), guard, accum, nthreads, _p(out))
    del kk
    return out
