"""ctypes binding of libfinchcuda.so (the C ABI declared in include/finch_cuda.h).

There is no CPU fallback: if the shared library is missing or a symbol cannot
be resolved, importing the library raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
SO_PATH = os.path.join(PKG, "libfinchcuda.so")
SO_PATH = os.environ.get("FINCH_CUDA_SO", SO_PATH)   # another build of the same sources (e.g. one with phase stamps)
HEADER = os.path.join(os.path.dirname(PKG), "include", "finch_cuda.h")

OK, E_ARG, E_NOSLOT, E_CUDA, E_NCCL, E_TIMEOUT, E_UNSUPPORTED, E_NOMEM = range(8)
BF16, FP16, F32 = 0, 1, 2
BITS_BF16, BITS_Q4_K, BITS_Q6_K = 0, 10, 11


class FinchError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"finch status {status}: {msg}")
        self.status = status


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("device", "hidden", "n_experts", "top_k", "moe_inter", "shared_inter",
                                       "group_size", "n_layers", "expert_bits", "scale_dtype", "act_dtype",
                                       "max_tokens")]


class WDesc(C.Structure):
    _fields_ = [("W", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p), ("out_dim", C.c_int),
                ("in_dim", C.c_int), ("group_size", C.c_int), ("bits", C.c_int), ("scale_dtype", C.c_int)]


class Shared(C.Structure):
    _fields_ = [("gate", WDesc), ("up", WDesc), ("down", WDesc), ("gate_score", C.c_void_p)]


class GgufExperts(C.Structure):
    _fields_ = [("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p), ("gate_slab", C.c_size_t), ("up_slab", C.c_size_t),
                ("down_slab", C.c_size_t), ("gate_type", C.c_int), ("up_type", C.c_int), ("down_type", C.c_int)]


class PoolStats(C.Structure):
    _fields_ = [("hits", C.c_uint64), ("misses", C.c_uint64), ("evictions", C.c_uint64), ("slots", C.c_int),
                ("used", C.c_int), ("slot_bytes", C.c_size_t)]


_vp, _i, _sz = C.c_void_p, C.c_int, C.c_size_t
_PROTOS = {
    "finch_ctx_create": (_i, [C.POINTER(Config), C.POINTER(_vp)]),
    "finch_ctx_destroy": (None, [_vp]),
    "finch_last_error": (C.c_char_p, [_vp]),
    "finch_status_str": (C.c_char_p, [_i]),
    "finch_expert_bytes": (_sz, [_vp]),
    "finch_weights_upload": (_i, [_vp, _vp, _sz, C.POINTER(_vp)]),
    "finch_buf_alloc": (_i, [_vp, _sz, C.POINTER(_vp)]),
    "finch_buf_free": (_i, [_vp, _vp]),
    "finch_pool_create": (_i, [_vp, _i, _i, _i, C.POINTER(_vp)]),
    "finch_pool_destroy": (None, [_vp]),
    "finch_pool_put": (_i, [_vp, _i, _i, _vp]),
    "finch_pool_get": (_i, [_vp, _i, _i, _vp]),
    "finch_pool_lookup": (_i, [_vp, _i, _i, C.POINTER(_i), C.POINTER(_vp)]),
    "finch_pool_get_stats": (_i, [_vp, C.POINTER(PoolStats)]),
    "finch_pool_fill_synthetic": (_i, [_vp, _i, _i, C.c_uint64]),
    "finch_matvec": (_i, [_vp, C.POINTER(WDesc), _vp, _vp, _i]),
    "finch_matvec_noalloc": (_i, [C.POINTER(WDesc), _vp, _vp, _i, _vp]),
    "finch_encode_batch_matvec": (_i, [_vp, _vp, _vp, _i, C.POINTER(WDesc), C.POINTER(_vp), _i, _i]),
    "finch_encode_route_topk": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _i]),
    "finch_encode_moe_decode": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, C.POINTER(Shared), _vp, _vp, _i]),
    "finch_encode_moe_decode_multi": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _i, C.POINTER(Shared), _vp, _vp, _vp]),
    "finch_encode_moe_prefill": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, C.POINTER(Shared), _vp, _vp, _i]),
    "finch_set_prefill_mode": (_i, [_vp, _i]),
    "finch_set_prefill_chunk": (_i, [_vp, _i]),
    "finch_encode_dense_gemm": (_i, [_vp, _vp, C.POINTER(WDesc), _vp, _vp, _i]),
    "finch_ep_record_bytes": (_i, [_vp]),
    "finch_encode_ep_plan": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "finch_encode_ep_pack": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    "finch_encode_ep_unpack": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp]),
    "finch_encode_ep_combine": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i]),
    "finch_ep_peer_create": (_i, [_vp, _i, _i, _i, C.POINTER(_vp)]),
    "finch_ep_peer_export": (_i, [_vp, _vp]),
    "finch_ep_peer_import": (_i, [_vp, _i, _vp]),
    "finch_ep_peer_area": (_vp, [_vp]),
    "finch_ep_peer_attach": (_i, [_vp, _i, _vp]),
    "finch_ep_peer_set_wait_limit": (_i, [_vp, C.c_longlong]),
    "finch_ep_peer_reset": (_i, [_vp]),
    "finch_ep_peer_destroy": (_i, [_vp]),
    "finch_encode_ep_peer_dispatch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "finch_encode_ep_peer_receive": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i]),
    "finch_encode_ep_peer_return": (_i, [_vp, _vp, _vp, _vp]),
    "finch_encode_ep_peer_decode": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "finch_encode_ep_peer_combine": (_i, [_vp, _vp, _vp, _vp]),
    "finch_pool_fill_synthetic_range": (_i, [_vp, _i, _i, _i, _i, C.c_uint64]),
    "finch_encode_residual_norm": (_i, [_vp, _vp, _vp, _vp, _vp, C.c_float, _vp, _vp, _i]),
    "finch_encode_router": (_i, [_vp, _vp, C.POINTER(WDesc), C.POINTER(WDesc), _vp, _vp, _vp, _vp, _i]),
    "finch_encode_moe_gguf": (_i, [_vp, _vp, C.POINTER(GgufExperts), _vp, _vp, _vp, _vp, _vp, _vp, _i]),
    "finch_moe_forward_host": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, C.POINTER(Shared), _vp, _vp, _vp, _i]),
    "finch_event_create": (_i, [_vp, C.POINTER(_vp)]),
    "finch_event_record": (_i, [_vp, _vp]),
    "finch_event_wait": (_i, [_vp, _i]),
    "finch_event_destroy": (None, [_vp]),
    "finch_sync": (_i, [_vp]),
    "finch_device_status": (_i, [_vp, C.POINTER(_i)]),
    "finch_device_status_clear": (_i, [_vp]),
    "finch_debug_dequant": (_i, [_vp, C.POINTER(WDesc), _vp, _vp, _vp, _i]),
    "finch_launch_count": (C.c_uint64, [_vp]),
    "finch_debug_fault": (_i, [_vp, _i]),
    "finch_profile_enable": (_i, [_vp, _i]),
    "finch_profile_read": (_i, [_vp, C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(_i)]),
}


def declared_symbols(header: str = HEADER) -> list[str]:
    """Every FINCH_API function the public header declares."""
    with open(header) as f:
        text = f.read()
    return sorted(set(re.findall(r"FINCH_API\s+[\w\s\*]+?\b(finch_\w+)\s*\(", text)))


_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(SO_PATH):
            raise ImportError(f"{SO_PATH} is missing: build it with `python -m finchmoe_b200.build` "
                              "(there is no CPU fallback)")
        lib = C.CDLL(SO_PATH)
        for name, (res, args) in _PROTOS.items():
            fn = getattr(lib, name)  # AttributeError if the symbol is not exported
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
