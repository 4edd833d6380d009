"""Host-side mirror of the reference's MoE dispatch seams on top of the C ABI.

Method names follow the functions of finchmoe/infer.m they stand in for
(``fast_dequant_matvec`` infer.m:3369, ``fast_batch_matvec`` 4477,
``expert_cache_*`` 6179-6291, ``gpu_encode_experts_batched`` 4065 ...); every
call goes through ``libfinchcuda.so`` -- there is no Python or CPU compute path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lib as L
from .synth import f32_to_bf16_rne


def _ptr(x):
    """numpy array / int / None / object with data_ptr() -> c_void_p value."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ptr"):
        return x.ptr
    raise TypeError(type(x))


class DeviceBuf:
    def __init__(self, ctx: "Context", ptr: int, nbytes: int):
        self.ctx, self.ptr, self.nbytes = ctx, ptr, nbytes

    def free(self):
        if self.ptr:
            self.ctx.lib.finch_buf_free(self.ctx.h, self.ptr)
            self.ptr = 0


class Pool:
    """expert_cache_new / lookup / insert / free (finchmoe/infer.m:6179-6291)."""

    def __init__(self, ctx: "Context", n_layers: int, n_experts: int, max_slots: int = 0):
        self.ctx = ctx
        h = C.c_void_p()
        ctx.check(ctx.lib.finch_pool_create(ctx.h, n_layers, n_experts, max_slots, C.byref(h)))
        self.h = h
        self.n_layers, self.n_experts = n_layers, n_experts

    def put(self, layer: int, expert: int, block: np.ndarray):
        block = np.ascontiguousarray(block, np.uint8)
        assert block.size == self.ctx.expert_bytes, (block.size, self.ctx.expert_bytes)
        self.ctx.check(self.ctx.lib.finch_pool_put(self.h, layer, expert, block.ctypes.data))

    def get(self, layer: int, expert: int) -> np.ndarray:
        out = np.empty(self.ctx.expert_bytes, np.uint8)
        self.ctx.check(self.ctx.lib.finch_pool_get(self.h, layer, expert, out.ctypes.data))
        return out

    def lookup(self, layer: int, expert: int):
        slot, ptr = C.c_int(-1), C.c_void_p()
        rc = self.ctx.lib.finch_pool_lookup(self.h, layer, expert, C.byref(slot), C.byref(ptr))
        if rc == L.E_NOSLOT:
            return None
        self.ctx.check(rc)
        return slot.value, ptr.value

    def stats(self) -> dict:
        st = L.PoolStats()
        self.ctx.check(self.ctx.lib.finch_pool_get_stats(self.h, C.byref(st)))
        return {n: getattr(st, n) for n, _ in L.PoolStats._fields_}

    def fill_synthetic(self, layer0: int, layer1: int, seed: int):
        self.ctx.check(self.ctx.lib.finch_pool_fill_synthetic(self.h, layer0, layer1, seed))

    def destroy(self):
        if self.h:
            self.ctx.lib.finch_pool_destroy(self.h)
            self.h = None


class Context:
    def __init__(self, *, hidden=2048, n_experts=256, top_k=8, moe_inter=512, shared_inter=512, group_size=64,
                 n_layers=40, expert_bits=3, scale_dtype=L.FP16, act_dtype=L.BF16, max_tokens=8, device=0):
        self.lib = L.load()
        self.cfg = L.Config(device, hidden, n_experts, top_k, moe_inter, shared_inter, group_size, n_layers,
                            expert_bits, scale_dtype, act_dtype, max_tokens)
        h = C.c_void_p()
        rc = self.lib.finch_ctx_create(C.byref(self.cfg), C.byref(h))
        if rc:
            raise L.FinchError(rc, self.lib.finch_status_str(rc).decode())
        self.h = h
        self.expert_bytes = self.lib.finch_expert_bytes(h)
        self._keep = []

    # -- plumbing
    def check(self, rc: int):
        if rc:
            raise L.FinchError(rc, self.lib.finch_last_error(self.h).decode() or self.lib.finch_status_str(rc).decode())

    def destroy(self):
        if self.h:
            self.lib.finch_ctx_destroy(self.h)
            self.h = None

    def sync(self):
        self.check(self.lib.finch_sync(self.h))

    def device_status(self) -> int:
        s = C.c_int(0)
        self.check(self.lib.finch_device_status(self.h, C.byref(s)))
        return s.value

    def device_status_clear(self):
        self.check(self.lib.finch_device_status_clear(self.h))

    def debug_fault(self, kind: int):
        """Failure injection for the tests of the bounded device-side waits (finch_debug_fault)."""
        self.check(self.lib.finch_debug_fault(self.h, kind))

    def launch_count(self) -> int:
        return int(self.lib.finch_launch_count(self.h))

    def alloc(self, nbytes: int) -> DeviceBuf:
        p = C.c_void_p()
        self.check(self.lib.finch_buf_alloc(self.h, nbytes, C.byref(p)))
        return DeviceBuf(self, p.value, nbytes)

    def upload(self, arr: np.ndarray) -> DeviceBuf:
        """metal_set_weights (finchmoe/infer.m:2813): host bytes -> device buffer."""
        arr = np.ascontiguousarray(arr)
        p = C.c_void_p()
        self.check(self.lib.finch_weights_upload(self.h, arr.ctypes.data, arr.nbytes, C.byref(p)))
        return DeviceBuf(self, p.value, arr.nbytes)

    def upload_tensor(self, t: dict) -> L.WDesc:
        """Uploads a tensor dict (W, S, B, out_dim, in_dim, bits, scale_dtype) and returns its descriptor."""
        w = self.upload(t["W"])
        s = self.upload(t["S"]) if t.get("S") is not None else None
        b = self.upload(t["B"]) if t.get("B") is not None else None
        self._keep += [w, s, b]
        return L.WDesc(w.ptr, s.ptr if s else None, b.ptr if b else None, t["out_dim"], t["in_dim"],
                       t.get("group", 64), t["bits"], t.get("scale_dtype", L.BF16))

    def pool(self, n_layers=None, n_experts=None, max_slots=0) -> Pool:
        return Pool(self, n_layers or self.cfg.n_layers, n_experts or self.cfg.n_experts, max_slots)

    def acts_to_wire(self, x: np.ndarray) -> np.ndarray:
        """fp32 activations -> the context's act_dtype as raw host bytes."""
        x = np.ascontiguousarray(x, np.float32)
        return f32_to_bf16_rne(x) if self.cfg.act_dtype == L.BF16 else x

    # -- matvec seams
    def fast_dequant_matvec(self, w: L.WDesc, x: np.ndarray) -> np.ndarray:
        """fast_dequant_matvec (finchmoe/infer.m:3369): host x [in] or [M, in] fp32 -> host out."""
        x = np.ascontiguousarray(x, np.float32)
        xs = x.reshape(-1, w.in_dim)
        out = np.empty((xs.shape[0], w.out_dim), np.float32)
        self.check(self.lib.finch_matvec(self.h, C.byref(w), xs.ctypes.data, out.ctypes.data, xs.shape[0]))
        return out.reshape(x.shape[:-1] + (w.out_dim,))

    def fast_batch_matvec(self, x, x_dtype: int, specs: list, outs: list, M: int = 1, stream=None):
        """gpu_encode_batch_matvec (finchmoe/infer.m:3528): device pointers, enqueues only."""
        arr = (L.WDesc * len(specs))(*specs)
        po = (C.c_void_p * len(outs))(*[_ptr(o) for o in outs])
        self.check(self.lib.finch_encode_batch_matvec(self.h, stream, _ptr(x), x_dtype, arr, po, len(specs), M))

    def route_topk(self, logits, n_experts: int, K: int, ids, weights, T: int, stream=None):
        self.check(self.lib.finch_encode_route_topk(self.h, stream, _ptr(logits), n_experts, K, _ptr(ids),
                                                    _ptr(weights), T))

    def debug_dequant(self, w: L.WDesc, w16_dtype: int = L.BF16):
        """--compare-experts probe: (codes u8, weights fp32, weights 16-bit) as numpy arrays."""
        n = (w.out_dim, w.in_dim)
        codes, w32, w16 = np.empty(n, np.uint8), np.empty(n, np.float32), np.empty(n, np.uint16)
        self.check(self.lib.finch_debug_dequant(self.h, C.byref(w), codes.ctypes.data, w32.ctypes.data,
                                                w16.ctypes.data, w16_dtype))
        return codes, w32, w16

    def dense_gemm(self, w: L.WDesc, x_bf16: np.ndarray) -> np.ndarray:
        """gpu_encode_prefill_matvec (finchmoe/infer.m:3672) on the tensor cores: host x as bf16 bits
        (uint16 [M, in]) -> host out fp32 [M, out].  torch holds the device buffers."""
        import torch
        x_bf16 = np.ascontiguousarray(x_bf16, np.uint16)
        M = x_bf16.shape[0]
        xd = torch.from_numpy(x_bf16.view(np.int16)).cuda()
        od = torch.empty((M, w.out_dim), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        self.check(self.lib.finch_encode_dense_gemm(self.h, None, C.byref(w), xd.data_ptr(), od.data_ptr(), M))
        self.sync()
        return od.cpu().numpy()

    # -- MoE layer
    def set_prefill_mode(self, mode: int):
        """0: by chunk length, 1: sub-batches through the decode kernels, 2: grouped dequant-GEMMs on tcgen05,
        3: grouped mma.sync passes (one unpack per unit for up to 16 tokens of an expert),
        4: grouped tcgen05 GEMMs whose A operand is the packed codes themselves (no dequantisation)."""
        self.check(self.lib.finch_set_prefill_mode(self.h, mode))
        self.prefill_mode = mode

    def set_prefill_chunk(self, tokens: int):
        """Tokens per pass of the tensor-core prefill path (0 = the default 512; at most max_tokens)."""
        self.check(self.lib.finch_set_prefill_chunk(self.h, tokens))
        self.prefill_chunk = tokens

    def make_shared(self, gate: L.WDesc, up: L.WDesc, down: L.WDesc, gate_score=None) -> L.Shared:
        return L.Shared(gate, up, down, _ptr(gate_score))

    def encode_moe_decode(self, pool: Pool, layer: int, h_post, ids, weights, valid, shared, h_mid, hidden_out,
                          B: int, stream=None, prefill=False):
        """gpu_encode_experts_batched + shared expert + moe_combine_residual (finchmoe/infer.m:4065, 9603-9703)."""
        fn = self.lib.finch_encode_moe_prefill if prefill else self.lib.finch_encode_moe_decode
        self.check(fn(self.h, stream, pool.h, layer, _ptr(h_post), _ptr(ids), _ptr(weights), _ptr(valid),
                      C.byref(shared) if shared is not None else None, _ptr(h_mid), _ptr(hidden_out), B))

    def encode_moe_gguf(self, experts: L.GgufExperts, h_post, ids, weights, valid, h_mid, hidden_out, B: int, stream=None):
        """gpu_gguf_experts_forward (finchmoe/infer.m:3153): device pointers, enqueues only."""
        self.check(self.lib.finch_encode_moe_gguf(self.h, stream, C.byref(experts), _ptr(h_post), _ptr(ids), _ptr(weights), _ptr(valid),
                                                  _ptr(h_mid), _ptr(hidden_out), B))

    def moe_forward_host_ptrs(self, pool: Pool, layer: int, h_post: int, ids: int, weights: int, valid: int | None, shared, gate_score: int | None,
                              h_mid: int | None, hidden_out: int, T: int):
        """finch_moe_forward_host on raw host addresses (arrays the caller keeps alive and contiguous): the call a C
        host makes, without the per-call array conversions of moe_forward_host."""
        rc = self.lib.finch_moe_forward_host(self.h, pool.h, layer, h_post, ids, weights, valid, shared, gate_score, h_mid, hidden_out, T)
        if rc:
            self.check(rc)

    def moe_forward_host(self, pool: Pool, layer: int, h_post: np.ndarray, ids: np.ndarray, weights: np.ndarray,
                         valid=None, shared: L.Shared | None = None, gate_score=None, h_mid=None) -> np.ndarray:
        """Host buffers in, host buffer out (one H2D, the kernels, one D2H, wait)."""
        T = ids.shape[0]
        xw = self.acts_to_wire(h_post) if h_post.dtype != np.uint16 else np.ascontiguousarray(h_post)
        ids = np.ascontiguousarray(ids, np.int32)
        weights = np.ascontiguousarray(weights, np.float32)
        valid = None if valid is None else np.ascontiguousarray(valid, np.uint8)
        gs = None if gate_score is None else np.ascontiguousarray(gate_score, np.float32)
        hm = None if h_mid is None else np.ascontiguousarray(h_mid, np.float32)
        out = np.empty((T, self.cfg.hidden), np.float32)
        self.check(self.lib.finch_moe_forward_host(self.h, pool.h, layer, xw.ctypes.data, ids.ctypes.data,
                                                   weights.ctypes.data, _ptr(valid),
                                                   C.byref(shared) if shared is not None else None, _ptr(gs),
                                                   _ptr(hm), out.ctypes.data, T))
        return out
