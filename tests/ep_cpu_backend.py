"""CPU stand-in for finchmoe_b200.ep.GpuBackend: the same five operations on numpy arrays, with the
oracle as the expert arithmetic.  Test infrastructure only."""
import numpy as np
import torch

from finchmoe_b200 import ep
from oracle import oracle


class _Plan:
    pass


class NumpyBackend:
    def __init__(self, cfg, local_blocks, shared_tensors):
        """cfg: dict(hidden, inter, n_experts, K, sd); local_blocks: {global expert id: packed block} held
        by this rank; shared_tensors: (gate, up, down) dicts or None."""
        self.cfg, self.blocks, self.shared_t = cfg, local_blocks, shared_tensors
        self.hidden, self.K = cfg["hidden"], cfg["K"]

    def stream_scope(self):
        import contextlib
        return contextlib.nullcontext()

    def record_bytes(self):
        return (self.hidden * 4 + 9 * self.K + 15) & ~15

    def empty_bytes(self, n):
        return torch.empty(n, dtype=torch.uint8)

    def empty_f32(self, n):
        return torch.empty(n, dtype=torch.float32)

    def plan(self, ids, valid, world):
        p = _Plan()
        p.world = world
        counts, offs, send_tok, slot_of = ep.plan_numpy(ids.numpy(), None if valid is None else valid.numpy(), self.cfg["n_experts"], world)
        p.counts, p.offs, p.send_tok, p.slot_of = torch.from_numpy(counts), offs, send_tok, slot_of
        return p

    def static_plan(self, T, world, skip=-1):
        p = _Plan()
        p.world = world
        counts, p.offs, p.send_tok, p.slot_of = ep.static_plan_numpy(T, world, skip)
        p.counts = torch.from_numpy(counts)
        return p

    def pack(self, p, x, ids, weights, valid, n_rows):
        rec, H, K = self.record_bytes(), self.hidden, self.K
        buf = np.zeros((n_rows, rec), np.uint8)
        xn, idn, wn = x.numpy(), ids.numpy(), weights.numpy()
        vn = np.ones_like(idn, dtype=np.uint8) if valid is None else valid.numpy()
        for i, t in enumerate(p.send_tok):
            buf[i, :H * 4] = xn[t].view(np.uint8)
            buf[i, H * 4:H * 4 + 4 * K] = idn[t].view(np.uint8)
            buf[i, H * 4 + 4 * K:H * 4 + 8 * K] = wn[t].view(np.uint8)
            buf[i, H * 4 + 8 * K:H * 4 + 9 * K] = vn[t]
        return torch.from_numpy(buf.reshape(-1))

    def local_moe(self, layer, recv_buf, n, skip=None):
        rec, H, K, c = self.record_bytes(), self.hidden, self.K, self.cfg
        buf = recv_buf.numpy().reshape(n, rec)
        out = np.zeros((n, H), np.float32)
        for i in range(n):
            x = buf[i, :H * 4].copy().view(np.float32)
            ids = buf[i, H * 4:H * 4 + 4 * K].copy().view(np.int32)
            w = buf[i, H * 4 + 4 * K:H * 4 + 8 * K].copy().view(np.float32)
            v = buf[i, H * 4 + 8 * K:H * 4 + 9 * K].copy()
            blocks = [self.blocks.get(int(e)) if v[k] else None for k, e in enumerate(ids)]
            vv = np.array([b is not None for b in blocks], np.uint8)
            out[i] = oracle.moe_layer(blocks, w, vv, x, bits=3, scale_dtype=c["sd"], hidden=H, inter=c["inter"])
        return torch.from_numpy(out)

    def base(self, layer, x, ids, weights, shared, h_mid, out):
        xn = x.numpy()
        o = np.zeros((xn.shape[0], self.hidden), np.float32) if h_mid is None else h_mid.numpy().copy()
        if shared is not None:   # shared = gate scores (fp32 [T]) in this backend
            for t in range(xn.shape[0]):
                so = oracle.shared_forward(*self.shared_t, xn[t])
                o[t] += (np.float32(1.0) / (np.float32(1.0) + np.exp(-np.float32(shared[t])))) * so
        out.copy_(torch.from_numpy(o))

    def combine(self, p, out, back):
        H = self.hidden
        b = back.numpy().reshape(-1, H)
        o = out.numpy()
        for t in range(o.shape[0]):
            for d in range(p.world):
                s = p.slot_of[t, d]
                if s >= 0:
                    o[t] += b[p.offs[d] + s]
