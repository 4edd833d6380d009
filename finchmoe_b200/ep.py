"""Expert-parallel MoE layer: one process per GPU, experts sharded in contiguous blocks.

Rank r of G owns experts [r*E/G, (r+1)*E/G) of every layer and keeps only those in its HBM pool;
tokens stay with the rank that owns them (each rank routes its own tokens).  One layer:

  1. plan      which of my tokens go to which rank -- a token goes to a rank once, with its whole row of
               expert ids and router weights, however many of its experts live there
  2. counts    all-to-all of the per-destination row counts (the only host synchronisation of the layer)
  3. dispatch  all-to-all of the packed records (activation row + ids + weights + mask)
  4. local     the rank's ordinary MoE path over the rows it received; experts that are not in its
               pool are skipped, so each output row is the weighted sum over the local experts
  5. return    all-to-all of the fp32 partial rows
  6. combine   hidden = h_mid + shared expert (computed where the token lives) + partial rows added in
               ascending rank order, so the result does not depend on arrival order

The collectives go through torch.distributed (NCCL on GPUs; gloo in the CPU tests).  `ep_layer` holds the
protocol and is backend-agnostic: the GPU backend drives the C-ABI steps (finch_encode_ep_*), the CPU
tests plug in a numpy backend with the same five operations.  With G = 1 the same code runs and the
all-to-alls degenerate to copies.

`ep_layer_static` is the same layer for decode-sized batches of equal size on every rank: the plan is fixed
(every token to every rank), so steps 1 and 2 and the host synchronisation disappear, the home rank works on its
own tokens while the records travel, and the layer can be recorded into a CUDA graph.

The reference runs on one device (finchmoe/infer.m:9597-9741 is the per-layer path this extends).
"""
from __future__ import annotations

import ctypes as C

import numpy as np


def owner_of(expert: int, n_experts: int, world: int) -> int:
    return expert // (n_experts // world)


def plan_numpy(ids: np.ndarray, valid, n_experts: int, world: int, skip: int = -1):
    """Host mirror of finch_encode_ep_plan: (counts[G], offs[G+1], send_tok, slot_of[T,G]).  Nothing goes to rank `skip`."""
    T, K = ids.shape
    per = n_experts // world
    ok = (ids >= 0) & (ids < n_experts)
    if valid is not None:
        ok &= valid.astype(bool)
    dest = np.where(ok, ids // per, -1)
    counts = np.zeros(world, np.int32)
    slot_of = np.full((T, world), -1, np.int32)
    lists = []
    for d in range(world):
        toks = np.nonzero((dest == d).any(axis=1))[0].astype(np.int32) if d != skip else np.zeros(0, np.int32)
        counts[d] = toks.size
        slot_of[toks, d] = np.arange(toks.size, dtype=np.int32)
        lists.append(toks)
    offs = np.zeros(world + 1, np.int32)
    offs[1:] = np.cumsum(counts)
    return counts, offs, np.concatenate(lists) if lists else np.zeros(0, np.int32), slot_of


def ep_layer(backend, dist, group, layer: int, x, ids, weights, valid, shared, h_mid, out):
    """The protocol.  `dist` is torch.distributed (or None for a single process); tensors are whatever
    the backend uses (torch tensors on the backend's device).  Returns `out`."""
    with backend.stream_scope():
        return _ep_layer(backend, dist, group, layer, x, ids, weights, valid, shared, h_mid, out)


def _ep_layer(backend, dist, group, layer, x, ids, weights, valid, shared, h_mid, out):
    import torch
    world = dist.get_world_size(group) if dist is not None else 1
    rank = dist.get_rank(group) if dist is not None else 0
    # Two ways to treat the tokens' experts that live on the home rank.  planned_direct: nothing is sent to the home
    # rank itself; one pass over its tokens gives h_mid + shared expert + the experts this rank holds while the
    # records travel, and a second pass serves the received rows.  Otherwise (the default) the rank's own rows take
    # the same route as everybody else's (a local copy inside the all-to-all) and ONE pass serves all rows of the
    # rank's experts -- the grouped GEMMs dequantise an expert's tile once per pass, so one fuller pass beats
    # two -- while h_mid + shared expert is computed during the exchange.
    direct = getattr(backend, "planned_direct", False) or (world == 1 and getattr(backend, "home_direct", False))
    overlap = hasattr(backend, "home")             # the GPU backend: collectives run beside its stream
    h = backend.plan(ids, valid, world, rank) if direct else backend.plan(ids, valid, world)   # .counts: int32 [G] tensor
    recv_counts = torch.empty_like(h.counts)
    if world > 1:
        dist.all_to_all_single(recv_counts, h.counts, group=group)
    else:
        recv_counts.copy_(h.counts)
    c_send = h.counts.cpu().tolist()                           # host sync: split sizes must be host integers
    c_recv = recv_counts.cpu().tolist()
    if getattr(backend, "stats", None) is not None:            # rows that left for / arrived from every rank, this layer
        backend.stats.append((c_send, c_recv))
    rec = backend.record_bytes()
    send_buf = backend.pack(h, x, ids, weights, valid, sum(c_send))            # uint8 [sum(c_send) * rec]
    recv_buf = backend.empty_bytes(sum(c_recv) * rec)
    work = None
    if world > 1:
        work = dist.all_to_all_single(recv_buf, send_buf, [c * rec for c in c_recv], [c * rec for c in c_send], group=group, async_op=overlap)
    else:
        recv_buf.copy_(send_buf)
    if direct:
        backend.home(layer, x, ids, weights, valid, shared, h_mid, out)
    elif overlap:
        backend.base(layer, x, ids, weights, shared, h_mid, out)                # h_mid + shared expert, no routed expert
    if work is not None:
        work.wait()
    part = backend.local_moe(layer, recv_buf, sum(c_recv))                      # fp32 [sum(c_recv), H]
    H = backend.hidden
    back = backend.empty_f32(sum(c_send) * H)
    if world > 1:
        dist.all_to_all_single(back, part.reshape(-1), [c * H for c in c_send], [c * H for c in c_recv], group=group)
    else:
        back.copy_(part.reshape(-1))
    if not direct and not overlap:
        backend.base(layer, x, ids, weights, shared, h_mid, out)
    backend.combine(h, out, back)
    return out


def static_plan_numpy(T: int, world: int, skip: int = -1):
    """The plan of the fixed-capacity exchange: every token goes to every rank, in token order.  Same
    four arrays as plan_numpy.  skip: a rank whose returned rows the combine step leaves out (the home
    rank, when it adds its own experts' share to the output directly)."""
    counts = np.full(world, T, np.int32)
    offs = (np.arange(world + 1, dtype=np.int32) * T).astype(np.int32)
    send_tok = np.tile(np.arange(T, dtype=np.int32), world)
    slot_of = np.repeat(np.arange(T, dtype=np.int32)[:, None], world, axis=1)
    if skip >= 0:
        slot_of[:, skip] = -1
    return counts, offs, send_tok, slot_of


def ep_layer_static(backend, dist, group, layer: int, x, ids, weights, valid, shared, h_mid, out, in_scope=False):
    """The same layer with a fixed-capacity exchange: every rank owns the same number of tokens T and sends
    each of them to every rank, so all message sizes are known beforehand.  No row counts are exchanged and
    the host never waits for the device: the whole layer is a fixed sequence of launches and two
    all-to-alls with equal splits, which can also be recorded into a CUDA graph (in_scope=True: the caller
    has already made the backend's stream current, as a graph capture does).  A rank skips the experts
    it does not hold, so rows that have no expert there cost it no weight traffic and come back as zeros.
    Meant for decode-sized batches, where the rows are few and latency is what matters; the planned
    exchange (ep_layer) sends less when batches are large."""
    if in_scope:
        return _ep_layer_static(backend, dist, group, layer, x, ids, weights, valid, shared, h_mid, out)
    with backend.stream_scope():
        return _ep_layer_static(backend, dist, group, layer, x, ids, weights, valid, shared, h_mid, out)


def _ep_layer_static(backend, dist, group, layer, x, ids, weights, valid, shared, h_mid, out):
    world = dist.get_world_size(group) if dist is not None else 1
    rank = dist.get_rank(group) if dist is not None else 0
    T = ids.shape[0]
    # A backend that can run the home rank's own tokens straight from their buffers does so while the records
    # are in flight: one pass gives h_mid + shared expert + the experts this rank holds, and the rows the rank
    # would have sent to itself are neither processed a second time nor added again.
    direct = getattr(backend, "home_direct", False)
    if direct and world == 1:      # every expert is here: the rank's ordinary pass over its own tokens is the layer
        backend.home(layer, x, ids, weights, valid, shared, h_mid, out)
        return out
    peer = getattr(backend, "peer", None)
    if peer is not None and direct and peer.world == world and peer.T == T:
        # The ranks' own kernels move the records and the partial rows through each other's memory (NVLink), each
        # slot with its flag: no collective and no host step, the whole layer is launches on the backend's stream.
        backend.peer_dispatch(x, ids, weights, valid)
        if backend.can_multi(T, world) and getattr(backend, "fuse_return", False):
            # the same launch sequence, whose last kernel also stores the other ranks' rows into their areas: the
            # return step without a kernel of its own
            backend.peer_decode(layer, shared, h_mid, out)
            backend.peer_combine(out)
            return out
        if backend.can_multi(T, world):
            # one launch sequence serves every rank's batch of T rows, the rank's own among them (with h_mid and the
            # shared expert): batch c = the tokens of rank c, of which only the experts held here are computed
            part = backend.peer_local_multi(layer, T, world, rank, shared, h_mid, out)
        else:
            backend.home(layer, x, ids, weights, valid, shared, h_mid, out)      # while the peers' records arrive
            part = backend.peer_local_moe(layer, T * world, (rank * T, T))
        backend.peer_return(part)
        backend.peer_combine(out)
        return out
    h = backend.static_plan(T, world, rank if direct else -1)
    rec, H, n = backend.record_bytes(), backend.hidden, T * world
    send_buf = backend.pack(h, x, ids, weights, valid, n)
    multi = direct and hasattr(backend, "can_multi") and backend.can_multi(T, world)
    if world > 1:
        recv_buf = backend.empty_bytes(n * rec)
        work = dist.all_to_all_single(recv_buf, send_buf, group=group, async_op=True)    # equal splits: T records per peer
        if direct and not multi:
            backend.home(layer, x, ids, weights, valid, shared, h_mid, out)
        work.wait()
    else:
        recv_buf = send_buf
    if multi:      # every rank's batch, the rank's own among them (h_mid, shared expert), in one launch sequence
        part = backend.local_multi(layer, recv_buf, T, world, rank, shared, h_mid, out)
    else:
        part = backend.local_moe(layer, recv_buf, n, (rank * T, T) if direct else None)   # fp32 [n, H], source-major
    if world > 1:
        back = backend.empty_f32(n * H)
        dist.all_to_all_single(back, part.reshape(-1), group=group)
    else:
        back = part.reshape(-1)
    if not direct:
        backend.base(layer, x, ids, weights, shared, h_mid, out)
    backend.combine(h, out, back)
    return out


class _Plan:
    pass


class PeerExchange:
    """This rank's receive area for the fixed-capacity layer and the other ranks' areas mapped into this process
    (finch_ep_peer_*): T tokens per rank, `world` ranks on one node."""

    def __init__(self, ctx, rank: int, world: int, T: int):
        self.ctx, self.rank, self.world, self.T = ctx, rank, world, T
        self.h = C.c_void_p()
        ctx.check(ctx.lib.finch_ep_peer_create(ctx.h, rank, world, T, C.byref(self.h)))

    def export(self) -> bytes:
        buf = C.create_string_buffer(64)
        self.ctx.check(self.ctx.lib.finch_ep_peer_export(self.h, buf))
        return buf.raw

    def import_handle(self, src_rank: int, handle: bytes):
        self.ctx.check(self.ctx.lib.finch_ep_peer_import(self.h, src_rank, C.create_string_buffer(handle, 64)))

    def area(self) -> int:
        return self.ctx.lib.finch_ep_peer_area(self.h)

    def attach(self, src_rank: int, area: int):
        self.ctx.check(self.ctx.lib.finch_ep_peer_attach(self.h, src_rank, C.c_void_p(area)))

    def set_wait_limit(self, polls: int):
        self.ctx.check(self.ctx.lib.finch_ep_peer_set_wait_limit(self.h, polls))

    def reset(self):
        self.ctx.check(self.ctx.lib.finch_ep_peer_reset(self.h))

    def destroy(self):
        if self.h:
            self.ctx.lib.finch_ep_peer_destroy(self.h)
            self.h = None

    @classmethod
    def connect(cls, ctx, dist, group, T: int):
        """Collective over the group: every rank creates its area and maps the others'.  Returns None on every rank
        when any rank could not (no peer access between the devices, handles that cannot cross the processes)."""
        import torch
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        px, payload = None, None
        try:
            px = cls(ctx, rank, world, T)
            payload = px.export()
        except Exception:
            payload = None
        handles = [None] * world
        dist.all_gather_object(handles, payload, group=group)      # every rank takes part, whatever happened above
        ok = 1 if all(hd is not None for hd in handles) else 0
        if ok:
            try:
                for r, hd in enumerate(handles):
                    if r != rank:
                        px.import_handle(r, hd)
            except Exception:
                ok = 0
        flag = torch.tensor([ok], device=torch.device("cuda", ctx.cfg.device))
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        if int(flag.item()) == 0:
            if px is not None and px.h:
                px.destroy()
            return None
        dist.barrier(group)
        return px


class GpuBackend:
    """Drives the C-ABI steps on one GPU.  torch holds the device buffers."""

    def __init__(self, ctx, pool, max_rows: int):
        """max_rows: the most rows this rank may receive in one layer (sum over sources)."""
        import torch
        self.torch, self.ctx, self.pool, self.lib = torch, ctx, pool, ctx.lib
        self.hidden, self.K = ctx.cfg.hidden, ctx.cfg.top_k
        self.elt = 2 if ctx.cfg.act_dtype == 0 else 4
        self.max_rows = max_rows
        dev = torch.device("cuda", ctx.cfg.device)
        self.dev = dev
        self.rx = torch.empty(max_rows * self.hidden * self.elt, dtype=torch.uint8, device=dev)
        self.rids = torch.empty((max_rows, self.K), dtype=torch.int32, device=dev)
        self.rw = torch.empty((max_rows, self.K), dtype=torch.float32, device=dev)
        self.rv = torch.empty((max_rows, self.K), dtype=torch.uint8, device=dev)
        self.rout = torch.empty((max_rows, self.hidden), dtype=torch.float32, device=dev)
        self.zero_valid = None
        self._static = {}
        self.multi = True            # decode-sized batches of all ranks in one launch sequence (finch_encode_moe_decode_multi)
        self.peer = None             # a connected PeerExchange routes the fixed-capacity layer through peer memory
        self.fuse_return = True      # ... and the decode pass's last kernel stores the other ranks' rows into their areas itself
        self.stats = None            # a list makes ep_layer append (rows sent per rank, rows received per rank) per layer
        # Received rows select few local experts each.  More than one decode-sized batch of them goes through the
        # tensor-core path in passes of `tc_chunk` rows (one sort and one pair of grouped GEMMs per pass) instead of
        # one decode pass per 8 rows.
        self.tc_rows_min = 9
        # how the received rows' experts run: 2 = tcgen05 grouped GEMMs, 3 = grouped mma.sync passes, 0 = by the tokens an
        # expert sees on average (rows * top_k / n_experts): the GEMMs from 64 up, where a 64-token tile fills
        self.tc_mode = 0
        self.tc_chunk = min(ctx.cfg.max_tokens, max_rows, 4096)

        self.stream = torch.cuda.Stream(device=dev)   # kernels, copies and collectives of a layer are ordered on it

    def _stream(self):
        return self.stream.cuda_stream

    def stream_scope(self):
        """Runs the layer on the backend's stream: it first waits for what the caller's stream has queued
        (the inputs), and the caller's stream waits for it afterwards."""
        import contextlib
        torch = self.torch

        @contextlib.contextmanager
        def scope():
            outer = torch.cuda.current_stream(self.dev)
            self.stream.wait_stream(outer)
            with torch.cuda.stream(self.stream):
                yield
            outer.wait_stream(self.stream)
        return scope()

    def record_bytes(self):
        return self.lib.finch_ep_record_bytes(self.ctx.h)

    def empty_bytes(self, n):
        return self.torch.empty(n, dtype=self.torch.uint8, device=self.dev)

    def empty_f32(self, n):
        return self.torch.empty(n, dtype=self.torch.float32, device=self.dev)

    def plan(self, ids, valid, world, skip=-1):
        torch = self.torch
        T = ids.shape[0]
        p = _Plan()
        p.T, p.world = T, world
        p.counts = torch.empty(world, dtype=torch.int32, device=self.dev)
        p.offs = torch.empty(world + 1, dtype=torch.int32, device=self.dev)
        p.send_tok = torch.empty(T * world, dtype=torch.int32, device=self.dev)
        p.slot_of = torch.empty((T, world), dtype=torch.int32, device=self.dev)
        self.ctx.check(self.lib.finch_encode_ep_plan(self.ctx.h, self._stream(), ids.data_ptr(), valid.data_ptr() if valid is not None else None,
                                                     T, world, skip, p.counts.data_ptr(), p.offs.data_ptr(), p.send_tok.data_ptr(),
                                                     p.slot_of.data_ptr()))
        return p

    home_direct = True        # fixed-capacity layer: the rank's own tokens in one in-place pass
    planned_direct = False    # planned layer: see _ep_layer

    def static_plan(self, T, world, skip=-1):
        """Device copy of static_plan_numpy, made once per (T, world, skip)."""
        torch = self.torch
        key = (T, world, skip)
        if key not in self._static:
            counts, offs, send_tok, slot_of = static_plan_numpy(T, world, skip)
            p = _Plan()
            p.T, p.world = T, world
            p.counts = torch.from_numpy(counts).to(self.dev)
            p.offs = torch.from_numpy(offs).to(self.dev)
            p.send_tok = torch.from_numpy(send_tok).to(self.dev)
            p.slot_of = torch.from_numpy(np.ascontiguousarray(slot_of)).to(self.dev)
            self._static[key] = p
        return self._static[key]

    def pack(self, p, x, ids, weights, valid, n_rows):
        buf = self.empty_bytes(n_rows * self.record_bytes())
        if n_rows == 0:   # nothing leaves this rank (no token picked an expert elsewhere, or every pair is masked)
            return buf
        self.ctx.check(self.lib.finch_encode_ep_pack(self.ctx.h, self._stream(), x.data_ptr(), ids.data_ptr(), weights.data_ptr(),
                                                     valid.data_ptr() if valid is not None else None, p.T, p.world, p.offs.data_ptr(),
                                                     p.send_tok.data_ptr(), buf.data_ptr()))
        return buf

    def home(self, layer, x, ids, weights, valid, shared, h_mid, out):
        """out = h_mid + shared expert + the experts of this rank's pool, for the rank's own tokens."""
        T = ids.shape[0]
        st = self._stream()
        step = self.ctx.cfg.max_tokens
        for t0 in range(0, T, step):
            m = min(step, T - t0)
            sh = None
            if shared is not None:
                from . import lib as L
                sh = L.Shared(shared.gate, shared.up, shared.down, shared.gate_score + 4 * t0)
            self.ctx.check(self.lib.finch_encode_moe_prefill(
                self.ctx.h, st, self.pool.h, layer, x.data_ptr() + t0 * self.hidden * self.elt, ids[t0:].data_ptr(), weights[t0:].data_ptr(),
                valid[t0:].data_ptr() if valid is not None else None, C.byref(sh) if sh is not None else None,
                h_mid[t0:].data_ptr() if h_mid is not None else None, out[t0:].data_ptr(), m))

    def local_moe(self, layer, recv_buf, n, skip=None):
        """skip = (first row, rows): a block of received rows that is left out (its output rows are not written)."""
        if n > self.max_rows:
            raise ValueError(f"received {n} rows, backend sized for {self.max_rows}")
        if n == 0:
            return self.rout[:0]
        st = self._stream()
        self.ctx.check(self.lib.finch_encode_ep_unpack(self.ctx.h, st, recv_buf.data_ptr(), n, self.rx.data_ptr(), self.rids.data_ptr(),
                                                       self.rw.data_ptr(), self.rv.data_ptr()))
        return self._moe_rows(layer, n, skip)

    def _moe_rows(self, layer, n, skip=None):
        """The rank's MoE path over rows [0, n) of rx / rids / rw / rv -> rout."""
        st = self._stream()
        step = self.ctx.cfg.max_tokens
        blocks = [(0, n)] if skip is None else [(0, skip[0]), (skip[0] + skip[1], n)]
        rows = sum(hi - lo for lo, hi in blocks)
        tc = rows >= self.tc_rows_min and step >= 16
        if tc:
            mode = self.tc_mode or (2 if rows * self.K >= 64 * self.ctx.cfg.n_experts else 3)
            self.ctx.check(self.lib.finch_set_prefill_mode(self.ctx.h, mode))
            self.ctx.check(self.lib.finch_set_prefill_chunk(self.ctx.h, min(self.tc_chunk, step)))
            if skip is not None:     # one pass over all rows; the block that is left out selects nothing
                self.rv[skip[0]:skip[0] + skip[1]].zero_()
                blocks = [(0, n)]
        try:
            for r0, m in ((r, min(step, hi - r)) for lo, hi in blocks for r in range(lo, hi, step)):
                self.ctx.check(self.lib.finch_encode_moe_prefill(
                    self.ctx.h, st, self.pool.h, layer, self.rx.data_ptr() + r0 * self.hidden * self.elt, self.rids[r0:].data_ptr(),
                    self.rw[r0:].data_ptr(), self.rv[r0:].data_ptr(), None, None, self.rout[r0:].data_ptr(), m))
        finally:
            if tc:
                self.ctx.check(self.lib.finch_set_prefill_mode(self.ctx.h, getattr(self.ctx, "prefill_mode", 0)))
                self.ctx.check(self.lib.finch_set_prefill_chunk(self.ctx.h, getattr(self.ctx, "prefill_chunk", 0)))
        return self.rout[:n]

    # -- the exchange through peer memory (PeerExchange)
    def peer_dispatch(self, x, ids, weights, valid):
        self.ctx.check(self.lib.finch_encode_ep_peer_dispatch(self.ctx.h, self._stream(), self.peer.h, x.data_ptr(), ids.data_ptr(), weights.data_ptr(),
                                                              valid.data_ptr() if valid is not None else None))

    def peer_receive(self, mask_own: bool):
        self.ctx.check(self.lib.finch_encode_ep_peer_receive(self.ctx.h, self._stream(), self.peer.h, self.rx.data_ptr(), self.rids.data_ptr(),
                                                             self.rw.data_ptr(), self.rv.data_ptr(), 1 if mask_own else 0))

    def peer_local_moe(self, layer, n, skip):
        if n > self.max_rows:
            raise ValueError(f"{n} rows, backend sized for {self.max_rows}")
        self.peer_receive(True)
        return self._moe_rows(layer, n, skip)

    def can_multi(self, T, world):
        """finch_encode_moe_decode_multi takes the layer: decode-sized batches, one per rank."""
        c = self.ctx.cfg
        return self.multi and T <= 8 and T * self.K <= 64 and world <= 16 and T * world <= min(c.max_tokens, self.max_rows)

    def local_multi(self, layer, recv_buf, T, world, rank, shared, h_mid, out):
        self.ctx.check(self.lib.finch_encode_ep_unpack(self.ctx.h, self._stream(), recv_buf.data_ptr(), T * world, self.rx.data_ptr(),
                                                       self.rids.data_ptr(), self.rw.data_ptr(), self.rv.data_ptr()))
        return self._multi_rows(layer, T, world, rank, shared, h_mid, out)

    def peer_local_multi(self, layer, T, world, rank, shared, h_mid, out):
        self.peer_receive(False)
        return self._multi_rows(layer, T, world, rank, shared, h_mid, out)

    def _multi_rows(self, layer, T, world, rank, shared, h_mid, out):
        self.ctx.check(self.lib.finch_encode_moe_decode_multi(
            self.ctx.h, self._stream(), self.pool.h, layer, world, T, self.rx.data_ptr(), self.rids.data_ptr(), self.rw.data_ptr(), self.rv.data_ptr(),
            rank, C.byref(shared) if shared is not None else None, h_mid.data_ptr() if h_mid is not None else None, out.data_ptr(),
            self.rout.data_ptr()))
        return self.rout[:T * world]

    def peer_decode(self, layer, shared, h_mid, out):
        """receive + finch_encode_ep_peer_decode: the layer on this rank, the other ranks' rows stored into their areas
        by the decode pass itself."""
        self.peer_receive(False)
        self.ctx.check(self.lib.finch_encode_ep_peer_decode(
            self.ctx.h, self._stream(), self.peer.h, self.pool.h, layer, self.rx.data_ptr(), self.rids.data_ptr(), self.rw.data_ptr(),
            self.rv.data_ptr(), C.byref(shared) if shared is not None else None, h_mid.data_ptr() if h_mid is not None else None, out.data_ptr()))

    def peer_return(self, part):
        self.ctx.check(self.lib.finch_encode_ep_peer_return(self.ctx.h, self._stream(), self.peer.h, part.data_ptr()))

    def peer_combine(self, out):
        self.ctx.check(self.lib.finch_encode_ep_peer_combine(self.ctx.h, self._stream(), self.peer.h, out.data_ptr()))

    def base(self, layer, x, ids, weights, shared, h_mid, out):
        torch = self.torch
        T = ids.shape[0]
        if self.zero_valid is None or self.zero_valid.shape[0] < T:
            self.zero_valid = torch.zeros((T, self.K), dtype=torch.uint8, device=self.dev)
        st = self._stream()
        step = self.ctx.cfg.max_tokens
        for t0 in range(0, T, step):
            m = min(step, T - t0)
            sh = None
            if shared is not None:
                from . import lib as L
                sh = L.Shared(shared.gate, shared.up, shared.down, shared.gate_score + 4 * t0)
            self.ctx.check(self.lib.finch_encode_moe_prefill(
                self.ctx.h, st, self.pool.h, layer, x.data_ptr() + t0 * self.hidden * self.elt, ids[t0:].data_ptr(), weights[t0:].data_ptr(),
                self.zero_valid.data_ptr(), C.byref(sh) if sh is not None else None,
                h_mid[t0:].data_ptr() if h_mid is not None else None, out[t0:].data_ptr(), m))

    def combine(self, p, out, back):
        if back.numel() == 0:   # no row left this rank: nothing comes back
            return
        self.ctx.check(self.lib.finch_encode_ep_combine(self.ctx.h, self._stream(), out.data_ptr(), back.data_ptr(), p.slot_of.data_ptr(),
                                                        p.offs.data_ptr(), p.T, p.world))
