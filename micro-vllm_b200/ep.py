"""Expert-parallel routed MoE layer: one rank per GPU, experts sharded.

By default expert e lives on rank e % nranks as that rank's local expert
e // nranks (strided placement balances Zipf-skewed routing far better than
contiguous blocks).  A `Placement` may also replicate hot experts on every
rank: each rank then serves those experts for its own tokens, so a handful
of very popular experts no longer pile their rows onto one rank
(`balance_replicas` picks them from routing statistics).  One layer step on
rank r, for r's own tokens:

  1. plan      which ranks need each token, and its row in the
               destination-major send buffer        (mvllm_moe_ep_plan_dev)
  2. counts    all-to-all of the per-destination row counts      (NCCL)
  3. pack      token rows, per-slot local expert ids (-1 where another rank
               owns the slot) and weights into the send buffer
                                                     (mvllm_moe_ep_pack_dev)
  4. dispatch  all-to-all of the rows, and one of ids + weights (one int32
               buffer)                                           (NCCL)
  5. compute   the received rows through r's local experts: the routed layer
               on device (mvllm_moe_layer_dev) with E = r's expert count;
               slots marked -1 are skipped by its permutation
  6. return    all-to-all of the partial sums back to the token owners (f16
               rows with a power-of-two scale per row; f32 for one rank)
  7. combine   out[c] += partials of token c in ascending rank order
                                                     (mvllm_moe_ep_combine_dev)

The reference runs every expert on one host; the partition, the exchanges
and the combine order belong to this layer.  Every sum has a fixed order, so
runs are bit-reproducible; the association differs from the single-GPU
order, within the parity tolerance.

The device steps go through an ``ops`` object so that the orchestration
(counts, splits, buffers, exchange order) is the same code whether the ops
are the CUDA library (``CudaOps``) or a CPU test double, and whether the
exchange is torch.distributed (NCCL on GPUs, gloo on CPU) or an in-process
emulation of several ranks.
"""
from __future__ import annotations

import mvllm_moe as moe


def owner(e, nranks):
    return e % nranks


def local_id(e, nranks):
    return e // nranks


def local_experts(rank, nranks, E):
    """Global ids of the experts rank `rank` holds (strided), in local-id order."""
    return list(range(rank, E, nranks))


class Placement:
    """Which rank serves each expert, and under which local id.

    Replicated experts come first in every rank's local table (local id j =
    position in `replicated`), then the rank's strided own experts (e on rank
    e % nranks, replicated ones left out).  dest[e] = serving rank, or -1 for
    a replicated expert (the token's own rank serves it)."""

    def __init__(self, E, nranks, replicated=()):
        self.E, self.nranks = E, nranks
        self.replicated = sorted({int(e) for e in replicated if 0 <= int(e) < E})
        rep = set(self.replicated)
        R = len(self.replicated)
        self.dest = [-1 if e in rep else e % nranks for e in range(E)]
        self.lid = [0] * E
        for j, e in enumerate(self.replicated):
            self.lid[e] = j
        self._local = []
        for r in range(nranks):
            own = [e for e in range(r, E, nranks) if e not in rep]
            for i, e in enumerate(own):
                self.lid[e] = R + i
            self._local.append(self.replicated + own)

    @property
    def strided(self):
        return not self.replicated

    def local_experts(self, rank):
        """Global ids rank `rank` holds, in local-id order."""
        return list(self._local[rank])

    def serving_rank(self, e, token_rank):
        d = self.dest[e]
        return token_rank if d < 0 else d


def rank_loads(load, placement):
    """Routed rows each rank serves under `placement`, for per-expert row
    counts `load` summed over ranks whose tokens are alike (a replicated
    expert's rows split evenly over the ranks)."""
    N = placement.nranks
    per = [0.0] * N
    for e, n in enumerate(load):
        if placement.dest[e] < 0:
            for r in range(N):
                per[r] += n / N
        else:
            per[placement.dest[e]] += n
    return per


def balance_replicas(load, nranks, max_replicas, tol=0.05):
    """Experts to replicate, hottest first, until no rank serves more than
    (1 + tol) x the mean routed rows or `max_replicas` are taken."""
    E = len(load)
    mean = sum(load) / nranks
    order = sorted(range(E), key=lambda e: (-load[e], e))
    rep = []
    while len(rep) < max_replicas:
        if max(rank_loads(load, Placement(E, nranks, rep))) <= (1.0 + tol) * mean:
            break
        rep.append(order[len(rep)])
    return rep


class CudaOps:
    """Device steps of a rank through the sm_100a library."""

    def __init__(self, torch, E, K, D, I, fmt, act, act_a, act_b, local_tables, nranks,
                 max_recv_rows, placement=None, rank=0, partial16=None):
        self.torch = torch
        self.rank = rank
        # Return the partial sums as f16 rows with a power-of-two scale per row
        # (half the bytes of f32 over NVLink, relative error <= 2^-11); one
        # rank keeps f32, so it matches the single-GPU layer bit for bit.
        self.partial16 = (nranks > 1) if partial16 is None else partial16
        self.dest = self.lid = None
        if placement is not None and not placement.strided:
            self.dest = torch.tensor(placement.dest, dtype=torch.int32, device="cuda")
            self.lid = torch.tensor(placement.lid, dtype=torch.int32, device="cuda")
        self.E, self.K, self.D, self.I, self.fmt = E, K, D, I, fmt
        self.act, self.act_a, self.act_b = act, act_a, act_b
        self.tables = local_tables
        self.nranks = nranks
        self.E_local = len(local_tables[0]) if local_tables else 0
        self.ws = torch.empty(moe.layer_workspace_bytes(max(max_recv_rows, 1), K,
                                                        max(self.E_local, 1), 0, D, I, fmt),
                              dtype=torch.uint8, device="cuda")
        self.max_recv_rows = max_recv_rows

    def plan(self, idx):
        T = idx.shape[0]
        pos = self.torch.empty((T, self.nranks), dtype=self.torch.int32, device=idx.device)
        cnt = self.torch.empty(self.nranks, dtype=self.torch.int32, device=idx.device)
        moe.ep_plan_dev(idx, self.E, self.nranks, pos, cnt, self.dest, self.rank)
        return pos, cnt

    def plan_fixed(self, idx, capacity):
        T = idx.shape[0]
        pos = self.torch.empty((T, self.nranks), dtype=self.torch.int32, device=idx.device)
        cnt = self.torch.empty(self.nranks, dtype=self.torch.int32, device=idx.device)
        moe.ep_plan_fixed_dev(idx, self.E, self.nranks, capacity, pos, cnt, self.dest, self.rank)
        return pos, cnt

    def pack_fixed(self, x, idx, wt, pos, rows):
        """pack() into segments of a fixed size: rows without a token keep
        send_idx -1 (no expert), so the receiver skips them."""
        send_x, send_idx, send_wt = self.pack(x, idx, wt, pos, rows, fill_idx=True)
        return send_x, send_idx, send_wt

    def pack(self, x, idx, wt, pos, rows, fill_idx=False):
        t = self.torch
        send_x = t.empty((rows, self.D), dtype=x.dtype, device=x.device)
        send_idx = (t.full((rows, self.K), -1, dtype=t.int32, device=x.device) if fill_idx else
                    t.empty((rows, self.K), dtype=t.int32, device=x.device))
        send_wt = t.empty((rows, self.K), dtype=t.float32, device=x.device)
        if rows:
            moe.ep_pack_dev(x, idx, wt, self.E, self.nranks, pos, send_x, send_idx, send_wt,
                            self.dest, self.lid, self.rank)
        return send_x, send_idx, send_wt

    def compute(self, rx, ridx, rwt):
        R = rx.shape[0]
        if R > self.max_recv_rows:
            raise ValueError(f"received {R} rows, above the {self.max_recv_rows} sized for")
        t = self.torch
        if self.partial16:
            part = t.empty((R, moe.partial_row_bytes(self.D)), dtype=t.uint8, device=rx.device)
            if R and self.E_local:
                moe.layer_partial_dev(R, self.K, self.E_local, 0, self.D, self.I, self.fmt, ridx,
                                      rwt, rx, self.tables, part, self.act, self.act_a,
                                      self.act_b, self.ws)
            elif R:
                part.zero_()
            return part
        part = t.zeros((R, self.D), dtype=t.float32, device=rx.device)
        if R and self.E_local:
            moe.layer_dev(R, self.K, self.E_local, 0, self.D, self.I, self.fmt, ridx, rwt, rx,
                          self.tables, part, self.act, self.act_a, self.act_b, self.ws)
        return part

    def combine(self, back, pos, out):
        if self.partial16:
            moe.ep_combine16_dev(back, pos, out)
        else:
            moe.ep_combine_dev(back, pos, out)

    # ---- the exchange over peer memory (EPLayer.forward_peer)
    def dispatch_peer(self, x, idx, wt, pos, cnt, win, rank):
        moe.ep_dispatch_peer_dev(x, idx, wt, self.E, self.nranks, win.seg, pos, cnt, win.table,
                                 self.dest, self.lid, rank)

    def compute_peer(self, win, rank):
        R = self.nranks * win.seg
        if R > self.max_recv_rows:
            raise ValueError(f"{R} window rows, above the {self.max_recv_rows} sized for")
        if self.E_local:
            moe.layer_partial_peer_dev(self.nranks, win.seg, rank, self.K, self.E_local, self.D,
                                       self.I, self.fmt, win.x_dtype, win.addr, win.table,
                                       self.tables, self.act, self.act_a, self.act_b, self.ws)

    def combine_peer(self, win, pos, out):
        moe.ep_combine16_dev(win.addr + win.off["back"], pos, out)

    def set_sm_reserve(self, n):
        """Leave n SMs out of the expert kernels (0: use them all)."""
        if n <= 0:
            moe.set_sm_limit(0)
        else:
            sms = self.torch.cuda.get_device_properties(
                self.torch.cuda.current_device()).multi_processor_count
            moe.set_sm_limit(max(2, sms - n))


class PeerWindows:
    """The exchange window of one rank for `EPLayer.forward_peer`: one
    cudaMalloc'd block (mvllm_moe_peer_alloc) of nranks * seg rows -- token
    rows, local ids and weights received, and the partial rows returned to
    this rank -- that every other rank maps through CUDA IPC and writes over
    NVLink.  `table` is the device array of every rank's window address."""

    def __init__(self, torch, nranks, seg, K, D, x_dtype=moe.DTYPE_BF16):
        self.torch, self.nranks, self.seg, self.x_dtype = torch, nranks, seg, x_dtype
        self.total, self.off = moe.ep_window_layout(nranks, seg, K, D, x_dtype)
        self.addr, self.handle = moe.peer_alloc(self.total)
        self.opened, self.table = [], None

    def connect(self, rank, dist=None, group=None, peers=None):
        """Builds `table`: from the other processes' IPC handles (an all-gather
        of the 64-byte handles over `dist`, each peer's window mapped here) or,
        for ranks emulated in one process, from their PeerWindows (`peers`)."""
        t = self.torch
        if peers is not None:
            addrs = [p.addr for p in peers]
        else:
            n = moe.PEER_HANDLE_BYTES
            mine = t.tensor(list(self.handle), dtype=t.uint8, device="cuda")
            every = t.empty(self.nranks * n, dtype=t.uint8, device="cuda")
            dist.all_gather_into_tensor(every, mine, group=group)
            raw = bytes(every.cpu().tolist())
            addrs = []
            for r in range(self.nranks):
                if r == rank:
                    addrs.append(self.addr)
                else:
                    a = moe.peer_open(raw[r * n:(r + 1) * n])
                    self.opened.append(a)
                    addrs.append(a)
        self.table = t.tensor(addrs, dtype=t.int64, device="cuda")
        return self

    def close(self, dist=None, group=None):
        """Unmaps the peers' windows, waits for every rank to have done the
        same (dist), then frees this rank's own."""
        self.torch.cuda.synchronize()
        for a in self.opened:
            moe.peer_close(a)
        self.opened = []
        if dist is not None and self.nranks > 1:
            dist.barrier(group=group)
        if self.addr:
            moe.peer_free(self.addr)
            self.addr = 0


class EPLayer:
    """The layer step of one rank; `ops` holds the device steps."""

    def __init__(self, ops, rank, nranks, D, K):
        self.ops, self.rank, self.nranks, self.D, self.K = ops, rank, nranks, D, K
        self._flag = None

    def _barrier(self, dist, group):
        """Orders every rank's preceding kernels before every rank's following
        ones: an all-reduce of one word, queued on the stream like a kernel
        (no host synchronisation)."""
        if self.nranks > 1:
            t = self.ops.torch
            if self._flag is None:
                self._flag = t.zeros(1, dtype=t.int32, device="cuda")
            dist.all_reduce(self._flag, group=group)

    def forward_peer(self, x, idx, wt, out, dist, win, group=None, timing=None):
        """The step with the exchanges as stores over NVLink (no NCCL transfer
        carries rows): the fixed plan (segments of win.seg rows), the dispatch
        kernel storing each token row, its local ids and weights into the
        destinations' windows, a barrier, the rank's experts over its window
        with each partial row stored into its owner's window, a barrier, and
        the combine of the rows returned to this rank (ranks ascending).  The
        same rows and sums as `forward_fixed`, so the same bits."""
        T = x.shape[0]
        if T > win.seg:
            raise ValueError(f"{T} tokens, above the window's {win.seg} per rank")
        t, ev = self.ops.torch, []

        def mark():
            if timing is not None:
                e = t.cuda.Event(enable_timing=True)
                e.record()
                ev.append(e)

        mark()
        pos, cnt = self.ops.plan_fixed(idx, win.seg)
        mark()
        self.ops.dispatch_peer(x, idx, wt, pos, cnt, win, self.rank)
        mark()
        self._barrier(dist, group)
        mark()
        self.ops.compute_peer(win, self.rank)
        mark()
        self._barrier(dist, group)
        mark()
        self.ops.combine_peer(win, pos, out)
        mark()
        if timing is not None:
            t.cuda.synchronize()
            names = ("plan", "dispatch_stores", "barrier1", "experts_and_return_stores",
                     "barrier2", "combine")
            for n, a, b in zip(names, ev[:-1], ev[1:]):
                timing[n] = timing.get(n, 0.0) + a.elapsed_time(b)
        return {"sent_rows": self.nranks * win.seg, "received_rows": self.nranks * win.seg}

    # ---- phases (the distributed forward and the in-process emulation both use them)
    def prepare(self, x, idx, wt):
        pos, cnt = self.ops.plan(idx)
        return pos, cnt

    def pack(self, x, idx, wt, pos, send_splits):
        return self.ops.pack(x, idx, wt, pos, int(sum(send_splits)))

    def _meta(self, sidx, swt):
        """The send rows' expert ids and weights in one int32 buffer [rows, 2K]
        (the weights as their f32 bits), so both travel in one exchange.  The
        token rows stay a buffer of their own: they are the experts' operand,
        read in place on arrival."""
        t = self.ops.torch
        return t.cat([sidx, swt.view(t.int32)], dim=1)

    def _split_meta(self, rmeta):
        t = self.ops.torch
        return rmeta[:, :self.K].contiguous(), rmeta[:, self.K:].contiguous().view(t.float32)

    def forward_local(self, x, idx, wt, out):
        """One rank: the single-GPU routed layer (mvllm_moe_layer_dev over all
        experts, out += layer(x)); no plan, pack, exchange or combine."""
        if self.nranks != 1:
            raise ValueError("forward_local is the one-rank step")
        o = self.ops
        T = x.shape[0]
        if T > o.max_recv_rows:
            raise ValueError(f"{T} tokens, above the {o.max_recv_rows} sized for")
        moe.layer_dev(T, self.K, o.E_local, 0, self.D, o.I, o.fmt, idx, wt, x, o.tables, out,
                      o.act, o.act_a, o.act_b, o.ws)
        return {"sent_rows": 0, "received_rows": T}

    def forward_fixed(self, x, idx, wt, out, dist, group=None):
        """The step with fixed-size exchange segments: every rank sends each
        destination `T` rows (a token goes to a rank at most once; rows
        without a token carry expert ids -1), so no counts travel to the host
        and the step never waits on the GPU from the CPU.  Costs the padding
        rows' bytes on the links; the received rows without an expert cost
        nothing in the expert kernels (their permutation skips them).  Same
        results as `forward`."""
        t = self.ops.torch
        T = x.shape[0]
        N = self.nranks
        pos, _ = self.ops.plan_fixed(idx, T)
        sx, sidx, swt = self.ops.pack_fixed(x, idx, wt, pos, N * T)
        smeta = self._meta(sidx, swt)
        rx, rmeta = t.empty_like(sx), t.empty_like(smeta)
        dist.all_to_all_single(rx, sx, group=group)
        dist.all_to_all_single(rmeta, smeta, group=group)
        ridx, rwt = self._split_meta(rmeta)
        part = self.ops.compute(rx, ridx, rwt)
        back = t.empty_like(part)
        dist.all_to_all_single(back, part, group=group)
        self.ops.combine(back, pos, out)
        return {"sent_rows": N * T, "received_rows": N * T}

    def forward_chunked(self, x, idx, wt, out, dist, chunks=2, group=None, sm_reserve=16):
        """The step in `chunks` slices of the rank's tokens, pipelined so the
        exchanges overlap the expert kernels: the dispatches of every slice
        are queued at once (NCCL runs them on its own stream), slice c's
        experts start when its dispatch has landed, and its return starts as
        soon as its experts finish, under slice c + 1's experts.  The expert
        kernels leave `sm_reserve` SMs to NCCL meanwhile.  All slices' counts
        go in one exchange (one host synchronisation per step).  Same
        results as `forward`: every row is computed by the same kernels and
        combined in the same order per slice."""
        t = self.ops.torch
        T = x.shape[0]
        C = max(1, min(chunks, T))
        cuts = [T * c // C for c in range(C + 1)]
        sl = [slice(cuts[c], cuts[c + 1]) for c in range(C)]
        plans = [self.prepare(x[s], idx[s], wt[s]) for s in sl]
        N = self.nranks
        cnt = t.stack([p[1] for p in plans], dim=1).reshape(-1)  # destination-major [N, C]
        rcnt = t.empty_like(cnt)
        dist.all_to_all_single(rcnt, cnt, group=group)
        sc_all = [int(v) for v in cnt.tolist()]
        rc_all = [int(v) for v in rcnt.tolist()]
        sc = [[sc_all[d * C + c] for d in range(N)] for c in range(C)]  # sc[c][d]
        rc = [[rc_all[s * C + c] for s in range(N)] for c in range(C)]  # rc[c][s]
        recv, works = [], []
        for c in range(C):
            sx, sidx, swt = self.pack(x[sl[c]], idx[sl[c]], wt[sl[c]], plans[c][0], sc[c])
            smeta = self._meta(sidx, swt)
            R = sum(rc[c])
            rx = t.empty((R, self.D), dtype=x.dtype, device=x.device)
            rmeta = t.empty((R, 2 * self.K), dtype=t.int32, device=x.device)
            works.append([dist.all_to_all_single(rx, sx, rc[c], sc[c], group=group,
                                                 async_op=True),
                          dist.all_to_all_single(rmeta, smeta, rc[c], sc[c], group=group,
                                                 async_op=True)])
            recv.append((rx, rmeta, sx, smeta))
        backs = []
        lim = getattr(self.ops, "set_sm_reserve", None)
        if lim and N > 1:
            lim(sm_reserve)
        try:
            for c in range(C):
                for w in works[c]:
                    w.wait()
                rx, rmeta = recv[c][:2]
                ridx, rwt = self._split_meta(rmeta)
                part = self.ops.compute(rx, ridx, rwt)
                back = t.empty((sum(sc[c]),) + tuple(part.shape[1:]), dtype=part.dtype,
                               device=x.device)
                backs.append((back, part, dist.all_to_all_single(back, part, sc[c], rc[c],
                                                                 group=group, async_op=True)))
        finally:
            if lim and N > 1:
                lim(0)
        for c in range(C):
            back, _, w = backs[c]
            w.wait()
            self.ops.combine(back, plans[c][0], out[sl[c]])
        return {"sent_rows": sum(sum(v) for v in sc), "received_rows": sum(sum(v) for v in rc)}

    def forward(self, x, idx, wt, out, dist, group=None, timing=None):
        """One step through torch.distributed (all ranks call it in step).
        With ``timing`` (a dict), CUDA events on the current stream split the
        step into its phases; the dict receives their device milliseconds."""
        t = self.ops.torch
        ev = []

        def mark():
            if timing is not None:
                e = t.cuda.Event(enable_timing=True)
                e.record()
                ev.append(e)

        mark()
        pos, cnt = self.prepare(x, idx, wt)
        mark()
        rcnt = t.empty_like(cnt)
        dist.all_to_all_single(rcnt, cnt, group=group)
        sc = [int(v) for v in cnt.tolist()]
        rc = [int(v) for v in rcnt.tolist()]
        mark()
        sx, sidx, swt = self.pack(x, idx, wt, pos, sc)
        smeta = self._meta(sidx, swt)
        R = sum(rc)
        rx = t.empty((R, self.D), dtype=x.dtype, device=x.device)
        rmeta = t.empty((R, 2 * self.K), dtype=t.int32, device=x.device)
        mark()
        dist.all_to_all_single(rx, sx, rc, sc, group=group)
        dist.all_to_all_single(rmeta, smeta, rc, sc, group=group)
        ridx, rwt = self._split_meta(rmeta)
        mark()
        part = self.ops.compute(rx, ridx, rwt)
        mark()
        back = t.empty((sum(sc),) + tuple(part.shape[1:]), dtype=part.dtype, device=x.device)
        dist.all_to_all_single(back, part, sc, rc, group=group)
        mark()
        self.ops.combine(back, pos, out)
        mark()
        if timing is not None:
            t.cuda.synchronize()
            names = ("plan", "counts", "pack", "dispatch", "experts", "return", "combine")
            for n, a, b in zip(names, ev[:-1], ev[1:]):
                timing[n] = timing.get(n, 0.0) + a.elapsed_time(b)
        return {"sent_rows": sum(sc), "received_rows": R}


def emulate_step_peer(layers, wins, xs, idxs, wts, outs):
    """forward_peer for all ranks in one process on one GPU: the windows are
    the ranks' own allocations (PeerWindows.connect with `peers`), and the
    stream order of the phases (every rank's dispatch, then every rank's
    experts, then every rank's combine) stands in for the barriers."""
    plans = []
    for L, w, x, i, t in zip(layers, wins, xs, idxs, wts):
        pos, cnt = L.ops.plan_fixed(i, w.seg)
        L.ops.dispatch_peer(x, i, t, pos, cnt, w, L.rank)
        plans.append(pos)
    for L, w in zip(layers, wins):
        L.ops.compute_peer(w, L.rank)
    for L, w, pos, o in zip(layers, wins, plans, outs):
        L.ops.combine_peer(w, pos, o)


def emulate_step(layers, xs, idxs, wts, outs, torch):
    """All ranks' steps in one process: the exchanges become slicing and
    concatenation of the ranks' buffers in the order NCCL's all-to-all uses
    (rank d receives, from each source s ascending, s's rows for d)."""
    N = len(layers)
    plans = [L.prepare(x, i, w) for L, x, i, w in zip(layers, xs, idxs, wts)]
    sc = [[int(v) for v in cnt.tolist()] for (_, cnt) in plans]  # sc[s][d]
    packs = [L.pack(x, i, w, pos, sc[s]) for s, (L, x, i, w, (pos, _)) in
             enumerate(zip(layers, xs, idxs, wts, plans))]

    def chunk(buf, splits, d):
        a = sum(splits[:d])
        return buf[a:a + splits[d]]

    parts = []
    for d in range(N):
        rx = torch.cat([chunk(packs[s][0], sc[s], d) for s in range(N)])
        ridx = torch.cat([chunk(packs[s][1], sc[s], d) for s in range(N)])
        rwt = torch.cat([chunk(packs[s][2], sc[s], d) for s in range(N)])
        parts.append(layers[d].ops.compute(rx, ridx, rwt))
    rc = [[sc[s][d] for s in range(N)] for d in range(N)]  # rc[d][s]
    for s in range(N):
        back = torch.cat([chunk(parts[d], rc[d], s) for d in range(N)])
        layers[s].ops.combine(back, plans[s][0], outs[s])
