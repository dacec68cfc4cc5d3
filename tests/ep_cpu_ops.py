"""CPU test double of ep.CudaOps (test infrastructure only).

The same four steps as the device path, on torch CPU tensors, with the expert
FFN through the CPU oracle (oracle.Oracle moe_block).  It lets the expert-
parallel orchestration (ep.EPLayer: counts, splits, buffers, exchange order)
run as gloo ranks on CPU.
"""
import numpy as np

from oracle import permute  # test infrastructure only


class CpuOps:
    def __init__(self, torch, codec, E, K, D, I, fmt, act, act_a, act_b, local_experts, nranks,
                 placement=None, rank=0):
        self.torch, self.codec = torch, codec
        self.placement, self.rank = placement, rank
        self.E, self.K, self.D, self.I, self.fmt = E, K, D, I, fmt
        self.act, self.act_a, self.act_b = act, act_a, act_b
        self.local = local_experts  # [(gate, up, down)] of (packed, scales), local-id order
        self.nranks = nranks

    def _serving(self, e):
        if self.placement is None:
            return e % self.nranks
        return self.placement.serving_rank(e, self.rank)

    def _lid(self, e):
        return e // self.nranks if self.placement is None else self.placement.lid[e]

    def plan(self, idx):
        ids = idx.numpy()
        T = ids.shape[0]
        need = np.zeros((T, self.nranks), bool)
        for c in range(T):
            for e in ids[c]:
                if 0 <= e < self.E:
                    need[c, self._serving(e)] = True
        cnt = need.sum(axis=0).astype(np.int32)
        off = np.concatenate([[0], np.cumsum(cnt)[:-1]])
        pos = np.full((T, self.nranks), -1, np.int32)
        for d in range(self.nranks):
            rows = np.nonzero(need[:, d])[0]
            pos[rows, d] = off[d] + np.arange(len(rows))
        return self.torch.from_numpy(pos), self.torch.from_numpy(cnt)

    def plan_fixed(self, idx, capacity):
        pos, cnt = self.plan(idx)
        P = pos.numpy().copy()
        off = np.concatenate([[0], np.cumsum(cnt.numpy())[:-1]])
        for d in range(self.nranks):
            m = P[:, d] >= 0
            P[m, d] = P[m, d] - off[d] + d * capacity
        return self.torch.from_numpy(P), cnt

    def pack_fixed(self, x, idx, wt, pos, rows):
        return self.pack(x, idx, wt, pos, rows)

    def pack(self, x, idx, wt, pos, rows):
        t = self.torch
        sx = t.zeros((rows, self.D), dtype=x.dtype)
        sidx = t.full((rows, self.K), -1, dtype=t.int32)
        swt = t.zeros((rows, self.K), dtype=t.float32)
        P = pos.numpy()
        ids = idx.numpy()
        for c in range(P.shape[0]):
            for d in range(self.nranks):
                p = P[c, d]
                if p < 0:
                    continue
                sx[p] = x[c]
                for k in range(self.K):
                    e = int(ids[c, k])
                    mine = 0 <= e < self.E and self._serving(e) == d
                    sidx[p, k] = self._lid(e) if mine else -1
                swt[p] = wt[c]
        return sx, sidx, swt

    def compute(self, rx, ridx, rwt):
        R = rx.shape[0]
        out = np.zeros((max(R, 1), self.D), np.float32)
        if R == 0 or not self.local:
            return self.torch.from_numpy(out[:R])
        idx = ridx.numpy().astype(np.int32)
        wt = rwt.numpy().astype(np.float32)
        uniq = self.codec.moe_union_ids(idx)
        nr, xoff, rows, rw = permute(idx, wt, uniq)
        x = rx.numpy().astype(np.float32)
        xg = np.ascontiguousarray(x[rows]) if rows.size else np.zeros((1, self.D), np.float32)
        sel = [self.local[e] for e in uniq]
        if sel:
            f32 = self.fmt == 0
            ok = self.codec.moe_block(
                len(sel), self.D, self.I, self.fmt, [s[0][0] for s in sel],
                [s[1][0] for s in sel], [s[2][0] for s in sel],
                None if f32 else [s[0][1] for s in sel], None if f32 else [s[1][1] for s in sel],
                None if f32 else [s[2][1] for s in sel], xg, xoff, nr, rows, rw, out, R,
                self.act, self.act_a, self.act_b)
            assert ok
        return self.torch.from_numpy(out[:R].copy())

    def combine(self, back, pos, out):
        P = pos.numpy()
        for c in range(P.shape[0]):
            for d in range(self.nranks):
                if P[c, d] >= 0:
                    out[c] += back[P[c, d]]

    # ---- the exchange over peer memory (ep.EPLayer.forward_peer): the
    # windows are CPU buffers of ranks emulated in one process, written with
    # the index arithmetic of the device kernels (ep_dispatch_peer_kernel and
    # the peer form of combine_tokens_f16_kernel).
    def dispatch_peer(self, x, idx, wt, pos, cnt, win, rank):
        P, ids, seg = pos.numpy(), idx.numpy(), win.seg
        for c in range(P.shape[0]):
            for d in range(self.nranks):
                p = P[c, d]
                if p < 0:
                    continue
                q = rank * seg + (p - d * seg)
                w = win.table[d]
                w.x[q] = x[c]
                for k in range(self.K):
                    e = int(ids[c, k])
                    mine = 0 <= e < self.E and self._serving(e) == d
                    w.ids[q, k] = self._lid(e) if mine else -1
                w.wt[q] = wt[c]
        for d in range(self.nranks):
            for j in range(int(cnt[d]), seg):
                win.table[d].ids[rank * seg + j] = -1

    def compute_peer(self, win, rank):
        part = self.compute(win.x, win.ids, win.wt)
        live = (win.ids.numpy() >= 0).any(axis=1)
        for c in range(part.shape[0]):
            if live[c]:
                o, j = divmod(c, win.seg)
                win.table[o].back[rank * win.seg + j] = part[c]

    def combine_peer(self, win, pos, out):
        self.combine(win.back, pos, out)


class CpuWindow:
    """A rank's exchange window for the CPU double: the regions of the device
    window (x, ids, wt, back) as CPU tensors; `table` lists every rank's."""

    def __init__(self, torch, nranks, seg, K, D, x_dtype):
        rows = nranks * seg
        self.seg = seg
        self.x = torch.zeros((rows, D), dtype=x_dtype)
        self.ids = torch.full((rows, K), 7, dtype=torch.int32)  # stale ids until written
        self.wt = torch.zeros((rows, K), dtype=torch.float32)
        self.back = torch.full((rows, D), float("nan"))  # unread unless returned
        self.table = None

    def connect(self, rank, peers):
        self.table = list(peers)
        return self
