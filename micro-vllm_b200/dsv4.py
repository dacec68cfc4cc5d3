"""DeepSeek-V4 routed MoE step with the experts split over ranks and the
ranks' partial outputs summed by an all-reduce (the reference's EP2).

The reference (dsv4.cpp:2863-3010, moe_layer_ep2) runs, per token,
dsv4_cuda::route_moe_ep2 (dsv4_cuda.cpp:1841-1906): both ranks route the same
input, rank r runs the routed slots whose expert id has parity r
(map_ep_expert, :1356-1369) through moe_routed_parity (:1371-1404; the bank's
FP8 shared expert on one rank only), and allreduce_pair (:1195-1204) adds the
two partial outputs on the host.  The layer then adds acc * routed_scale and
the dense shared MLP's output to the residual stream (dsv4.cpp:2993-3008).

Here every step works on all T tokens at once, on rank r of N (one GPU each;
N = 2 with strided placement is the reference's parity split):

  1. route       every rank routes all T tokens identically: sqrt(softplus)
                 scores + bias, top 6, weights x route_scale
                                                  (mvllm_moe_route_ex_dev)
  2. local ids   the slots rank r serves become local ids, the rest -1
                                                  (mvllm_moe_ep_local_ids_dev)
  3. experts     the routed layer for all T tokens through r's MXFP4 experts
                 with clamped SwiGLU              (mvllm_moe_layer_dev)
  4. shared      rank 0 adds the bank's FP8 shared expert, if any
                                                  (mvllm_moe_dense_ffn_dev)
  5. all-reduce  sum of the partial outputs (NCCL).  With two ranks the sum is
                 one addition per element, so every rank holds exactly the
                 reference's rank0 + rank1.
  6. tail        h += acc * routed_scale, then the dense shared MLP's output
                 (mvllm_moe_epilogue_dev; the MLP through mvllm_moe_layer_dev as
                 one expert, or exactly with mvllm_moe_dense_ffn_dev)

The device steps go through an ``ops`` object, so the orchestration is the
same code over the CUDA library (``CudaOps``) or a CPU test double, and over
torch.distributed (NCCL on GPUs, gloo on CPU) or the in-process emulation of
the ranks on one device (``emulate_step``).
"""
from __future__ import annotations

import mvllm_moe as moe

TOPK = 6  # DeepSeek-V4 routes every token to 6 experts (dsv4_cuda.cpp:1561)


def mx_geom(H, O):
    """Byte sizes of one DeepSeek-V4 expert blob's parts (make_mx_geom,
    dsv4.cpp:64-80): packed gate/up rows [O, H/2] and their ue8m0 scales
    [O, H/32], packed down rows [H, O/2] and scales [H, O/32] (rounded up
    when H or O is not a multiple of 32).  Returns (w1p, w1s, w2p, w2s, slot)."""
    H, O = max(H, 1), max(O, 1)
    if H >= 32 and O >= 32 and H % 32 == 0 and O % 32 == 0:
        w1p, w1s, w2p, w2s = O * (H // 2), O * (H // 32), H * (O // 2), H * (O // 32)
    else:
        w1p, w1s = O * ((H + 1) // 2), O * ((H + 31) // 32)
        w2p, w2s = H * ((O + 1) // 2), H * ((O + 31) // 32)
    return w1p, w1s, w2p, w2s, 2 * (w1p + w1s) + w2p + w2s


def blob_pointers(base, H, O):
    """The six array addresses of an expert blob at address `base`, in the
    order the pointer tables take them (gate, up, down, gate scales, up
    scales, down scales).  The blob is w1 (gate) packed, w1 scales, w2 (down)
    packed, w2 scales, w3 (up) packed, w3 scales (dsv4.cpp:2958-2965)."""
    w1p, w1s, w2p, w2s, _ = mx_geom(H, O)
    gate = base
    gate_s = gate + w1p
    down = gate_s + w1s
    down_s = down + w2p
    up = down_s + w2s
    up_s = up + w1p
    return gate, up, down, gate_s, up_s, down_s


class CudaOps:
    """Device steps of one rank through the sm_100a library.

    router f32 [E, H], bias f32 [E] or None (device tensors); local_tables:
    the six int64 device tensors of the rank's expert pointers (gate, up,
    down, gate scales, up scales, down scales) in local-id order (strided:
    global experts rank, rank + nranks, ...), MXFP4 gate
    and up [I, H] and down [H, I]; shared_fp8: the bank's shared expert
    ((w, scales) x 3, FP8 tiles, device) on the rank that holds it, else
    None; dense_shared: (fmt, gate, up, down) of the layer's shared MLP
    (each (w, scales-or-None), device), or None.  An int4-g64 or MXFP4 shared
    MLP (QuantMat 4-bit is the reference's default, config.hpp:143) runs
    through the MoE kernels as one expert that every token takes with weight
    1, within the MoE tolerance; with dense_exact, and for the other formats,
    it runs on the sequential-order GEMM in the reference's exact arithmetic.
    """

    def __init__(self, torch, E, H, I, limit, router, bias, local_tables, rank, nranks,
                 max_tokens, route_scale=1.0, routed_scale=1.0, shared_fp8=None,
                 dense_shared=None, dense_exact=False):
        self.torch = torch
        self.E, self.H, self.I, self.limit = E, H, I, limit
        self.router, self.bias = router, bias
        self.tables = local_tables
        self.E_local = int(local_tables[0].numel()) if local_tables else 0
        self.rank, self.nranks = rank, nranks
        self.route_scale, self.routed_scale = route_scale, routed_scale
        self.shared_fp8, self.dense_shared = shared_fp8, dense_shared
        T = max(max_tokens, 1)
        self.max_tokens = T
        dev = router.device
        self.ws = torch.empty(moe.layer_workspace_bytes(T, TOPK, max(self.E_local, 1), 0, H, I,
                                                        moe.FMT_MXFP4),
                              dtype=torch.uint8, device=dev)
        self.ffn_ws = torch.empty(moe.dense_ffn_workspace_bytes(T, H, I), dtype=torch.uint8,
                                  device=dev)
        self.idx = torch.empty((T, TOPK), dtype=torch.int32, device=dev)
        self.wt = torch.empty((T, TOPK), dtype=torch.float32, device=dev)
        self.lidx = torch.empty((T, TOPK), dtype=torch.int32, device=dev)
        self.scores = torch.empty((T, E), dtype=torch.float32, device=dev)
        self.choice = torch.empty((T, E), dtype=torch.float32, device=dev)
        self.acc = torch.empty((T, H), dtype=torch.float32, device=dev)
        self.sd = torch.empty((T, H), dtype=torch.float32, device=dev)
        self.dense_moe = None
        if (dense_shared is not None and not dense_exact
                and dense_shared[0] in (moe.FMT_INT4_G64, moe.FMT_MXFP4)):
            fmt, g, u, d = dense_shared
            tabs = [torch.tensor([a.data_ptr()], dtype=torch.int64, device=dev)
                    for a in (g[0], u[0], d[0], g[1], u[1], d[1])]
            self.dense_moe = dict(
                fmt=fmt, tables=tabs,
                idx=torch.zeros((T, 1), dtype=torch.int32, device=dev),
                wt=torch.ones((T, 1), dtype=torch.float32, device=dev),
                ws=torch.empty(moe.layer_workspace_bytes(T, 1, 1, 0, H, I, fmt),
                               dtype=torch.uint8, device=dev))

    def _rows(self, x):
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens, above the {self.max_tokens} sized for")
        return T

    def route(self, x):
        T = self._rows(x)
        idx, wt = self.idx[:T], self.wt[:T]
        moe.route_ex_dev(x, self.router, self.bias, TOPK, idx, wt, self.scores[:T],
                         self.choice[:T], moe.SCORE_SQRT_SOFTPLUS, self.route_scale)
        return idx, wt

    def local_ids(self, idx):
        T = idx.shape[0]
        lidx = self.lidx[:T]
        moe.ep_local_ids_dev(idx, self.E, self.nranks, self.rank, lidx)  # strided
        return lidx

    def experts(self, x, lidx, wt):
        T = self._rows(x)
        acc = self.acc[:T]
        acc.zero_()
        if self.E_local:
            moe.layer_dev(T, TOPK, self.E_local, 0, self.H, self.I, moe.FMT_MXFP4, lidx, wt, x,
                          self.tables, acc, moe.ACT_CLAMP_SWIGLU, self.limit, 0.0, self.ws)
        return acc

    def add_shared(self, x, acc):
        if self.shared_fp8 is not None:
            moe.dense_ffn_dev(moe.FMT_FP8_B128, x, *self.shared_fp8, acc, moe.ACT_CLAMP_SWIGLU,
                              self.limit, 0.0, accumulate=True, workspace=self.ffn_ws)

    def tail(self, x, acc, h):
        sd = None
        if self.dense_shared is not None:
            T = x.shape[0]
            sd = self.sd[:T]
            if self.dense_moe is not None:
                m = self.dense_moe
                sd.zero_()
                moe.layer_dev(T, 1, 1, 0, self.H, self.I, m["fmt"], m["idx"][:T], m["wt"][:T],
                              x, m["tables"], sd, moe.ACT_CLAMP_SWIGLU, self.limit, 0.0,
                              m["ws"])
            else:
                fmt, g, u, d = self.dense_shared
                moe.dense_ffn_dev(fmt, x, g, u, d, sd, moe.ACT_CLAMP_SWIGLU, self.limit, 0.0,
                                  workspace=self.ffn_ws)
        moe.epilogue_dev(acc, h, self.routed_scale, shared=sd)


class EP2Layer:
    """The MoE step of one rank; `ops` holds the device steps."""

    def __init__(self, ops, rank, nranks):
        self.ops, self.rank, self.nranks = ops, rank, nranks

    def partial(self, x):
        """Steps 1-4: this rank's partial output for all tokens of x."""
        idx, wt = self.ops.route(x)
        acc = self.ops.experts(x, self.ops.local_ids(idx), wt)
        if self.rank == 0:
            self.ops.add_shared(x, acc)
        return acc

    def forward(self, x, h, dist, group=None):
        """One step through torch.distributed (all ranks call it in step, with
        the same x); h [T, H] f32 is updated in place.  Returns the summed
        routed output."""
        acc = self.partial(x)
        if self.nranks > 1:
            dist.all_reduce(acc, group=group)
        self.ops.tail(x, acc, h)
        return acc


def emulate_step(layers, x, h):
    """All ranks of one step on one device: the partial outputs are added in
    rank order (for two ranks, the all-reduce's single addition)."""
    acc = None
    for ly in layers:
        p = ly.partial(x)
        acc = p.clone() if acc is None else acc.add_(p)
    layers[0].ops.tail(x, acc, h)
    return acc
