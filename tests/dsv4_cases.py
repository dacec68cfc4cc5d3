"""DeepSeek-V4 MoE test cases and the CPU test double of dsv4.CudaOps
(test infrastructure only).

``dsv4_case`` builds a seeded layer: tokens, router and bias, a bank of MXFP4
experts (gate/up [I, H], down [H, I]), the bank's FP8 shared expert and the
layer's dense shared MLP (int8 rows), in the reference's formats.
``expected`` is the oracle's result for a whole step: per token
dsv4_route_moe_ep2 (route, the two parity partials, their sum), then the
layer tail of moe_layer_ep2 (dsv4.cpp:2993-3008).  ``CpuOps`` runs the device
steps of one rank on the oracle, so dsv4.EP2Layer's orchestration can run as
gloo ranks on CPU.
"""
import numpy as np

import cases

LIMIT = 7.0


def fp8_codes(rng, shape):
    """Random e4m3fn codes with exponent field <= 8 (|value| <= 3.75), no NaN."""
    sign = rng.integers(0, 2, shape) << 7
    ex = rng.integers(0, 9, shape) << 3
    man = rng.integers(0, 8, shape)
    return (sign | ex | man).astype(np.uint8)


def fp8_tensor(rng, O, I, base=120):
    """(codes [O, I], e8m0 tiles [ceil(O/128), ceil(I/128)])."""
    tiles = rng.integers(base - 1, base + 2, ((O + 127) // 128, (I + 127) // 128))
    return fp8_codes(rng, (O, I)), tiles.astype(np.uint8)


def dsv4_case(port, seed, H, I, E, T, shared=True, dense=True, absent=(), dense_fmt=8):
    rng = np.random.default_rng(seed)
    c = dict(H=H, I=I, E=E, T=T)
    c["x"] = rng.standard_normal((T, H)).astype(np.float32)
    c["h"] = rng.standard_normal((T, H)).astype(np.float32)
    c["router"] = (rng.standard_normal((E, H)) * (2.0 / np.sqrt(H))).astype(np.float32)
    c["bias"] = (rng.standard_normal(E) * 0.1).astype(np.float32)
    ex = cases.make_experts(port, rng, cases.FMT_MXFP4, E, H, I)
    c["experts"] = [None if e in absent else ex[e] for e in range(E)]
    c["shared_fp8"] = ([fp8_tensor(rng, I, H), fp8_tensor(rng, I, H), fp8_tensor(rng, H, I)]
                       if shared else None)
    c["dense"], c["dense_fmt"] = None, dense_fmt
    if dense:
        ws = [(rng.standard_normal(s) * 0.05).astype(np.float32) for s in ((I, H), (I, H), (H, I))]
        q = port.quantize_int8_row if dense_fmt == 8 else port.quantize_int4_g64
        c["dense"] = [q(w) for w in ws]
    c["route_scale"], c["routed_scale"] = 1.0, 2.5
    return c


def clamped(port, g, u):
    out = np.empty_like(g)
    for i, (a, b) in enumerate(zip(g.ravel(), u.ravel())):
        out.ravel()[i] = port.clamped_swiglu(float(a), float(b), LIMIT)
    return out


def fp8_shared_out(port, x, shared):
    """expert_fp8 for rows x: down . clamped_swiglu(gate . x, up . x)."""
    (gw, gs), (uw, us), (dw, ds) = shared
    I, H = gw.shape
    g = port.matmul_fp8_b128(x, gw, gs, I)
    u = port.matmul_fp8_b128(x, uw, us, I)
    return port.matmul_fp8_b128(clamped(port, g, u), dw, ds, H)


def dense_out(port, x, dense, fmt=8):
    """The layer's shared MLP (QuantMat int8 rows or int4-g64) for rows x."""
    (gq, gs), (uq, us), (dq, ds) = dense
    I, H = gq.shape[0], dq.shape[0]
    mm = port.matmul_int8_row if fmt == 8 else port.matmul_int4_g64
    g = mm(x, gq, gs, I)
    u = mm(x, uq, us, I)
    return mm(clamped(port, g, u), dq, ds, H)


def expected(port, c):
    """(acc [T, H] the summed routed output, h [T, H] after the tail)."""
    acc = np.zeros((c["T"], c["H"]), np.float32)
    for t in range(c["T"]):
        out, peer = port.dsv4_route_moe_ep2(c["x"][t], c["router"], c["bias"], c["route_scale"],
                                            c["I"], c["experts"], c["shared_fp8"], LIMIT)
        assert np.array_equal(out, peer)
        acc[t] = out
    sd = dense_out(port, c["x"], c["dense"], c["dense_fmt"]) if c["dense"] is not None else None
    h = port.moe_epilogue(acc, c["h"], c["routed_scale"], shared=sd)
    return acc, h


class CpuOps:
    """dsv4.CudaOps on the oracle, for rank `rank` of `nranks` (strided)."""

    def __init__(self, torch, port, c, rank, nranks, shared_fp8=None):
        self.torch, self.port, self.c = torch, port, c
        self.rank, self.nranks = rank, nranks
        self.local = [c["experts"][e] for e in range(rank, c["E"], nranks)]
        self.shared_fp8 = shared_fp8

    def route(self, x):
        ids, w = self.port.dsv4_route(x.numpy(), self.c["router"], self.c["bias"],
                                      self.c["route_scale"])
        return self.torch.from_numpy(ids), self.torch.from_numpy(w)

    def local_ids(self, idx):
        ids = idx.numpy()
        mine = (ids >= 0) & (ids < self.c["E"]) & (ids % self.nranks == self.rank)
        return self.torch.from_numpy(np.where(mine, ids // self.nranks, -1).astype(np.int32))

    def experts(self, x, lidx, wt):
        xs, L, W = x.numpy(), lidx.numpy(), wt.numpy()
        acc = np.zeros((xs.shape[0], self.c["H"]), np.float32)
        for t in range(xs.shape[0]):
            sel = [(self.local[l], W[t, k]) for k, l in enumerate(L[t])
                   if l >= 0 and self.local[l] is not None]
            if sel:
                acc[t] = self.port.dsv4_moe(xs[t], self.c["I"], [s[0] for s in sel],
                                            [s[1] for s in sel], None, LIMIT)
        return self.torch.from_numpy(acc)

    def add_shared(self, x, acc):
        if self.shared_fp8 is not None:
            acc += self.torch.from_numpy(fp8_shared_out(self.port, x.numpy(), self.shared_fp8))

    def tail(self, x, acc, h):
        sd = (dense_out(self.port, x.numpy(), self.c["dense"], self.c["dense_fmt"])
              if self.c["dense"] else None)
        h.copy_(self.torch.from_numpy(self.port.moe_epilogue(acc.numpy(), h.numpy(),
                                                             self.c["routed_scale"],
                                                             shared=sd)))
