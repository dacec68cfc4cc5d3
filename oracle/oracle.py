"""ctypes front end for the CPU parity checker (TEST INFRASTRUCTURE ONLY).

Two interchangeable back ends with the same call shape:

* ``Oracle("port")`` -- ``_build/libmoe_oracle.so``, the C restatement in
  ``moe_oracle.c`` of the reference's hot path.
* ``Oracle("reference")`` -- ``_ref/libmvllm_ref.so``, the reference's own
  sources (``src/gpu/metal_ops.cpp``, ``src/quant/quant.cpp``,
  ``src/model/ops.cpp``, ``src/model/moe_pick.cpp``) behind ``ref_shim.cpp``.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBS = {
    "port": (os.path.join(HERE, "_build", "libmoe_oracle.so"), "orc_"),
    "reference": (os.path.join(HERE, "_ref", "libmvllm_ref.so"), "ref_"),
}

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build(reference: bool = False) -> None:
    """Compile the port (and, when the reference tree exists, the reference)."""
    targets = ["oracle"]
    if reference:
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def available(kind: str) -> bool:
    return os.path.exists(LIBS[kind][0])


def _ptr(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _ptr_array(arrs):
    if arrs is None:
        return None
    out = (C.c_void_p * len(arrs))()
    for i, a in enumerate(arrs):
        out[i] = None if a is None else a.ctypes.data
    return out


class Oracle:
    """CPU moe_block and helpers; ``kind`` is "port" or "reference"."""

    def __init__(self, kind: str = "port"):
        path, pre = LIBS[kind]
        if not os.path.exists(path):
            build(reference=(kind == "reference"))
        self.kind = kind
        self.lib = C.CDLL(path)
        L, p = self.lib, pre
        self._moe = getattr(L, p + "moe_block")
        self._moe.restype = C.c_int
        self._moe.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int] + [C.c_void_p] * 6 + [
            C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
            C.c_int, C.c_float, C.c_float]
        self._q4 = getattr(L, p + "quantize_int4_g64")
        self._q4.argtypes = [_f32p, C.c_int, C.c_int, _u8p, _f32p]
        self._mx = getattr(L, p + "pack_mxfp4")
        self._mx.argtypes = [_f32p, C.c_int, C.c_int, _u8p, _u8p]
        self._mm32 = getattr(L, p + "matmul_f32")
        self._mm32.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]
        self._mm4 = getattr(L, p + "matmul_int4_g64")
        self._mm4.argtypes = [_f32p, _f32p, _u8p, _f32p, C.c_int, C.c_int, C.c_int]
        self._mmx = getattr(L, p + "matmul_mxfp4")
        self._mmx.argtypes = [_f32p, _f32p, _u8p, _u8p, C.c_int, C.c_int, C.c_int]
        self._q8 = getattr(L, p + "quantize_int8_row")
        self._q8.argtypes = [_f32p, C.c_int, C.c_int, C.c_void_p, _f32p]
        self._mm8 = getattr(L, p + "matmul_int8_row")
        self._mm8.argtypes = [_f32p, _f32p, C.c_void_p, _f32p, C.c_int, C.c_int, C.c_int]
        self._rms = getattr(L, p + "rmsnorm")
        self._rms.argtypes = [_f32p, C.c_void_p, _f32p, C.c_int, C.c_float]
        self._epi = getattr(L, "orc_moe_epilogue", None)  # the port only
        if self._epi is not None:
            self._epi.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, C.c_void_p, C.c_float,
                                  C.c_int, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, _f32p]
        for name in ("situ_glu", "clamped_swiglu", "sigmoid"):
            f = getattr(L, p + name)
            f.restype = C.c_float
            setattr(self, "_" + name, f)
        self._situ_glu.argtypes = [C.c_float] * 4
        self._clamped_swiglu.argtypes = [C.c_float] * 3
        self._sigmoid.argtypes = [C.c_float]
        self._softmax = getattr(L, p + "softmax_inplace")
        self._softmax.argtypes = [_f32p, C.c_int]
        self._topk = getattr(L, p + "moe_topk")
        self._topk.restype = C.c_int
        self._topk.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p, C.c_void_p]
        self._union = getattr(L, p + "moe_union_ids")
        self._union.restype = C.c_int
        self._union.argtypes = [_i32p, C.c_int, C.c_int, _i32p, C.c_int]
        self._pick = getattr(L, p + "moe_topk_pick")
        self._pick.restype = C.c_int
        self._pick.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p]
        # DeepSeek-V4 (dsv4_cuda.cpp, native_act.cpp)
        for name in ("e8m0_decode", "e4m3fn_decode"):
            f = getattr(L, p + name)
            f.restype = C.c_float
            f.argtypes = [C.c_uint8]
            setattr(self, "_" + name, f)
        self._mm8b = getattr(L, p + "matmul_fp8_b128")
        self._mm8b.argtypes = [_f32p, _f32p, _u8p, _u8p, C.c_int, C.c_int, C.c_int]
        self._d4route = getattr(L, p + "dsv4_route")
        self._d4route.restype = C.c_int
        self._d4route.argtypes = [_f32p, C.c_int, _f32p, C.c_void_p, C.c_int, C.c_void_p,
                                  C.c_float, _i32p, _f32p]
        self._d4moe = getattr(L, p + "dsv4_moe")
        self._d4moe.restype = C.c_int
        self._d4moe.argtypes = [_f32p, C.c_int, C.c_int, C.c_int] + [C.c_void_p] * 6 + [
            C.c_void_p, C.c_void_p, C.c_float, _f32p]
        self._d4ep2 = getattr(L, p + "dsv4_route_moe_ep2")
        self._d4ep2.restype = C.c_int
        self._d4ep2.argtypes = [_f32p, C.c_int, _f32p, C.c_void_p, C.c_int, C.c_float,
                                C.c_int] + [C.c_void_p] * 7 + [C.c_float, _f32p, _f32p]
        self._ssp = getattr(L, "orc_sqrt_softplus", None)  # the port only
        if self._ssp is not None:
            self._ssp.restype = C.c_float
            self._ssp.argtypes = [C.c_float]

    # ---- codecs -----------------------------------------------------------
    def quantize_int4_g64(self, w):
        w = np.ascontiguousarray(w, np.float32)
        O, I = w.shape
        p = np.zeros((O, (I + 1) // 2), np.uint8)
        s = np.zeros((O, (I + 63) // 64), np.float32)
        self._q4(w, O, I, p, s)
        return p, s

    def pack_mxfp4(self, w):
        w = np.ascontiguousarray(w, np.float32)
        O, I = w.shape
        p = np.zeros((O, (I + 1) // 2), np.uint8)
        s = np.zeros((O, (I + 31) // 32), np.uint8)
        self._mx(w, O, I, p, s)
        return p, s

    def matmul_f32(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        S, I = x.shape
        O = w.shape[0]
        y = np.zeros((S, O), np.float32)
        self._mm32(y, x, w, S, I, O)
        return y

    def matmul_int4_g64(self, x, p, s, O):
        x = np.ascontiguousarray(x, np.float32)
        S, I = x.shape
        y = np.zeros((S, O), np.float32)
        self._mm4(y, x, np.ascontiguousarray(p), np.ascontiguousarray(s, np.float32), S, I, O)
        return y

    def matmul_mxfp4(self, x, p, s, O):
        x = np.ascontiguousarray(x, np.float32)
        S, I = x.shape
        y = np.zeros((S, O), np.float32)
        self._mmx(y, x, np.ascontiguousarray(p), np.ascontiguousarray(s), S, I, O)
        return y

    def quantize_int8_row(self, w):
        w = np.ascontiguousarray(w, np.float32)
        O, I = w.shape
        q = np.zeros((O, I), np.int8)
        s = np.zeros(O, np.float32)
        self._q8(w, O, I, q.ctypes.data, s)
        return q, s

    def matmul_int8_row(self, x, q, s, O):
        x = np.ascontiguousarray(x, np.float32)
        S, I = x.shape
        y = np.zeros((S, O), np.float32)
        q = np.ascontiguousarray(q, np.int8)
        self._mm8(y, x, q.ctypes.data, np.ascontiguousarray(s, np.float32), S, I, O)
        return y

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        wp = None if w is None else np.ascontiguousarray(w, np.float32)
        self._rms(x, None if wp is None else wp.ctypes.data, y, x.shape[0], eps)
        return y

    def moe_epilogue(self, acc, h, routed_scale, lat_n=None, eps=1e-6, up_fmt=0, up_w=None,
                     up_scales=None, shared=None):
        """Returns h + epilogue(acc) (kimi_k3.cpp:2074-2108 order); port only."""
        acc = np.ascontiguousarray(acc, np.float32)
        out = np.array(h, np.float32, copy=True)
        T, L = acc.shape
        H = out.shape[1]
        keep = [None if a is None else np.ascontiguousarray(a) for a in
                (lat_n, up_w, up_scales, shared)]
        ptr = [None if a is None else a.ctypes.data for a in keep]
        self._epi(T, H, L, acc, ptr[0], eps, up_fmt, ptr[1], ptr[2], routed_scale, ptr[3], out)
        return out

    def situ_glu(self, g, u, b1, b2):
        return self._situ_glu(g, u, b1, b2)

    def clamped_swiglu(self, g, u, limit):
        return self._clamped_swiglu(g, u, limit)

    def sigmoid(self, x):
        return self._sigmoid(x)

    def softmax(self, x):
        y = np.array(x, np.float32, copy=True)
        self._softmax(y, y.shape[0])
        return y

    # ---- moe_block ---------------------------------------------------------
    def moe_block(self, nb, D, Iinter, fmt, g, u, d, gs, us, ds, xg, xoff, nr, rows, rw, out, S,
                  act=0, act_a=0.0, act_b=0.0, qgs=0):
        """Calls moe_block in place on ``out`` (float32, accumulated); returns 0/1."""
        keep = [_ptr_array(g), _ptr_array(u), _ptr_array(d), _ptr_array(gs), _ptr_array(us),
                _ptr_array(ds)]
        args = [nb, D, Iinter, fmt, qgs] + keep + [
            _ptr(xg), _ptr(xoff), _ptr(nr), _ptr(rows), _ptr(rw), _ptr(out), S, act, act_a, act_b]
        return self._moe(*args)

    # ---- routing -----------------------------------------------------------
    def moe_topk(self, choice, k, mix=None):
        choice = np.ascontiguousarray(choice, np.float32)
        n = choice.shape[0]
        kk = min(k, n)
        idx = np.zeros(max(kk, 1), np.int32)
        w = np.zeros(max(kk, 1), np.float32)
        mixa = None if mix is None else np.ascontiguousarray(mix, np.float32)
        r = self._topk(choice, n, k, idx, w, None if mixa is None else mixa.ctypes.data)
        return idx[:r], w[:r]

    def moe_union_ids(self, idx, cap=None):
        idx = np.ascontiguousarray(idx, np.int32)
        n_tok, topk = idx.shape
        cap = cap if cap is not None else max(n_tok * topk, 1)
        out = np.zeros(cap, np.int32)
        n = self._union(idx.reshape(-1), n_tok, topk, out, cap)
        return out[:n]

    def moe_topk_pick(self, scores, k):
        scores = np.ascontiguousarray(scores, np.float32)
        idx = np.zeros(max(k, 1), np.int32)
        w = np.zeros(max(k, 1), np.float32)
        r = self._pick(scores, scores.shape[0], k, idx, w)
        return idx[:r], w[:r]

    # ---- DeepSeek-V4 -------------------------------------------------------
    def e8m0_decode(self, v):
        return self._e8m0_decode(v)

    def e4m3fn_decode(self, v):
        return self._e4m3fn_decode(v)

    def sqrt_softplus(self, z):
        """Port only (the reference's is file-local)."""
        return self._ssp(z)

    def matmul_fp8_b128(self, x, w, s, O):
        """y = x . dequant(W)^T, W e4m3fn [O, I] with 128x128 e8m0 tiles."""
        x = np.ascontiguousarray(x, np.float32)
        S, I = x.shape
        y = np.zeros((S, O), np.float32)
        self._mm8b(y, x, np.ascontiguousarray(w, np.uint8), np.ascontiguousarray(s, np.uint8), S,
                   I, O)
        return y

    def dsv4_route(self, x, router, bias, routed_scale, fixed=None):
        """dsv4_cuda::route per row of x [T, H]: ids [T, 6] int32, w [T, 6]."""
        x = np.ascontiguousarray(x, np.float32)
        router = np.ascontiguousarray(router, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        T, H = x.shape
        E = router.shape[0]
        ids = np.full((T, 6), -1, np.int32)
        w = np.zeros((T, 6), np.float32)
        fx = None if fixed is None else np.ascontiguousarray(fixed, np.int32)
        for t in range(T):
            i6 = np.zeros(6, np.int32)
            w6 = np.zeros(6, np.float32)
            ok = self._d4route(x[t], H, router, _ptr(b), E, _ptr(fx), routed_scale, i6, w6)
            assert ok
            ids[t], w[t] = i6, w6
        return ids, w

    @staticmethod
    def _tables(experts, E=None):
        """Six pointer arrays (gate, up, down, gate scales, up scales, down
        scales) from [(gate, up, down)] of (packed, scales); None = absent."""
        n = len(experts) if E is None else E
        cols = [[None] * n for _ in range(6)]
        for e, ex in enumerate(experts):
            if ex is None:
                continue
            (gp, gsc), (up, usc), (dp, dsc) = ex
            for j, a in enumerate((gp, up, dp, gsc, usc, dsc)):
                cols[j][e] = a
        return [_ptr_array(c) for c in cols]

    @staticmethod
    def _shared(shared):
        if shared is None:
            return None
        (gw, gs), (uw, us), (dw, ds) = shared
        return _ptr_array([gw, gs, uw, us, dw, ds])

    def dsv4_moe(self, x, O, experts, weights, shared=None, limit=0.0):
        """dsv4_cuda::moe for one token x [H]: MXFP4 experts [(gate, up, down)]
        of (packed, scales) with their weights, then the FP8 shared expert
        ((w, scales) x 3) if given.  Returns y [H] (None = reference false)."""
        x = np.ascontiguousarray(x, np.float32)
        H = x.shape[0]
        t = self._tables(experts)
        sh = self._shared(shared)
        wv = np.ascontiguousarray(weights, np.float32)
        y = np.zeros(H, np.float32)
        ok = self._d4moe(x, H, O, len(experts), *t, wv.ctypes.data, sh, limit, y)
        return y if ok else None

    def dsv4_route_moe_ep2(self, x, router, bias, routed_scale, O, experts, shared=None,
                           limit=0.0):
        """dsv4_cuda::route_moe_ep2 for one token x [H] over a bank of
        len(experts) MXFP4 experts (None = absent): (out, peer_out)."""
        x = np.ascontiguousarray(x, np.float32)
        router = np.ascontiguousarray(router, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        H = x.shape[0]
        E = len(experts)
        t = self._tables(experts)
        sh = self._shared(shared)
        out = np.zeros(H, np.float32)
        peer = np.zeros(H, np.float32)
        ok = self._d4ep2(x, H, router, _ptr(b), E, routed_scale, O, *t, sh, limit, out, peer)
        assert ok
        return out, peer


def permute(idx, wt, uniq):
    """Caller-side gather order (glm53.cpp:1958-1971): returns nr, xoff, rows, rw.

    Pure restatement in Python loops over the per-token top-k lists; each
    wsum is accumulated in f32, t ascending, exactly like the reference.
    """
    idx = np.asarray(idx, np.int32)
    wt = np.asarray(wt, np.float32)
    C_, K = idx.shape
    nr, xoff, rows, rw = [], [], [], []
    for eid in uniq:
        xoff.append(len(rows))
        n = 0
        for c in range(C_):
            wsum = np.float32(0.0)
            for t in range(K):
                if idx[c, t] == eid:
                    wsum = np.float32(wsum + wt[c, t])
            if wsum == 0.0:
                continue
            rows.append(c)
            rw.append(wsum)
            n += 1
        nr.append(n)
    return (np.array(nr, np.int32), np.array(xoff, np.int32), np.array(rows, np.int32),
            np.array(rw, np.float32))


def glm_geom(hidden, inter):
    """GLM int4-g64 blob offsets (glm53.cpp:56-78): (g, gs, u, us, d, ds), slot."""
    if hidden > 0 and inter > 0 and hidden % 64 == 0 and inter % 64 == 0:
        pack_go = inter * hidden // 2
        sc_go = inter * hidden // 64 * 4
        pack_d = pack_go
    else:
        pack_go = inter * ((hidden + 1) // 2)
        sc_go = inter * ((hidden + 63) // 64) * 4
        pack_d = hidden * ((inter + 1) // 2)
    sc_d = (hidden * ((inter + 63) // 64) * 4) if not (
        hidden % 64 == 0 and inter % 64 == 0) else sc_go
    g = 0
    gs = pack_go
    u = gs + sc_go
    us = u + pack_go
    d = us + sc_go
    ds = d + pack_d
    return (g, gs, u, us, d, ds), ds + sc_d


def k3_geom(latent, inter):
    """K3 MXFP4 blob offsets (kimi_k3.cpp:83-102, order w1 w1s w2 w2s w3 w3s)."""
    if latent >= 32 and inter >= 32 and latent % 32 == 0 and inter % 32 == 0:
        w1p, w1s = inter * (latent // 2), inter * (latent // 32)
        w2p, w2s = latent * (inter // 2), latent * (inter // 32)
    else:
        w1p, w1s = inter * ((latent + 1) // 2), inter * ((latent + 31) // 32)
        w2p, w2s = latent * ((inter + 1) // 2), latent * ((inter + 31) // 32)
    g, gs = 0, w1p
    d = w1p + w1s
    ds = d + w2p
    u = ds + w2s
    us = u + w1p
    return (g, gs, u, us, d, ds), 2 * (w1p + w1s) + w2p + w2s
