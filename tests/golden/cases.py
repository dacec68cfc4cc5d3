"""Seeded synthetic moe_block cases shared by gen_golden.py and the tests.

Every case is a dict of numpy inputs in the reference's moe_block layout
(src/gpu/metal_ops.hpp:104-108).  Weights are drawn N(0, 0.02) and packed by
the given CPU codec object (the reference build or the C restatement, which
are bit-identical; tests check that through stored SHA-256 digests of the
packed bytes).  Routing follows the callers: choice -> moe_topk -> union ->
gather order (src/model/glm53.cpp:1921-1971).

The public benchmark suites of the reference are not used
are synthetic by definition, and these generators produce them from seeds.
"""
from __future__ import annotations

import hashlib

import numpy as np

FMT_F32, FMT_INT4, FMT_MXFP4 = 0, 4, 7
ACT_SILU, ACT_CLAMP, ACT_SITU = 0, 1, 2


def bf16_round(a):
    """Round f32 to the nearest bf16 (ties to even), returned as f32."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def pack(codec, fmt, w):
    if fmt == FMT_INT4:
        return codec.quantize_int4_g64(w)
    if fmt == FMT_MXFP4:
        return codec.pack_mxfp4(w)
    return np.ascontiguousarray(w, np.float32), None


def make_experts(codec, rng, fmt, n, D, I):
    """n experts of (gate [I,D], up [I,D], down [D,I]) packed as fmt."""
    ex = []
    for _ in range(n):
        ws = [(rng.standard_normal(s) * 0.02).astype(np.float32) for s in ((I, D), (I, D), (D, I))]
        ex.append([pack(codec, fmt, w) for w in ws])
    return ex


def digest(experts):
    h = hashlib.sha256()
    for e in experts:
        for p, s in e:
            h.update(np.ascontiguousarray(p).tobytes())
            if s is not None:
                h.update(np.ascontiguousarray(s).tobytes())
    return h.hexdigest()


def route(codec, choice, K, mix=None):
    """Per-token moe_topk (ops.cpp:860-890) -> idx [T,K], wt [T,K]."""
    T = choice.shape[0]
    idx = np.zeros((T, K), np.int32)
    wt = np.zeros((T, K), np.float32)
    for c in range(T):
        i, w = codec.moe_topk(choice[c], K, None if mix is None else mix[c])
        idx[c, :len(i)] = i
        wt[c, :len(w)] = w
    return idx, wt


def layer_case(codec, seed, D, I, E, K, T, fmt, act, act_a, act_b, n_shared=0, router="softmax",
               bf16_x=False):
    """A routed layer: routing, the reference gather order, moe_block arguments."""
    from oracle import permute  # test infrastructure only

    rng = np.random.default_rng(seed)
    if router == "softmax":
        logits = rng.standard_normal((T, E)).astype(np.float32)
        choice = np.stack([codec.softmax(l) for l in logits])
    else:  # uniform(0,1) router draws used directly as choice
        choice = rng.random((T, E), dtype=np.float32)
    x = rng.standard_normal((T, D)).astype(np.float32)
    if bf16_x:
        x = bf16_round(x)
    experts = make_experts(codec, rng, fmt, E + n_shared, D, I)
    idx, wt = route(codec, choice, K)
    uniq = codec.moe_union_ids(idx)
    nr, xoff, rows, rw = permute(idx, wt, uniq)
    ids = list(uniq)
    if n_shared:
        # The always-on shared expert runs after the routed ones with weight 1
        # for every token (one more moe_block expert).
        ids.append(E)
        xoff = np.append(xoff, rows.shape[0]).astype(np.int32)
        nr = np.append(nr, T).astype(np.int32)
        rows = np.append(rows, np.arange(T, dtype=np.int32))
        rw = np.append(rw, np.ones(T, np.float32))
    xg = np.ascontiguousarray(x[rows]) if rows.size else np.zeros((1, D), np.float32)
    sel = [experts[e] for e in ids]
    return dict(
        D=D, I=I, E=E, K=K, T=T, fmt=fmt, act=act, act_a=act_a, act_b=act_b, n_shared=n_shared,
        x=x, idx=idx, wt=wt, experts=experts, ids=np.array(ids, np.int32), nb=len(ids),
        g=[s[0][0] for s in sel], u=[s[1][0] for s in sel], d=[s[2][0] for s in sel],
        gs=None if fmt == FMT_F32 else [s[0][1] for s in sel],
        us=None if fmt == FMT_F32 else [s[1][1] for s in sel],
        ds=None if fmt == FMT_F32 else [s[2][1] for s in sel],
        xg=xg, xoff=xoff, nr=nr, rows=rows, rw=rw, S=T, digest=digest(experts))


def run_block(codec, c, out=None):
    """moe_block of a case through a CPU codec (port or reference)."""
    o = np.zeros((max(c["S"], 1), c["D"]), np.float32) if out is None else out
    ok = codec.moe_block(c["nb"], c["D"], c["I"], c["fmt"], c["g"], c["u"], c["d"], c["gs"],
                         c["us"], c["ds"], c["xg"], c["xoff"], c["nr"], c["rows"], c["rw"], o,
                         c["S"], c["act"], c["act_a"], c["act_b"])
    return ok, o


# --------------------------------------------------------------- named cases --
def kat_identity(act, act_a):
    """tests/test_host.cpp:2567-2601 and :2627-2651: 4x4 identity f32 weights."""
    ident = np.eye(4, dtype=np.float32)
    return dict(D=4, I=4, fmt=FMT_F32, act=act, act_a=act_a, act_b=0.0, nb=1, g=[ident],
                u=[ident], d=[ident], gs=None, us=None, ds=None,
                xg=np.array([[0.5, -0.25, 1.0, -1.0]], np.float32),
                xoff=np.array([0], np.int32), nr=np.array([1], np.int32),
                rows=np.array([0], np.int32), rw=np.array([1.0], np.float32), S=1)


def kat_mxfp4_diag(codec):
    """tests/test_host.cpp:2743-2790: I=O=32 MXFP4 diag(0.5), x = e0, SiTU(4,25)."""
    wf = np.zeros((32, 32), np.float32)
    np.fill_diagonal(wf, 0.5)
    (gp, gs), (up, us), (dp, ds) = [codec.pack_mxfp4(wf) for _ in range(3)]
    x = np.zeros((1, 32), np.float32)
    x[0, 0] = 1.0
    return dict(D=32, I=32, fmt=FMT_MXFP4, act=ACT_SITU, act_a=4.0, act_b=25.0, nb=1, g=[gp],
                u=[up], d=[dp], gs=[gs], us=[us], ds=[ds], xg=x, xoff=np.array([0], np.int32),
                nr=np.array([1], np.int32), rows=np.array([0], np.int32),
                rw=np.array([1.0], np.float32), S=1)


def edge_case(codec, seed=7):
    """Reference skip rules: nr<=0 (base not advanced), null weights (base
    advanced), destinations < 0 or >= S dropped, repeated destinations."""
    rng = np.random.default_rng(seed)
    D, I = 128, 64
    ex = make_experts(codec, rng, FMT_INT4, 5, D, I)
    nr = np.array([2, 0, 3, -1, 2], np.int32)
    xoff = np.array([0, 0, 2, 0, 5], np.int32)
    xg = rng.standard_normal((7, D)).astype(np.float32)
    rows = np.array([0, 3, -1, 2, 5, 1, 1], np.int32)  # 7 rows; -1 and 5 (>= S=4) dropped
    rw = rng.random(7).astype(np.float32)
    g = [e[0][0] for e in ex]
    g[2] = None  # expert 2 skipped for a null weight, its 3 rows still advance base
    return dict(D=D, I=I, fmt=FMT_INT4, act=ACT_CLAMP, act_a=7.0, act_b=0.0, nb=5, g=g,
                u=[e[1][0] for e in ex], d=[e[2][0] for e in ex], gs=[e[0][1] for e in ex],
                us=[e[1][1] for e in ex], ds=[e[2][1] for e in ex], xg=xg, xoff=xoff, nr=nr,
                rows=rows, rw=rw, S=4)


CONFIG0 = dict(seed=0, D=1024, I=512, E=16, K=4, T=4, fmt=FMT_INT4, act=ACT_CLAMP, act_a=7.0,
               act_b=0.0, n_shared=0, router="softmax", bf16_x=False)
SMALL_MXFP4 = dict(seed=11, D=512, I=512, E=8, K=2, T=3, fmt=FMT_MXFP4, act=ACT_SITU, act_a=4.0,
                   act_b=25.0, n_shared=1, router="uniform", bf16_x=True)
SMALL_INT4 = dict(seed=12, D=1024, I=512, E=12, K=3, T=9, fmt=FMT_INT4, act=ACT_CLAMP, act_a=7.0,
                  act_b=0.0, n_shared=0, router="softmax", bf16_x=True)
ODD_INT4 = dict(seed=13, D=192, I=96, E=4, K=2, T=5, fmt=FMT_INT4, act=ACT_CLAMP, act_a=7.0,
                act_b=0.0, n_shared=0, router="softmax", bf16_x=False)
ODD_MXFP4 = dict(seed=14, D=96, I=160, E=5, K=2, T=4, fmt=FMT_MXFP4, act=ACT_SITU, act_a=4.0,
                 act_b=25.0, n_shared=0, router="uniform", bf16_x=False)
F32_SILU = dict(seed=15, D=64, I=48, E=3, K=2, T=3, fmt=FMT_F32, act=ACT_SILU, act_a=0.0,
                act_b=0.0, n_shared=0, router="softmax", bf16_x=False)

LAYER_CASES = {"config0": CONFIG0, "small_mxfp4": SMALL_MXFP4, "small_int4": SMALL_INT4,
               "odd_int4": ODD_INT4, "odd_mxfp4": ODD_MXFP4, "f32_silu": F32_SILU}


def make_layer(codec, name):
    kw = dict(LAYER_CASES[name])
    seed = kw.pop("seed")
    return layer_case(codec, seed, **kw)
