"""Parity at the exact shapes bench.py measures, every token where the oracle
can afford it.

* config[1] (MXFP4 decode, 256 experts top-8 + the shared expert, SiTU) at
  B = 1 and B = 32 (the decode headline batch): every token.
* config[2] (int4-g64, 160 experts top-8, clamped SwiGLU) at B = 1 and
  B = 64: every token.
* config[3] (4096 tokens, Zipf routing) in the library's default tensor-core
  mode: 32 tokens spread over the batch.
* config[4] (384 experts, 8192 tokens) through the expert-parallel layer
  with 8 ranks emulated on one GPU (exchanges as slicing): 32 tokens.

The CPU oracle (moe_block of the reference restated, metal_ops.cpp:278-342)
checks each token on its own: tokens are independent, so a token's output
row against the oracle's is a complete check of that row.  Oracle calls run
on host threads (ctypes releases the GIL).  Tolerance as everywhere:
<= 1e-2 relative L2 and <= 2e-2 max-abs.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import cases
from conftest import assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _experts(moe, fmt, ids, D, I, seed):
    """Expert weights drawn N(0, 0.02) and packed on the GPU, per global id."""
    gs_ = 64 if fmt == cases.FMT_INT4 else 32
    sdt = torch.float32 if fmt == cases.FMT_INT4 else torch.uint8
    pack = moe.quantize_int4_g64_dev if fmt == cases.FMT_INT4 else moe.pack_mxfp4_dev
    out = {}
    for e in ids:
        g = torch.Generator(device="cuda").manual_seed(seed * 100003 + e)
        mats = []
        for (O_, I_) in ((I, D), (I, D), (D, I)):
            w = torch.randn((O_, I_), generator=g, device="cuda") * 0.02
            p = torch.empty((O_, I_ // 2), dtype=torch.uint8, device="cuda")
            s = torch.empty((O_, I_ // gs_), dtype=sdt, device="cuda")
            pack(w, p, s)
            mats.append((p, s))
        out[e] = mats
    return out


def _tables(experts, order):
    tabs = [[experts[e][k % 3][k // 3].data_ptr() for e in order] for k in range(6)]
    return [torch.tensor(t, dtype=torch.int64, device="cuda") for t in tabs]


def _oracle_rows(port, host, tokens, idx, wt, x, D, I, fmt, act, a, b, shared=None):
    """Each token's output row from the oracle, on host threads.  host[e] is
    the expert's six arrays on the host; `shared` (an id) is added to every
    token with weight 1, ordered after the routed experts as the layer's
    combine orders it (ascending id, the shared expert last)."""
    def one(t):
        ids = [int(e) for e in idx[t]]
        ws = [float(w) for w in wt[t]]
        pairs = {}
        for e, w in zip(ids, ws):
            pairs[e] = np.float32(pairs.get(e, np.float32(0)) + np.float32(w))
        order = sorted(pairs)
        wl = [pairs[e] for e in order]
        if shared is not None:
            order.append(shared)
            wl.append(1.0)
        nb = len(order)
        o = np.zeros((1, D), np.float32)
        ok = port.moe_block(nb, D, I, fmt, [host[e][0] for e in order],
                            [host[e][1] for e in order], [host[e][2] for e in order],
                            [host[e][3] for e in order], [host[e][4] for e in order],
                            [host[e][5] for e in order], x[t:t + 1], np.zeros(nb, np.int32),
                            np.ones(nb, np.int32), np.zeros(nb, np.int32),
                            np.array(wl, np.float32), o, 1, act, a, b)
        assert ok
        return o[0]

    with ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 4)) as ex:
        return np.stack(list(ex.map(one, tokens)))


def _host(experts, ids):
    return {e: [experts[e][k][0].cpu().numpy() for k in range(3)] +
               [experts[e][k][1].cpu().numpy() for k in range(3)] for e in ids}


def _layer(moe, port, D, I, E, K, T, fmt, act, a, b, n_shared, seed, tokens=None,
           router="uniform"):
    rng = np.random.default_rng(seed)
    if router == "uniform":
        choice = rng.random((T, E), dtype=np.float32)
    elif router == "softmax":
        logits = rng.standard_normal((T, E)).astype(np.float32)
        choice = np.exp(logits - logits.max(1, keepdims=True))
        choice = (choice / choice.sum(1, keepdims=True)).astype(np.float32)
    else:  # config[3]'s Zipf s=1.1 over a ranking of the experts, Gumbel noise per token
        rank = rng.permutation(E) + 1
        logits = -1.1 * np.log(rank)[None, :] - np.log(-np.log(rng.random((T, E)) + 1e-20))
        p = np.exp(logits - logits.max(1, keepdims=True))
        choice = (p / p.sum(1, keepdims=True)).astype(np.float32)
    idx, wt = cases.route(port, choice, K)
    x = cases.bf16_round(rng.standard_normal((T, D)).astype(np.float32))
    used = sorted(set(idx.reshape(-1).tolist()))
    ids = used + ([E] if n_shared else [])
    ex = _experts(moe, fmt, ids, D, I, seed)
    order = list(range(E + n_shared))
    zero = (ex[ids[0]][0][0], ex[ids[0]][0][1])  # never read: experts no token routes to
    full = {e: ex.get(e, [zero, zero, zero]) for e in order}
    tables = _tables(full, order)
    ws = torch.empty(moe.layer_workspace_bytes(T, K, E, n_shared, D, I, fmt), dtype=torch.uint8,
                     device="cuda")
    out = torch.zeros((T, D), dtype=torch.float32, device="cuda")
    moe.layer_dev(T, K, E, n_shared, D, I, fmt, torch.from_numpy(idx).cuda(),
                  torch.from_numpy(wt).cuda(), torch.from_numpy(x).cuda().to(torch.bfloat16),
                  tables, out, act, a, b, ws)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    tokens = list(range(T)) if tokens is None else tokens
    want = _oracle_rows(port, _host(ex, ids), tokens, idx, wt, x, D, I, fmt, act, a, b,
                        shared=E if n_shared else None)
    return got[tokens], want


@pytest.mark.parametrize("B", [1, 32])
def test_config1_every_token(moe, port, B):
    got, want = _layer(moe, port, 7168, 2048, 256, 8, B, cases.FMT_MXFP4, cases.ACT_SITU, 4.0,
                       25.0, 1, 61 + B)
    assert_close(got, want, f"config[1] B={B}")


@pytest.mark.parametrize("B", [1, 64])
def test_config2_every_token(moe, port, B):
    got, want = _layer(moe, port, 6144, 1536, 160, 8, B, cases.FMT_INT4, cases.ACT_CLAMP, 7.0,
                       0.0, 0, 71 + B, router="softmax")
    assert_close(got, want, f"config[2] B={B}")


def test_config3_default_mode(moe, port):
    """4096 tokens, Zipf routing: pair, ragged, single-CTA and decode tiles in
    one call, in the library's default tensor-core mode."""
    T = 4096
    tokens = [int(t) for t in np.linspace(0, T - 1, 32)]
    got, want = _layer(moe, port, 7168, 2048, 256, 8, T, cases.FMT_MXFP4, cases.ACT_SITU, 4.0,
                       25.0, 0, 81, tokens=tokens, router="zipf")
    assert_close(got, want, f"config[3] ({moe.PREFILL_NAMES[moe.get_prefill_mode()]})")


def test_config4_ep_eight_ranks_emulated(moe, port):
    """384 experts strided over 8 ranks (e % 8), 8192 tokens, 1024 per rank,
    exchanges emulated by slicing on one GPU; sampled tokens of every rank."""
    import ep
    D, I, E, K, N, T = 7168, 2048, 384, 8, 8, 8192
    rng = np.random.default_rng(91)
    choice = rng.random((T, E), dtype=np.float32)
    idx, wt = cases.route(port, choice, K)
    x = cases.bf16_round(rng.standard_normal((T, D)).astype(np.float32))
    ex = _experts(moe, cases.FMT_MXFP4, list(range(E)), D, I, 91)
    T_loc = T // N
    layers, xs, idxs, wts, outs = [], [], [], [], []
    for r in range(N):
        mine = ep.local_experts(r, N, E)
        ops = ep.CudaOps(torch, E, K, D, I, cases.FMT_MXFP4, cases.ACT_SITU, 4.0, 25.0,
                         _tables(ex, mine), N, T)
        layers.append(ep.EPLayer(ops, r, N, D, K))
        sl = slice(r * T_loc, (r + 1) * T_loc)
        xs.append(torch.from_numpy(x[sl]).cuda().to(torch.bfloat16))
        idxs.append(torch.from_numpy(idx[sl]).cuda())
        wts.append(torch.from_numpy(wt[sl]).cuda())
        outs.append(torch.zeros((T_loc, D), device="cuda"))
    ep.emulate_step(layers, xs, idxs, wts, outs, torch)
    # The exchange over peer memory (forward_peer's kernels, windows as
    # separate allocations on this GPU): the same bits.
    wins = [ep.PeerWindows(torch, N, T_loc, K, D) for _ in range(N)]
    for r, w in enumerate(wins):
        w.connect(r, peers=wins)
    peer = [torch.zeros_like(o) for o in outs]
    ep.emulate_step_peer(layers, wins, xs, idxs, wts, peer)
    torch.cuda.synchronize()
    for w in wins:
        w.close()
    for o, p in zip(outs, peer):
        assert torch.equal(o, p)
    got = torch.cat(outs).cpu().numpy()
    tokens = [int(t) for t in np.linspace(0, T - 1, 32)]
    used = sorted(set(idx[tokens].reshape(-1).tolist()))
    want = _oracle_rows(port, _host(ex, used), tokens, idx, wt, x, D, I, cases.FMT_MXFP4,
                        cases.ACT_SITU, 4.0, 25.0)
    assert_close(got[tokens], want, "config[4] EP, 8 emulated ranks")
