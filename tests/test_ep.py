"""Expert-parallel layer (micro-vllm_b200/ep.py) on CPU: the orchestration with
the CPU test double of the device steps.

* In-process emulation of 3 ranks (the exchanges as slicing / concatenation).
* Two gloo ranks through torch.distributed all-to-all (spawned processes,
  127.0.0.1 rendezvous).
Both against the oracle's single-host moe_block of the whole layer; tolerance
as everywhere (the sum association differs from the single-host order).
"""
import os
import socket
import sys

import numpy as np
import pytest

import cases
from conftest import assert_close

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "micro-vllm_b200"))

CASE = dict(D=128, I=64, E=6, K=2, fmt=cases.FMT_INT4, act=cases.ACT_CLAMP, act_a=7.0,
            act_b=0.0)


def layer(port, T, seed=41):
    c = cases.layer_case(port, seed, CASE["D"], CASE["I"], CASE["E"], CASE["K"], T, CASE["fmt"],
                         CASE["act"], CASE["act_a"], CASE["act_b"])
    _, want = cases.run_block(port, c)
    return c, want


def rank_ops(port, c, rank, nranks, placement=None):
    from ep_cpu_ops import CpuOps
    import ep
    ids = (ep.local_experts(rank, nranks, CASE["E"]) if placement is None
           else placement.local_experts(rank))
    local = [c["experts"][e] for e in ids]
    return CpuOps(torch, port, CASE["E"], CASE["K"], CASE["D"], CASE["I"], CASE["fmt"],
                  CASE["act"], CASE["act_a"], CASE["act_b"], local, nranks, placement, rank)


def test_ep_emulated_replicated_experts(port):
    """Experts 1 and 4 on every rank (each rank serves them for its own
    tokens), the rest strided: same layer output."""
    import ep
    N, T_loc = 3, 7
    c, want = layer(port, N * T_loc, seed=43)
    pl = ep.Placement(CASE["E"], N, replicated=[4, 1])
    assert pl.replicated == [1, 4] and pl.dest == [0, -1, 2, 0, -1, 2]
    assert pl.local_experts(0) == [1, 4, 0, 3] and pl.local_experts(1) == [1, 4]
    assert [pl.lid[e] for e in range(6)] == [2, 0, 2, 3, 1, 3]
    layers, xs, idxs, wts, outs = [], [], [], [], []
    for r in range(N):
        sl = slice(r * T_loc, (r + 1) * T_loc)
        layers.append(ep.EPLayer(rank_ops(port, c, r, N, pl), r, N, CASE["D"], CASE["K"]))
        xs.append(torch.from_numpy(np.ascontiguousarray(c["x"][sl])))
        idxs.append(torch.from_numpy(np.ascontiguousarray(c["idx"][sl])))
        wts.append(torch.from_numpy(np.ascontiguousarray(c["wt"][sl])))
        outs.append(torch.zeros((T_loc, CASE["D"])))
    ep.emulate_step(layers, xs, idxs, wts, outs, torch)
    assert_close(torch.cat(outs).numpy(), want, "emulated 3-rank EP, replicated experts")


def test_balance_replicas():
    import ep
    # one expert with half of all rows: replicating it alone balances 4 ranks
    load = [400] + [25] * 16
    rep = ep.balance_replicas(load, 4, max_replicas=8)
    assert rep == [0]
    per = ep.rank_loads(load, ep.Placement(17, 4, rep))
    assert max(per) <= 1.05 * sum(load) / 4
    # uniform loads need no replica; the cap is honoured
    assert ep.balance_replicas([10] * 16, 4, max_replicas=8) == []
    zipf = [1000.0 / (i + 1) ** 1.1 for i in range(64)]
    assert len(ep.balance_replicas(zipf, 8, max_replicas=3)) == 3


def test_ep_emulated_three_ranks(port):
    import ep
    N, T_loc = 3, 7
    c, want = layer(port, N * T_loc)
    layers, xs, idxs, wts, outs = [], [], [], [], []
    for r in range(N):
        sl = slice(r * T_loc, (r + 1) * T_loc)
        layers.append(ep.EPLayer(rank_ops(port, c, r, N), r, N, CASE["D"], CASE["K"]))
        xs.append(torch.from_numpy(np.ascontiguousarray(c["x"][sl])))
        idxs.append(torch.from_numpy(np.ascontiguousarray(c["idx"][sl])))
        wts.append(torch.from_numpy(np.ascontiguousarray(c["wt"][sl])))
        outs.append(torch.zeros((T_loc, CASE["D"])))
    ep.emulate_step(layers, xs, idxs, wts, outs, torch)
    got = torch.cat(outs).numpy()
    assert_close(got, want, "emulated 3-rank EP")


def test_ep_emulated_peer_windows(port):
    """The peer-memory step (forward_peer's dispatch into the destinations'
    windows, experts over the own window, partial rows into the owners'
    windows, combine) on the CPU double: the same output as the exchange
    through send buffers, exactly; windows start with stale ids, which the
    dispatch must overwrite (-1 for unused segment rows)."""
    import ep
    from ep_cpu_ops import CpuWindow
    N, T_loc = 3, 7
    c, want = layer(port, N * T_loc)
    layers, xs, idxs, wts, outs, ref = [], [], [], [], [], []
    for r in range(N):
        sl = slice(r * T_loc, (r + 1) * T_loc)
        layers.append(ep.EPLayer(rank_ops(port, c, r, N), r, N, CASE["D"], CASE["K"]))
        xs.append(torch.from_numpy(np.ascontiguousarray(c["x"][sl])))
        idxs.append(torch.from_numpy(np.ascontiguousarray(c["idx"][sl])))
        wts.append(torch.from_numpy(np.ascontiguousarray(c["wt"][sl])))
        outs.append(torch.zeros((T_loc, CASE["D"])))
        ref.append(torch.zeros((T_loc, CASE["D"])))
    wins = [CpuWindow(torch, N, T_loc + 2, CASE["K"], CASE["D"], xs[0].dtype) for _ in range(N)]
    for r, w in enumerate(wins):
        w.connect(r, wins)
    ep.emulate_step_peer(layers, wins, xs, idxs, wts, outs)
    ep.emulate_step(layers, xs, idxs, wts, ref, torch)
    for o, f in zip(outs, ref):
        assert torch.equal(o, f)
    assert_close(torch.cat(outs).numpy(), want, "emulated 3-rank EP, peer windows")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gloo_rank(rank, nranks, port_no, T_loc, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "micro-vllm_b200"))
    from datetime import timedelta
    from oracle import Oracle
    import ep
    dist.init_process_group("gloo", rank=rank, world_size=nranks, timeout=timedelta(seconds=60))
    port = Oracle("port")
    c, _ = layer(port, nranks * T_loc)
    sl = slice(rank * T_loc, (rank + 1) * T_loc)
    L = ep.EPLayer(rank_ops(port, c, rank, nranks), rank, nranks, CASE["D"], CASE["K"])
    args = (torch.from_numpy(np.ascontiguousarray(c["x"][sl])),
            torch.from_numpy(np.ascontiguousarray(c["idx"][sl])),
            torch.from_numpy(np.ascontiguousarray(c["wt"][sl])))
    out = torch.zeros((T_loc, CASE["D"]))
    L.forward(*args, out, dist)
    np.save(os.path.join(out_dir, f"out{rank}.npy"), out.numpy())
    # The chunked step (exchanges queued per slice, overlapping the experts
    # on a GPU): the same rows through the same computation, slice by slice.
    for chunks in (2, 3):
        outc = torch.zeros((T_loc, CASE["D"]))
        L.forward_chunked(*args, outc, dist, chunks=chunks)
        np.save(os.path.join(out_dir, f"out{rank}_c{chunks}.npy"), outc.numpy())
    # Fixed-size exchange segments (no counts on the host).
    outf = torch.zeros((T_loc, CASE["D"]))
    L.forward_fixed(*args, outf, dist)
    np.save(os.path.join(out_dir, f"out{rank}_fixed.npy"), outf.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_ep_two_gloo_ranks(port, tmp_path):
    import multiprocessing as mp
    N, T_loc = 2, 9
    ctx = mp.get_context("spawn")
    p_no = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, N, p_no, T_loc, str(tmp_path)))
             for r in range(N)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(N)])
    _, want = layer(port, N * T_loc)
    assert_close(got, want, "2 gloo ranks EP")
    for chunks in (2, 3):
        gc = np.concatenate([np.load(tmp_path / f"out{r}_c{chunks}.npy") for r in range(N)])
        assert_close(gc, want, f"2 gloo ranks EP, {chunks} slices")
    gf = np.concatenate([np.load(tmp_path / f"out{r}_fixed.npy") for r in range(N)])
    assert_close(gf, want, "2 gloo ranks EP, fixed-size segments")


def test_ep_plan_positions(port):
    """The plan's send-buffer layout: destination-major, tokens ascending, one
    row per (token, destination) however many of its experts the rank owns."""
    c, _ = layer(port, 10)
    ops = rank_ops(port, c, 0, 4)
    pos, cnt = ops.plan(torch.from_numpy(c["idx"]))
    P, idx = pos.numpy(), c["idx"]
    expect_rows = 0
    for d in range(4):
        toks = [t for t in range(10) if any(e % 4 == d for e in idx[t])]
        assert cnt[d] == len(toks)
        for j, t in enumerate(toks):
            assert P[t, d] == expect_rows + j
        expect_rows += len(toks)
