"""Expert-parallel layer on the GPU: plan / pack / combine kernels and the
local expert compute through the library.

* 4 ranks emulated in one process on one GPU (exchanges as slicing), against
  the oracle and against the single-GPU layer.
* 2 ranks on 2 GPUs over NCCL (torchrun), when the box has 2 GPUs.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import cases
from conftest import assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "micro-vllm_b200"))

CASE = dict(D=512, I=512, E=8, K=2, fmt=cases.FMT_MXFP4, act=cases.ACT_SITU, act_a=4.0,
            act_b=25.0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def tables_of(experts):
    keep, tabs = [], [[], [], [], [], [], []]
    for (gp, gsc), (up, usc), (dp, dsc) in experts:
        for k, a in enumerate((gp, up, dp, gsc, usc, dsc)):
            t = dev(a)
            keep.append(t)
            tabs[k].append(t.data_ptr())
    return [torch.tensor(t, dtype=torch.int64, device="cuda") for t in tabs], keep


def test_ep_emulated_four_ranks_gpu(moe, port):
    import ep
    N, T_loc = 4, 40
    c = cases.layer_case(port, 51, CASE["D"], CASE["I"], CASE["E"], CASE["K"], N * T_loc,
                         CASE["fmt"], CASE["act"], CASE["act_a"], CASE["act_b"], bf16_x=True)
    _, want = cases.run_block(port, c)
    layers, xs, idxs, wts, outs, keep = [], [], [], [], [], []
    for r in range(N):
        tabs, k = tables_of([c["experts"][e] for e in ep.local_experts(r, N, CASE["E"])])
        keep.append(k)
        ops = ep.CudaOps(torch, CASE["E"], CASE["K"], CASE["D"], CASE["I"], CASE["fmt"],
                         CASE["act"], CASE["act_a"], CASE["act_b"], tabs, N, N * T_loc)
        layers.append(ep.EPLayer(ops, r, N, CASE["D"], CASE["K"]))
        sl = slice(r * T_loc, (r + 1) * T_loc)
        xs.append(dev(c["x"][sl]).to(torch.bfloat16))
        idxs.append(dev(c["idx"][sl]))
        wts.append(dev(c["wt"][sl]))
        outs.append(torch.zeros((T_loc, CASE["D"]), device="cuda"))
    ep.emulate_step(layers, xs, idxs, wts, outs, torch)
    torch.cuda.synchronize()
    got = torch.cat(outs).cpu().numpy()
    assert_close(got, want, "emulated 4-rank EP")
    # The plan kernel against its definition.
    pos, cnt = layers[0].ops.plan(idxs[0])
    P, idx = pos.cpu().numpy(), c["idx"][:T_loc]
    row = 0
    for d in range(N):
        toks = [t for t in range(T_loc) if any(e % N == d for e in idx[t])]
        assert int(cnt[d]) == len(toks)
        for j, t in enumerate(toks):
            assert P[t, d] == row + j
        row += len(toks)
    # One rank holding every expert is the single-GPU layer, bit for bit.
    tabs, k = tables_of(c["experts"])
    ops = ep.CudaOps(torch, CASE["E"], CASE["K"], CASE["D"], CASE["I"], CASE["fmt"], CASE["act"],
                     CASE["act_a"], CASE["act_b"], tabs, 1, N * T_loc)
    one = torch.zeros((N * T_loc, CASE["D"]), device="cuda")
    ep.emulate_step([ep.EPLayer(ops, 0, 1, CASE["D"], CASE["K"])],
                    [dev(c["x"]).to(torch.bfloat16)], [dev(c["idx"])], [dev(c["wt"])], [one], torch)
    direct = torch.zeros_like(one)
    ws = torch.empty(moe.layer_workspace_bytes(N * T_loc, CASE["K"], CASE["E"], 0, CASE["D"],
                                               CASE["I"], CASE["fmt"]), dtype=torch.uint8,
                     device="cuda")
    moe.layer_dev(N * T_loc, CASE["K"], CASE["E"], 0, CASE["D"], CASE["I"], CASE["fmt"],
                  dev(c["idx"]), dev(c["wt"]), dev(c["x"]).to(torch.bfloat16), tabs, direct,
                  CASE["act"], CASE["act_a"], CASE["act_b"], ws)
    torch.cuda.synchronize()
    assert torch.equal(one, direct)
    # ... and EPLayer.forward_local (the one-rank step bench.py times) is that layer.
    local = torch.zeros_like(one)
    ep.EPLayer(ops, 0, 1, CASE["D"], CASE["K"]).forward_local(
        dev(c["x"]).to(torch.bfloat16), dev(c["idx"]), dev(c["wt"]), local)
    torch.cuda.synchronize()
    assert torch.equal(local, direct)


@pytest.mark.parametrize("replicated", [(), (5, 1)])
def test_ep_peer_windows_emulated_gpu(moe, port, replicated):
    """The exchange over peer memory (forward_peer's kernels: dispatch stores
    into the destinations' windows, experts with partial rows stored into the
    owners' windows, combine) with 4 ranks emulated on one GPU, their windows
    separate allocations: bit-identical to the exchange through send buffers
    (emulate_step) and within tolerance of the oracle; two steps with
    different routing through the same windows (the first step's rows and ids
    must not leak into the second)."""
    import ep
    N, T_loc = 4, 40
    pl = ep.Placement(CASE["E"], N, replicated=list(replicated))
    wins = [ep.PeerWindows(torch, N, T_loc, CASE["K"], CASE["D"]) for _ in range(N)]
    for r, w in enumerate(wins):
        w.connect(r, peers=wins)
    keep = []
    try:
        for seed in (61, 62):
            c = cases.layer_case(port, seed, CASE["D"], CASE["I"], CASE["E"], CASE["K"],
                                 N * T_loc, CASE["fmt"], CASE["act"], CASE["act_a"],
                                 CASE["act_b"], bf16_x=True)
            _, want = cases.run_block(port, c)
            layers, xs, idxs, wts, outs, ref = [], [], [], [], [], []
            for r in range(N):
                tabs, k = tables_of([c["experts"][e] for e in pl.local_experts(r)])
                keep.append(k)
                ops = ep.CudaOps(torch, CASE["E"], CASE["K"], CASE["D"], CASE["I"], CASE["fmt"],
                                 CASE["act"], CASE["act_a"], CASE["act_b"], tabs, N, N * T_loc,
                                 placement=pl, rank=r)
                layers.append(ep.EPLayer(ops, r, N, CASE["D"], CASE["K"]))
                sl = slice(r * T_loc, (r + 1) * T_loc)
                xs.append(dev(c["x"][sl]).to(torch.bfloat16))
                idxs.append(dev(c["idx"][sl]))
                wts.append(dev(c["wt"][sl]))
                outs.append(torch.zeros((T_loc, CASE["D"]), device="cuda"))
                ref.append(torch.zeros((T_loc, CASE["D"]), device="cuda"))
            ep.emulate_step_peer(layers, wins, xs, idxs, wts, outs)
            ep.emulate_step(layers, xs, idxs, wts, ref, torch)
            torch.cuda.synchronize()
            for o, f in zip(outs, ref):
                assert torch.equal(o, f)
            assert_close(torch.cat(outs).cpu().numpy(), want, "4-rank EP over peer windows")
    finally:
        for w in wins:
            w.close()


def test_ep_emulated_replicated_experts_gpu(moe, port):
    """Experts 1 and 5 replicated on every rank (served locally for each
    rank's own tokens), the rest strided: the layer output is unchanged."""
    import ep
    N, T_loc = 4, 40
    c = cases.layer_case(port, 53, CASE["D"], CASE["I"], CASE["E"], CASE["K"], N * T_loc,
                         CASE["fmt"], CASE["act"], CASE["act_a"], CASE["act_b"], bf16_x=True)
    _, want = cases.run_block(port, c)
    pl = ep.Placement(CASE["E"], N, replicated=[5, 1])
    layers, xs, idxs, wts, outs, keep = [], [], [], [], [], []
    for r in range(N):
        tabs, k = tables_of([c["experts"][e] for e in pl.local_experts(r)])
        keep.append(k)
        ops = ep.CudaOps(torch, CASE["E"], CASE["K"], CASE["D"], CASE["I"], CASE["fmt"],
                         CASE["act"], CASE["act_a"], CASE["act_b"], tabs, N, N * T_loc,
                         placement=pl, rank=r)
        layers.append(ep.EPLayer(ops, r, N, CASE["D"], CASE["K"]))
        sl = slice(r * T_loc, (r + 1) * T_loc)
        xs.append(dev(c["x"][sl]).to(torch.bfloat16))
        idxs.append(dev(c["idx"][sl]))
        wts.append(dev(c["wt"][sl]))
        outs.append(torch.zeros((T_loc, CASE["D"]), device="cuda"))
    ep.emulate_step(layers, xs, idxs, wts, outs, torch)
    torch.cuda.synchronize()
    assert_close(torch.cat(outs).cpu().numpy(), want, "emulated 4-rank EP, replicated experts")
    # rank 2's plan: a token goes to itself for experts 1/5, to e % 4 otherwise
    pos, cnt = layers[2].ops.plan(idxs[2])
    P, idx = pos.cpu().numpy(), c["idx"][2 * T_loc:3 * T_loc]
    for t in range(T_loc):
        need = {2 if e in (1, 5) else e % N for e in idx[t] if 0 <= e < CASE["E"]}
        assert {d for d in range(N) if P[t, d] >= 0} == need


def test_layer_partial_rows(moe, port):
    """mvllm_moe_layer_partial_dev: each row is the f32 layer result rounded
    once to f16 after a power-of-two scale that puts the row maximum in
    [2^14, 2^15); tokens without a slot give zero rows."""
    T = 48
    c = cases.layer_case(port, 57, CASE["D"], CASE["I"], CASE["E"], CASE["K"], T, CASE["fmt"],
                         CASE["act"], CASE["act_a"], CASE["act_b"], bf16_x=True)
    idx = c["idx"].copy()
    idx[5] = -1  # a token routed nowhere
    tabs, keep = tables_of(c["experts"])
    ws = torch.empty(moe.layer_workspace_bytes(T, CASE["K"], CASE["E"], 0, CASE["D"], CASE["I"],
                                               CASE["fmt"]), dtype=torch.uint8, device="cuda")
    args = (T, CASE["K"], CASE["E"], 0, CASE["D"], CASE["I"], CASE["fmt"], dev(idx), dev(c["wt"]),
            dev(c["x"]).to(torch.bfloat16), tabs)
    ref = torch.zeros((T, CASE["D"]), device="cuda")
    moe.layer_dev(*args, ref, CASE["act"], CASE["act_a"], CASE["act_b"], ws)
    rows = torch.full((T, moe.partial_row_bytes(CASE["D"])), 0xAB, dtype=torch.uint8,
                      device="cuda")
    moe.layer_partial_dev(*args, rows, CASE["act"], CASE["act_a"], CASE["act_b"], ws)
    torch.cuda.synchronize()
    got = moe.decode_partial_rows(torch, rows, CASE["D"])
    sc = rows[:, 2 * CASE["D"]:2 * CASE["D"] + 4].contiguous().view(torch.float32).flatten()
    assert torch.all(got[5] == 0) and float(sc[5]) == 1.0
    m = ref.abs().amax(dim=1)
    live = m > 0
    q = (m[live] / sc[live]).cpu().numpy()
    assert np.all(q >= 2.0 ** 14) and np.all(q < 2.0 ** 15)
    assert np.all(np.log2(sc.cpu().numpy()) == np.round(np.log2(sc.cpu().numpy())))
    # one f16 rounding of v / 2^s: |err| <= 2^-11 |v| (normal range) or half an f16 ulp
    err = (got - ref).abs()
    bound = torch.maximum(ref.abs() * 2.0 ** -11, sc[:, None] * 2.0 ** -25)
    assert torch.all(err <= bound), float((err - bound).max())


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_ep_nccl_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29561",
           os.path.join(ROOT, "tests", "ep_nccl_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=330)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "EP-NCCL-OK" in r.stdout
