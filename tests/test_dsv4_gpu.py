"""DeepSeek-V4 routed experts on the GPU against the oracle (which
tests/test_dsv4.py pins to the reference's DeepSeek-V4 CPU tier).

* mvllm_moe_route_ex_dev with sqrt(softplus) scores: router dot products in
  the reference's order, e^x and log1p correctly rounded.  The host's log1pf
  is not correctly rounded (a few percent of its results are off by an ulp or
  two), so scores match the host's within 4 ulp, most to the last bit; ids
  identical for every token, weights to 1e-6.
* mvllm_matmul_dev on FP8 128x128 tiles: bit-identical.
* mvllm_moe_dense_ffn_dev (FP8 shared expert, int8-row dense MLP): the
  reference's arithmetic, equal up to the activation's exponential.
* mvllm_moe_ep_local_ids_dev: the parity split, exactly.
* dsv4.EP2Layer, both ranks emulated on one GPU: against route_moe_ep2 plus
  the layer tail, within the MoE tolerance (rel-L2 1e-2, max-abs 2e-2).
* Two ranks on two GPUs over NCCL (torchrun), when the box has two GPUs.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import dsv4_cases as dc
from conftest import assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "micro-vllm_b200"))


def dev(a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("E,H,rs,dtype", [(256, 1024, 1.0, "f32"), (64, 512, 2.5, "f32"),
                                          (5, 256, 1.0, "f32"), (256, 1024, 1.0, "bf16"),
                                          (96, 300, 1.0, "f32")])
def test_route_sqrt_softplus(exact, port, E, H, rs, dtype):
    """f32 and bf16 activations; H = 300 is not a whole number of 16-byte
    pieces, so the router takes the register-staged tile instead of the
    cp.async ring.  Exact mode."""
    moe = exact
    rng = np.random.default_rng(E * 7 + H)
    T = 96
    x = rng.standard_normal((T, H)).astype(np.float32)
    if dtype == "bf16":
        x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)  # bf16-exact values
    router = (rng.standard_normal((E, H)) * (3.0 / np.sqrt(H))).astype(np.float32)
    router[0] *= 30.0  # logits past the +-20 cut-offs
    router[1] *= -30.0
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    K = 6
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wt = torch.empty((T, K), dtype=torch.float32, device="cuda")
    scores = torch.empty((T, E), dtype=torch.float32, device="cuda")
    choice = torch.empty((T, E), dtype=torch.float32, device="cuda")
    xd = dev(x) if dtype == "f32" else dev(x).to(torch.bfloat16)
    moe.route_ex_dev(xd, dev(router), dev(bias), K, idx, wt, scores, choice,
                     moe.SCORE_SQRT_SOFTPLUS, rs)
    torch.cuda.synchronize()
    ri, rw = port.dsv4_route(x, router, bias, rs)
    logits = port.matmul_f32(x, router)
    sc = np.array([[port.sqrt_softplus(float(v)) for v in row] for row in logits], np.float32)
    gs = scores.cpu().numpy()
    ulps = np.abs(gs.view(np.int32).astype(np.int64) - sc.view(np.int32).astype(np.int64))
    assert ulps.max() <= 4, ulps.max()
    assert (ulps > 0).mean() < 0.05, (ulps > 0).mean()
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(wt.cpu().numpy(), rw, rtol=1e-6, atol=0)


def test_route_ex_sigmoid_is_route(moe):
    """score_fn sigmoid with routed_scale 1 is mvllm_moe_route_dev, bit for bit."""
    rng = np.random.default_rng(2)
    T, H, E, K = 33, 256, 160, 8
    x, router = dev(rng.standard_normal((T, H)).astype(np.float32)), dev(
        (rng.standard_normal((E, H)) * 0.05).astype(np.float32))
    outs = []
    for ex in (False, True):
        o = [torch.empty((T, K), dtype=torch.int32, device="cuda"),
             torch.empty((T, K), dtype=torch.float32, device="cuda"),
             torch.empty((T, E), device="cuda"), torch.empty((T, E), device="cuda")]
        if ex:
            moe.route_ex_dev(x, router, None, K, *o, moe.SCORE_SIGMOID, 1.0)
        else:
            moe.route_dev(x, router, None, K, *o)
        outs.append([t.cpu() for t in o])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_matmul_fp8_bit_exact(moe, port):
    rng = np.random.default_rng(12)
    for S, I, O in ((1, 256, 40), (37, 300, 200), (5, 2048, 384)):
        w, s = dc.fp8_tensor(rng, O, I)
        x = rng.standard_normal((S, I)).astype(np.float32)
        y = torch.zeros((S, O), device="cuda")
        moe.matmul_dev(moe.FMT_FP8_B128, y, dev(x), dev(w), dev(s))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), port.matmul_fp8_b128(x, w, s, O))


def _close_to_last_bit(got, want, what):
    """Equal except where one exponential misrounds on the host: a few
    ulp-level differences carried through the down projection."""
    bad = got != want
    assert bad.mean() < 0.02, (what, bad.mean())
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6, err_msg=what)


def test_dense_ffn(moe, port):
    rng = np.random.default_rng(21)
    T, H, I = 9, 512, 256
    x = rng.standard_normal((T, H)).astype(np.float32)
    sh = [dc.fp8_tensor(rng, I, H), dc.fp8_tensor(rng, I, H), dc.fp8_tensor(rng, H, I)]
    want = dc.fp8_shared_out(port, x, sh)
    y = torch.zeros((T, H), device="cuda")
    moe.dense_ffn_dev(moe.FMT_FP8_B128, dev(x), *[(dev(w), dev(s)) for w, s in sh], y,
                      moe.ACT_CLAMP_SWIGLU, dc.LIMIT)
    torch.cuda.synchronize()
    _close_to_last_bit(y.cpu().numpy(), want, "fp8 shared expert")
    # accumulate: y + d, one rounding per element
    base = rng.standard_normal((T, H)).astype(np.float32)
    y2 = dev(base)
    moe.dense_ffn_dev(moe.FMT_FP8_B128, dev(x), *[(dev(w), dev(s)) for w, s in sh], y2,
                      moe.ACT_CLAMP_SWIGLU, dc.LIMIT, accumulate=True)
    torch.cuda.synchronize()
    _close_to_last_bit(y2.cpu().numpy(), (base + want).astype(np.float32), "accumulate")
    # int8-row dense MLP (the layer's QuantMat shared MLP)
    ws = [(rng.standard_normal(s) * 0.05).astype(np.float32) for s in ((I, H), (I, H), (H, I))]
    q = [port.quantize_int8_row(w) for w in ws]
    y3 = torch.zeros((T, H), device="cuda")
    moe.dense_ffn_dev(moe.FMT_INT8_ROW, dev(x), *[(dev(a), dev(b)) for a, b in q], y3,
                      moe.ACT_CLAMP_SWIGLU, dc.LIMIT)
    torch.cuda.synchronize()
    _close_to_last_bit(y3.cpu().numpy(), dc.dense_out(port, x, q), "int8 dense")


def test_local_ids(moe):
    rng = np.random.default_rng(5)
    E, T, K = 20, 50, 6
    idx = rng.integers(-2, E + 3, (T, K)).astype(np.int32)
    for n in (1, 2, 3):
        for r in range(n):
            out = torch.empty((T, K), dtype=torch.int32, device="cuda")
            moe.ep_local_ids_dev(dev(idx), E, n, r, out)
            mine = (idx >= 0) & (idx < E) & (idx % n == r)
            np.testing.assert_array_equal(out.cpu().numpy(), np.where(mine, idx // n, -1))


def rank_ops(moe, c, rank, nranks, keep):
    import dsv4
    tabs = [[], [], [], [], [], []]
    for e in range(rank, c["E"], nranks):
        (gp, gsc), (up, usc), (dp, dsc) = c["experts"][e]
        for k, a in enumerate((gp, up, dp, gsc, usc, dsc)):
            t = dev(a)
            keep.append(t)
            tabs[k].append(t.data_ptr())
    tables = [torch.tensor(t, dtype=torch.int64, device="cuda") for t in tabs]
    sh = None
    if rank == 0 and c["shared_fp8"] is not None:
        sh = [(dev(w), dev(s)) for w, s in c["shared_fp8"]]
    dense = (c["dense_fmt"],) + tuple((dev(a), dev(b)) for a, b in c["dense"])
    return dsv4.CudaOps(torch, c["E"], c["H"], c["I"], dc.LIMIT, dev(c["router"]),
                        dev(c["bias"]), tables, rank, nranks, c["T"], c["route_scale"],
                        c["routed_scale"], sh, dense)


@pytest.mark.parametrize("H,I,E,T,dfmt", [(512, 256, 16, 40, 8), (1024, 512, 32, 8, 8),
                                          (512, 256, 16, 24, 4)])
def test_ep2_emulated(moe, port, H, I, E, T, dfmt):
    """int8-row dense MLP: the exact sequential path; int4-g64 (the reference's
    default dense_bits): through the MoE kernels as one expert."""
    import dsv4
    c = dc.dsv4_case(port, H + T, H, I, E, T, dense_fmt=dfmt)
    acc_w, h_w = dc.expected(port, c)
    keep = []
    layers = [dsv4.EP2Layer(rank_ops(moe, c, r, 2, keep), r, 2) for r in range(2)]
    assert (layers[0].ops.dense_moe is not None) == (dfmt == 4)
    h = dev(c["h"])
    acc = dsv4.emulate_step(layers, dev(c["x"]), h)
    torch.cuda.synchronize()
    assert_close(acc.cpu().numpy(), acc_w, "EP2 routed sum")
    assert_close(h.cpu().numpy(), h_w, "EP2 layer output")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_ep2_nccl_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29563",
           os.path.join(ROOT, "tests", "dsv4_nccl_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=330)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "DSV4-EP2-NCCL-OK" in r.stdout
