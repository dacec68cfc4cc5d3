"""Routing on the device against the oracle and the reference goldens.

* mvllm_moe_topk_dev is bit-identical to moe_topk (ops.cpp:860-890): ids
  and weights, with ties, negative choices, mix on and off, K > E.
* mvllm_moe_route_dev: the router dot products follow the reference's order
  exactly; the sigmoid's exponential is the correctly rounded one, so scores
  match the host's to the last bit except where the host expf misrounds (then
  by at most 2 ulp, in under 0.1% of the scores).
  Routing ids must match for every token; weights to 1e-6.  (Exact mode.)
* Tolerance mode (the default): the cluster kernel's scores within 1e-5
  relative (5e-6 absolute) of the reference's; ids equal wherever the reference's K-th and
  (K+1)-th choices are more than 1e-5 apart.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_topk(moe, choice, K, mix=None):
    T, E = choice.shape
    idx = torch.full((T, K), -7, dtype=torch.int32, device="cuda")
    wt = torch.full((T, K), -7.0, dtype=torch.float32, device="cuda")
    moe.topk_dev(dev(choice), K, idx, wt, None if mix is None else dev(mix))
    torch.cuda.synchronize()
    return idx.cpu().numpy(), wt.cpu().numpy()


def ref_topk(port, choice, K, mix=None):
    T = choice.shape[0]
    idx = np.full((T, K), -1, np.int32)
    wt = np.zeros((T, K), np.float32)
    for t in range(T):
        i, w = port.moe_topk(choice[t], K, None if mix is None else mix[t])
        idx[t, :len(i)] = i
        wt[t, :len(w)] = w
    return idx, wt


@pytest.mark.parametrize("E,K", [(16, 4), (160, 8), (256, 8), (384, 8), (1000, 32), (5, 8)])
def test_topk_dev_bit_exact(moe, port, E, K):
    rng = np.random.default_rng(E * 100 + K)
    T = 200
    choice = rng.standard_normal((T, E)).astype(np.float32)
    # ties: quantise some rows to a few levels, repeat values across ids
    choice[::3] = np.round(choice[::3] * 2) / 2
    choice[1::5] = 0.25
    mix = rng.random((T, E), dtype=np.float32) - 0.1  # some negative -> clamped
    for m in (None, mix):
        gi, gw = run_topk(moe, choice, K, m)
        ri, rw = ref_topk(port, choice, K, m)
        np.testing.assert_array_equal(gi, ri)
        np.testing.assert_array_equal(gw.view(np.uint32), rw.view(np.uint32))


def test_topk_dev_golden(moe, golden):
    """The reference's routing known answer (tests/test_host.cpp:4916-4931;
    fixture written by the reference build, tests/golden/gen_golden.py)."""
    arrays, _ = golden
    choice = np.array([[0.1, 0.4, 10.3, 0.2]], np.float32)
    mix = np.array([[0.1, 0.4, 0.3, 0.2]], np.float32)
    gi, gw = run_topk(moe, choice, 2, mix)
    np.testing.assert_array_equal(gi[0], arrays["topk/idx"])
    np.testing.assert_array_equal(gw[0], arrays["topk/w"])


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_route_dev_matches_reference(exact, port, dtype):
    moe = exact
    rng = np.random.default_rng(5 if dtype == "f32" else 6)
    T, H, E, K = 64, 1024, 160, 8
    x = rng.standard_normal((T, H)).astype(np.float32)
    if dtype == "bf16":
        x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)  # bf16-exact
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    xd = dev(x) if dtype == "f32" else dev(x).to(torch.bfloat16)
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wt = torch.empty((T, K), dtype=torch.float32, device="cuda")
    scores = torch.empty((T, E), dtype=torch.float32, device="cuda")
    choice = torch.empty((T, E), dtype=torch.float32, device="cuda")
    moe.route_dev(xd, dev(router), dev(bias), K, idx, wt, scores, choice)
    torch.cuda.synchronize()
    # the reference: matmul_f32, sigmoid, + bias, moe_topk(choice, mix=scores)
    logits = port.matmul_f32(x, router)
    sc = np.array([[port.sigmoid(v) for v in row] for row in logits], np.float32)
    ch = (sc + bias[None, :]).astype(np.float32)
    ri, rw = ref_topk(port, ch, K, sc)
    gs = scores.cpu().numpy()
    ulps = np.abs(gs.view(np.int32).astype(np.int64) - sc.view(np.int32).astype(np.int64))
    # One ulp of difference in e^x (where the host expf misrounds) can move the
    # sigmoid's quotient by up to two.
    assert ulps.max() <= 2, ulps.max()
    assert (ulps > 0).mean() < 1e-3, (ulps > 0).mean()
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(wt.cpu().numpy(), rw, rtol=1e-6, atol=0)


def _route_case(seed, T, H, E, dtype):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H)).astype(np.float32)
    if dtype == "bf16":
        x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)
    router = (rng.standard_normal((E, H)) * (1.0 / np.sqrt(H))).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    xd = dev(x) if dtype == "f32" else dev(x).to(torch.bfloat16)
    return x, router, bias, xd


@pytest.mark.parametrize("T,H,E,K,dtype", [(64, 1024, 160, 8, "f32"), (32, 7168, 256, 8, "bf16"),
                                           (40, 6144, 160, 8, "bf16"), (5, 512, 37, 4, "f32")])
def test_route_dev_tolerance(moe, port, T, H, E, K, dtype):
    assert not moe.get_exact()
    x, router, bias, xd = _route_case(T + H + E, T, H, E, dtype)
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wt = torch.empty((T, K), dtype=torch.float32, device="cuda")
    scores = torch.empty((T, E), dtype=torch.float32, device="cuda")
    choice = torch.empty((T, E), dtype=torch.float32, device="cuda")
    moe.route_dev(xd, dev(router), dev(bias), K, idx, wt, scores, choice)
    torch.cuda.synchronize()
    logits = port.matmul_f32(x, router)
    sc = np.array([[port.sigmoid(v) for v in row] for row in logits], np.float32)
    ch = (sc + bias[None, :]).astype(np.float32)
    ri, rw = ref_topk(port, ch, K, sc)
    gs = scores.cpu().numpy()
    np.testing.assert_allclose(gs, sc, rtol=1e-5, atol=5e-6)
    np.testing.assert_allclose(choice.cpu().numpy(), ch, rtol=1e-5, atol=5e-6)
    srt = -np.sort(-ch, axis=1)
    clear = (srt[:, K - 1] - srt[:, K]) > 1e-5 if E > K else np.ones(T, bool)
    assert clear.mean() > 0.9
    np.testing.assert_array_equal(idx.cpu().numpy()[clear], ri[clear])
    np.testing.assert_allclose(wt.cpu().numpy()[clear], rw[clear], rtol=1e-4, atol=1e-7)
