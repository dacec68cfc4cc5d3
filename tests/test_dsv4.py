"""DeepSeek-V4 routed experts on CPU: the oracle pinned to the reference's own
DeepSeek-V4 CPU tier (src/gpu/dsv4_cuda.cpp built into oracle/_ref), and the
expert-split step (micro-vllm_b200/dsv4.py) run as two gloo ranks.

* route (sqrt(softplus) scores, top 6, routed_scale): the reference test's
  known answer (tests/test_host.cpp:1700-1775) and random cases, bit for bit.
* e4m3fn / e8m0 decoders for every code; the FP8 128x128-tile matvec.
* moe (MXFP4 expert group + FP8 shared expert): the reference test's case
  (tests/test_host.cpp:1617-1680) and a random one, bit for bit.
* route_moe_ep2 (parity split + allreduce_pair), bit for bit, with absent
  bank slots and with and without the shared expert.
* dsv4.EP2Layer over two gloo ranks and emulated: bit-identical to the
  oracle's route_moe_ep2 plus the layer tail; over three gloo ranks, the same
  result on every rank, within tolerance.
* the expert blob geometry (make_mx_geom and the blob order).
"""
import os
import socket
import sys

import numpy as np
import pytest

import dsv4_cases as dc

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "micro-vllm_b200"))


def test_route_known_answer(port, ref):
    """tests/test_host.cpp:1700-1775: E 16, H 8, W[e][h] = 0.01 ((e+h) % 3),
    bias[e] = e, x = 1, routed_scale 1.5, free and fixed ids."""
    E, H, rs = 16, 8, 1.5
    W = np.array([[0.01 * ((e + h) % 3) for h in range(H)] for e in range(E)], np.float32)
    b = np.arange(E, dtype=np.float32)
    x = np.ones((1, H), np.float32)
    logits = port.matmul_f32(x, W)[0]
    scores = np.array([port.sqrt_softplus(float(v)) for v in logits], np.float32)
    choice = (scores + b).astype(np.float32)
    order = sorted(range(E), key=lambda e: (-choice[e], e))[:6]
    for fixed, want_ids in ((None, order), ([1, 3, 5, 7, 9, 11], [1, 3, 5, 7, 9, 11])):
        w = np.maximum(scores[want_ids], 0)
        want_w = w / w.sum() * rs
        pi, pw = port.dsv4_route(x, W, b, rs, fixed)
        ri, rw = ref.dsv4_route(x, W, b, rs, fixed)
        np.testing.assert_array_equal(pi[0], want_ids)
        np.testing.assert_allclose(pw[0], want_w, atol=1e-4)  # the test's CHECK_NEAR
        np.testing.assert_array_equal(pi, ri)
        np.testing.assert_array_equal(pw.view(np.uint32), rw.view(np.uint32))


@pytest.mark.parametrize("E,H,rs", [(64, 96, 1.0), (5, 40, 2.5), (256, 64, 1.0)])
def test_route_pinned(port, ref, E, H, rs):
    rng = np.random.default_rng(E + H)
    T = 40
    x = rng.standard_normal((T, H)).astype(np.float32)
    router = (rng.standard_normal((E, H)) * (3.0 / np.sqrt(H))).astype(np.float32)
    router[0] *= 30.0  # logits past the +-20 cut-offs
    router[1] *= -30.0
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    x[3] = 0.0  # all logits 0: equal scores, ties to the lower id
    for b in (bias, None):
        pi, pw = port.dsv4_route(x, router, b, rs)
        ri, rw = ref.dsv4_route(x, router, b, rs)
        np.testing.assert_array_equal(pi, ri)
        np.testing.assert_array_equal(pw.view(np.uint32), rw.view(np.uint32))
    if E < 6:
        assert (pi[:, E:] == -1).all() and (pw[:, E:] == 0).all()


def test_fp8_decoders_pinned(port, ref):
    for v in range(256):
        for f in ("e4m3fn_decode", "e8m0_decode"):
            a, b = getattr(port, f)(v), getattr(ref, f)(v)
            assert (np.isnan(a) and np.isnan(b)) or np.float32(a).view(np.uint32) == \
                np.float32(b).view(np.uint32), (f, v, a, b)


def test_matmul_fp8_pinned(port, ref):
    rng = np.random.default_rng(8)
    for S, I, O in ((3, 300, 200), (1, 32, 32), (2, 128, 129)):
        w, s = dc.fp8_tensor(rng, O, I)
        x = rng.standard_normal((S, I)).astype(np.float32)
        np.testing.assert_array_equal(port.matmul_fp8_b128(x, w, s, O),
                                      ref.matmul_fp8_b128(x, w, s, O))
    # the reference test's FP8 pattern (tests/test_host.cpp:1670-1676)
    O = I = 32
    sw = np.array([(i * 11 + 5) % 120 + 1 for i in range(O * I)], np.uint8).reshape(O, I)
    ssc = np.full((1, 1), 127, np.uint8)
    x = (0.05 * ((np.arange(I) % 7) - 3)).astype(np.float32)[None]
    np.testing.assert_array_equal(port.matmul_fp8_b128(x, sw, ssc, O),
                                  ref.matmul_fp8_b128(x, sw, ssc, O))


def _kat_experts():
    """The reference test's two MXFP4 experts and FP8 shared expert
    (tests/test_host.cpp:1617-1676), O = I = 32."""
    O = I = 32
    ex = []
    for e in range(2):
        pg = np.array([(i * 19 + e * 5 + 3) & 0xFF for i in range(O * I // 2)], np.uint8)
        pu = np.array([(i * 23 + e * 7 + 9) & 0xFF for i in range(O * I // 2)], np.uint8)
        pd = np.array([(i * 29 + e * 11 + 1) & 0xFF for i in range(I * O // 2)], np.uint8)
        sc = np.full((O, 1), 127, np.uint8)
        ex.append(((pg.reshape(O, I // 2), sc), (pu.reshape(O, I // 2), sc),
                   (pd.reshape(I, O // 2), sc)))
    sw = np.array([(i * 11 + 5) % 120 + 1 for i in range(O * I)], np.uint8).reshape(O, I)
    ssc = np.full((1, 1), 127, np.uint8)
    shared = ((sw, ssc), (sw, ssc), (sw, ssc))
    x = (0.05 * ((np.arange(I) % 7) - 3)).astype(np.float32)
    return ex, shared, x


def test_moe_known_answer(port, ref):
    ex, shared, x = _kat_experts()
    ew = np.array([0.7, 0.3], np.float32)
    grp_p = port.dsv4_moe(x, 32, ex, ew, None, 7.0)
    grp_r = ref.dsv4_moe(x, 32, ex, ew, None, 7.0)
    np.testing.assert_array_equal(grp_p, grp_r)
    # expert_group against the experts one by one (the test's y_seq, 1e-3)
    seq = np.zeros(32, np.float32)
    for e in range(2):
        seq += port.dsv4_moe(x, 32, [ex[e]], [1.0], None, 7.0) * ew[e]
    np.testing.assert_allclose(grp_p, seq, atol=1e-3)
    moe_p = port.dsv4_moe(x, 32, ex, ew, shared, 7.0)
    np.testing.assert_array_equal(moe_p, ref.dsv4_moe(x, 32, ex, ew, shared, 7.0))
    sh = dc.fp8_shared_out(port, x[None], shared)[0]
    np.testing.assert_allclose(moe_p, grp_p + sh, atol=1e-3)  # the test's y_moe check
    assert port.dsv4_moe(x, 32, [], [], shared, 7.0) is None  # count 0: false
    assert ref.dsv4_moe(x, 32, [], [], shared, 7.0) is None


def test_moe_pinned_random(port, ref):
    rng = np.random.default_rng(4)
    H, I = 160, 96
    ex = cases_experts(port, rng, 6, H, I)
    shared = [dc.fp8_tensor(rng, I, H), dc.fp8_tensor(rng, I, H), dc.fp8_tensor(rng, H, I)]
    x = rng.standard_normal(H).astype(np.float32)
    w = rng.random(6).astype(np.float32)
    for sh in (None, shared):
        np.testing.assert_array_equal(port.dsv4_moe(x, I, ex, w, sh, 7.0),
                                      ref.dsv4_moe(x, I, ex, w, sh, 7.0))


def cases_experts(port, rng, n, H, I):
    import cases
    return cases.make_experts(port, rng, cases.FMT_MXFP4, n, H, I)


@pytest.mark.parametrize("shared,absent", [(True, ()), (False, ()), (True, (3, 8)),
                                           (False, (0, 5, 11))])
def test_route_moe_ep2_pinned(port, ref, shared, absent):
    c = dc.dsv4_case(port, 17 + len(absent), 96, 64, 12, 6, shared=shared, dense=False,
                     absent=absent)
    for t in range(c["T"]):
        args = (c["x"][t], c["router"], c["bias"], 1.0, c["I"], c["experts"], c["shared_fp8"],
                dc.LIMIT)
        po, pp = port.dsv4_route_moe_ep2(*args)
        ro, rp = ref.dsv4_route_moe_ep2(*args)
        np.testing.assert_array_equal(po, ro)
        np.testing.assert_array_equal(pp, rp)
        np.testing.assert_array_equal(po, pp)


def _layers(port, c, nranks):
    import dsv4
    return [dsv4.EP2Layer(dc.CpuOps(torch, port, c, r, nranks,
                                    c["shared_fp8"] if r == 0 else None), r, nranks)
            for r in range(nranks)]


def test_ep2_emulated_bit_exact(port):
    import dsv4
    c = dc.dsv4_case(port, 23, 96, 64, 12, 7)
    acc_w, h_w = dc.expected(port, c)
    h = torch.from_numpy(c["h"].copy())
    acc = dsv4.emulate_step(_layers(port, c, 2), torch.from_numpy(c["x"]), h)
    np.testing.assert_array_equal(acc.numpy(), acc_w)
    np.testing.assert_array_equal(h.numpy(), h_w)


def test_ep2_emulated_more_ranks(port):
    """Beyond the reference's two ranks: three and one, within tolerance of
    the two-rank result (the partial sums associate differently)."""
    import dsv4
    from conftest import assert_close
    c = dc.dsv4_case(port, 29, 96, 64, 12, 5)
    acc_w, _ = dc.expected(port, c)
    for n in (1, 3):
        h = torch.from_numpy(c["h"].copy())
        acc = dsv4.emulate_step(_layers(port, c, n), torch.from_numpy(c["x"]), h)
        assert_close(acc.numpy(), acc_w, f"{n} ranks")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gloo_rank(rank, nranks, port_no, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no))
    for p in ("tests", os.path.join("tests", "golden"), "oracle", "micro-vllm_b200"):
        sys.path.insert(0, os.path.join(ROOT, p))
    from oracle import Oracle
    import dsv4
    dist.init_process_group("gloo", rank=rank, world_size=nranks, timeout=timedelta(seconds=60))
    port = Oracle("port")
    c = dc.dsv4_case(port, 31, 96, 64, 12, 6)
    L = dsv4.EP2Layer(dc.CpuOps(torch, port, c, rank, nranks,
                                c["shared_fp8"] if rank == 0 else None), rank, nranks)
    h = torch.from_numpy(c["h"].copy())
    L.forward(torch.from_numpy(c["x"]), h, dist)
    np.save(os.path.join(out_dir, f"h{rank}.npy"), h.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("N", [2, 3])
def test_ep2_gloo_ranks(port, tmp_path, N):
    """Two ranks: the reference's EP2, bit for bit.  Three ranks (beyond the
    reference): every rank holds the same result, within tolerance of it."""
    import multiprocessing as mp
    from conftest import assert_close
    ctx = mp.get_context("spawn")
    p_no = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, N, p_no, str(tmp_path))) for r in range(N)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    c = dc.dsv4_case(port, 31, 96, 64, 12, 6)
    _, h_w = dc.expected(port, c)
    got = [np.load(tmp_path / f"h{r}.npy") for r in range(N)]
    for g in got[1:]:
        np.testing.assert_array_equal(g, got[0])
    if N == 2:  # the reference's result, bit for bit
        np.testing.assert_array_equal(got[0], h_w)
    else:
        assert_close(got[0], h_w, f"{N} gloo ranks")


def test_blob_geometry():
    """make_mx_geom (dsv4.cpp:64-80) and the blob order of moe_layer_ep2
    (dsv4.cpp:2958-2965): gate packed, gate scales, down packed, down scales,
    up packed, up scales."""
    import dsv4
    H, O = 7168, 2048
    w1p, w1s, w2p, w2s, slot = dsv4.mx_geom(H, O)
    assert (w1p, w1s, w2p, w2s) == (O * H // 2, O * H // 32, H * O // 2, H * O // 32)
    assert slot == 2 * (w1p + w1s) + w2p + w2s
    g, u, d, gs, us, ds = dsv4.blob_pointers(1000, H, O)
    assert (g, gs, d, ds, u, us) == (1000, 1000 + w1p, 1000 + w1p + w1s,
                                     1000 + w1p + w1s + w2p, 1000 + w1p + w1s + w2p + w2s,
                                     1000 + 2 * w1p + w1s + w2p + w2s)
    assert us + w1s == 1000 + slot
    # shapes off the 32 grid round up per row
    w1p, w1s, w2p, w2s, _ = dsv4.mx_geom(40, 24)
    assert (w1p, w1s, w2p, w2s) == (24 * 20, 24 * 2, 40 * 12, 40 * 1)
