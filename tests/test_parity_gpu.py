"""Parity of the sm_100a path against the CPU oracle / reference goldens.

Tolerance (north star): <= 1e-2 relative L2 and <= 2e-2 max-abs for the
f32-accumulated outputs (conftest.REL_L2_TOL / MAX_ABS_TOL); routing,
permutation and weight packing bit-exact.
"""
import numpy as np
import pytest

import cases
from conftest import assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


class DeviceExperts:
    """Uploads per-expert packed arrays; exposes the six device pointer tables."""

    def __init__(self, experts):
        self.keep = []
        tabs = [[], [], [], [], [], []]
        for (gp, gsc), (up, usc), (dp, dsc) in experts:
            for k, a in enumerate((gp, up, dp, gsc, usc, dsc)):
                if a is None:
                    tabs[k].append(0)
                    continue
                t = dev(a)
                self.keep.append(t)
                tabs[k].append(t.data_ptr())
        self.tables = [torch.tensor(t, dtype=torch.int64, device="cuda") for t in tabs]
        self.host_tables = tabs


def run_host_block(moe, c):
    out = np.zeros((max(c["S"], 1), c["D"]), np.float32)
    ok = moe.moe_block(c["nb"], c["D"], c["I"], c["fmt"], c["g"], c["u"], c["d"], c["gs"],
                       c["us"], c["ds"], c["xg"], c["xoff"], c["nr"], c["rows"], c["rw"], out,
                       c["S"], c["act"], c["act_a"], c["act_b"])
    return ok, out


def test_kat_goldens(moe, port, golden):
    arrays, _ = golden
    for name, (act, a) in {"kat_silu": (cases.ACT_SILU, 0.0),
                           "kat_clamp10": (cases.ACT_CLAMP, 10.0)}.items():
        ok, out = run_host_block(moe, cases.kat_identity(act, a))
        assert ok
        assert np.allclose(out, arrays[name + "/out"], atol=1e-4), name
    ok, out = run_host_block(moe, cases.kat_mxfp4_diag(port))
    assert ok
    assert np.allclose(out, arrays["kat_mxfp4_diag/out"], atol=1e-4)
    ok, out = run_host_block(moe, cases.edge_case(port))
    assert ok
    assert_close(out, arrays["edge/out"], "edge")


@pytest.mark.parametrize("name", list(cases.LAYER_CASES))
def test_layer_goldens_host_abi(moe, port, golden, name):
    arrays, meta = golden
    c = cases.make_layer(port, name)
    assert c["digest"] == meta[name]["digest"]
    ok, out = run_host_block(moe, c)
    assert ok
    assert_close(out, arrays[name + "/out"], name)
    # Unregistered weights were uploaded per call; registering them gives the same bits.
    regs = [a for e in c["experts"] for p in e for a in p if a is not None]
    for a in regs:
        moe.cache_register(a, 1)
    ok, out2 = run_host_block(moe, c)
    moe.cache_clear()
    assert ok
    np.testing.assert_array_equal(out, out2)


@pytest.mark.parametrize("name", list(cases.LAYER_CASES))
def test_layer_goldens_device_layer(moe, port, golden, name):
    arrays, _ = golden
    c = cases.make_layer(port, name)
    T, K, E, ns, D, I = c["T"], c["K"], c["E"], c["n_shared"], c["D"], c["I"]
    de = DeviceExperts(c["experts"])
    ws = torch.empty(moe.layer_workspace_bytes(T, K, E, ns, D, I, c["fmt"]), dtype=torch.uint8,
                     device="cuda")
    out = torch.zeros((T, D), dtype=torch.float32, device="cuda")
    moe.layer_dev(T, K, E, ns, D, I, c["fmt"], dev(c["idx"]), dev(c["wt"]), dev(c["x"]),
                  de.tables, out, c["act"], c["act_a"], c["act_b"], ws)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), arrays[name + "/out"], name)
    # bf16 activations give the same result when x is bf16-exact.
    if name in ("small_mxfp4", "small_int4"):
        out2 = torch.zeros_like(out)
        moe.layer_dev(T, K, E, ns, D, I, c["fmt"], dev(c["idx"]), dev(c["wt"]),
                      dev(c["x"]).to(torch.bfloat16), de.tables, out2, c["act"], c["act_a"],
                      c["act_b"], ws)
        torch.cuda.synchronize()
        assert torch.equal(out, out2)


def test_block_dev_matches_host(moe, port, golden):
    arrays, _ = golden
    c = cases.make_layer(port, "config0")
    sel = [c["experts"][e] for e in c["ids"]]
    de = DeviceExperts(sel)
    R = int(c["rows"].shape[0])
    ws = torch.empty(moe.block_dev_workspace_bytes(c["nb"], c["D"], c["I"], c["fmt"], R, R,
                                                   c["S"]), dtype=torch.uint8, device="cuda")
    out = torch.zeros((c["S"], c["D"]), dtype=torch.float32, device="cuda")
    moe.block_dev(c["nb"], c["D"], c["I"], c["fmt"], de.tables, dev(c["xg"]), R, dev(c["xoff"]),
                  dev(c["nr"]), dev(c["rows"]), dev(c["rw"]), out, c["S"], c["act"], c["act_a"],
                  c["act_b"], R, ws)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), arrays["config0/out"], "block_dev")


def test_permute_bit_exact(moe, port):
    from oracle import permute
    rng = np.random.default_rng(3)
    for T, K, E, ns in [(1, 8, 256, 1), (5, 4, 16, 0), (37, 8, 64, 1), (300, 6, 40, 0),
                        (64, 8, 160, 0)]:
        idx = rng.integers(-1, E + 2, (T, K)).astype(np.int32)  # out-of-range and -1 ids
        idx[:, 1] = idx[:, 0]                                   # duplicate ids in a token
        wt = rng.random((T, K)).astype(np.float32)
        wt[rng.random((T, K)) < 0.1] = 0.0                      # zero weights are skipped
        valid = np.where((idx >= 0) & (idx < E), idx, -1)
        uniq = port.moe_union_ids(valid)
        nr, xoff, rows, rw = permute(valid, wt, uniq)
        EE, KK = E + ns, K + ns
        d_nr = torch.zeros(EE, dtype=torch.int32, device="cuda")
        d_xoff = torch.zeros(EE, dtype=torch.int32, device="cuda")
        d_rows = torch.full((T * KK,), -7, dtype=torch.int32, device="cuda")
        d_rw = torch.zeros(T * KK, dtype=torch.float32, device="cuda")
        d_pos = torch.zeros(T * KK, dtype=torch.int32, device="cuda")
        d_n = torch.zeros(1, dtype=torch.int32, device="cuda")
        ws = torch.empty(moe.permute_workspace_bytes(T, K, E, ns), dtype=torch.uint8,
                         device="cuda")
        moe.permute_dev(dev(idx), dev(wt), E, ns, d_nr, d_xoff, d_rows, d_rw, d_pos, d_n, ws)
        torch.cuda.synchronize()
        n = int(d_n.item())
        want_n = int(rows.shape[0]) + (T if ns else 0)
        assert n == want_n
        got_nr = d_nr.cpu().numpy()
        full_nr = np.zeros(EE, np.int32)
        full_nr[uniq] = nr
        if ns:
            full_nr[E] = T
        np.testing.assert_array_equal(got_nr, full_nr)
        got_rows = d_rows.cpu().numpy()[:n]
        got_rw = d_rw.cpu().numpy()[:n]
        R0 = rows.shape[0]
        np.testing.assert_array_equal(got_rows[:R0], rows)
        np.testing.assert_array_equal(got_rw[:R0], rw)
        if ns:
            np.testing.assert_array_equal(got_rows[R0:], np.arange(T))
            assert np.all(got_rw[R0:] == 1.0)


def test_device_packers_bit_exact(moe, port):
    rng = np.random.default_rng(4)
    for O, I, scale in [(64, 7168, 0.02), (33, 200, 1.0), (8, 96, 1e-7), (5, 64, 0.0),
                        (16, 2048, 30.0)]:
        w = (rng.standard_normal((O, I)) * scale).astype(np.float32)
        w[0, :5] = [0.0, -0.0, 1e-30, -3.5, 6.0]
        wd = dev(w)
        for fmt, fn, sdt, g in ((4, moe.quantize_int4_g64_dev, torch.float32, 64),
                                (7, moe.pack_mxfp4_dev, torch.uint8, 32)):
            p = torch.zeros((O, (I + 1) // 2), dtype=torch.uint8, device="cuda")
            s = torch.zeros((O, (I + g - 1) // g), dtype=sdt, device="cuda")
            fn(wd, p, s)
            torch.cuda.synchronize()
            want = port.quantize_int4_g64(w) if fmt == 4 else port.pack_mxfp4(w)
            np.testing.assert_array_equal(p.cpu().numpy(), want[0])
            np.testing.assert_array_equal(s.cpu().numpy(), want[1])


def test_matmul_dev(moe, port):
    rng = np.random.default_rng(6)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    w = (rng.standard_normal((40, 256)) * 0.02).astype(np.float32)
    for fmt in (0, 4, 7):
        if fmt == 0:
            p, s, want = w, None, port.matmul_f32(x, w)
        elif fmt == 4:
            p, s = port.quantize_int4_g64(w)
            want = port.matmul_int4_g64(x, p, s, 40)
        else:
            p, s = port.pack_mxfp4(w)
            want = port.matmul_mxfp4(x, p, s, 40)
        y = torch.zeros((3, 40), dtype=torch.float32, device="cuda")
        moe.matmul_dev(fmt, y, dev(x), dev(p), None if s is None else dev(s))
        torch.cuda.synchronize()
        assert np.allclose(y.cpu().numpy(), want, atol=1e-4, rtol=1e-4)


def _full_size(moe, port, D, I, E, K, T, fmt, act, a, b, n_shared, check_tokens, seed,
               zipf=False):
    """Full BASELINE shapes: weights generated and packed on the GPU for the
    experts the routing touches; the oracle checks a sample of tokens (tokens
    are independent, so any subset is a complete check of those rows).
    `zipf`: config[3]'s skewed routing (softmax of -1.1 ln(rank) + Gumbel noise,
    then the reference's top-k), so the tensor-core tiles of every size run."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    rng = np.random.default_rng(seed)
    if zipf:
        rank = rng.permutation(E) + 1
        logits = -1.1 * np.log(rank)[None, :] - np.log(-np.log(rng.random((T, E)) + 1e-20))
        logits = logits - logits.max(axis=1, keepdims=True)
        p = np.exp(logits)
        choice = (p / p.sum(axis=1, keepdims=True)).astype(np.float32)
    else:
        choice = rng.random((T, E), dtype=np.float32)
    idx, wt = cases.route(port, choice, K)
    x = cases.bf16_round(rng.standard_normal((T, D)).astype(np.float32))
    used = sorted(set(idx.reshape(-1).tolist())) + ([E] if n_shared else [])
    gs_ = 64 if fmt == 4 else 32
    sdt = torch.float32 if fmt == 4 else torch.uint8
    pack = moe.quantize_int4_g64_dev if fmt == 4 else moe.pack_mxfp4_dev
    tabs = [[0] * (E + n_shared) for _ in range(6)]
    keep, host = {}, {}
    for e in used:
        mats = []
        for (O_, I_) in ((I, D), (I, D), (D, I)):
            w = torch.randn((O_, I_), generator=g, device="cuda") * 0.02
            p = torch.empty((O_, (I_ + 1) // 2), dtype=torch.uint8, device="cuda")
            s = torch.empty((O_, (I_ + gs_ - 1) // gs_), dtype=sdt, device="cuda")
            pack(w, p, s)
            mats.append((p, s))
        keep[e] = mats
        for k, (p, s) in enumerate(mats):
            tabs[k][e] = p.data_ptr()
            tabs[3 + k][e] = s.data_ptr()
    tables = [torch.tensor(t, dtype=torch.int64, device="cuda") for t in tabs]
    ws = torch.empty(moe.layer_workspace_bytes(T, K, E, n_shared, D, I, fmt), dtype=torch.uint8,
                     device="cuda")
    out = torch.zeros((T, D), dtype=torch.float32, device="cuda")
    xd = dev(x).to(torch.bfloat16)
    moe.layer_dev(T, K, E, n_shared, D, I, fmt, dev(idx), dev(wt), xd, tables, out, act, a, b, ws)
    out2 = torch.zeros_like(out)
    moe.layer_dev(T, K, E, n_shared, D, I, fmt, dev(idx), dev(wt), xd, tables, out2, act, a, b, ws)
    torch.cuda.synchronize()
    assert torch.equal(out, out2), "run-to-run results differ"
    got = out.cpu().numpy()
    for c in check_tokens:
        ids = list(idx[c]) + ([E] if n_shared else [])
        ws_ = list(wt[c]) + ([1.0] if n_shared else [])
        order = sorted(range(len(ids)), key=lambda j: ids[j])
        ids = [ids[j] for j in order]
        ws_ = [ws_[j] for j in order]
        mats = [[(keep[e][k][0].cpu().numpy(), keep[e][k][1].cpu().numpy()) for k in range(3)]
                for e in ids]
        o = np.zeros((1, D), np.float32)
        nb = len(ids)
        ok = port.moe_block(nb, D, I, fmt, [m[0][0] for m in mats], [m[1][0] for m in mats],
                            [m[2][0] for m in mats], [m[0][1] for m in mats],
                            [m[1][1] for m in mats], [m[2][1] for m in mats], x[c:c + 1],
                            np.zeros(nb, np.int32), np.ones(nb, np.int32),
                            np.zeros(nb, np.int32), np.array(ws_, np.float32), o, 1, act, a, b)
        assert ok
        assert_close(got[c:c + 1], o, f"token {c}")


def test_full_size_config1_mxfp4(moe, port):
    _full_size(moe, port, 7168, 2048, 256, 8, 8, 7, cases.ACT_SITU, 4.0, 25.0, 1, [0, 5], 21)


def test_full_size_config2_int4(moe, port):
    _full_size(moe, port, 6144, 1536, 160, 8, 16, 4, cases.ACT_CLAMP, 7.0, 0.0, 0, [3, 15], 22)


def test_full_size_config3_prefill(moe, port):
    """config[3]: 4096 tokens over 256 MXFP4 experts, Zipf routing: 256-row pair
    tiles, ragged pair tiles, single-CTA tiles and the decode kernels for the
    smallest experts, all in one call; sampled tokens against the oracle."""
    _full_size(moe, port, 7168, 2048, 256, 8, 4096, 7, cases.ACT_SITU, 4.0, 25.0, 0,
               [0, 1234, 4095], 23, zipf=True)


def test_layer_host_registered_buffers(moe, port, golden):
    """mvllm_moe_layer_host with the caller's x / out page-locked (direct copies)
    gives the same bits as through the pinned staging copy."""
    c = cases.make_layer(port, "small_mxfp4")
    keep, tabs = [], [[], [], [], [], [], []]
    for (gp, gsc), (up, usc), (dp, dsc) in c["experts"]:
        for k, a in enumerate((gp, up, dp, gsc, usc, dsc)):
            t = dev(a)
            keep.append(t)
            tabs[k].append(t.data_ptr())
    T, D = c["T"], c["D"]
    args = (T, c["K"], c["E"], c["n_shared"], D, c["I"], c["fmt"], c["idx"], c["wt"])
    x = np.ascontiguousarray(c["x"], np.float32)
    base = np.random.default_rng(5).standard_normal((T, D)).astype(np.float32)
    out_a = base.copy()
    moe.layer_host(*args, x, tabs, out_a, c["act"], c["act_a"], c["act_b"])
    x_r, out_b = x.copy(), base.copy()
    moe.host_register(x_r)
    moe.host_register(out_b)
    try:
        moe.layer_host(*args, x_r, tabs, out_b, c["act"], c["act_a"], c["act_b"])
    finally:
        moe.host_unregister(x_r)
        moe.host_unregister(out_b)
    np.testing.assert_array_equal(out_b, out_a)


def test_moe_block_registered_buffers(moe, port):
    """mvllm_moe_block with the caller's xg / out page-locked (direct copies)
    gives the same bits as through the pinned staging copy."""
    c = cases.make_layer(port, "small_int4")
    ok, want = run_host_block(moe, c)
    assert ok
    xg = np.ascontiguousarray(c["xg"], np.float32).copy()
    out = np.zeros((max(c["S"], 1), c["D"]), np.float32)
    moe.host_register(xg)
    moe.host_register(out)
    try:
        assert moe.moe_block(c["nb"], c["D"], c["I"], c["fmt"], c["g"], c["u"], c["d"], c["gs"],
                             c["us"], c["ds"], xg, c["xoff"], c["nr"], c["rows"], c["rw"], out,
                             c["S"], c["act"], c["act_a"], c["act_b"])
    finally:
        moe.host_unregister(xg)
        moe.host_unregister(out)
    np.testing.assert_array_equal(out, want)


def test_combine_linearity(moe, port):
    """Doubling every routing weight doubles the routed output exactly."""
    c = cases.make_layer(port, "small_int4")
    ok, out1 = run_host_block(moe, c)
    c2 = dict(c, rw=(c["rw"] * 2).astype(np.float32))
    ok2, out2 = run_host_block(moe, c2)
    assert ok and ok2
    np.testing.assert_array_equal(out2, 2 * out1)


def test_moe_block_large_rows(moe, port):
    """A moe_block call with more than 4 MB of activation rows, 16 experts and
    200 destination rows accumulated into: against the oracle, with the
    caller's rows page-locked (direct copies on the copy stream, out read
    back with the error word) and without (pinned staging); the two agree
    bit for bit."""
    rng = np.random.default_rng(77)
    D, I, nb = 2048, 512, 16
    ex = cases.make_experts(port, rng, cases.FMT_MXFP4, nb, D, I)
    nr = rng.integers(20, 45, nb).astype(np.int32)
    R = int(nr.sum())
    assert R * D * 4 >= 4 << 20
    xoff = np.concatenate([[0], np.cumsum(nr)[:-1]]).astype(np.int32)
    xg = cases.bf16_round(rng.standard_normal((R, D)).astype(np.float32))
    S = 200
    rows = rng.integers(0, S, R).astype(np.int32)
    rw = rng.random(R).astype(np.float32)
    c = dict(D=D, I=I, fmt=cases.FMT_MXFP4, act=cases.ACT_SILU, act_a=0.0, act_b=0.0, nb=nb,
             g=[e[0][0] for e in ex], u=[e[1][0] for e in ex], d=[e[2][0] for e in ex],
             gs=[e[0][1] for e in ex], us=[e[1][1] for e in ex], ds=[e[2][1] for e in ex],
             xg=xg, xoff=xoff, nr=nr, rows=rows, rw=rw, S=S)
    base = rng.standard_normal((S, D)).astype(np.float32)
    _, want = cases.run_block(port, c, out=base.copy())
    args = (nb, D, I, cases.FMT_MXFP4, c["g"], c["u"], c["d"], c["gs"], c["us"], c["ds"])
    out_a = base.copy()
    assert moe.moe_block(*args, xg, xoff, nr, rows, rw, out_a, S, cases.ACT_SILU, 0.0, 0.0)
    assert_close(out_a, want, "large rows")
    x_r, out_b = xg.copy(), base.copy()
    moe.host_register(x_r)
    moe.host_register(out_b)
    try:
        assert moe.moe_block(*args, x_r, xoff, nr, rows, rw, out_b, S, cases.ACT_SILU, 0.0, 0.0)
    finally:
        moe.host_unregister(x_r)
        moe.host_unregister(out_b)
    np.testing.assert_array_equal(out_b, out_a)
