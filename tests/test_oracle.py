"""Pins the CPU oracle (the C restatement) before it is trusted as the checker.

* against the golden fixtures written by the reference build (bit-exact);
* against the reference build itself on random cases, when oracle/_ref exists;
* against the reference's own known-answer tests (tests/test_host.cpp), restated.
"""
import math

import numpy as np
import pytest

import cases


def test_layer_goldens_bit_exact(port, golden):
    arrays, meta = golden
    for name in cases.LAYER_CASES:
        c = cases.make_layer(port, name)
        assert c["digest"] == meta[name]["digest"], f"{name}: packed weights differ from reference"
        np.testing.assert_array_equal(c["idx"], arrays[name + "/idx"])
        np.testing.assert_array_equal(c["wt"], arrays[name + "/wt"])
        np.testing.assert_array_equal(c["rows"], arrays[name + "/rows"])
        np.testing.assert_array_equal(c["rw"], arrays[name + "/rw"])
        np.testing.assert_array_equal(c["nr"], arrays[name + "/nr"])
        ok, out = cases.run_block(port, c)
        assert ok == meta[name]["ok"]
        np.testing.assert_array_equal(out, arrays[name + "/out"], err_msg=name)


def test_kat_goldens_bit_exact(port, golden):
    arrays, meta = golden
    for name, (act, a) in {"kat_silu": (cases.ACT_SILU, 0.0),
                           "kat_clamp10": (cases.ACT_CLAMP, 10.0)}.items():
        ok, out = cases.run_block(port, cases.kat_identity(act, a))
        assert ok == meta[name]["ok"]
        np.testing.assert_array_equal(out, arrays[name + "/out"])
    ok, out = cases.run_block(port, cases.kat_mxfp4_diag(port))
    np.testing.assert_array_equal(out, arrays["kat_mxfp4_diag/out"])
    ok, out = cases.run_block(port, cases.edge_case(port))
    np.testing.assert_array_equal(out, arrays["edge/out"])


def test_reference_kat_closed_forms(port):
    # tests/test_host.cpp:2567-2601: identity weights, SiLU -> silu(x)*x within 1e-4.
    c = cases.kat_identity(cases.ACT_SILU, 0.0)
    ok, out = cases.run_block(port, c)
    x = c["xg"][0]
    want = [(v * (1 / (1 + math.exp(-v)))) * v for v in x]
    assert ok and np.allclose(out[0], want, atol=1e-4)
    # :2627-2651: ClampSwiGLU(limit 10) vs clamped_swiglu(x, x, 10).
    ok, out = cases.run_block(port, cases.kat_identity(cases.ACT_CLAMP, 10.0))
    want = [port.clamped_swiglu(float(v), float(v), 10.0) for v in x]
    assert ok and np.allclose(out[0], want, atol=1e-4)
    # :2743-2790: MXFP4 diag, SiTU: finite and non-zero energy.
    ok, out = cases.run_block(port, cases.kat_mxfp4_diag(port))
    assert ok and np.all(np.isfinite(out)) and float((out ** 2).sum()) > 0
    # :133-180: activation known answers.
    assert abs(port.situ_glu(0, 0, 4, 25)) <= 1e-6
    assert abs(port.clamped_swiglu(100.0, 1.0, 7.0) - 7.0 * port.sigmoid(7.0)) <= 1e-4


def test_reference_quant_kats(port):
    # tests/test_host.cpp:133-180: int4 roundtrip within 0.6 ("4-bit, loose"), MXFP4 finite.
    O, I = 4, 64
    W = np.array([((i * 17) % 11 - 5) * 0.1 for i in range(O * I)], np.float32).reshape(O, I)
    X = np.array([((i * 3) % 7 - 3) * 0.2 for i in range(I)], np.float32).reshape(1, I)
    yf = port.matmul_f32(X, W)
    p, s = port.quantize_int4_g64(W)
    yq = port.matmul_int4_g64(X, p, s, O)
    assert np.all(np.abs(yf - yq) < 0.6)
    p, s = port.pack_mxfp4(W)
    assert np.all(np.isfinite(port.matmul_mxfp4(X, p, s, O)))
    # :2160-2230: patterned MXFP4 bytes, scale code 127.
    packed = np.array([(i * 37 + 11) & 0xFF for i in range(32 * 16)], np.uint8).reshape(32, 16)
    e8 = np.full((32, 1), 127, np.uint8)
    x = (0.1 * np.arange(1, 33, dtype=np.float32)).reshape(1, 32)
    y = port.matmul_mxfp4(x, packed, e8, 32)
    lut = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], np.float32)
    nib = np.stack([packed & 15, packed >> 4], -1).reshape(32, 32)
    assert np.allclose(y[0], (lut[nib] * x).sum(1), atol=1e-4)


def test_routing_goldens(port, golden):
    arrays, _ = golden
    # tests/test_host.cpp:4916-4931: bias-selected, mixed with unbiased sigma.
    i, w = port.moe_topk(np.array([0.1, 0.4, 10.3, 0.2], np.float32), 2,
                         np.array([0.1, 0.4, 0.3, 0.2], np.float32))
    assert list(i) == [2, 1]
    assert abs(w[0] - 0.3 / 0.7) < 1e-5 and abs(w[1] - 0.4 / 0.7) < 1e-5
    np.testing.assert_array_equal(i, arrays["topk/idx"])
    np.testing.assert_array_equal(w, arrays["topk/w"])
    u = port.moe_union_ids(np.array([[3, 1], [3, 2], [1, -1]], np.int32), 8)
    assert list(u) == [1, 2, 3]
    np.testing.assert_array_equal(u, arrays["union/out"])
    # :8255-8275: moe_topk_pick, NaN-safe.
    i, w = port.moe_topk_pick(np.array([0.1, 0.8, 0.3, 0.5], np.float32), 2)
    assert list(i) == [1, 3] and abs(w.sum() - 1) < 1e-5 and w[0] > w[1]
    np.testing.assert_array_equal(i, arrays["pick/idx"])
    i, w = port.moe_topk_pick(np.full(4, np.nan, np.float32), 2)
    assert list(i) == [0, 1] and np.allclose(w, [0.5, 0.5])
    np.testing.assert_array_equal(w, arrays["pick_nan/w"])


def test_port_matches_reference_random(port, ref):
    rng = np.random.default_rng(123)
    for trial in range(6):
        fmt = [cases.FMT_INT4, cases.FMT_MXFP4, cases.FMT_F32][trial % 3]
        act = [cases.ACT_CLAMP, cases.ACT_SITU, cases.ACT_SILU][(trial // 3 + trial) % 3]
        D = int(rng.choice([64, 96, 130, 256]))
        I = int(rng.choice([32, 64, 100]))
        c = cases.layer_case(ref, int(rng.integers(1 << 30)), D, I, E=6, K=2, T=5, fmt=fmt,
                             act=act, act_a=7.0 if act == cases.ACT_CLAMP else 4.0, act_b=25.0)
        ok_r, out_r = cases.run_block(ref, c)
        ok_p, out_p = cases.run_block(port, c)
        assert ok_r == ok_p == 1
        np.testing.assert_array_equal(out_p, out_r)


def test_port_codecs_match_reference(port, ref):
    rng = np.random.default_rng(5)
    for shape in [(7, 200), (64, 64), (3, 33), (5, 1)]:
        w = (rng.standard_normal(shape) * rng.choice([0.02, 1.0, 1e-6])).astype(np.float32)
        w.flat[0] = 0.0
        for f in ("quantize_int4_g64", "pack_mxfp4"):
            a, b = getattr(port, f)(w), getattr(ref, f)(w)
            np.testing.assert_array_equal(a[0], b[0])
            np.testing.assert_array_equal(a[1], b[1])


def test_port_topk_union_match_reference(port, ref):
    rng = np.random.default_rng(9)
    for _ in range(300):
        n = int(rng.integers(1, 40))
        k = int(rng.integers(1, 10))
        c = rng.random(n).astype(np.float32)
        c[rng.integers(0, n, 3)] = c[0]  # ties
        mix = rng.standard_normal(n).astype(np.float32) if rng.random() < 0.5 else None
        a, b = port.moe_topk(c, k, mix), ref.moe_topk(c, k, mix)
        np.testing.assert_array_equal(a[0], b[0])
        np.testing.assert_array_equal(a[1], b[1])
        idx = rng.integers(-1, 12, (int(rng.integers(1, 6)), 3)).astype(np.int32)
        np.testing.assert_array_equal(port.moe_union_ids(idx), ref.moe_union_ids(idx))


def test_invalid_args_return_false(port):
    c = cases.kat_identity(cases.ACT_SILU, 0.0)
    out = np.zeros((1, 4), np.float32)
    # metal_ops.cpp:452-457: nb<1, D<1, bad fmt, missing xoff/nr -> false.
    assert port.moe_block(0, 4, 4, 0, c["g"], c["u"], c["d"], None, None, None, c["xg"],
                          c["xoff"], c["nr"], c["rows"], c["rw"], out, 1) == 0
    assert port.moe_block(1, 4, 4, 5, c["g"], c["u"], c["d"], None, None, None, c["xg"],
                          c["xoff"], c["nr"], c["rows"], c["rw"], out, 1) == 0
    assert port.moe_block(1, 4, 4, 0, c["g"], c["u"], c["d"], None, None, None, c["xg"], None,
                          c["nr"], c["rows"], c["rw"], out, 1) == 0
