"""Activation magnitudes at the edges of the f16 operand range.

The reference computes every activation in f32 (metal_ops.cpp:278-342), so it
accepts any finite x.  The CUDA path stages token rows (and h = act(gate, up))
as f16 operands: values below the f16 normal range lose relative precision
but stay within the absolute tolerance, and values beyond 65504 cannot be
represented at all.  Those calls are refused with MVLLM_ERR_ACT_RANGE (the
caller's `out` is left as it was) instead of returning inf.  Tolerance as
everywhere: <= 1e-2 relative L2 and <= 2e-2 max-abs.
"""
import numpy as np
import pytest

import cases
from conftest import assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _case(port, seed, scale_rows, fmt=cases.FMT_MXFP4, n=48, D=512, I=512):
    rng = np.random.default_rng(seed)
    ex = cases.make_experts(port, rng, fmt, 2, D, I)
    x = cases.bf16_round(rng.standard_normal((n, D)).astype(np.float32))
    for r, s in scale_rows.items():
        x[r] *= np.float32(s)
    nr = np.array([n // 2, n - n // 2], np.int32)
    xoff = np.array([0, n // 2], np.int32)
    act = cases.ACT_SITU if fmt == cases.FMT_MXFP4 else cases.ACT_CLAMP
    return dict(D=D, I=I, fmt=fmt, act=act, act_a=4.0 if act == cases.ACT_SITU else 7.0,
                act_b=25.0 if act == cases.ACT_SITU else 0.0, nb=2,
                g=[e[0][0] for e in ex], u=[e[1][0] for e in ex], d=[e[2][0] for e in ex],
                gs=[e[0][1] for e in ex], us=[e[1][1] for e in ex], ds=[e[2][1] for e in ex],
                xg=x, xoff=xoff, nr=nr, rows=np.arange(n, dtype=np.int32),
                rw=np.ones(n, np.float32), S=n)


def _run(moe, c, out):
    return moe.moe_block(c["nb"], c["D"], c["I"], c["fmt"], c["g"], c["u"], c["d"], c["gs"],
                         c["us"], c["ds"], c["xg"], c["xoff"], c["nr"], c["rows"], c["rw"], out,
                         c["S"], c["act"], c["act_a"], c["act_b"])


@pytest.mark.parametrize("fmt", [cases.FMT_MXFP4, cases.FMT_INT4])
def test_tiny_and_subnormal_rows_within_tolerance(moe, port, fmt):
    """Rows scaled to 1e-3, 1e-6 (below the f16 normal range) and 1e-40 (an
    f32 subnormal; f16 rounds it to zero) and an all-zero row: the outputs of
    those rows are tiny and the whole batch stays within tolerance."""
    c = _case(port, 51, {1: 1e-3, 2: 1e-6, 3: 1e-40, 30: 1e-6, 31: 0.0}, fmt=fmt)
    _, want = cases.run_block(port, c)
    out = np.zeros_like(want)
    assert _run(moe, c, out)
    assert_close(out, want, "tiny rows")
    assert np.abs(out[2]).max() < 1e-4 and np.abs(out[3]).max() < 1e-30


@pytest.mark.parametrize("where", ["x", "h"])
def test_beyond_f16_is_refused(moe, port, where):
    """A finite activation beyond the f16 range is refused with
    MVLLM_ERR_ACT_RANGE and the caller's rows are left untouched: a token row
    with |x| = 1e5 (where="x"), or moderate x whose SiLU(gate) * up exceeds
    65504 (where="h")."""
    if where == "x":
        c = _case(port, 52, {5: 1e5 / 3.0})
    else:
        c = _case(port, 53, {7: 1000.0})
        c["act"], c["act_a"], c["act_b"] = cases.ACT_SILU, 0.0, 0.0
        assert np.abs(c["xg"]).max() < 65504  # x itself fits f16
        # The reference's f32 h = silu(gate) * up of row 7 is beyond the f16 range.
        g = port.matmul_mxfp4(c["xg"][7:8], c["g"][0], c["gs"][0], c["I"])
        u = port.matmul_mxfp4(c["xg"][7:8], c["u"][0], c["us"][0], c["I"])
        h = g / (1.0 + np.exp(-g.astype(np.float64))) * u
        assert np.abs(h).max() > 65504
    base = np.random.default_rng(3).standard_normal((c["S"], c["D"])).astype(np.float32)
    out = base.copy()
    with pytest.raises(moe.MoeError) as e:
        _run(moe, c, out)
    assert e.value.code == moe.ERR_ACT_RANGE
    np.testing.assert_array_equal(out, base)


@pytest.mark.parametrize("T", [24, 300])
def test_layer_dev_error_leaves_out(moe, port, T):
    """A device-pointer call (no host sync) with a token row beyond the f16
    range: the combine does not run, so `out` keeps the caller's rows, and
    mvllm_moe_layer_error reports MVLLM_ERR_ACT_RANGE; the next clean call
    on the same workspace reports MVLLM_OK.  T = 24 takes the decode-sized
    chain (row-order staging), T = 300 the large one (token-order staging).
    In both, a token routed to no expert is not staged, so a huge value in
    it is not an error (the clean call carries one)."""
    D, I, E, K = 512, 512, 4, 2
    rng = np.random.default_rng(57)
    ex = cases.make_experts(port, rng, cases.FMT_MXFP4, E, D, I)
    tabs = [[], [], [], [], [], []]
    keep = []
    for (gp, gsc), (up, usc), (dp, dsc) in ex:
        for k, a in enumerate((gp, up, dp, gsc, usc, dsc)):
            t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
            keep.append(t)
            tabs[k].append(t.data_ptr())
    tables = [torch.tensor(t, dtype=torch.int64, device="cuda") for t in tabs]
    idx_h = rng.integers(0, E, (T, K)).astype(np.int32)
    idx_h[T - 2] = -1  # token T-2 goes to no expert
    idx = torch.from_numpy(idx_h).cuda()
    wt = torch.full((T, K), 0.5, device="cuda")
    x = rng.standard_normal((T, D)).astype(np.float32)
    x[T - 2] *= np.float32(1e6)
    ws = torch.empty(moe.layer_workspace_bytes(T, K, E, 0, D, I, cases.FMT_MXFP4),
                     dtype=torch.uint8, device="cuda")
    base = torch.from_numpy(rng.standard_normal((T, D)).astype(np.float32)).cuda()
    for bad, want_code in ((True, moe.ERR_ACT_RANGE), (False, 0)):
        xx = x.copy()
        if bad:
            xx[3] *= np.float32(1e5 / 3.0)
        out = base.clone()
        moe.layer_dev(T, K, E, 0, D, I, cases.FMT_MXFP4, idx, wt, torch.from_numpy(xx).cuda(),
                      tables, out, cases.ACT_SITU, 4.0, 25.0, ws)
        assert moe.layer_error(ws) == want_code
        if bad:
            assert torch.equal(out, base)
        else:
            assert not torch.equal(out, base)
