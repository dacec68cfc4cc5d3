"""Layer epilogue after the routed combine (kimi_k3.cpp:2074-2108, glm53.cpp:1993-2027):
rmsnorm of the routed sum, the latent up-projection (QuantMat fmt 0 / 4 / 8), the
routed scale and the shared expert's output added to the residual stream.

* CPU: the oracle's int8-row codec, rmsnorm and epilogue against the reference build
  (bit-exact; the epilogue against the reference's own pieces composed in its order).
* GPU, exact mode: mvllm_moe_epilogue_dev and the int8-row mvllm_matmul_dev against the
  oracle, bit for bit (the device keeps the reference's summation order and roundings).
* GPU, tolerance mode (the default): the fused epilogue kernel against the oracle within
  <= 1e-2 relative L2 and <= 2e-2 max-abs, on the update h_out - h_in (the part the
  kernel computes) as well as on h_out; run-to-run identical.
"""
import numpy as np
import pytest


torch = pytest.importorskip("torch")


def _case(seed, T, H, L, up_fmt, norm, shared, port):
    rng = np.random.default_rng(seed)
    acc = rng.standard_normal((T, L)).astype(np.float32)
    h = rng.standard_normal((T, H)).astype(np.float32)
    lat_n = (1.0 + 0.1 * rng.standard_normal(L)).astype(np.float32) if norm else None
    up_w = up_s = None
    if up_fmt is not None:
        w = (rng.standard_normal((H, L)) * (1.0 / np.sqrt(L))).astype(np.float32)
        if up_fmt == 0:
            up_w = w
        elif up_fmt == 4:
            up_w, up_s = port.quantize_int4_g64(w)
        else:
            up_w, up_s = port.quantize_int8_row(w)
    sh = rng.standard_normal((T, H)).astype(np.float32) if shared else None
    return acc, h, lat_n, up_w, up_s, sh


CASES = [  # (T, H, L, up_fmt, norm, shared, routed_scale)
    (5, 256, 256, None, False, True, 2.5),   # GLM: no latent, shared expert
    (4, 256, 128, 8, True, True, 1.75),      # K3: norm, int8 up-projection, shared
    (3, 192, 128, 4, True, False, 1.0),      # int4-g64 up-projection
    (2, 160, 96, 0, False, True, 0.5),       # f32 up-projection, no norm
]


@pytest.mark.parametrize("T,H,L,fmt,norm,shared,scale", CASES)
def test_epilogue_oracle_pinned(port, ref, T, H, L, fmt, norm, shared, scale):
    acc, h, lat_n, up_w, up_s, sh = _case(T * 7 + H, T, H, L, fmt, norm, shared, port)
    got = port.moe_epilogue(acc, h, scale, lat_n, 1e-6, 0 if fmt is None else fmt, up_w, up_s, sh)
    # the reference's pieces in the reference's order
    want = h.copy()
    for c in range(T):
        a = ref.rmsnorm(acc[c], lat_n, 1e-6) if norm else acc[c]
        if fmt is None:
            u = a
        elif fmt == 0:
            u = ref.matmul_f32(a[None], up_w)[0]
        elif fmt == 4:
            u = ref.matmul_int4_g64(a[None], up_w, up_s, H)[0]
        else:
            u = ref.matmul_int8_row(a[None], up_w, up_s, H)[0]
        want[c] = (want[c] + (u * np.float32(scale)).astype(np.float32)).astype(np.float32)
        if shared:
            want[c] = (want[c] + sh[c]).astype(np.float32)
    np.testing.assert_array_equal(got, want)


def test_int8_row_codec_pinned(port, ref):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((40, 192)) * 0.05).astype(np.float32)
    w[7] = 0.0  # a zero row: scale 0, all codes 0
    qp, sp = port.quantize_int8_row(w)
    qr, sr = ref.quantize_int8_row(w)
    np.testing.assert_array_equal(qp, qr)
    np.testing.assert_array_equal(sp, sr)
    x = rng.standard_normal((3, 192)).astype(np.float32)
    np.testing.assert_array_equal(port.matmul_int8_row(x, qp, sp, 40),
                                  ref.matmul_int8_row(x, qr, sr, 40))
    v = rng.standard_normal(777).astype(np.float32)
    np.testing.assert_array_equal(port.rmsnorm(v, None, 1e-5), ref.rmsnorm(v, None, 1e-5))


def _dev(a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,L,fmt,norm,shared,scale", CASES + [(32, 7168, 2048, 8, True, True, 2.0)])
def test_epilogue_dev(exact, port, T, H, L, fmt, norm, shared, scale):
    moe = exact
    acc, h, lat_n, up_w, up_s, sh = _case(T * 11 + L, T, H, L, fmt, norm, shared, port)
    want = port.moe_epilogue(acc, h, scale, lat_n, 1e-6, 0 if fmt is None else fmt, up_w, up_s,
                             sh)
    hd = _dev(h)
    ws = torch.empty(moe.epilogue_workspace_bytes(T, H, L), dtype=torch.uint8, device="cuda")
    moe.epilogue_dev(_dev(acc), hd, scale, _dev(lat_n), 1e-6, 0 if fmt is None else fmt,
                     _dev(up_w), _dev(up_s), _dev(sh), ws)
    torch.cuda.synchronize()
    # every operation in the reference's order and rounding: bit-identical
    np.testing.assert_array_equal(hd.cpu().numpy(), want)


@pytest.mark.gpu
def test_matmul_int8_row_dev(moe, port):
    rng = np.random.default_rng(9)
    for S, I, O in ((1, 256, 40), (37, 512, 96)):  # 37 rows: two passes of 32
        w = (rng.standard_normal((O, I)) * 0.05).astype(np.float32)
        q, s = port.quantize_int8_row(w)
        x = rng.standard_normal((S, I)).astype(np.float32)
        y = torch.zeros((S, O), device="cuda")
        moe.matmul_dev(8, y, _dev(x), _dev(q), _dev(s))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), port.matmul_int8_row(x, q, s, O))


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [0, 4, 7, 8, 9])
def test_matmul_dev_every_format(moe, port, fmt):
    """mvllm_matmul_dev in every format, bit-identical to the reference's
    matmul: shapes on the cp.async ring (whole 16-byte row pieces) and off it
    (the register-staged tile), 1 to 40 rows of x, ragged W-row tiles."""
    import dsv4_cases as dc
    rng = np.random.default_rng(100 + fmt)
    shapes = [(1, 256, 40), (40, 512, 200), (7, 2048, 129)]
    if fmt in (0, 8, 9):
        shapes.append((5, 300, 33))  # rows not whole 16-byte pieces
    for S, I, O in shapes:
        w = (rng.standard_normal((O, I)) * 0.05).astype(np.float32)
        x = rng.standard_normal((S, I)).astype(np.float32)
        if fmt == 0:
            q, s, want = w, None, port.matmul_f32(x, w)
        elif fmt == 4:
            q, s = port.quantize_int4_g64(w)
            want = port.matmul_int4_g64(x, q, s, O)
        elif fmt == 7:
            q, s = port.pack_mxfp4(w)
            want = port.matmul_mxfp4(x, q, s, O)
        elif fmt == 8:
            q, s = port.quantize_int8_row(w)
            want = port.matmul_int8_row(x, q, s, O)
        else:
            q, s = dc.fp8_tensor(rng, O, I)
            want = port.matmul_fp8_b128(x, q, s, O)
        y = torch.zeros((S, O), device="cuda")
        moe.matmul_dev(fmt, y, _dev(x), _dev(q), _dev(s))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), want, err_msg=f"{S}x{I}->{O}")


TOL_CASES = CASES + [
    (32, 7168, 2048, 8, True, True, 2.0),   # the K3 decode step (bench.py's epilogue leg)
    (37, 7168, 2048, 8, True, False, 2.0),  # two token groups of the fused kernel
    (1, 1024, 512, 8, False, True, 1.0),    # no norm: the row's own range scaling
    (3, 512, 512, None, True, True, 1.5),   # norm + residual, no up-projection
    (6, 256, 2560, 8, True, True, 1.0),     # latent 2560: eight slices per row block
    (4, 512, 3072, 8, True, True, 1.0),     # latent 3072: beyond shared memory, exact path
]


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,L,fmt,norm,shared,scale", TOL_CASES)
def test_epilogue_dev_tolerance(moe, port, T, H, L, fmt, norm, shared, scale):
    from conftest import assert_close
    assert not moe.get_exact()
    acc, h, lat_n, up_w, up_s, sh = _case(T * 13 + L, T, H, L, fmt, norm, shared, port)
    if T == 1:
        acc *= np.float32(3e4)  # large rows: the f16 operands are scaled per row
    want = port.moe_epilogue(acc, h, scale, lat_n, 1e-6, 0 if fmt is None else fmt, up_w, up_s,
                             sh)
    ws = torch.empty(moe.epilogue_workspace_bytes(T, H, L), dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(2):
        hd = _dev(h)
        moe.epilogue_dev(_dev(acc), hd, scale, _dev(lat_n), 1e-6, 0 if fmt is None else fmt,
                         _dev(up_w), _dev(up_s), _dev(sh), ws)
        torch.cuda.synchronize()
        outs.append(hd.cpu().numpy())
    np.testing.assert_array_equal(outs[0], outs[1])
    got = outs[0]
    # Rows scaled by 3e4 (beyond f16 without the kernel's per-row scaling):
    # compared at the scale of N(0, 1) rows, the tolerance being absolute.
    s = np.float32(3e4 if T == 1 else 1.0)
    assert_close((got - h) / s, (want - h) / s, "epilogue update")
    assert_close(got / s, want / s, "epilogue output")
