"""The allocation-free permutation entry, mvllm_moe_permute_dev_noalloc.

Some callers of this library cannot allocate device memory when they permute
tokens: serving engines that split HBM once at start-up and forbid allocation
in the serving loop, and plugins inside a host process whose own allocator
owns the GPU's memory.  For them the entry keeps its scratch in a 1 MiB
file-scope device array instead of a caller workspace.

The test calls it through the C ABI several times in a row -- the array keeps
each call's contents, so every later call starts from a dirty array, the
multi-kernel path (T > 256) included -- and checks every output bit for bit
against the workspace entry mvllm_moe_permute_dev and, at the smaller sizes,
against the CPU oracle's caller-order permutation (bit-exact is the tolerance
the permutation tests use everywhere).  It also checks the size limit at its
edge: the documented example (exactly 1 MiB of scratch) runs, one more token
is refused before any launch.  The file sorts last so a failure here cannot
stop the rest of the suite, and it initialises the library itself so it also
passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _outputs(T, K, E, ns):
    KK, EE = K + ns, E + ns
    i32 = dict(dtype=torch.int32, device="cuda")
    return dict(nr=torch.full((EE,), -5, **i32), xoff=torch.full((EE,), -5, **i32),
                rows=torch.full((T * KK,), -5, **i32),
                rw=torch.full((T * KK,), -5.0, dtype=torch.float32, device="cuda"),
                tok_pos=torch.full((T * KK,), -5, **i32), n_rows=torch.zeros(1, **i32))


def _ptrs(o):
    return [C.c_void_p(o[k].data_ptr()) for k in ("nr", "xoff", "rows", "rw", "tok_pos",
                                                   "n_rows")]


def _compare(a, b):
    n = int(a["n_rows"].item())
    assert n == int(b["n_rows"].item())
    for k in ("nr", "xoff", "tok_pos"):
        assert torch.equal(a[k], b[k]), k
    assert torch.equal(a["rows"][:n], b["rows"][:n])
    assert torch.equal(a["rw"][:n], b["rw"][:n])


def _check_oracle(got, idx, wt, E, ns):
    """The routed rows against the oracle's caller-order gather (glm53.cpp:1958-1971)."""
    from oracle import Oracle, permute
    T = idx.shape[0]
    valid = np.where((idx >= 0) & (idx < E), idx, -1).astype(np.int32)
    uniq = Oracle("port").moe_union_ids(valid)
    nr, xoff, rows, rw = permute(valid, wt, uniq)
    full_nr = np.zeros(E + ns, np.int32)
    full_nr[uniq] = nr
    if ns:
        full_nr[E] = T
    np.testing.assert_array_equal(got["nr"].cpu().numpy(), full_nr)
    R0 = rows.shape[0]
    n = int(got["n_rows"].item())
    assert n == R0 + (T if ns else 0)
    np.testing.assert_array_equal(got["rows"].cpu().numpy()[:R0], rows)
    np.testing.assert_array_equal(got["rw"].cpu().numpy()[:R0], rw)


def test_noalloc_permute_matches_workspace_entry_and_oracle():
    import build as mvbuild
    mvbuild.build()
    import mvllm_moe as moe
    moe.init(0)
    L = moe.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(2024)
    # Calls in a row on the one shared array: the multi-kernel path (T > 256)
    # on the fresh array, the one-CTA path after it, the multi-kernel path
    # again on the array both left dirty (different E and K, so stale bits
    # would land in live words), and the documented size limit, exactly
    # 1 MiB of scratch.
    for T, K, E, ns in [(512, 8, 256, 1), (37, 6, 384, 0), (300, 4, 160, 0),
                        (8192, 8, 384, 0)]:
        idx = rng.integers(-1, E + 1, (T, K)).astype(np.int32)
        idx[:, 2] = idx[:, 0]
        wt = rng.random((T, K)).astype(np.float32)
        wt[rng.random((T, K)) < 0.05] = 0.0
        d_idx = torch.from_numpy(idx).cuda()
        d_wt = torch.from_numpy(wt).cuda()

        want = _outputs(T, K, E, ns)
        ws = torch.empty(moe.permute_workspace_bytes(T, K, E, ns), dtype=torch.uint8,
                         device="cuda")
        rc = L.mvllm_moe_permute_dev(stream, C.c_void_p(d_idx.data_ptr()),
                                     C.c_void_p(d_wt.data_ptr()), T, K, E, ns, *_ptrs(want),
                                     C.c_void_p(ws.data_ptr()), ws.numel())
        assert rc == moe.OK, moe.last_error()

        got = _outputs(T, K, E, ns)
        rc = L.mvllm_moe_permute_dev_noalloc(stream, C.c_void_p(d_idx.data_ptr()),
                                             C.c_void_p(d_wt.data_ptr()), T, K, E, ns,
                                             *_ptrs(got))
        assert rc == moe.OK, moe.last_error()
        torch.cuda.synchronize()
        _compare(got, want)
        if T <= 512:
            _check_oracle(got, idx, wt, E, ns)

    # One token more than the documented example needs more than the static
    # maximum: refused, no launch (the output buffers stay untouched).
    big = _outputs(1, 1, 1, 0)
    b_idx = torch.zeros((8193, 8), dtype=torch.int32, device="cuda")
    b_wt = torch.ones((8193, 8), dtype=torch.float32, device="cuda")
    rc = L.mvllm_moe_permute_dev_noalloc(stream, C.c_void_p(b_idx.data_ptr()),
                                         C.c_void_p(b_wt.data_ptr()), 8193, 8, 384, 0,
                                         *_ptrs(big))
    assert rc == moe.ERR_WORKSPACE
    assert "static maximum" in moe.last_error()
    torch.cuda.synchronize()
    assert int(big["nr"][0].item()) == -5
