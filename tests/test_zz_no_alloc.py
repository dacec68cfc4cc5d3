"""The allocation-free permutation entry, mvllm_moe_permute_dev_noalloc.

It serves callers that cannot allocate device memory when they permute
tokens: code running inside a CUDA graph capture, engines whose HBM budget is
fixed at start-up, plugins whose host process owns the GPU allocator.  Its
scratch is a 1 MiB file-scope device array instead of a caller workspace.
The test calls it through the C ABI twice in a row (the array keeps the first
call's contents, so the second call shows the scratch is cleared) and checks
every output against the workspace entry mvllm_moe_permute_dev, with the
tolerance the permutation tests use everywhere: bit-exact.  It also checks
that a size beyond the static maximum is refused.  The file sorts last so a
failure here cannot stop the rest of the suite, and it initialises the
library itself so it also passes alone in a fresh process.
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


def test_noalloc_permute_matches_workspace_entry():
    import build as mvbuild
    mvbuild.build()
    import mvllm_moe as moe
    moe.init(0)
    L = moe.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(2024)
    # Two calls in a row; the second one routes fewer tokens to more experts,
    # so stale bits from the first call would show up if the scratch were not
    # cleared.
    for T, K, E, ns in [(512, 8, 256, 1), (37, 6, 384, 0)]:
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

    # A size whose scratch exceeds the static maximum is refused, no launch.
    big = _outputs(1, 1, 1, 0)
    rc = L.mvllm_moe_permute_dev_noalloc(stream, C.c_void_p(d_idx.data_ptr()),
                                         C.c_void_p(d_wt.data_ptr()), 1 << 16, 8, 4096, 0,
                                         *_ptrs(big))
    assert rc == moe.ERR_WORKSPACE
    assert "static maximum" in moe.last_error()
