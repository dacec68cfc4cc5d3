"""Failure path of the device pipelines, without a GPU fault.

Every mbarrier wait in the library's kernels is bounded: when a copy or a peer
never completes, the wait gives up after its time limit, records
MVLLM_ERR_TIMEOUT in the launch's error word and the kernel returns.  The
health-check entry runs that path on purpose (an mbarrier nothing arrives at)
and the test checks the status and that the context is still usable after it.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_bounded_wait_gives_up_and_context_survives(moe, port):
    completed, timed_out = moe.wait_selftest()
    assert completed, "a wait whose barrier completes must succeed"
    assert timed_out, "a wait nothing completes must give up with MVLLM_ERR_TIMEOUT"
    # the same context keeps working: a bit-exact matmul right after
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((64, 256)) * 0.05).astype(np.float32)
    q, s = port.quantize_int8_row(w)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    y = torch.zeros((3, 64), device="cuda")
    moe.matmul_dev(8, y, torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(),
                   torch.from_numpy(s).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), port.matmul_int8_row(x, q, s, 64))
