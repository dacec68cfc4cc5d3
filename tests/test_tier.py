"""Device expert tier.

* CPU: the residency policy (csrc/expert_tier.hpp) through a small C++ driver
  (tests/test_tier_policy.cpp): hits, LRU eviction that spares the blobs the
  call uses, overflow, generations, overlapping bindings.
* GPU: mvllm_moe_block with bound blobs and a budget smaller than the call's
  experts -- cold blobs stream in while resident ones compute; the output is
  bit-identical to the same call without the tier, and the counters follow the
  policy.
"""
import os
import subprocess

import numpy as np
import pytest

import cases

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_tier_policy_cpu():
    out = os.path.join(ROOT, "tests", "_build")
    os.makedirs(out, exist_ok=True)
    exe = os.path.join(out, "test_tier_policy")
    src = os.path.join(ROOT, "tests", "test_tier_policy.cpp")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", src, "-o", exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "TIER-POLICY-OK" in r.stdout


def _blobs(c):
    """One host blob per expert holding its six arrays (64-byte aligned
    offsets), as an ExpertStore slot does; returns the blobs and the six
    per-expert pointer views into them."""
    blobs, views = [], []
    for (gp, gsc), (up, usc), (dp, dsc) in c["experts"]:
        arrs = [gp, up, dp, gsc, usc, dsc]
        offs, n = [], 0
        for a in arrs:
            offs.append(n)
            n += (a.nbytes + 63) // 64 * 64
        blob = np.zeros(n + 64, np.uint8)
        base = (-blob.ctypes.data) % 64
        blob = blob[base:base + n]
        for a, o in zip(arrs, offs):
            blob[o:o + a.nbytes] = np.frombuffer(np.ascontiguousarray(a).tobytes(), np.uint8)
        blobs.append(blob)
        views.append([blob[o:o + a.nbytes].view(a.dtype).reshape(a.shape)
                      for a, o in zip(arrs, offs)])
    return blobs, views


@pytest.mark.gpu
def test_tier_moe_block_gpu(moe, port):
    from oracle import permute
    D, I = 512, 256
    c = cases.layer_case(port, 61, D, I, 6, 2, 24, cases.FMT_MXFP4, cases.ACT_SITU, 4.0, 25.0)
    blobs, views = _blobs(c)
    slot = max(b.nbytes for b in blobs)
    uniq = sorted({int(e) for e in c["idx"].flatten() if e >= 0})
    assert len(uniq) >= 4
    T = c["x"].shape[0]

    def call(sel):
        """moe_block over experts `sel` (ascending) with the case's routing."""
        idx = c["idx"].copy()
        idx[~np.isin(idx, sel)] = -1
        nr, xoff, rows, rw = permute(idx, c["wt"], np.array(sel, np.int32))
        xg = np.ascontiguousarray(c["x"][rows]) if rows.size else np.zeros((1, D), np.float32)
        out = np.zeros((T, D), np.float32)
        v = [views[e] for e in sel]
        moe.moe_block(len(sel), D, I, cases.FMT_MXFP4, [a[0] for a in v], [a[1] for a in v],
                      [a[2] for a in v], [a[3] for a in v], [a[4] for a in v], [a[5] for a in v],
                      xg, xoff, nr, rows, rw, out, T, cases.ACT_SITU, 4.0, 25.0)
        return out

    sets = [uniq[:3], uniq[:2], uniq, [uniq[2]], uniq[:1]]
    want = [call(s_) for s_ in sets]  # tier off: per-call uploads
    moe.tier_configure(2 * slot, slot)  # two slots
    try:
        for b in blobs:
            moe.expert_bind(b, 1)
        st = [moe.tier_stats()]
        for s_, w_ in zip(sets, want):
            assert np.array_equal(call(s_), w_), s_
            st.append(moe.tier_stats())
            if s_ is sets[3]:
                # a refilled RAM slot (new generation) must be copied again
                moe.expert_bind(blobs[uniq[0]], 2)
        d = [{k: b[k] - a[k] for k in a} for a, b in zip(st[:-1], st[1:])]
        # 3 cold blobs, 2 slots: two stream in, the third is uploaded for the call
        assert (d[0]["misses"], d[0]["overflow"], d[0]["hits"]) == (2, 1, 0)
        # both resident now: two hits, no copy
        assert (d[1]["hits"], d[1]["misses"]) == (2, 0)
        # every expert: two hits, the rest find only slots this call holds
        assert (d[2]["hits"], d[2]["misses"], d[2]["overflow"]) == (2, 0, len(uniq) - 2)
        # expert uniq[2] alone: copied in, evicting the least recently used
        assert (d[3]["misses"], d[3]["evictions"]) == (1, 1)
        # uniq[0] again after its RAM slot was refilled: copied again
        assert d[4]["misses"] == 1
        assert st[-1]["resident_bytes"] <= 2 * slot
    finally:
        for b in blobs:
            moe.expert_unbind(b)
        moe.tier_configure(0, 0)
