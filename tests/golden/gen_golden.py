"""Generates tests/golden/golden.npz + golden.json with the REFERENCE build.

Runs the reference's own moe_block / codecs / routing (oracle/_ref, compiled
from the reference sources by oracle/Makefile) on the seeded cases of
cases.py and stores the outputs, the routing and a SHA-256 digest of every
packed expert set.  Inputs are not stored: tests regenerate them from the
seeds and check the digest first.  Re-run with ``python tests/golden/gen_golden.py``
in a container where the reference tree exists.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, HERE)

import cases  # noqa: E402
from oracle import Oracle, build  # noqa: E402


def main():
    build(reference=True)
    ref = Oracle("reference")
    arrays, meta = {}, {}

    for name, (act, a) in {"kat_silu": (cases.ACT_SILU, 0.0),
                           "kat_clamp10": (cases.ACT_CLAMP, 10.0)}.items():
        c = cases.kat_identity(act, a)
        ok, out = cases.run_block(ref, c)
        arrays[name + "/out"] = out
        meta[name] = {"ok": int(ok)}
    c = cases.kat_mxfp4_diag(ref)
    ok, out = cases.run_block(ref, c)
    arrays["kat_mxfp4_diag/out"] = out
    meta["kat_mxfp4_diag"] = {"ok": int(ok)}
    c = cases.edge_case(ref)
    ok, out = cases.run_block(ref, c)
    arrays["edge/out"] = out
    meta["edge"] = {"ok": int(ok)}

    for name in cases.LAYER_CASES:
        c = cases.make_layer(ref, name)
        ok, out = cases.run_block(ref, c)
        arrays[name + "/out"] = out
        arrays[name + "/idx"] = c["idx"]
        arrays[name + "/wt"] = c["wt"]
        arrays[name + "/rows"] = c["rows"]
        arrays[name + "/rw"] = c["rw"]
        arrays[name + "/nr"] = c["nr"]
        meta[name] = {"ok": int(ok), "digest": c["digest"], "nb": c["nb"]}

    # Routing known answers of tests/test_host.cpp:4916-4931 and :8255-8275.
    sig = np.array([0.1, 0.4, 0.3, 0.2], np.float32)
    choice = np.array([0.1, 0.4, 10.3, 0.2], np.float32)
    i, w = ref.moe_topk(choice, 2, sig)
    arrays["topk/idx"], arrays["topk/w"] = i, w
    arrays["union/out"] = ref.moe_union_ids(np.array([[3, 1], [3, 2], [1, -1]], np.int32), 8)
    i, w = ref.moe_topk_pick(np.array([0.1, 0.8, 0.3, 0.5], np.float32), 2)
    arrays["pick/idx"], arrays["pick/w"] = i, w
    i, w = ref.moe_topk_pick(np.full(4, np.nan, np.float32), 2)
    arrays["pick_nan/idx"], arrays["pick_nan/w"] = i, w

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump({"generator": "tests/golden/gen_golden.py", "source": "reference build "
                   "(oracle/_ref/libmvllm_ref.so from the reference's own sources)",
                   "cases": meta}, f, indent=1, sort_keys=True)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main()
