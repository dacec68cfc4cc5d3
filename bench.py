#!/usr/bin/env python
"""MoE-block tokens/s on B200 -- BASELINE config[4], the expert-parallel layer.

One step = one routed MoE layer over 8192 tokens: 384 MXFP4 experts (e2m1 +
ue8m0 per 32, drawn N(0, 0.02) and packed on the GPU), hidden 7168, expert
intermediate 2048, top-8, SiTU(4,25), bf16 activations N(0, 1), uniform
router draws.  At N GPUs (torchrun, one process per GPU, NCCL) the experts
are strided over the ranks (e on rank e % N, hot experts replicated), each
rank routes its 8192 / N tokens, dispatches them over an NCCL all-to-all,
runs its experts and returns the partial sums (strong scaling); tokens/s
over the slowest rank's step time.  At one GPU the same layer runs whole.
Weights total 9.0 GB, far above L2, so no flush is needed between steps.

Beside the headline: the Zipf run and weak scaling of config[4], the
decode path (config[1], HBM-bound, with its roofline), the prefill path
(config[3], every tensor-core mode with its measured error), config[0] and
config[2], the device expert tier, the layer epilogue, and the DeepSeek-V4
expert split.  `--impl reference` times the reference's own CPU moe_block
(oracle/_ref) on the host cores for config[4]'s metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "micro-vllm_b200"))

CFG = dict(D=7168, I=2048, E=256, K=8, n_shared=1, fmt=7, act=2, act_a=4.0, act_b=25.0)
EXPERT_BYTES = 3 * (CFG["I"] * CFG["D"] // 2 + CFG["I"] * CFG["D"] // 32)  # 23,396,352
METRIC = "MoE-block tokens/sec (config[4] expert-parallel MXFP4 layer, 8192 tokens per step)"
N_INPUTS = 16
PROFILE_HEADLINE = False  # --profile-headline: two headline steps for ncu, nothing timed


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--no-tier", action="store_true",
                    help="skip the device expert tier measurement (host moe_block entry)")
    ap.add_argument("--tier-steps", type=int, default=16)
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the config[3] prefill measurement")
    ap.add_argument("--prefill-steps", type=int, default=10)
    ap.add_argument("--no-ep", action="store_true", help="skip the config[4] expert-parallel leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the config[1] decode leg")
    ap.add_argument("--decode-steps", type=int, default=200)
    ap.add_argument("--no-decode-configs", action="store_true",
                    help="skip the config[0] and config[2] decode legs")
    ap.add_argument("--ep-steps", type=int, default=20)
    ap.add_argument("--ep-mode", default="auto", choices=["auto", "compact", "fixed", "peer"],
                    help="NCCL exchange with segments sized by host counts (compact) or fixed "
                         "(no host synchronisation), or stores over NVLink into the ranks' "
                         "IPC-mapped windows (peer); auto: peer")
    ap.add_argument("--ep-chunks", type=int, default=1,
                    help="token slices per expert-parallel step (N > 1): the exchanges of one "
                         "slice overlap the experts of another")
    ap.add_argument("--no-dsv4", action="store_true",
                    help="skip the DeepSeek-V4 expert-split (EP2) leg")
    ap.add_argument("--dsv4-steps", type=int, default=100)
    ap.add_argument("--dsv4-all-ranks", action="store_true",
                    help="run the DeepSeek-V4 leg on more than two ranks too")
    ap.add_argument("--prefill-tokens", type=int, default=4096,
                    help="config[3]: 4096; fewer only to size a profiler capture")
    ap.add_argument("--profile-decode-batch", type=int, default=0,
                    help="only build the config[1] decode workload at this batch, time it from "
                         "CUDA-graph replays, and run three layer steps between "
                         "cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--profile-headline", action="store_true",
                    help="only build the headline config[4] layer and run two steps between "
                         "cudaProfilerStart/Stop after the warm-up (for ncu)")
    ap.add_argument("--profile-scale", type=int, default=1,
                    help="with --profile-headline: divide config[4]'s experts and tokens by "
                         "this factor (the same rows per expert) to size an ncu capture")
    ap.add_argument("--profile-epilogue-router", action="store_true",
                    help="only run the layer epilogue and the router at the K3 / DeepSeek-V4 "
                         "decode shape, two calls each between cudaProfilerStart/Stop")
    ap.add_argument("--profile-prefill-modes", default="",
                    help="only build the config[3] prefill layer and, per listed tensor-core "
                         "mode (comma-separated names), time five steps and run one between "
                         "cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--mma-rates", action="store_true",
                    help="only print the tensor pipes' measured rates over MMA widths: "
                         "kind::f16 on single CTAs (A and B from shared memory) and "
                         "kind::mxf8f6f4 on single CTAs and CTA pairs")
    ap.add_argument("--experts", type=int, default=256,
                    help="routed experts (BASELINE config[1]: 256); fewer only to size a "
                         "profiler capture")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def bf16_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"])
    return 1590.0


def traffic_ratio():
    """DRAM bytes per algorithmic byte of the expert kernels, from the
    committed ncu summary (profiles/decode_ffn_config1.txt), or None."""
    p = os.path.join(ROOT, "profiles", "decode_ffn_config1.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("dram_bytes_per_algorithmic_byte:"):
                return float(line.split(":", 1)[1])
    return None


def headline_traffic():
    """DRAM bytes per launch of the headline's dominant kernel (phase-1 CTA
    pairs) at full size, from the committed ncu summary
    (profiles/headline_config4_one_gpu.txt), or None."""
    p = os.path.join(ROOT, "profiles", "headline_config4_one_gpu.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("phase1_wide_dram_bytes_per_launch_full_size:"):
                return float(line.split(":", 1)[1])
    return None


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during a region."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index):
        self.samples, self.reasons = [], 0
        self.stop_ev = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML missing: report no clocks
            self.nv = None
            self.max_mhz = None

    def _run(self):
        while not self.stop_ev.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h) & ~0x1
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self.stop_ev.set()
        if self.nv:
            self.t.join()

    def report(self):
        if not self.nv or not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "samples": len(self.samples),
                "reasons": [n for b, n in self.REASONS.items() if self.reasons & b]}


# ---------------------------------------------------------------- workload --
class Workload:
    """Config[1] weights on the device and N_INPUTS routed batches."""

    def __init__(self, moe, torch, B, seed):
        D, I, E, K, ns = CFG["D"], CFG["I"], CFG["E"], CFG["K"], CFG["n_shared"]
        EE = E + ns
        self.B = B
        g = torch.Generator(device="cuda").manual_seed(seed)
        u8 = torch.uint8
        self.gp = torch.empty((EE, I, D // 2), dtype=u8, device="cuda")
        self.up = torch.empty((EE, I, D // 2), dtype=u8, device="cuda")
        self.dp = torch.empty((EE, D, I // 2), dtype=u8, device="cuda")
        self.gs = torch.empty((EE, I, D // 32), dtype=u8, device="cuda")
        self.us = torch.empty((EE, I, D // 32), dtype=u8, device="cuda")
        self.ds = torch.empty((EE, D, I // 32), dtype=u8, device="cuda")
        for e in range(EE):
            for p, s, shape in ((self.gp, self.gs, (I, D)), (self.up, self.us, (I, D)),
                                (self.dp, self.ds, (D, I))):
                w = torch.randn(shape, generator=g, device="cuda").mul_(0.02)
                moe.pack_mxfp4_dev(w, p[e], s[e])
        torch.cuda.synchronize()
        self.host_tables = [[t[e].data_ptr() for e in range(EE)]
                            for t in (self.gp, self.up, self.dp, self.gs, self.us, self.ds)]
        self.tables = [torch.tensor(t, dtype=torch.int64, device="cuda")
                       for t in self.host_tables]
        # The host API's address tables as int64 arrays (passed without a copy).
        self.host_tables = [np.asarray(t, dtype=np.int64) for t in self.host_tables]
        self.inputs = []
        for _ in range(N_INPUTS):
            choice = torch.rand((B, E), generator=g, device="cuda")
            vals, idx = torch.topk(choice, K, dim=1)  # moe_topk with mix = null
            wt = (vals / vals.sum(dim=1, keepdim=True)).float()
            x = torch.randn((B, D), generator=g, device="cuda").to(torch.bfloat16)
            self.inputs.append((idx.int().contiguous(), wt.contiguous(), x))
        self.out = torch.zeros((B, D), dtype=torch.float32, device="cuda")
        self.ws = torch.empty(moe.layer_workspace_bytes(B, K, E, ns, D, I, CFG["fmt"]),
                              dtype=torch.uint8, device="cuda")
        # Experts each step touches (routed union + shared) -> algorithmic bytes.
        self.experts_per_input = [len(set(i.flatten().tolist())) + ns
                                  for (i, _, _) in self.inputs]

    def step(self, moe, i):
        idx, wt, x = self.inputs[i % N_INPUTS]
        self.out.zero_()
        moe.layer_dev(self.B, CFG["K"], CFG["E"], CFG["n_shared"], CFG["D"], CFG["I"], CFG["fmt"],
                      idx, wt, x, self.tables, self.out, CFG["act"], CFG["act_a"], CFG["act_b"],
                      self.ws)


def graph_throughput(moe, torch, wl, steps, warmup):
    """Tokens/s of `steps` steps replayed from a CUDA graph of N_INPUTS steps."""
    for i in range(3):
        wl.step(moe, i)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for i in range(N_INPUTS):
                wl.step(moe, i)
    torch.cuda.synchronize()
    reps = max(1, steps // N_INPUTS)
    for _ in range(max(1, warmup // N_INPUTS)):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    del graph
    return wl.B * reps * N_INPUTS / (ms / 1e3), ms / (reps * N_INPUTS)


# --------------------------------------------------- other decode configs --
def decode_leg(moe, torch, name, D, I, E, K, fmt, act, a, b, batches, router, peak_gbs, seed,
               reps=320):
    """A decode config of BASELINE at each batch size through the device
    layer (mvllm_moe_layer_dev), CUDA-graph replays of 16 routings: tokens/s,
    ms per step and the HBM fraction of the step (the touched experts' weight
    bytes + the activation rows in and out, over the step time).  Weights are
    drawn N(0, 0.02) and packed on the GPU; activations bf16 N(0, 1)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    gs_ = 64 if fmt == 4 else 32
    sdt = torch.float32 if fmt == 4 else torch.uint8
    pack = moe.quantize_int4_g64_dev if fmt == 4 else moe.pack_mxfp4_dev
    per_expert = 3 * (I * D // 2 + I * D // gs_ * (4 if fmt == 4 else 1))
    mats = []
    for e in range(E):
        m = []
        for shape in ((I, D), (I, D), (D, I)):
            w = torch.randn(shape, generator=g, device="cuda").mul_(0.02)
            pk = torch.empty((shape[0], shape[1] // 2), dtype=torch.uint8, device="cuda")
            sc = torch.empty((shape[0], shape[1] // gs_), dtype=sdt, device="cuda")
            pack(w, pk, sc)
            m.append((pk, sc))
        mats.append(m)
    tables = [torch.tensor([mats[e][k % 3][k // 3].data_ptr() for e in range(E)],
                           dtype=torch.int64, device="cuda") for k in range(6)]
    res = {}
    for B in batches:
        inputs, touched = [], []
        for _ in range(N_INPUTS):
            if router == "softmax":  # N(0,1) logits, softmax (temperature 1), top-K renormalised
                choice = torch.softmax(torch.randn((B, E), generator=g, device="cuda"), dim=1)
            else:
                choice = torch.rand((B, E), generator=g, device="cuda")
            vals, idx = torch.topk(choice, K, dim=1)
            wt = (vals / vals.sum(1, keepdim=True)).float().contiguous()
            x = torch.randn((B, D), generator=g, device="cuda").to(torch.bfloat16)
            inputs.append((idx.int().contiguous(), wt, x))
            touched.append(len(set(idx.flatten().tolist())))
        out = torch.zeros((B, D), dtype=torch.float32, device="cuda")
        ws = torch.empty(moe.layer_workspace_bytes(B, K, E, 0, D, I, fmt), dtype=torch.uint8,
                         device="cuda")

        def step(i):
            idx, wt, x = inputs[i % N_INPUTS]
            moe.layer_dev(B, K, E, 0, D, I, fmt, idx, wt, x, tables, out, act, a, b, ws)

        for i in range(3):
            step(i)
        torch.cuda.synchronize()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(graph, stream=st):
                for i in range(N_INPUTS):
                    step(i)
        torch.cuda.synchronize()
        n = max(1, reps // N_INPUTS)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (n * N_INPUTS)
        del graph
        nbytes = sum(touched) / len(touched) * per_expert + B * D * (2 + 4)
        res[f"B{B}"] = {"tokens_per_s": B / (ms / 1e3), "ms_per_step": ms,
                        "us_per_step": ms * 1e3, "experts_touched_mean": sum(touched) / len(touched),
                        "algorithmic_bytes_per_step": nbytes,
                        "hbm_gbs": nbytes / (ms / 1e3) / 1e9,
                        "hbm_frac_of_step": nbytes / (ms / 1e3) / 1e9 / peak_gbs}
    del mats, tables
    torch.cuda.empty_cache()
    return {"workload": name, "expert_bytes": per_expert,
            "timing": "CUDA-graph replays of 16 routings through mvllm_moe_layer_dev; HBM "
                      "fraction over the whole step (permutation, gather, plan, maps, both "
                      "expert phases, combine)", **res}


# ------------------------------------------------------------ prefill --
PREFILL_T = 4096


def zipf_routing(torch, T, E, K, g, s=1.1, perm=None):
    """BASELINE config[3] routing: logits = -s ln(rank) + Gumbel noise per token
    over a seeded random ranking of the experts, softmax, top-K renormalised.
    `perm` (optional) fixes the ranking, so that draws with different token
    noise share the same popular experts."""
    if perm is None:
        perm = torch.randperm(E, generator=g, device="cuda")
    rank = torch.empty(E, device="cuda")
    rank[perm] = torch.arange(1, E + 1, device="cuda", dtype=torch.float32)
    u = torch.rand((T, E), generator=g, device="cuda").clamp_min(1e-20)
    logits = -s * torch.log(rank)[None, :] - torch.log(-torch.log(u))
    vals, idx = torch.topk(torch.softmax(logits, dim=1), K, dim=1)
    return idx.int().contiguous(), (vals / vals.sum(1, keepdim=True)).float().contiguous()


def host_routing(idx, wt, E, with_shared):
    """The caller's side of moe_block for one batch (glm53.cpp:1958-1971 /
    kimi_k3.cpp:2036-2050 order): experts ascending, tokens ascending inside
    each, wsum = sum of the token's weights for that expert; the shared expert
    (id E) last with weight 1.  Returns ids, nr, xoff, rows, rw."""
    B, K = idx.shape
    ids = sorted({int(e) for e in idx.flatten() if 0 <= e < E})
    nr, rows, rw = [], [], []
    for e in ids:
        n = 0
        for c in range(B):
            m = idx[c] == e
            if m.any():
                rows.append(c)
                rw.append(float(np.float32(wt[c][m].sum(dtype=np.float32))))
                n += 1
        nr.append(n)
    if with_shared:
        ids.append(E)
        nr.append(B)
        rows.extend(range(B))
        rw.extend([1.0] * B)
    nr = np.array(nr, np.int32)
    xoff = np.concatenate([[0], np.cumsum(nr)[:-1]]).astype(np.int32)
    return ids, nr, xoff, np.array(rows, np.int32), np.array(rw, np.float32)


def pinned_h2d_gbs(torch):
    """Pinned host -> device copy bandwidth (1 GiB, best of 3, CUDA events)."""
    n = 1 << 30
    h = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(n, dtype=torch.uint8, device="cuda")
    best = 0.0
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        d.copy_(h, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        best = max(best, n / (a.elapsed_time(b) / 1e3) / 1e9)
    del h, d
    return best


def tier_bench(moe, torch, wl, steps):
    """Device expert tier: config[1] decode (batch wl.B) through the
    reference-facing mvllm_moe_block, each expert's six arrays in one pinned
    host blob (an ExpertStore slot) bound to the tier.  VRAM budgets: every
    expert fits; half of them fit (least recently used blobs give their slots
    up, cold ones stream over PCIe while the resident ones compute); and no
    tier (every call uploads its experts).  The routing/permutation is the
    caller's work and is prepared outside the timed region."""
    D, I, E, ns = CFG["D"], CFG["I"], CFG["E"], CFG["n_shared"]
    EE = E + ns
    parts = (wl.gp, wl.up, wl.dp, wl.gs, wl.us, wl.ds)
    sizes = [t[0].numel() for t in parts]
    offs, n = [], 0
    for z in sizes:
        offs.append(n)
        n += (z + 255) // 256 * 256
    blob = n
    host = torch.empty((EE, blob), dtype=torch.uint8, pin_memory=True)
    for e in range(EE):
        for t, o, z in zip(parts, offs, sizes):
            host[e, o:o + z].copy_(t[e].flatten())
    torch.cuda.synchronize()
    hn = host.numpy()
    views = [[hn[e, o:o + z] for o, z in zip(offs, sizes)] for e in range(EE)]
    batches = []
    for (idx, wt, x) in wl.inputs:
        ih, wh, xh = idx.cpu().numpy(), wt.cpu().numpy(), x.float().cpu().numpy()
        ids, nr, xoff, rows, rw = host_routing(ih, wh, E, ns > 0)
        # the caller's six pointer arrays for the batch, built once
        ptrs = [np.array([views[e][k].ctypes.data for e in ids], np.int64) for k in range(6)]
        batches.append((ids, nr, xoff, rows, rw, np.ascontiguousarray(xh[rows]), ptrs))
    out = np.zeros((wl.B, D), np.float32)
    # activation rows and the output in page-locked memory, as the engine's I/O buffers
    for b in batches:
        moe.host_register(b[5])
    moe.host_register(out)

    def call(b):
        # out += moe_block(...): the call's contract; the timed loop adds into
        # the same rows (no host memset inside it)
        ids, nr, xoff, rows, rw, xg, ptrs = b
        moe.moe_block(len(ids), D, I, CFG["fmt"], *ptrs, xg, xoff, nr, rows, rw, out, wl.B,
                      CFG["act"], CFG["act_a"], CFG["act_b"])

    res = {"blob_bytes": blob, "experts": EE, "batch": wl.B,
           "pinned_h2d_gbs": pinned_h2d_gbs(torch)}
    for name, nslots, n_steps in (("all_resident", EE, steps), ("half_resident", EE // 2, steps),
                                  ("no_tier", 0, max(2, steps // 4))):
        moe.tier_configure(nslots * blob, blob)
        if nslots:
            for e in range(EE):
                moe.expert_bind(hn[e], 1)
        for i in range(len(batches)):  # warm: fills the slots
            call(batches[i])
        s0 = moe.tier_stats()
        c0 = moe.stats()
        t0 = time.perf_counter()
        for i in range(n_steps):
            call(batches[i % len(batches)])
        dt = time.perf_counter() - t0
        s1 = moe.tier_stats()
        c1 = moe.stats()
        dev_split = {k: (c1[k] - c0[k]) / n_steps for k in ("h2d_ms", "kernel_ms", "d2h_ms")}
        bin_ = (s1["bytes_in"] - s0["bytes_in"]) / n_steps
        bov = (s1["overflow_bytes"] - s0["overflow_bytes"]) / n_steps
        if not nslots:  # no tier: every touched expert's blob is uploaded per call
            bov = sum(len(batches[i % len(batches)][0]) for i in range(n_steps)) * blob / n_steps
        acq = (s1["hits"] - s0["hits"]) + (s1["misses"] - s0["misses"]) + \
              (s1["overflow"] - s0["overflow"])
        h2d = (bin_ + bov) * n_steps / dt / 1e9
        res[name] = {"slots": nslots, "steps": n_steps, "ms_per_step": dt / n_steps * 1e3,
                     "tokens_per_s": wl.B * n_steps / dt,
                     "hit_rate": (s1["hits"] - s0["hits"]) / acq if acq else None,
                     "streamed_bytes_per_step": bin_, "uploaded_bytes_per_step": bov,
                     "h2d_gbs": h2d, "h2d_frac_of_pinned_peak": h2d / res["pinned_h2d_gbs"],
                     "device_split_ms_per_call": dev_split,
                     "host_only_ms_per_call": dt / n_steps * 1e3 - sum(dev_split.values())}
        if nslots:
            for e in range(EE):
                moe.expert_unbind(hn[e])
        moe.tier_configure(0, 0)
    for b in batches:
        moe.host_unregister(b[5])
    moe.host_unregister(out)
    del host
    return res


def graph_us_per_call(torch, step, ncalls, reps):
    """Device microseconds per call of `step(i)`, i = 0..ncalls-1 captured once
    in a CUDA graph and replayed `reps` times (no host launch cost inside)."""
    for i in range(ncalls):
        step(i)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for i in range(ncalls):
                step(i)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / (reps * ncalls)
    del graph
    return us


def epilogue_bench(moe, torch, peak_gbs, reps=200):
    """Layer epilogue after the routed combine, Kimi-K3 form at config[1]'s
    decode batch: rmsnorm over a 2048-wide latent, int8-row up-projection to
    7168 (QuantMat fmt 8), routed scale, shared-expert add, residual update.
    Bound by the up-projection's weight bytes (14.7 MB per call).  Calls cycle
    over 10 copies of the weights (147 MB, more than L2), in the tolerance
    mode (one fused kernel, the default) and the exact mode (the reference's
    order: serial rmsnorm, sequential dot products, residual)."""
    T, H, L = 32, CFG["D"], 2048
    g = torch.Generator(device="cuda").manual_seed(31)
    acc = torch.randn((T, L), generator=g, device="cuda")
    h = torch.randn((T, H), generator=g, device="cuda")
    sh = torch.randn((T, H), generator=g, device="cuda")
    lat_n = torch.ones(L, device="cuda")
    ncopy = 10
    qs = [torch.randint(-127, 128, (H, L), generator=g, device="cuda", dtype=torch.int32).to(
        torch.int8) for _ in range(ncopy)]
    sc = torch.full((H,), 0.01, device="cuda")
    ws = torch.empty(moe.epilogue_workspace_bytes(T, H, L), dtype=torch.uint8, device="cuda")
    nbytes = H * L + H * 4 + T * L * 4 + T * H * 4 * 3  # weights, scales, acc, h in/out, shared
    res = {"workload": f"K3 epilogue: {T} tokens, latent {L} -> hidden {H}, int8-row "
                       "up-projection, rmsnorm, routed scale, shared add",
           "algorithmic_bytes": nbytes, "l2": f"{ncopy} weight copies cycled (> L2)"}
    for mode, exact, n in (("tolerance", False, reps), ("exact", True, max(20, reps // 10))):
        moe.set_exact(exact)

        def step(i):
            moe.epilogue_dev(acc, h, 2.0, lat_n, 1e-6, 8, qs[i % ncopy], sc, sh, ws)

        us = graph_us_per_call(torch, step, ncopy, max(1, n // ncopy))
        res[mode] = {"us_per_call": us, "achieved_gbs": nbytes / (us / 1e6) / 1e9,
                     "frac_of_hbm": nbytes / (us / 1e6) / 1e9 / peak_gbs if peak_gbs else None,
                     "launches_per_call": 1 if not exact else 3, "calls": n,
                     "timing": "CUDA-graph replays of one call per weight copy"}
    moe.set_exact(None)
    res["us_per_call"] = res["tolerance"]["us_per_call"]
    res["frac_of_hbm"] = res["tolerance"]["frac_of_hbm"]
    return res


def router_bench(moe, torch, peak_gbs, reps=200):
    """Router scores + top-k at the DeepSeek-V4 / K3 decode shape: 32 tokens,
    hidden 7168, 256 experts f32 router (7.3 MB), sqrt(softplus) + bias, top 6
    times routed_scale.  Calls cycle over 20 router copies (147 MB, more than
    L2); tolerance mode (cluster kernel) and exact mode (the reference's
    sequential order)."""
    T, H, E, K = 32, CFG["D"], 256, 6
    g = torch.Generator(device="cuda").manual_seed(37)
    x = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
    ncopy = 20
    rs = [torch.randn((E, H), generator=g, device="cuda") * (1.0 / H ** 0.5)
          for _ in range(ncopy)]
    bias = torch.randn(E, generator=g, device="cuda") * 0.01
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wt = torch.empty((T, K), device="cuda")
    scores = torch.empty((T, E), device="cuda")
    choice = torch.empty((T, E), device="cuda")
    nbytes = E * H * 4 + T * H * 2 + T * E * 8 + T * K * 8
    res = {"workload": f"router: {T} tokens, hidden {H}, {E} experts f32, sqrt(softplus) + bias, "
                       f"top-{K}", "algorithmic_bytes": nbytes,
           "l2": f"{ncopy} router copies cycled (> L2)"}
    for mode, exact, n in (("tolerance", False, reps), ("exact", True, max(20, reps // 10))):
        moe.set_exact(exact)

        def step(i):
            moe.route_ex_dev(x, rs[i % ncopy], bias, K, idx, wt, scores, choice,
                             moe.SCORE_SQRT_SOFTPLUS, 2.5)

        us = graph_us_per_call(torch, step, ncopy, max(1, n // ncopy))
        res[mode] = {"us_per_call": us, "achieved_gbs": nbytes / (us / 1e6) / 1e9,
                     "frac_of_hbm": nbytes / (us / 1e6) / 1e9 / peak_gbs if peak_gbs else None,
                     "launches_per_call": 2, "calls": n,
                     "timing": "CUDA-graph replays of one call per router copy"}
    moe.set_exact(None)
    return res


PREFILL_MODES = ("f16", "mxf4x1", "mxf4x2", "mxf4x3", "mxf8x1", "mxf8x2")
# The tensor pipe each mode issues on (kind for mvllm_moe_mma_rate) and its
# token terms; f16 dequantises the weights and runs kind::f16.
MODE_PIPE = {"f16": ("f16", 2, 1), "mxf4x1": ("mxf4", 0, 1), "mxf4x2": ("mxf4", 0, 2),
             "mxf4x3": ("mxf4", 0, 3), "mxf8x1": ("mxf8f6f4", 1, 1),
             "mxf8x2": ("mxf8f6f4", 1, 2)}


def mxfp4_dequant(torch, p, s):
    """MXFP4 rows (packed e2m1 [O, I/2], ue8m0 [O, I/32]) as f64 values, the
    reference's decoding (quant.hpp:12-20: code 0 -> +0, 255 -> +inf)."""
    lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6],
                       dtype=torch.float64, device=p.device)
    O = p.shape[0]
    v = torch.stack([lut[(p & 15).long()], lut[(p >> 4).long()]], -1).reshape(O, -1)
    sc = torch.where(s == 0, torch.zeros((), dtype=torch.float64, device=p.device),
                     torch.exp2(s.double() - 127))
    return v * sc.repeat_interleave(32, dim=1)


def prefill_reference(torch, wl, idx, wt, x, sample):
    """The layer's output rows for `sample` tokens in f64 (torch on the GPU,
    weights decoded as the reference decodes them): the yardstick of each
    tensor-core mode's measured error."""
    D, I, a, b = CFG["D"], CFG["I"], CFG["act_a"], CFG["act_b"]
    xs = x[sample].double()
    ids, ws = idx[sample].long(), wt[sample].double()
    out = torch.zeros((len(sample), D), dtype=torch.float64, device="cuda")
    for e in sorted(set(ids.flatten().tolist())):
        m = (ids == e)
        rows = m.any(1).nonzero().flatten()
        w_e = (ws * m).sum(1)[rows]
        g = xs[rows] @ mxfp4_dequant(torch, wl.gp[e], wl.gs[e]).T
        u = xs[rows] @ mxfp4_dequant(torch, wl.up[e], wl.us[e]).T
        h = a * torch.tanh(g / a) * torch.sigmoid(g) * b * torch.tanh(u / b)
        y = h @ mxfp4_dequant(torch, wl.dp[e], wl.ds[e]).T
        out[rows] += w_e[:, None] * y
    return out


def prefill_bench(moe, torch, wl, steps, peak_tf, peak_gbs, T=PREFILL_T):
    """Config[3]: 4096 tokens, the 256 routed MXFP4 experts of the decode
    workload (same shape and format), Zipf s=1.1 routing, no shared expert,
    bf16 activations, f32 accumulation.  Large experts run on the tensor-core
    kernels, the smallest on the decode kernels.  Every tensor-core mode is
    timed and its error measured against an f64 evaluation of the same
    layer on every token; the headline is the library's default mode
    (the fastest within the 1e-2 / 2e-2 tolerance).  Tensor fractions are
    against the tensor pipe's rate measured in this run (mvllm_moe_mma_rate,
    back-to-back MMAs of the same kind on every SM)."""
    D, I, E, K = CFG["D"], CFG["I"], CFG["E"], CFG["K"]
    g = torch.Generator(device="cuda").manual_seed(4242)
    idx, wt = zipf_routing(torch, T, E, K, g)
    x = torch.randn((T, D), generator=g, device="cuda").to(torch.bfloat16)
    out = torch.zeros((T, D), dtype=torch.float32, device="cuda")
    ws = torch.empty(moe.layer_workspace_bytes(T, K, E, 0, D, I, CFG["fmt"]), dtype=torch.uint8,
                     device="cuda")
    cnt = torch.bincount(idx.flatten().long(), minlength=E).cpu()
    sample = torch.arange(T, device="cuda")
    ref = prefill_reference(torch, wl, idx, wt, x, sample)
    pipes = {"mxf4": moe.mma_rate(0, 256, 1), "mxf8f6f4": moe.mma_rate(1, 256, 1),
             "f16": moe.mma_rate(2, 128, 0)}

    def step():
        out.zero_()
        moe.layer_dev(T, K, E, 0, D, I, CFG["fmt"], idx, wt, x, wl.tables, out, CFG["act"],
                      CFG["act_a"], CFG["act_b"], ws)

    flops = 2.0 * T * K * 3 * D * I
    touched = int((cnt > 0).sum())
    alg_bytes = touched * EXPERT_BYTES + T * D * 2 + T * D * 4
    default = moe.PREFILL_NAMES[moe.get_prefill_mode()]
    modes = {}
    for mode in PREFILL_MODES:
        moe.set_prefill_mode(mode)
        for _ in range(2):
            step()
        torch.cuda.synchronize()
        got = out[sample].double()
        rel = float(torch.linalg.norm(got - ref) / torch.linalg.norm(ref))
        mabs = float((got - ref).abs().max())
        moe.profile_enable(True)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
        ph = moe.profile_read()
        moe.profile_enable(False)
        ms = a.elapsed_time(b) / steps
        e_ms = (ph["expert_phase1"][0] + ph["expert_phase2"][0]) / steps
        pipe, _, nterm = MODE_PIPE[mode]
        tf = flops / (e_ms / 1e3) / 1e12
        modes[mode] = {
            "tokens_per_s": T / (ms / 1e3), "ms_per_step": ms,
            "expert_kernels_ms_per_step": e_ms,
            "rel_l2": rel, "max_abs": mabs, "within_tolerance": rel <= 1e-2 and mabs <= 2e-2,
            "achieved_tflops": tf, "pipe": pipe, "token_terms": nterm,
            "pipe_tflops_issued": tf * nterm, "pipe_peak_tflops": pipes[pipe],
            "pipe_frac": tf * nterm / pipes[pipe],
            "hbm_frac": alg_bytes / (ms / 1e3) / 1e9 / peak_gbs,
            "phases_ms_per_step": {k: v[0] / steps for k, v in ph.items()},
        }
    moe.set_prefill_mode(None)
    best = max((m for m in modes if modes[m]["within_tolerance"]),
               key=lambda m: modes[m]["tokens_per_s"], default=None)
    d = modes[default]
    return {
        "workload": f"config[3] MXFP4 prefill: {T} tokens, hidden 7168, inter 2048, {E} experts "
                    "top-8 (Zipf s=1.1 routing), SiTU(4,25), bf16 activations",
        "mode": default, "fastest_mode_within_tolerance": best,
        "tokens_per_s": d["tokens_per_s"], "ms_per_step": d["ms_per_step"], "steps": steps,
        "rel_l2": d["rel_l2"], "max_abs": d["max_abs"],
        "error_sample": f"all {T} tokens, against an f64 evaluation of the layer with the "
                        "weights decoded as the reference decodes them",
        "expert_rows_per_expert": {"min": int(cnt.min()), "max": int(cnt.max()),
                                   "below_128": int((cnt < 128).sum())},
        "tensor": {"flops_per_step": flops, "achieved_tflops": d["achieved_tflops"],
                   "pipe": d["pipe"], "pipe_peak_tflops": d["pipe_peak_tflops"],
                   "pipe_frac": d["pipe_frac"],
                   "peak_kind": "measured in this run: back-to-back MMAs of the pipe's kind on "
                                "every SM (mvllm_moe_mma_rate)",
                   "kernel_ms_per_step": d["expert_kernels_ms_per_step"],
                   "bf16_cublas_peak_tflops": peak_tf},
        "hbm": {"algorithmic_bytes_per_step": alg_bytes,
                "achieved_gbs": alg_bytes / (d["ms_per_step"] / 1e3) / 1e9, "peak_gbs": peak_gbs,
                "frac": alg_bytes / (d["ms_per_step"] / 1e3) / 1e9 / peak_gbs},
        "pipe_peaks_tflops": pipes,
        "modes": modes,
    }


# ----------------------------------------------------- expert parallelism --
EP_E, EP_T = 384, 8192


def ep_routing(torch, name, T, K, seed):
    """Config[4] routing draws; every Zipf draw ranks the experts the same way
    (the model's popular experts), the token noise comes from `seed`."""
    gr = torch.Generator(device="cuda").manual_seed(seed)
    if name == "uniform":
        choice = torch.rand((T, EP_E), generator=gr, device="cuda")
        vals, idx = torch.topk(choice, K, dim=1)
        wt = (vals / vals.sum(1, keepdim=True)).float()
        return idx.int(), wt
    perm = torch.randperm(EP_E, generator=torch.Generator(device="cuda").manual_seed(779),
                          device="cuda")
    return zipf_routing(torch, T, EP_E, K, gr, perm=perm)


def ep_bench(moe, torch, dist, rank, world, steps, warmup=3, weak=False, clk=None, e2e_steps=0,
             chunks=1, ep_mode="compact"):
    """Config[4]: 384 MXFP4 experts sharded over the ranks (expert e on rank
    e % world), top-8; uniform and Zipf s=1.1 routing.  Weights are drawn per
    global expert id, so the model is the same whatever the rank count.
    Strong scaling (default): 8192 tokens per step split evenly over the
    ranks.  Weak scaling (`weak`): 8192 tokens per rank per step (each rank
    brings its own batch, as data-parallel attention feeds an expert-parallel
    layer).  tokens/s = all ranks' tokens / step time (max over ranks).
    Hot experts are replicated on every rank (ep.balance_replicas, at most
    2 per rank) from the loads of a separate calibration draw of the same
    routing distribution; each rank serves its own tokens' rows for them.
    The uniform run's timed region is sampled by `clk`; its expert kernels'
    device time (phase events, max over ranks) gives the roofline; with
    `e2e_steps` the same step also runs from host buffers (pinned x, idx, wt
    copied in, out copied back inside the timed region).  With `chunks` > 1
    (N > 1) each step runs as that many token slices whose exchanges overlap
    the expert kernels (EPLayer.forward_chunked); with `ep_mode` "fixed" the
    exchanges use fixed-size segments and no counts reach the host
    (EPLayer.forward_fixed); with "peer" the dispatch and return are stores
    over NVLink into the ranks' IPC-mapped windows inside the dispatch kernel
    and the experts' combine kernel (EPLayer.forward_peer)."""
    import ep
    D, I, K = CFG["D"], CFG["I"], CFG["K"]
    u8 = torch.uint8
    T_loc = EP_T if weak else EP_T // world
    T_all = T_loc * world
    wcache = {}

    def expert(e):  # the same weights for a global id on every rank and rank count
        if e not in wcache:
            g = torch.Generator(device="cuda").manual_seed(100000 + e)
            mats = []
            for shape in ((I, D), (I, D), (D, I)):
                w = torch.randn(shape, generator=g, device="cuda").mul_(0.02)
                pk = torch.empty((shape[0], shape[1] // 2), dtype=u8, device="cuda")
                sc = torch.empty((shape[0], shape[1] // 32), dtype=u8, device="cuda")
                moe.pack_mxfp4_dev(w, pk, sc)
                mats.append((pk, sc))
            wcache[e] = mats
        return wcache[e]

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    g = torch.Generator(device="cuda").manual_seed(777)
    x_all = torch.randn((T_all, D), generator=g, device="cuda").to(torch.bfloat16)
    x = x_all[rank * T_loc:(rank + 1) * T_loc].contiguous()
    del x_all
    out = torch.zeros((T_loc, D), dtype=torch.float32, device="cuda")
    res = {}
    for name in ("uniform", "zipf"):
        # Placement from a calibration draw of the same distribution.
        cal, _ = ep_routing(torch, name, T_all, K, 990 if name == "uniform" else 991)
        load = torch.bincount(cal.flatten().long(), minlength=EP_E).tolist()
        del cal
        rep = ep.balance_replicas(load, world, max_replicas=2 * world) if world > 1 else []
        pl = ep.Placement(EP_E, world, rep)
        mine = pl.local_experts(rank)
        for e in list(wcache):
            if e not in mine:
                del wcache[e]
        mats = [expert(e) for e in mine]
        # (g, u, d, gs, us, ds) address tables in local-id order
        tabs = [torch.tensor([m[j % 3][j // 3].data_ptr() for m in mats], dtype=torch.int64,
                             device="cuda") for j in range(6)]
        ops = ep.CudaOps(torch, EP_E, K, D, I, CFG["fmt"], CFG["act"], CFG["act_a"],
                         CFG["act_b"], tabs, world, T_all, placement=pl, rank=rank)
        layer = ep.EPLayer(ops, rank, world, D, K)
        idx, wt = ep_routing(torch, name, T_all, K, 778 if name == "uniform" else 779)
        idx = idx[rank * T_loc:(rank + 1) * T_loc].contiguous()
        wt = wt[rank * T_loc:(rank + 1) * T_loc].contiguous()

        win = (ep.PeerWindows(torch, world, T_loc, K, D).connect(rank, dist)
               if world > 1 and ep_mode == "peer" else None)

        def step(xx=x, ii=idx, ww=wt, oo=out):
            # out += layer(x): the layer's contract (the residual stream); the
            # rows stay the same buffer from step to step
            if win is not None:
                return layer.forward_peer(xx, ii, ww, oo, dist, win)
            if world > 1 and ep_mode == "fixed":
                return layer.forward_fixed(xx, ii, ww, oo, dist)
            if world > 1 and chunks > 1:
                return layer.forward_chunked(xx, ii, ww, oo, dist, chunks=chunks)
            if world > 1:
                return layer.forward(xx, ii, ww, oo, dist)
            layer.forward_local(xx, ii, ww, oo)  # one rank: the single-GPU layer
            return None

        for _ in range(max(warmup, 2)):
            step()
        barrier()
        if PROFILE_HEADLINE:  # two steps for an ncu launch list, nothing timed
            torch.cuda.profiler.start()
            for _ in range(2):
                step()
            barrier()
            torch.cuda.profiler.stop()
            return {"profiled": name}
        moe.profile_enable(True)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler = clk if (clk is not None and name == "uniform") else None
        if sampler:
            sampler.__enter__()
        a.record()
        info = None
        for _ in range(steps):
            info = step()
        b.record()
        barrier()
        if sampler:
            sampler.__exit__(None, None, None)
        ph = moe.profile_read()
        moe.profile_enable(False)
        ms, e_ms = max_over_ranks([a.elapsed_time(b) / steps,
                                   (ph["expert_phase1"][0] + ph["expert_phase2"][0]) / steps])
        res[name] = {"tokens_per_s": T_all / (ms / 1e3), "ms_per_step": ms, "steps": steps,
                     "expert_kernels_ms_per_step_max_over_ranks": e_ms,
                     "replicated_experts": len(rep), "experts_per_rank": len(mine)}
        if world > 1:
            # One more step with phase events (not part of the timed steps).
            tm = {}
            out.zero_()
            if win is not None:
                layer.forward_peer(x, idx, wt, out, dist, win, timing=tm)
            else:
                layer.forward(x, idx, wt, out, dist, timing=tm)
            keys = sorted(tm)
            res[name]["phase_ms_max_over_ranks"] = dict(zip(keys, max_over_ranks(
                [tm[k] for k in keys])))
        if info:
            res[name]["rank0_sent_rows"] = info["sent_rows"]
            res[name]["rank0_received_rows"] = info["received_rows"]
        if e2e_steps and name == "uniform":
            # The same step from host buffers: x / idx / wt in pinned host
            # memory copied in, out copied back, inside the timed region.
            xh = x.cpu().pin_memory()
            ih = idx.cpu().pin_memory()
            wh = wt.cpu().pin_memory()
            oh = torch.empty((T_loc, D), dtype=torch.float32).pin_memory()
            xd, idd, wd = torch.empty_like(x), torch.empty_like(idx), torch.empty_like(wt)

            def e2e_step():
                xd.copy_(xh, non_blocking=True)
                idd.copy_(ih, non_blocking=True)
                wd.copy_(wh, non_blocking=True)
                step(xd, idd, wd, out)
                oh.copy_(out, non_blocking=True)

            for _ in range(2):
                e2e_step()
            barrier()
            a2, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            a2.record()
            for _ in range(e2e_steps):
                e2e_step()
            b2.record()
            barrier()
            wall = time.perf_counter() - t0
            ems, wall = max_over_ranks([a2.elapsed_time(b2) / e2e_steps, wall / e2e_steps])
            serial = {"value": T_all / (ems / 1e3), "ms_per_step": ems,
                      "host_wall_ms_per_step": wall * 1e3}

            # Pipelined: the same copies, each step's inputs and outputs in one
            # of two device buffer sets, H2D on one copy stream and D2H on
            # another, so step i's output read and step i+1's input copy run
            # while step i+1 / i computes (PCIe is full duplex).
            cs = torch.cuda.current_stream()
            s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
            bufs = [(torch.empty_like(x), torch.empty_like(idx), torch.empty_like(wt),
                     torch.zeros_like(out)) for _ in range(2)]
            ohs = [oh, torch.empty_like(oh).pin_memory()]
            ev = {k: [torch.cuda.Event() for _ in range(2)]
                  for k in ("in_ready", "in_free", "out_ready", "out_free")}
            for j in range(2):
                ev["in_free"][j].record(cs)
                ev["out_free"][j].record(cs)

            def e2e_pipe_step(i):
                j = i % 2
                xb, ib, wb, ob = bufs[j]
                with torch.cuda.stream(s_in):
                    s_in.wait_event(ev["in_free"][j])
                    xb.copy_(xh, non_blocking=True)
                    ib.copy_(ih, non_blocking=True)
                    wb.copy_(wh, non_blocking=True)
                    ev["in_ready"][j].record(s_in)
                cs.wait_event(ev["in_ready"][j])
                cs.wait_event(ev["out_free"][j])
                step(xb, ib, wb, ob)
                ev["in_free"][j].record(cs)
                ev["out_ready"][j].record(cs)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev["out_ready"][j])
                    ohs[j].copy_(ob, non_blocking=True)
                    ev["out_free"][j].record(s_out)

            for i in range(2):
                e2e_pipe_step(i)
            torch.cuda.synchronize()
            barrier()
            a3, b3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            a3.record()
            for i in range(e2e_steps):
                e2e_pipe_step(i)
            cs.wait_stream(s_out)  # the last step's output is on the host
            b3.record()
            barrier()
            wall3 = time.perf_counter() - t0
            pms, wall3 = max_over_ranks([a3.elapsed_time(b3) / e2e_steps, wall3 / e2e_steps])
            res["e2e"] = {"value": T_all / (pms / 1e3), "unit": "tokens/s",
                          "ms_per_step": pms, "host_wall_ms_per_step": wall3 * 1e3,
                          "h2d_bytes_per_step": T_all * (D * 2 + K * 8),
                          "d2h_bytes_per_step": T_all * D * 4,
                          "api": "EPLayer.forward over the library's device entries (one rank: "
                                 "the single-GPU layer), host buffers pinned",
                          "copies": "every step copies its x / idx / wt in and its out back; "
                                    "two device buffer sets, H2D and D2H on their own streams "
                                    "overlapping the neighbouring steps' compute",
                          "serial": serial}
        if win is not None:
            win.close(dist)
        del layer, ops, tabs, mats
    wcache.clear()
    torch.cuda.empty_cache()
    per = "8192 tokens per rank per step" if weak else "8192 tokens per step"
    return {"workload": "config[4] expert-parallel MXFP4 layer: 384 experts strided over the "
                        f"ranks (hot experts replicated), hidden 7168, inter 2048, top-8, {per}, "
                        "bf16 activations; "
                        + ("one rank: the single-GPU layer, no exchange" if world == 1 else
                           "dispatch and return as stores over NVLink into IPC-mapped windows"
                           if ep_mode == "peer" else "dispatch and return over NCCL all-to-all"),
            "n_gpus": world, "scaling": "weak" if weak else "strong", "tokens_per_step": T_all,
            "slices_per_step": chunks if world > 1 else 1,
            "exchange": ep_mode if world > 1 else "none (one rank)",
            **res}


# ------------------------------------------------------------ CPU baseline --
def dsv4_bench(moe, torch, dist, rank, world, wl, steps, T=32):
    """DeepSeek-V4 MoE step (the reference's moe_layer_ep2 with
    route_moe_ep2, dsv4.cpp:2863-3010) at decode: T tokens, hidden 7168, 256
    MXFP4 experts of intermediate 2048 (the config[1] bank), top-6 by
    sqrt(softplus) + bias, clamped SwiGLU (limit 7), an int4-g64 dense shared
    MLP in the tail (QuantMat 4-bit, the reference's default dense_bits; run
    through the MoE kernels as one expert) and routed_scale 2.5.  The
    reference names no DeepSeek-V4
    shape; these are stand-in sizes of that class.  The experts are split
    over the ranks (e on rank e % world; two ranks is the reference's EP2)
    and the partial outputs all-reduced over NCCL; every rank processes the
    same T tokens, so tokens/s = T / step time (max over ranks)."""
    import dsv4
    D, I, E = CFG["D"], CFG["I"], CFG["E"]
    g = torch.Generator(device="cuda").manual_seed(4242)  # the same on every rank
    x = torch.randn((T, D), generator=g, device="cuda")
    h0 = torch.randn((T, D), generator=g, device="cuda")
    router = torch.randn((E, D), generator=g, device="cuda").mul_(2.0 / D ** 0.5)
    bias = torch.randn((E,), generator=g, device="cuda").mul_(0.1)
    dense = [moe.FMT_INT4_G64]
    for shape in ((I, D), (I, D), (D, I)):
        w = torch.randn(shape, generator=g, device="cuda").mul_(0.02)
        pk = torch.empty((shape[0], shape[1] // 2), dtype=torch.uint8, device="cuda")
        sc = torch.empty((shape[0], shape[1] // 64), dtype=torch.float32, device="cuda")
        moe.quantize_int4_g64_dev(w, pk, sc)
        dense.append((pk, sc))
    del w
    mine = list(range(rank, E, world))
    tables = [t[mine].contiguous() for t in wl.tables]
    ops = dsv4.CudaOps(torch, E, D, I, 7.0, router, bias, tables, rank, world, T,
                       routed_scale=2.5, dense_shared=tuple(dense))
    layer = dsv4.EP2Layer(ops, rank, world)
    h = h0.clone()

    def step():
        layer.forward(x, h, dist)

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("dsv4_step")  # lets a profiler select these launches
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    idx, _ = ops.route(x)
    experts_touched = len(set(idx.flatten().tolist()))
    local_touched = len([e for e in set(idx.flatten().tolist()) if e % world == rank])
    ebytes = 3 * (I * D // 2 + I * D // 32)
    res = {"workload": f"DeepSeek-V4-class MoE step: {T} tokens, hidden {D}, {E} MXFP4 experts "
                       f"(inter {I}) top-6 sqrt(softplus)+bias, clamped SwiGLU, int4-g64 dense "
                       "shared MLP, routed_scale 2.5",
           "ranks": world, "placement": "strided e % ranks (2 ranks = the reference's EP2 "
                                        "parity split)",
           "tokens_per_s": T / (ms / 1e3), "ms_per_step": ms,
           "experts_touched": experts_touched, "rank0_experts_touched": local_touched,
           "rank0_expert_bytes_per_step": local_touched * ebytes,
           "allreduce_bytes_per_step": T * D * 4 if world > 1 else 0,
           "steps": steps, "warmup": 5}
    if rank == 0 and world == 1:
        res["cpu_reference"] = dsv4_cpu_reference(torch, wl, x, router, bias, idx)
    return res


def dsv4_cpu_reference(torch, wl, x, router, bias, idx, tokens=2):
    """The reference's DeepSeek-V4 CPU tier (dsv4_cuda::route_moe_ep2 in
    oracle/_ref, one thread) on the first tokens of the step: the bank holds
    only the experts those tokens route to (host copies), the rest absent."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from oracle import Oracle
        ref = Oracle("reference")
        E = CFG["E"]
        used = sorted({int(e) for e in idx[:tokens].flatten().tolist()})
        bank = [None] * E
        for e in used:
            bank[e] = [(wl.gp[e].cpu().numpy(), wl.gs[e].cpu().numpy()),
                       (wl.up[e].cpu().numpy(), wl.us[e].cpu().numpy()),
                       (wl.dp[e].cpu().numpy(), wl.ds[e].cpu().numpy())]
        xs, rs, bs = x.cpu().numpy(), router.cpu().numpy(), bias.cpu().numpy()
        t0 = time.perf_counter()
        for t in range(tokens):
            ref.dsv4_route_moe_ep2(xs[t], rs, bs, 1.0, CFG["I"], bank, None, 7.0)
        sec = time.perf_counter() - t0
        return {"tokens_per_s": tokens / sec, "cores": 1, "kind": "reference",
                "sample": f"{tokens} tokens through route_moe_ep2 (both parity ranks in one "
                          f"host process, as the reference runs them), {sec:.1f} s"}
    except Exception as ex:  # the reference build may be absent
        return {"tokens_per_s": None, "sample": f"unavailable: {ex}"}


def cpu_reference_rate(n_threads, rounds, expert_rows_per_call, host_experts=None,
                       rows_per_token=9.0):
    """Reference moe_block (oracle/_ref) on host threads.

    Each thread calls the reference moe_block on one token row through
    `expert_rows_per_call` MXFP4 experts (7168 / 2048); returns (tokens/s,
    seconds, tokens) with `rows_per_token` expert rows per token (config[1]:
    9, 8 routed + shared; config[4]: 8)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle
    ref = Oracle("reference")
    D, I = CFG["D"], CFG["I"]
    if host_experts is None:
        rng = np.random.default_rng(7)
        host_experts = []
        for _ in range(min(expert_rows_per_call, 9)):
            mats = [ref.pack_mxfp4((rng.standard_normal(s) * 0.02).astype(np.float32))
                    for s in ((I, D), (I, D), (D, I))]
            host_experts.append(mats)
    ne = expert_rows_per_call
    mats = [host_experts[e % len(host_experts)] for e in range(ne)]
    g = [m[0][0] for m in mats]
    u = [m[1][0] for m in mats]
    d = [m[2][0] for m in mats]
    gs = [m[0][1] for m in mats]
    us = [m[1][1] for m in mats]
    ds = [m[2][1] for m in mats]
    xs = [np.random.default_rng(t).standard_normal((1, D)).astype(np.float32)
          for t in range(n_threads)]

    def work(t):
        out = np.zeros((1, D), np.float32)
        ref.moe_block(ne, D, I, 7, g, u, d, gs, us, ds, xs[t], np.zeros(ne, np.int32),
                      np.ones(ne, np.int32), np.zeros(ne, np.int32), np.full(ne, 1.0 / 9,
                                                                               np.float32),
                      out, 1, 2, 4.0, 25.0)

    def one_round():
        ths = [threading.Thread(target=work, args=(t,)) for t in range(n_threads)]
        for th in ths:
            th.start()
        for th in ths:
            th.join()

    t0 = time.perf_counter()
    for _ in range(rounds):
        one_round()
    sec = time.perf_counter() - t0
    tokens = rounds * n_threads * ne / rows_per_token
    return tokens / sec, sec, tokens


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    """The reference's own CPU moe_block (oracle/_ref) on all host threads, on
    config[4]'s expert rows (8 MXFP4 experts of 7168 / 2048 per token, SiTU):
    each step a bounded sample of the workload, `threads` parallel calls of
    one token row through a few experts, sized so the run ends in about 90 s.
    Under torchrun rank 0 alone runs and prints."""
    rank, _, world = dist_env()
    if rank != 0:
        return
    threads = host_threads()
    per_step_budget = 90.0 / max(args.steps + args.warmup, 1)
    rows = max(1, int(per_step_budget / 0.05))
    cpu_reference_rate(threads, max(args.warmup, 0) and 1, rows, rows_per_token=8.0)  # warm-up
    rate, sec, tokens = cpu_reference_rate(threads, args.steps, rows, rows_per_token=8.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3 / max(args.steps, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config[4] expert-parallel MXFP4 MoE layer: 384 experts, hidden "
                               "7168, inter 2048, top-8, 8192 tokens per step, SiTU(4,25)",
                   "global_batch": EP_T, "parallelism": "host threads"},
        "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": threads,
                         "kind": "reference",
                         "sample": f"per step {threads} threads x 1 token row through {rows} "
                                   f"expert(s) of config[4] (8 expert rows = 1 token)"},
        "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------------- ours --
def auto_ep_mode(world):
    """The exchange form `--ep-mode auto` picks: stores over NVLink into the
    ranks' IPC-mapped windows (EPLayer.forward_peer), the fastest measured at
    2, 4 and 8 GPUs."""
    return "peer"


def launches_per_ep_step(world, mode):
    """This library's kernels in one config[4] step (NCCL's and torch's own
    kernels not counted): EP plan and pack (N > 1), the routed layer over the
    received rows (permutation: 4 kernels at these sizes; gather; expert plan;
    2 tensor-map builds; each phase on the decode kernel, the tensor-core
    kernels (f16: pairs, wide and small single CTAs; block-scaled: pairs and
    single CTAs, plus one term-quantisation kernel) and the redo launch;
    combine), and the EP combine (N > 1).  19 per step at one GPU, as the
    committed launch list (profiles/headline_config4_one_gpu.txt) shows."""
    per_phase = 5  # decode, 3 (f16) or 2 + terms (block-scaled) tensor-core launches, redo
    layer = 4 + 1 + 1 + 2 + 2 * per_phase + 1
    return layer + (3 if world > 1 else 0)


def profile_only(moe, torch, args):
    """A small, fixed workload for an ncu launch list or capture: the decode
    layer at one batch size, or the layer epilogue and the router."""
    if args.profile_decode_batch:
        wl = Workload(moe, torch, args.profile_decode_batch, seed=7)
        for i in range(20):
            wl.step(moe, i)
        torch.cuda.synchronize()
        _, ms = graph_throughput(moe, torch, wl, 320, 32)
        print(json.dumps({"profile": "decode", "batch": wl.B, "graph_ms_per_step": ms}),
              flush=True)
        torch.cuda.profiler.start()
        for i in range(3):
            wl.step(moe, i)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        return
    T, H, L, E, K = 32, CFG["D"], 2048, 256, 6
    g = torch.Generator(device="cuda").manual_seed(3)
    acc = torch.randn((T, L), generator=g, device="cuda")
    h = torch.randn((T, H), generator=g, device="cuda")
    sh = torch.randn((T, H), generator=g, device="cuda")
    lat_n = torch.ones(L, device="cuda")
    q = torch.randint(-127, 128, (H, L), generator=g, device="cuda", dtype=torch.int32).to(
        torch.int8)
    sc = torch.full((H,), 0.01, device="cuda")
    ws = torch.empty(moe.epilogue_workspace_bytes(T, H, L), dtype=torch.uint8, device="cuda")
    x = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
    r = torch.randn((E, H), generator=g, device="cuda") * (1.0 / H ** 0.5)
    bias = torch.randn(E, generator=g, device="cuda") * 0.01
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wt = torch.empty((T, K), device="cuda")
    scores, choice = torch.empty((T, E), device="cuda"), torch.empty((T, E), device="cuda")

    def epi():
        moe.epilogue_dev(acc, h, 2.0, lat_n, 1e-6, 8, q, sc, sh, ws)

    def rte():
        moe.route_ex_dev(x, r, bias, K, idx, wt, scores, choice, moe.SCORE_SQRT_SOFTPLUS, 2.5)

    for _ in range(10):
        epi()
        rte()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(2):
        epi()
        rte()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"profile": "epilogue+router", "tokens": T}), flush=True)


def profile_prefill_modes(moe, torch, modes):
    """Config[3] (the prefill leg's workload: 4096 tokens, Zipf routing) in
    each listed tensor-core mode: five timed steps, then one step between
    cudaProfilerStart/Stop, so an ncu launch list holds one step per mode in
    the order given."""
    D, I, E, K = CFG["D"], CFG["I"], CFG["E"], CFG["K"]
    wl = Workload(moe, torch, 32, seed=1234)
    g = torch.Generator(device="cuda").manual_seed(4242)
    idx, wt = zipf_routing(torch, PREFILL_T, E, K, g)
    x = torch.randn((PREFILL_T, D), generator=g, device="cuda").to(torch.bfloat16)
    out = torch.zeros((PREFILL_T, D), dtype=torch.float32, device="cuda")
    ws = torch.empty(moe.layer_workspace_bytes(PREFILL_T, K, E, 0, D, I, CFG["fmt"]),
                     dtype=torch.uint8, device="cuda")

    def step():
        moe.layer_dev(PREFILL_T, K, E, 0, D, I, CFG["fmt"], idx, wt, x, wl.tables, out,
                      CFG["act"], CFG["act_a"], CFG["act_b"], ws)

    res = {}
    for mode in modes:
        moe.set_prefill_mode(mode)
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(5):
            step()
        b.record()
        torch.cuda.synchronize()
        res[mode] = a.elapsed_time(b) / 5
        torch.cuda.profiler.start()
        step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    moe.set_prefill_mode(None)
    print(json.dumps({"profile": "prefill modes", "tokens": PREFILL_T, "ms_per_step": res}),
          flush=True)


def mma_rates(moe):
    """The tensor pipes' measured rates (TFLOP/s, back-to-back MMAs on every
    SM) over the MMA's N: kind::f16 on single CTAs (M = 128), kind::mxf8f6f4
    on single CTAs and CTA pairs."""
    res = {"f16_solo": {n: moe.mma_rate(2, n, 0) for n in (64, 128, 176, 192, 256)},
           "mxf8f6f4_solo": {n: moe.mma_rate(1, n, 0) for n in (128, 176, 192, 256)},
           "mxf8f6f4_pair": {n: moe.mma_rate(1, n, 1) for n in (128, 176, 192, 256)}}
    print(json.dumps({"profile": "mma rates", "tflops": res}), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    import build as mvbuild
    mvbuild.build()
    import mvllm_moe as moe

    CFG["E"] = args.experts
    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    moe.init(local_rank)
    peak, peak_kind = peaks()
    mode = moe.PREFILL_NAMES[moe.get_prefill_mode()]
    if args.profile_decode_batch or args.profile_epilogue_router:
        profile_only(moe, torch, args)
        return
    if args.profile_prefill_modes:
        profile_prefill_modes(moe, torch, args.profile_prefill_modes.split(","))
        return
    if args.mma_rates:
        mma_rates(moe)
        return
    if args.profile_headline:
        global PROFILE_HEADLINE, EP_E, EP_T
        PROFILE_HEADLINE = True
        EP_E, EP_T = EP_E // args.profile_scale, EP_T // args.profile_scale
        print(json.dumps(ep_bench(moe, torch, dist, rank, world, 2, args.warmup,
                                  ep_mode=auto_ep_mode(world))), flush=True)
        return

    # ---- headline: config[4], the expert-parallel layer at N GPUs (strong
    # scaling: 8192 tokens per step over all ranks), uniform routing; the Zipf
    # run and, at N > 1, weak scaling beside it.
    clk = ClockSampler(local_rank)
    if args.ep_mode == "auto":
        args.ep_mode = auto_ep_mode(world)
    ep_res = ep_bench(moe, torch, dist, rank, world, args.steps, args.warmup, clk=clk,
                      e2e_steps=args.e2e_steps, chunks=args.ep_chunks, ep_mode=args.ep_mode)
    uni = ep_res["uniform"]
    value, ms = uni["tokens_per_s"], uni["ms_per_step"]
    flops = 2.0 * EP_T * CFG["K"] * 3 * CFG["D"] * CFG["I"]  # per step, all ranks
    e_ms = uni["expert_kernels_ms_per_step_max_over_ranks"]
    if mode == "f16":
        tpeak, tpeak_kind = bf16_peak(), "measured (MEASURED_PEAKS.json bf16 dense, burst; the " \
                                         "expert kernels run kind::f16 MMAs at the same rate)"
    else:
        pk, _, _ = MODE_PIPE[mode]
        tpeak = moe.mma_rate(*((0, 256, 1) if pk == "mxf4" else (1, 256, 1)))
        tpeak_kind = f"measured in this run: back-to-back {pk} MMAs on every SM"
    achieved = flops / world / (e_ms / 1e3) / 1e12
    if world > 1:
        ep_res["weak_scaling"] = ep_bench(moe, torch, dist, rank, world, args.ep_steps,
                                          args.warmup, weak=True, chunks=args.ep_chunks,
                                          ep_mode=args.ep_mode)

    # ---- config[1] decode (N = 1): the HBM-bound path -------------------------
    decode = None
    if world == 1 and not args.no_decode:
        decode = decode_config1(moe, torch, args, peak)

    # config[2] (GLM-style int4-g64 decode) and config[0] (the reference's
    # CPU-runnable case) at N = 1
    glm = cfg0 = None
    if world == 1 and not args.no_decode_configs:
        glm = decode_leg(moe, torch, "config[2] int4-g64 decode: hidden 6144, inter 1536, 160 "
                         "experts top-8, clamped SwiGLU (7), softmax router, bf16 activations",
                         6144, 1536, 160, 8, 4, 1, 7.0, 0.0, (1, 16, 64), "softmax", peak, 2202)
        cfg0 = decode_leg(moe, torch, "config[0] int4-g64: hidden 1024, inter 512, 16 experts "
                          "top-4, 4 tokens, clamped SwiGLU (7), softmax router",
                          1024, 512, 16, 4, 4, 1, 7.0, 0.0, (4,), "softmax", peak, 2200)

    # DeepSeek-V4 MoE step, experts split over the ranks: one GPU, or the
    # reference's two-rank EP2 (more ranks with --dsv4-all-ranks)
    dsv4_res = None
    wl = decode["_workload"] if decode else None
    if not args.no_dsv4 and (world <= 2 or args.dsv4_all_ranks):
        if wl is None:
            wl = Workload(moe, torch, args.batch, seed=1234 + rank)
        dsv4_res = dsv4_bench(moe, torch, dist, rank, world, wl, args.dsv4_steps)

    # config[3] prefill, the device expert tier and the layer epilogue (N = 1)
    prefill = tier = epilogue = router = None
    if world == 1:
        if wl is None:
            wl = Workload(moe, torch, args.batch, seed=1234)
        if not args.no_tier:
            tier = tier_bench(moe, torch, wl, args.tier_steps)
        epilogue = epilogue_bench(moe, torch, peak)
        router = router_bench(moe, torch, peak)
        if not args.no_prefill:
            prefill = prefill_bench(moe, torch, wl, args.prefill_steps, bf16_peak(), peak,
                                    args.prefill_tokens)

    # CPU baseline (rank 0, N = 1): the reference moe_block on host threads,
    # config[4] expert rows (8 per token, no shared expert)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            nth = min(host_threads(), 16)
            rate, sec, toks = cpu_reference_rate(nth, 2, 8, rows_per_token=8.0)
            cpu = {"value": rate, "unit": "tokens/s", "cores": nth, "kind": "reference",
                   "sample": f"{toks:.0f} config[4] tokens: {nth} threads x 2 rounds of the "
                             f"reference moe_block on one token row through 8 MXFP4 experts "
                             f"(7168 / 2048), {sec:.1f} s wall"}
            # The reference moe_block is single-threaded: its one-core rate
            # is the primary CPU figure, the threaded one above a secondary.
            r1, s1, t1 = cpu_reference_rate(1, 2, 8, rows_per_token=8.0)
            cpu["single_core"] = {
                "value": r1, "unit": "tokens/s", "cores": 1,
                "sample": f"{t1:.0f} config[4] tokens, one after another on one thread, "
                          f"{s1:.1f} s wall"}
        except Exception as ex:  # the reference build may be absent
            cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                   "sample": f"unavailable: {ex}"}

    if decode:
        decode.pop("_workload", None)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": f"mxfp4 weights, {mode} tensor-core mode, f32 accumulate",
            "data": "synthetic",
            "config": {"workload": "config[4] expert-parallel MXFP4 MoE layer: 384 experts "
                                   "strided over the ranks (hot experts replicated), hidden "
                                   "7168, inter 2048, top-8, 8192 tokens per step (strong "
                                   "scaling), uniform routing, SiTU(4,25), bf16 activations",
                       "global_batch": EP_T, "parallelism": f"expert parallel x{world}",
                       "l2": "inputs larger than L2 (9.0 GB of expert weights over the ranks)"},
            "roofline": {"bound": "tensor", "kernel": "expert FFN (phase 1 + phase 2, tensor-core "
                                                     "and decode kernels), max over ranks",
                         "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s",
                         "frac": achieved / tpeak, "peak_kind": tpeak_kind,
                         "traffic": headline_traffic() if world == 1 and mode == "f16" else None,
                         "traffic_source": "DRAM read + write per launch of the dominant kernel "
                                           "(tc_ffn phase 1, wide single CTAs) at full size, "
                                           "from the "
                                           "committed ncu summary "
                                           "profiles/headline_config4_one_gpu.txt (a 48-expert "
                                           "capture with the same rows per expert, x 8); not "
                                           "measured in this run",
                         "algorithmic_flops_per_step_per_gpu": flops / world,
                         "kernel_ms_per_step": e_ms,
                         "limiter": "the dominant kernel (wide single-CTA tiles, N = 176 "
                                    "tokens per MMA) is bound by shared-memory bandwidth: per "
                                    "MMA its token slice is written by TMA and read by the MMA "
                                    "(5.6 KB each) with 1 KB of packed weights read by the "
                                    "dequant warps, about 96 cycles at 128 B/clk against 88 "
                                    "of tensor time; single-CTA f16 MMAs run at the full "
                                    "rate from N = 128 (bench.py --mma-rates)"},
            "gpu_launches": launches_per_ep_step(world, mode) * args.steps,
            "e2e": ep_res.get("e2e"),
            "cpu_baseline": cpu,
            "clocks": clk.report(),
            "expert_parallel": ep_res,
            "decode_config1": decode,
            "prefill": prefill,
            "config2_glm_int4_decode": glm,
            "config0_small_int4": cfg0,
            "expert_tier": tier,
            "epilogue": epilogue,
            "router": router,
            "dsv4_expert_split": dsv4_res,
        }
        if prefill and cpu and cpu.get("value"):
            prefill["cpu_reference_ms_per_step_extrapolated"] = (
                args.prefill_tokens / cpu["value"] * 1e3)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def decode_config1(moe, torch, args, peak):
    """Config[1] MXFP4 decode at the decode batch (32 tokens + the shared
    expert, 257 experts, 6 GB of weights): eager steps through
    mvllm_moe_layer_dev with the expert kernels' HBM roofline, the same
    batch end to end through mvllm_moe_layer_host, and batches 1 / 8 / 32
    from CUDA-graph replays."""
    import numpy as np
    B = args.batch
    wl = Workload(moe, torch, B, seed=1234)
    for i in range(max(args.warmup, 3)):
        wl.step(moe, i)
    torch.cuda.synchronize()
    steps = args.decode_steps
    moe.profile_enable(True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        wl.step(moe, i)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    phases = moe.profile_read()
    moe.profile_enable(False)
    e_steps = [wl.experts_per_input[i % N_INPUTS] for i in range(steps)]
    alg_bytes = sum(e_steps) * EXPERT_BYTES / steps
    k_ms = (phases["expert_phase1"][0] + phases["expert_phase2"][0]) / steps
    achieved = alg_bytes / (k_ms / 1e3) / 1e9
    ratio = traffic_ratio()
    # end to end through the host-pointer layer entry
    idx_h, wt_h, x_h = [], [], []
    for (idx, wt, x) in wl.inputs:
        idx_h.append(idx.cpu().numpy())
        wt_h.append(wt.cpu().numpy())
        x_h.append(x.float().cpu().numpy())
    out_h = np.zeros((B, CFG["D"]), np.float32)
    for arr in x_h + [out_h]:
        moe.host_register(arr)
    args_l = (B, CFG["K"], CFG["E"], CFG["n_shared"], CFG["D"], CFG["I"], CFG["fmt"])
    for i in range(3):
        moe.layer_host(*args_l, idx_h[i], wt_h[i], x_h[i], wl.host_tables, out_h, CFG["act"],
                       CFG["act_a"], CFG["act_b"])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        moe.layer_host(*args_l, idx_h[i % N_INPUTS], wt_h[i % N_INPUTS], x_h[i % N_INPUTS],
                       wl.host_tables, out_h, CFG["act"], CFG["act_a"], CFG["act_b"])
    e2e_s = time.perf_counter() - t0
    for arr in x_h + [out_h]:
        moe.host_unregister(arr)
    sweep = {}
    if not args.no_sweep:
        for bb in (1, 8, 32):
            wb = Workload.__new__(Workload)
            wb.__dict__.update({k: v for k, v in wl.__dict__.items()
                                if k not in ("inputs", "out", "ws", "B")})
            wb.B = bb
            g = torch.Generator(device="cuda").manual_seed(99 + bb)
            wb.inputs = []
            for _ in range(N_INPUTS):
                choice = torch.rand((bb, CFG["E"]), generator=g, device="cuda")
                vals, idx = torch.topk(choice, CFG["K"], dim=1)
                wt = (vals / vals.sum(dim=1, keepdim=True)).float()
                x = torch.randn((bb, CFG["D"]), generator=g, device="cuda").to(torch.bfloat16)
                wb.inputs.append((idx.int().contiguous(), wt.contiguous(), x))
            wb.out = torch.zeros((bb, CFG["D"]), dtype=torch.float32, device="cuda")
            wb.ws = torch.empty(moe.layer_workspace_bytes(bb, CFG["K"], CFG["E"], CFG["n_shared"],
                                                          CFG["D"], CFG["I"], CFG["fmt"]),
                                dtype=torch.uint8, device="cuda")
            tps, mstep = graph_throughput(moe, torch, wb, 320, 32)
            touched = [len(set(i.flatten().tolist())) + CFG["n_shared"] for (i, _, _) in wb.inputs]
            nb = sum(touched) / len(touched) * EXPERT_BYTES + bb * CFG["D"] * 6
            sweep[f"B{bb}"] = {"tokens_per_s": tps, "ms_per_step": mstep,
                               "algorithmic_bytes_per_step": nb,
                               "hbm_gbs": nb / (mstep / 1e3) / 1e9,
                               "hbm_frac_of_step": nb / (mstep / 1e3) / 1e9 / peak}
    EE = CFG["E"] + CFG["n_shared"]
    return {
        "workload": "config[1] MXFP4 decode MoE block: hidden 7168, inter 2048, 256 experts "
                    "top-8 + 1 shared, SiTU(4,25), bf16 activations",
        "batch": B, "tokens_per_s": B / (ms / 1e3), "ms_per_step": ms, "steps": steps,
        "roofline": {"bound": "hbm", "kernel": "decode_ffn (expert phase 1 + phase 2)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None if ratio is None else ratio * alg_bytes,
                     "traffic_source": "DRAM/algorithmic ratio of the committed ncu summary "
                                       "profiles/decode_ffn_config1.txt (64-expert capture, "
                                       "scaled), not measured in this run",
                     "algorithmic_bytes_per_step": alg_bytes, "kernel_ms_per_step": k_ms},
        "phases_ms_per_step": {k: v[0] / steps for k, v in phases.items()},
        "e2e": {"value": B * args.e2e_steps / e2e_s, "unit": "tokens/s",
                "h2d_bytes_per_step": 6 * EE * 8 + 2 * B * CFG["K"] * 4 + 2 * B * CFG["D"] * 4,
                "d2h_bytes_per_step": B * CFG["D"] * 4, "api": "mvllm_moe_layer_host",
                "host_buffers": "caller x / out page-locked with mvllm_moe_host_register"},
        "sweep": sweep, "_workload": wl,
    }


if __name__ == "__main__":
    main()
