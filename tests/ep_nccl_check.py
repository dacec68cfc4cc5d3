"""Two-rank expert-parallel check over NCCL (launched by tests/test_ep_gpu.py
through torchrun, one rank per GPU): each rank holds half of the experts
(strided), runs its tokens through ep.EPLayer.forward and through the other
exchange forms, which must give the same bits: the chunked, overlapped
forward_chunked, forward_fixed (fixed segments), and forward_peer (rows
stored over NVLink into the ranks' IPC-mapped windows, twice through the same
windows).  Rank 0 compares the gathered output with the single-GPU layer over
all tokens and experts.
Prints EP-NCCL-OK on success."""
import os
import sys
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in ("micro-vllm_b200", "oracle", "tests", os.path.join("tests", "golden")):
    sys.path.insert(0, os.path.join(ROOT, p))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import cases  # noqa: E402
import ep  # noqa: E402
import mvllm_moe as moe  # noqa: E402
from oracle import Oracle  # noqa: E402

D, I, E, K, T_LOC = 512, 512, 8, 2, 48
FMT, ACT, A, B = cases.FMT_MXFP4, cases.ACT_SITU, 4.0, 25.0


def tables_of(experts):
    keep, tabs = [], [[], [], [], [], [], []]
    for (gp, gsc), (up, usc), (dp, dsc) in experts:
        for k, a in enumerate((gp, up, dp, gsc, usc, dsc)):
            t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
            keep.append(t)
            tabs[k].append(t.data_ptr())
    return [torch.tensor(t, dtype=torch.int64, device="cuda") for t in tabs], keep


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    moe.init(local)
    port = Oracle("port")
    c = cases.layer_case(port, 77, D, I, E, K, world * T_LOC, FMT, ACT, A, B, bf16_x=True)
    tabs, keep = tables_of([c["experts"][e] for e in ep.local_experts(rank, world, E)])
    ops = ep.CudaOps(torch, E, K, D, I, FMT, ACT, A, B, tabs, world, world * T_LOC)
    layer = ep.EPLayer(ops, rank, world, D, K)
    sl = slice(rank * T_LOC, (rank + 1) * T_LOC)
    x = torch.from_numpy(np.ascontiguousarray(c["x"][sl])).cuda().to(torch.bfloat16)
    idx = torch.from_numpy(np.ascontiguousarray(c["idx"][sl])).cuda()
    wt = torch.from_numpy(np.ascontiguousarray(c["wt"][sl])).cuda()
    out = torch.zeros((T_LOC, D), device="cuda")
    layer.forward(x, idx, wt, out, dist)
    again = torch.zeros_like(out)
    layer.forward(x, idx, wt, again, dist)
    # The chunked step (exchanges on NCCL's stream overlapping the expert
    # kernels, which leave SMs free meanwhile): the same bits.
    sliced = torch.zeros_like(out)
    layer.forward_chunked(x, idx, wt, sliced, dist, chunks=2)
    # Fixed-size exchange segments (no counts on the host): the same bits.
    fixed = torch.zeros_like(out)
    layer.forward_fixed(x, idx, wt, fixed, dist)
    # The exchanges as stores over NVLink into the ranks' IPC-mapped windows:
    # the same bits, twice through the same windows.
    win = ep.PeerWindows(torch, world, T_LOC, K, D).connect(rank, dist)
    peer, peer2 = torch.zeros_like(out), torch.zeros_like(out)
    layer.forward_peer(x, idx, wt, peer, dist, win)
    layer.forward_peer(x, idx, wt, peer2, dist, win)
    torch.cuda.synchronize()
    win.close(dist)
    gathered = [torch.zeros_like(out) for _ in range(world)]
    dist.all_gather(gathered, out)
    ok = (torch.equal(out, again) and torch.equal(out, sliced) and torch.equal(out, fixed) and
          torch.equal(out, peer) and torch.equal(out, peer2))
    if not ok:
        print(f"rank {rank}: again {torch.equal(out, again)} sliced {torch.equal(out, sliced)} "
              f"fixed {torch.equal(out, fixed)} peer {torch.equal(out, peer)} "
              f"peer2 {torch.equal(out, peer2)}", flush=True)
    if rank == 0:
        tabs_all, keep_all = tables_of(c["experts"])
        ref = torch.zeros((world * T_LOC, D), device="cuda")
        ws = torch.empty(moe.layer_workspace_bytes(world * T_LOC, K, E, 0, D, I, FMT),
                         dtype=torch.uint8, device="cuda")
        moe.layer_dev(world * T_LOC, K, E, 0, D, I, FMT,
                      torch.from_numpy(c["idx"]).cuda(), torch.from_numpy(c["wt"]).cuda(),
                      torch.from_numpy(c["x"]).cuda().to(torch.bfloat16), tabs_all, ref, ACT, A,
                      B, ws)
        torch.cuda.synchronize()
        got = torch.cat(gathered)
        rel = float((got - ref).norm() / ref.norm())
        mx = float((got - ref).abs().max())
        print(f"rank 0: rel_l2 vs single GPU {rel:.3e}, max_abs {mx:.3e}, repeat equal {ok}",
              flush=True)
        ok = ok and rel <= 1e-2 and mx <= 2e-2
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0 and int(flag.item()) == 1:
        print("EP-NCCL-OK", flush=True)
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()
