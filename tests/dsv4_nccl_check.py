"""Two-rank DeepSeek-V4 expert split over NCCL (launched by
tests/test_dsv4_gpu.py through torchrun, one rank per GPU): each rank holds
the experts of its parity, both run dsv4.EP2Layer.forward on the same tokens,
and the all-reduced results must be identical on both ranks, identical to the
two ranks emulated on one GPU (the all-reduce of two is one addition), and
within the MoE tolerance of the oracle's route_moe_ep2 plus the layer tail.
Prints DSV4-EP2-NCCL-OK on success."""
import os
import sys
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in ("micro-vllm_b200", "oracle", "tests", os.path.join("tests", "golden")):
    sys.path.insert(0, os.path.join(ROOT, p))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import dsv4  # noqa: E402
import dsv4_cases as dc  # noqa: E402
import mvllm_moe as moe  # noqa: E402
from oracle import Oracle  # noqa: E402

H, I, E, T = 512, 256, 16, 24


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ops_for(c, rank, nranks, keep):
    tabs = [[], [], [], [], [], []]
    for e in range(rank, E, nranks):
        (gp, gsc), (up, usc), (dp, dsc) = c["experts"][e]
        for k, a in enumerate((gp, up, dp, gsc, usc, dsc)):
            t = dev(a)
            keep.append(t)
            tabs[k].append(t.data_ptr())
    tables = [torch.tensor(t, dtype=torch.int64, device="cuda") for t in tabs]
    sh = [(dev(w), dev(s)) for w, s in c["shared_fp8"]] if rank == 0 else None
    dense = (moe.FMT_INT8_ROW,) + tuple((dev(a), dev(b)) for a, b in c["dense"])
    return dsv4.CudaOps(torch, E, H, I, dc.LIMIT, dev(c["router"]), dev(c["bias"]), tables, rank,
                        nranks, T, c["route_scale"], c["routed_scale"], sh, dense)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    moe.init(local)
    port = Oracle("port")
    c = dc.dsv4_case(port, 91, H, I, E, T)
    keep = []
    layer = dsv4.EP2Layer(ops_for(c, rank, world, keep), rank, world)
    h = dev(c["h"])
    layer.forward(dev(c["x"]), h, dist)
    torch.cuda.synchronize()
    gathered = [torch.zeros_like(h) for _ in range(world)]
    dist.all_gather(gathered, h)
    ok = all(torch.equal(g, gathered[0]) for g in gathered)
    if rank == 0:
        emu = [dsv4.EP2Layer(ops_for(c, r, world, keep), r, world) for r in range(world)]
        he = dev(c["h"])
        dsv4.emulate_step(emu, dev(c["x"]), he)
        torch.cuda.synchronize()
        same = torch.equal(he, h)
        _, h_w = dc.expected(port, c)
        got = h.cpu().numpy()
        rel = float(np.linalg.norm(got - h_w) / np.linalg.norm(h_w))
        mx = float(np.abs(got - h_w).max())
        print(f"rank 0: ranks equal {ok}, equal to emulation {same}, rel_l2 vs oracle "
              f"{rel:.3e}, max_abs {mx:.3e}", flush=True)
        ok = ok and same and rel <= 1e-2 and mx <= 2e-2
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0 and int(flag.item()) == 1:
        print("DSV4-EP2-NCCL-OK", flush=True)
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()
