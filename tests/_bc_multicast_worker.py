"""Rank worker for test_multigpu_gpu.py (launched by torch.distributed.run).

d_inner sharding with B and C replicated: every rank scans a contiguous
channel slice, and the backward kernel sums dB / dC over the ranks through
NVLink multicast (parallel.MulticastBCSum).  Every rank also runs the
unsharded problem on its own GPU and the NCCL form (parallel.replicated_bc);
the worst relative errors (max over ranks) are printed by rank 0 as JSON.
"""

import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import selectssm_b200 as S  # noqa: E402
from selectssm_b200.parallel import MulticastBCSum, replicated_bc, shard_range  # noqa: E402

NAMES = ("u", "delta", "A", "B", "C", "D", "bias", "z")


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def inputs(Bsz, L, Dm, dtype, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)  # same draw on every rank

    def n(*s):
        return torch.randn(*s, generator=g, device=dev)

    t = {"u": n(Bsz, L, Dm), "delta": n(Bsz, L, Dm) - 4.0, "z": n(Bsz, L, Dm), "dout": n(Bsz, L, Dm),
         "B": n(Bsz, L, 16), "C": n(Bsz, L, 16), "A": -(1.0 + 15.0 * torch.rand(Dm, 16, generator=g, device=dev)),
         "D": 1.0 + 0.1 * n(Dm), "bias": 0.1 * n(Dm)}
    for k in ("u", "delta", "z", "dout", "B", "C"):
        t[k] = t[k].to(dtype)
    return t


def run(t, sl, bc_sum=None, nccl=False):
    """fwd + bwd on channel slice sl; returns (out, grads)."""
    per_ch = {"u", "delta", "z"}
    leaves = {}
    for k in NAMES:
        v = t[k]
        if k in per_ch:
            v = v[..., sl]
        elif k in ("A", "D", "bias"):
            v = v[sl]
        leaves[k] = v.detach().clone().requires_grad_()
    Bm, Cm = leaves["B"], leaves["C"]
    if nccl:
        Bm, Cm = replicated_bc(Bm, Cm)
    out = S.selective_scan(leaves["u"], leaves["delta"], leaves["A"], Bm, Cm, D=leaves["D"], z=leaves["z"],
                           delta_bias=leaves["bias"], delta_softplus=True, bc_sum=bc_sum)
    out.backward(t["dout"][..., sl])
    return out, {k: v.grad for k, v in leaves.items()}


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    Bsz, L, Dm = 2, 1000, 128 * world
    res = {}
    for dtype, name in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        t = inputs(Bsz, L, Dm, dtype, dev, 11)
        s, e = shard_range(Dm // 8, rank, world)
        sl = slice(8 * s, 8 * e)
        bcs = MulticastBCSum(Bsz, L, device=dev)
        if not bcs.available:
            if rank == 0:
                print(json.dumps({"skip": "the GPUs report no NVLink multicast support"}))
            dist.destroy_process_group()
            return
        full_out, full_g = run(t, slice(0, Dm))
        errs = {}
        for it in range(2):  # twice: the buffer is zeroed and reused
            out, g = run(t, sl, bc_sum=bcs)
            errs[f"out{it}"] = rel(out, full_out[..., sl])
            for k in ("u", "delta", "z"):
                errs[f"d{k}{it}"] = rel(g[k], full_g[k][..., sl])
            for k in ("A", "D", "bias"):
                errs[f"d{k}{it}"] = rel(g[k], full_g[k][sl])
            for k in ("B", "C"):  # the cross-rank sums
                errs[f"d{k}{it}"] = rel(g[k], full_g[k])
        _, gn = run(t, sl, nccl=True)
        for k in ("B", "C"):
            errs[f"d{k}_vs_nccl"] = rel(g[k], gn[k])
        worst = torch.tensor([max(errs.values())], device=dev)
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
        res[name] = {"worst": float(worst.item()), "rank0": errs}
    if rank == 0:
        print(json.dumps(res))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
