"""Worker for tests/test_gpu_ep.py: one process per GPU (torchrun), NCCL.

Every rank holds its own tokens and its block of the experts; the
expert-parallel layer (myelith_b200.ep over the MoE kernels, NCCL
all_to_all) must give, on every rank, the single-GPU MoE layer's output for
that rank's tokens bit for bit, and the CPU oracle's on a sample of them.
Rank 0 writes a JSON verdict to --out.
"""
import argparse
import json
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "golden"))

import moe_ref as R  # noqa: E402

import myelith_b200 as myl  # noqa: E402
from myelith_b200 import ep  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--tokens", type=int, default=512)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    verdict = {}
    try:
        ctx = myl.Context(local_rank)
        H, I, E, k, Is = 2048, 1408, 64, 4, 5632
        p, s = R.problem(H=H, I=I, E=E, k=k, shared_I=Is, seed=4)  # same weights on every rank
        first, last = ep.shard_range(E, rank, world)
        part = R.lib_moe(ctx, p, None, first_expert=first, num_local=last - first)
        shared = myl.Mlp(ctx, **s)
        layer = ep.ExpertParallelMoe(ep.LibMoeLocal(part, shared), E, k, H, rank, world)
        T = args.tokens + 37 * rank  # uneven token counts
        x = R.activations(np.random.default_rng(500 + rank), T, H)
        xt = torch.from_numpy(x).to(dev)
        out = layer(xt).cpu().numpy()
        out2 = layer(xt).cpu().numpy()
        # the same layer over peer memory (no collective library on the data path);
        # every rank passes the same token bound
        peer = ep.PeerExpertParallelMoe(ctx, ep.LibMoeLocal(part, shared), E, k, H, rank, world,
                                        max_tokens=args.tokens + 37 * (world - 1))
        outp = peer(xt).cpu().numpy()
        outp2 = peer(xt).cpu().numpy()
        ctx.synchronize()
        peer.close()
        full = R.lib_moe(ctx, p, s)
        single = full(x)
        sample = np.random.default_rng(7 + rank).choice(T, size=12, replace=False)
        ref = R.forward(p, s, x[sample])[0]
        ok = dict(single=bool(np.array_equal(out, single)), repeat=bool(np.array_equal(out, out2)),
                  peer=bool(np.array_equal(outp, single) and np.array_equal(outp2, single)),
                  oracle=bool(np.array_equal(out[sample], ref)))
        ok["all"] = all(ok.values())
        flag = torch.tensor([1 if ok["all"] else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok["all_ranks"] = bool(flag.item())
        verdict["moe"] = ok
        ctx.synchronize()
    finally:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank == 0:
        with open(args.out, "w") as f:
            json.dump({"world": world, **verdict}, f)


if __name__ == "__main__":
    main()
