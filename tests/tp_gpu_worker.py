"""Worker for tests/test_gpu_tp.py: one process per GPU (torchrun), NCCL.

Builds column-parallel, row-parallel and MLP layers of myelith_b200.tp over
the W8A16 kernels, runs them, and checks on every rank that the result equals
the unsharded single-GPU result of the same library (bit-identical at every
GPU count) and, for the linear layers, the CPU oracle. Rank 0 writes a JSON
verdict to --out.
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
sys.path.insert(0, os.path.join(HERE, "golden"))

import oracle as O  # noqa: E402
from make_golden import silu_lut_spec  # noqa: E402

import myelith_b200 as myl  # noqa: E402
from myelith_b200 import tp  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    verdict = {}
    try:
        ctx = myl.Context(local_rank)
        rng = np.random.default_rng(2024)  # same data on every rank
        M, K, N = 96, 3584, 1000
        W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        ws = rng.integers(11, 14, size=N).astype(np.uint8)
        of = rng.integers(6, 10, size=N).astype(np.uint8)
        x = np.clip(np.rint(rng.normal(0, 1024, size=(M, K))), -32767, 32767).astype(np.int16)
        H, I = 896, 4864
        mlp = dict(W_gate=rng.integers(-127, 128, size=(I, H), dtype=np.int8),
                   W_up=rng.integers(-127, 128, size=(I, H), dtype=np.int8),
                   W_down=rng.integers(-127, 128, size=(H, I), dtype=np.int8),
                   gate_w_shifts=rng.integers(11, 13, size=I).astype(np.uint8),
                   up_w_shifts=rng.integers(11, 13, size=I).astype(np.uint8),
                   down_w_shifts=rng.integers(12, 14, size=H).astype(np.uint8),
                   silu_lut=silu_lut_spec(), in_frac=8, gate_out_frac=7, up_out_frac=7,
                   down_in_frac=7, silu_in_frac=6, silu_lut_offset=8192, silu_out_frac=8,
                   out_frac=rng.integers(3, 7, size=H).astype(np.uint8))
        xm = np.clip(np.rint(rng.normal(0, 1500, size=(M, H))), -32767, 32767).astype(np.int16)

        V = 5003  # vocab-parallel LM head: uneven shards, a repeated half for cross-shard ties
        Wl = rng.integers(-127, 128, size=(V, K), dtype=np.int8)
        Wl[2502:5002] = Wl[:2500]
        wsl = rng.integers(12, 14, size=V).astype(np.uint8)

        local = tp.LibLocal(ctx)
        spec = tp.LinearSpec(W, ws, 8, of)
        head = tp.VocabParallelLMHead(local, "head", Wl, wsl, 8, 6, rank, world)
        xchg = tp.PeerExchange(ctx, M, N, rank, world)  # peer-memory row-parallel exchange
        col = tp.ColumnParallelLinear(local, "col", spec, rank, world)
        row = tp.RowParallelLinear(local, "row", spec, rank, world)
        pm = tp.ParallelMlp(local, "mlp", hidden=H, intermediate=I, rank=rank, world=world, **mlp)
        xt = torch.from_numpy(x).to(dev)
        xmt = torch.from_numpy(xm).to(dev)
        for Ms in (2, M):  # decode (GEMV) and prefill (tensor cores)
            y_col = col.gather(xt[:Ms]).cpu().numpy()
            y_row = row(row.x_shard(xt[:Ms])).cpu().numpy()
            y_ov = row.overlapped(row.x_shard(xt[:Ms]), chunks=4).cpu().numpy()
            y_mlp = pm(xmt[:Ms]).cpu().numpy()
            single = ctx.weight(W, K, ws).linear(x[:Ms], 8, of)
            single_mlp = myl.Mlp(ctx, mlp["W_gate"], mlp["W_up"], mlp["W_down"], H, I,
                                 mlp["gate_w_shifts"], mlp["up_w_shifts"], mlp["down_w_shifts"],
                                 mlp["silu_lut"], 8, 7, 7, 7, 6, 8192, 8, mlp["out_frac"])(xm[:Ms])
            ref = O.linear_w8a16_pc(x[:Ms], W.reshape(-1), K, ws, 8, of)
            tok, best = head.greedy(xt[:Ms])
            y_x = row.exchanged(row.x_shard(xt[:Ms]), xchg).cpu().numpy()
            logits = ctx.weight(Wl, K, wsl).lm_head(x[:Ms], 8, 6)
            ok = dict(col=bool(np.array_equal(y_col, single)), row=bool(np.array_equal(y_row, single)),
                      overlapped=bool(np.array_equal(y_ov, single)),
                      mlp=bool(np.array_equal(y_mlp, single_mlp)), oracle=bool(np.array_equal(single, ref)),
                      exchange=bool(np.array_equal(y_x, single)),
                      greedy=tok.cpu().tolist() == [O.argmax_int(r) for r in logits]
                      and best.cpu().tolist() == [int(r.max()) for r in logits])
            # every rank holds the same bytes
            h = torch.tensor([int(np.frombuffer(y_mlp.tobytes(), np.uint8).astype(np.int64).sum()),
                              int(np.frombuffer(y_row.tobytes(), np.uint8).astype(np.int64).sum())],
                             dtype=torch.int64, device=dev)
            hmax, hmin = h.clone(), h.clone()
            dist.all_reduce(hmax, op=dist.ReduceOp.MAX)
            dist.all_reduce(hmin, op=dist.ReduceOp.MIN)
            ok["ranks_agree"] = bool(torch.equal(hmax, hmin))
            ok["all"] = all(ok.values())
            flag = torch.tensor([1 if ok["all"] else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            ok["all_ranks"] = bool(flag.item())
            verdict[f"M{Ms}"] = ok
        ctx.synchronize()
        xchg.close()
    finally:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank == 0:
        with open(args.out, "w") as f:
            json.dump({"world": world, **verdict}, f)


if __name__ == "__main__":
    main()
