"""Worker for tests/test_gpu_tp_forward.py: tensor-parallel integer forward,
one process per GPU (torchrun).

Every rank builds the same synthetic model and its tensor-parallel share
(myl_model_create_tp); rank 0 also builds the unsharded single-GPU model. The
tensor-parallel greedy tokens must equal the single-GPU tokens and the CPU
oracle's, and the ranks' vocabulary slices of the logits, concatenated, must
equal the single-GPU logits: bit-identical at every GPU count. Cases: a model
whose 12 query heads over 2 KV heads split unevenly (ranks share a KV head),
and Qwen2.5-7B-shaped layers at batch 2. Rank 0 writes a JSON verdict.
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

import oracle as O  # noqa: E402

import myelith_b200 as myl  # noqa: E402
from myelith_b200 import model as M  # noqa: E402
from myelith_b200 import synthetic as S  # noqa: E402


def gather_logits(lg, vocab):
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, lg)
    return np.concatenate(parts, axis=1)


def check(ctx, spec, prompts, new, rank, world, use_oracle):
    B, P = prompts.shape
    tpm = M.IntegerModel(ctx, spec, world, rank)
    s = tpm.session(B, P + new)
    s.setup_tp()
    lg = s.forward(prompts)                       # logits of this rank's vocabulary rows
    full = gather_logits(lg, spec.vocab)
    toks = s.decode(new)[0]
    s.reset()
    toks_g, _, _ = tpm.generate(prompts, new, session=s)  # prefill + graph-replayed decode
    res = {}
    if rank == 0:
        ref = M.IntegerModel(ctx, spec)           # the unsharded model on this GPU
        rs = ref.session(B, P + new)
        ref_lg = rs.forward(prompts)
        ref_toks = rs.decode(new)[0]
        res["logits_equal"] = bool(np.array_equal(full, ref_lg))
        res["tokens_equal"] = bool(np.array_equal(toks, ref_toks) and np.array_equal(toks_g, ref_toks))
        if use_oracle:
            om = O.OracleModel(spec, P + new)
            wt, _ = om.generate(prompts[0], new)
            res["oracle_equal"] = bool(np.array_equal(toks[0], wt))
        rs.release()
        ref.release()
    ok = torch.tensor([int(all(res.values())) if rank == 0 else 1], device="cuda")
    dist.broadcast(ok, 0)
    s.release()
    tpm.release()
    return bool(ok.item()), res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    ctx = myl.Context(local)
    verdict = {"world": world}
    try:
        spec = S.synthetic_model("qwen2.5-0.5b", seed=21, num_layers=2, vocab=3001,
                                 dims=(2, 384, 12, 2, 32, 520, 3001, True))
        prompts = np.stack([S.prompt_tokens(spec.vocab, 37, seed=30 + b) for b in range(3)])
        ok, res = check(ctx, spec, prompts, 24, rank, world, True)
        verdict["uneven_heads"] = {"all_ranks": ok, **res}
        spec = S.synthetic_model("qwen2.5-7b", seed=22, num_layers=2)
        prompts = np.stack([S.prompt_tokens(spec.vocab, 300, seed=40 + b) for b in range(2)])
        ok, res = check(ctx, spec, prompts, 20, rank, world, False)
        verdict["qwen7b_layers"] = {"all_ranks": ok, **res}
    finally:
        dist.barrier()
        ctx.close()
        dist.destroy_process_group()
    if rank == 0:
        with open(args.out, "w") as f:
            json.dump(verdict, f)


if __name__ == "__main__":
    main()
