"""Runs one W8A16 linear shape, the config-4 MoE layer or an integer forward
repeatedly, for profiler captures (ncu). A measurement harness beside
bench.py, not part of the library.

    python profile_driver.py --M 1 --K 3584 --N 18944 --iters 6
    python profile_driver.py --moe --iters 4                 (config-4 MoE layer)
    python profile_driver.py --forward qwen2.5-7b --prompt 2048 --new 8 [--batch B] [--layers L]
        (synthetic model: prefill of the prompt, then greedy decode steps,
         twice; prints the prefill and decode times of each repetition)

Uses the device path (myl_linear_dev) with rotating weight sets whose total
size exceeds the 126 MB L2, so that DRAM counters reflect HBM traffic. Three
untimed warm-up calls come first (with ncu, skip their launches with -s).
Prints the average CUDA-event time per call (not a benchmark number when run
under a profiler).
"""
from __future__ import annotations

import argparse
import math

import numpy as np


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--K", type=int, default=3584)
    ap.add_argument("--N", type=int, default=18944)
    ap.add_argument("--iters", type=int, default=6)
    ap.add_argument("--sets", type=int, default=0, help="weight sets (0: enough to exceed 2x L2)")
    ap.add_argument("--moe", action="store_true", help="the config-4 MoE layer (myl_moe_dev)")
    ap.add_argument("--tokens", type=int, default=0, help="MoE tokens (0: 4096)")
    ap.add_argument("--forward", default="", help="synthetic model variant (qwen2.5-0.5b, qwen2.5-7b)")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--new", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=0, help="0: the variant's layer count")
    ap.add_argument("--reps", type=int, default=2)
    args = ap.parse_args()
    if args.moe:
        return moe(args)
    if args.forward:
        return forward(args)

    import torch

    import myelith_b200 as myl

    M, K, N = args.M, args.K, args.N
    ctx = myl.Context(0)
    rng = np.random.default_rng(5)
    sets = args.sets or max(2, math.ceil(2 * 126 * 2**20 / (N * K)))
    sh = int(round(math.log2(73.6 * math.sqrt(K))))
    ws = rng.integers(sh - 1, sh + 2, size=N).astype(np.uint8)
    Ws = [ctx.weight(rng.integers(-127, 128, size=(N, K), dtype=np.int8), K, ws) for _ in range(sets)]
    Rs = [w.requant(myl.RQ_SHIFT_I16, 8, 8) for w in Ws]
    x = torch.from_numpy(np.clip(np.rint(rng.normal(0, 1024, size=(M, K))), -32767, 32767)
                         .astype(np.int16)).cuda()
    y = torch.empty((M, N), dtype=torch.int16, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(3):  # warm-up: module loading and first-touch costs
            Ws[i % sets].linear_dev(Rs[i % sets], x, y, s)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(s)
        for i in range(args.iters):
            Ws[i % sets].linear_dev(Rs[i % sets], x, y, s)
        b.record(s)
        s.synchronize()
    ctx.synchronize()
    print(f"M={M} K={K} N={N} sets={sets}: {a.elapsed_time(b) / args.iters * 1e3:.2f} us/call, "
          f"{ctx.launch_count} launches")


def moe(args) -> None:
    import torch

    import myelith_b200 as myl
    from myelith_b200.synthetic import MOE_CONFIG4 as C, activations, moe_layer

    ctx = myl.Context(0)
    layer, shared = moe_layer(ctx, C["H"], C["I"], C["E"], C["k"], C["shared_I"])
    T = args.tokens or C["T"]
    x = torch.from_numpy(activations(np.random.default_rng(6), (T, C["H"]))).cuda()
    y = torch.empty_like(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(3):
            layer.dev(x, y, stream=s)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(s)
        for _ in range(args.iters):
            layer.dev(x, y, stream=s)
        b.record(s)
        s.synchronize()
    ctx.synchronize()
    print(f"moe T={T}: {a.elapsed_time(b) / args.iters * 1e3:.2f} us/layer, "
          f"{ctx.launch_count} launches")


def forward(args) -> None:
    import myelith_b200 as myl
    from myelith_b200 import model as M, synthetic as S

    ctx = myl.Context(0)
    spec = S.synthetic_model(args.forward, seed=2, num_layers=args.layers or None)
    gm = M.IntegerModel(ctx, spec)
    prompts = np.stack([S.prompt_tokens(spec.vocab, args.prompt, seed=100 + b) for b in range(args.batch)])
    sess = gm.session(args.batch, args.prompt + args.new)
    for rep in range(args.reps):
        sess.reset()
        sess.forward(prompts, want_logits=False)
        sess.decode(args.new)
        pre, dec = sess.timing()
        print(f"rep {rep}: prefill {pre:.3f} ms, decode {dec:.3f} ms for {args.new} steps", flush=True)


if __name__ == "__main__":
    main()
