#!/usr/bin/env python
"""W8A16 hot-path benchmark: prints one JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the W8A16 linear at the Qwen2.5-7B MLP shapes,
gate/up (K=3584 -> N=18944) and down (K=18944 -> N=3584), M=2048 activation
rows. One step = both shapes once: split x into byte planes, tcgen05 GEMM,
requant epilogue. Int8 weights uniform in [-127, 127], int16 activations
rounded N(0, 1024^2) clipped to +-32767, per-channel power-of-two requant;
synthetic, seeded, random-init.

N GPUs (torchrun): Megatron tensor parallelism of the same step. The gate/up
shape is column-parallel (N split), the down shape row-parallel (K split):
each rank produces exact int64 partial sums that are summed across the ranks
before the requant runs once, so the result is bit-identical at every GPU
count (tp_check compares the step with an int64 all-reduce step). With
--exchange p2p (default) the down GEMM's epilogue stores its partial rows
into the owning ranks' buffers over NVLink and a reduce kernel requantises and
all-gathers through peer memory (device barriers, no collective library on
the data path); --exchange nccl overlaps an NCCL reduce-scatter with the
gate/up GEMM and all-gathers after the requant. Total work is fixed: strong
scaling.

moe        the config-4 MoE layer (4096 tokens, 64 experts, top-4, shared
           expert): one GPU runs the fused layer; N GPUs split the experts
           (expert parallelism, dispatch and return through peer memory, or
           NCCL all_to_all with --exchange nccl), each rank 4096/N tokens.

value      whole-job algorithmic int TOPS (2*M*K*N per linear) over the timed
           steps, device time, max over ranks. Inputs are resident in HBM.
e2e        the same metric through the reference-facing host-pointer C ABI
           (myl_linear_w8a16 with pinned host buffers; at N>1 the host input
           and output copies around the tensor-parallel device step).
roofline   the tcgen05 GEMM kernel: algorithmic TOPS per launch from CUDA
           events around each launch, against the effective split-byte peak.
gemv       decode GEMV (M=1) at both shapes: weight-streaming GB/s vs HBM; and
           mlp_decode, the decode MLP as the forward runs it (interleaved
           gate/up GEMV with the SiLU epilogue, then down) at the 7B shapes.
cpu_baseline  the CPU oracle (C restatement of the reference's Rust loop) on a
           bounded row sample, all host cores, rank 0 at N=1.
L2: 4 rotating weight sets per shape (>= 4x the 126 MB L2 per step cycle), so
every weight byte comes from HBM.

--impl reference runs only the CPU oracle (the reference's algorithm; the Rust
original cannot be built here) with the same metric, config and unit.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from myelith_b200.synthetic import MOE_CONFIG4 as MOE, moe_layer  # noqa: E402

METRIC = "W8A16 GEMM TOPS & GEMV GB/s; 7B-shape int decode tok/s at 1/2/4/8 GPU"
SHAPES = [(3584, 18944), (18944, 3584)]  # (K, N): gate/up, down
M_HEAD = 2048
SWEEP_M = [1, 16, 128, 512, 2048]
L2_BYTES = 126 * 1024 * 1024
ACT_FRAC, OUT_FRAC = 8, 8


def kbits(K: int) -> int:
    """Per-row weight shift that keeps outputs unsaturated: round(log2(73.6*sqrt(K)))."""
    return int(round(math.log2(73.6 * math.sqrt(K))))


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic() -> dict:
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """SM clocks, power and clock-event reasons sampled DURING the timed region.

    NVML is polled from a thread every ~2 ms (a timed region of a few ms still
    gets samples); without NVML, nvidia-smi every 200 ms."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None
        self.nvml = None
        self.handle = None
        self.stop_flag = threading.Event()
        self.sm: list[float] = []
        self.power: list[float] = []
        self.reasons: set[str] = set()
        self.sm_max = None

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        self.nvml = pynvml
        try:  # the CUDA device's UUID names the same GPU under any CUDA_VISIBLE_DEVICES
            uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
            return pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def start(self):
        try:
            self.handle = self._nvml_handle()
            n = self.nvml
            self.sm_max = float(n.nvmlDeviceGetMaxClockInfo(self.handle, n.NVML_CLOCK_SM))
            self.masks = {
                "hw_slowdown": n.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": n.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": n.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": n.nvmlClocksEventReasonSwPowerCap,
            }
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.handle = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _poll_nvml(self):
        n, h = self.nvml, self.handle
        i = 0
        while not self.stop_flag.is_set():
            try:
                self.sm.append(float(n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM)))
                bits = n.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, mask in self.masks.items():
                    if bits & mask:
                        self.reasons.add(name)
                if i % 10 == 0:
                    self.power.append(n.nvmlDeviceGetPowerUsage(h) / 1000.0)
            except Exception:
                pass
            i += 1
            self.stop_flag.wait(0.002)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.handle is not None:
            self.stop_flag.set()
            self.thread.join(timeout=2)
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
            return {"sm_mhz": statistics.median(self.sm) if self.sm else None,
                    "sm_max_mhz": self.sm_max, "reasons": sorted(self.reasons),
                    "samples": len(self.sm), "power_w_max": max(self.power) if self.power else None,
                    "source": "nvml, every ~2 ms during the timed region"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons, power = [], None, set(), []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, v in zip(self.NAMES, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None,
                "source": "nvidia-smi every 200 ms"}


# ---------------------------------------------------------------------------------------
# CPU oracle (the reference's algorithm): bounded samples


def config1(tp: int, exchange: str = "p2p") -> dict:
    """The config object of the config-1 line, the same for both arms."""
    n1, k2 = SHAPES[0][1] // tp, SHAPES[1][0] // tp
    per_set = n1 * SHAPES[0][0] + SHAPES[1][1] * k2
    nsets = max(2, math.ceil(4 * L2_BYTES / per_set))
    par = f"tp{tp}" if tp == 1 else (f"tp{tp}, row-parallel exchange: " + (
        "peer memory from the GEMM epilogue" if exchange == "p2p" else "NCCL reduce-scatter + all-gather"))
    return {"workload": "config1: W8A16 linear at Qwen2.5-7B MLP shapes, gate/up + down per step",
            "M": M_HEAD, "shapes_KN": SHAPES, "parallelism": par,
            "l2": f"inputs larger than L2: {nsets} rotating weight sets "
                  f"({nsets * per_set / 2**20:.0f} MiB per rank)"}


def cpu_sample_tops(target_s: float, rng) -> dict:
    """Times the oracle's linear_w8a16 on a row sample of the step (both shapes),
    sized to about target_s seconds, on all host threads."""
    import oracle as O

    ws = {}
    for K, N in SHAPES:
        W = rng.integers(-127, 128, size=N * K, dtype=np.int8)
        s = rng.integers(kbits(K) - 1, kbits(K) + 2, size=N).astype(np.uint8)
        ws[(K, N)] = (W, s)

    def run(rows: int) -> float:
        t0 = time.perf_counter()
        for K, N in SHAPES:
            W, s = ws[(K, N)]
            x = np.clip(np.rint(rng.normal(0, 1024, size=(rows, K))), -32767, 32767).astype(np.int16)
            O.linear_w8a16(x, W, K, s, ACT_FRAC, OUT_FRAC)
        return time.perf_counter() - t0

    O.set_num_threads(os.cpu_count() or 1)  # torchrun sets OMP_NUM_THREADS=1 per process
    run(1)  # warm-up (page-in, thread pool)
    t1 = run(1)
    rows = max(1, min(M_HEAD, int(target_s / max(t1, 1e-6))))
    t = run(rows)
    ops = 2.0 * rows * sum(K * N for K, N in SHAPES)
    return {"value": ops / t / 1e12, "unit": "TOPS", "cores": O.num_threads(), "kind": "port",
            "sample": f"{rows} of {M_HEAD} rows at both shapes (K,N)={SHAPES}, {t:.1f} s",
            "seconds": t}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    rng = np.random.default_rng(1234)
    import oracle as O

    O.build()
    per_step = float(os.environ.get("MYL_REF_STEP_S", "4.0"))
    for _ in range(args.warmup):
        cpu_sample_tops(per_step / 4, rng)
    vals, secs = [], 0.0
    for _ in range(args.steps):
        r = cpu_sample_tops(per_step, rng)
        vals.append(r["value"])
        secs += r["seconds"]
    v = statistics.mean(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8xint16->int64", "data": "synthetic",
        "config": config1(world, args.exchange),
        "cpu_baseline": {"value": v, "unit": "TOPS", "cores": O.num_threads(), "kind": "port",
                         "sample": r["sample"]},
        "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU restatement of the reference's Rust loop (dot_scalar + rescale_i64 + clamp), "
                "OpenMP over output rows; the Rust crate cannot be built in this image",
    }
    emit(line)


# ---------------------------------------------------------------------------------------
# MoE layer

def moe_ops(T: int) -> float:
    """Algorithmic integer ops of one MoE layer over T tokens (2 per MAC):
    router, the top-k experts' gate/up/down and the shared expert."""
    H, I, E, k, Is = MOE["H"], MOE["I"], MOE["E"], MOE["k"], MOE["shared_I"]
    return 2.0 * T * (E * H + k * 3 * I * H + 3 * Is * H)


FWD_CFG2 = dict(variant="qwen2.5-0.5b", prompt=512, new=128, batch=(1,))
FWD_CFG3 = dict(variant="qwen2.5-7b", prompt=2048, new=256, batch=(1, 8, 32))


def bench_forward(ctx, cfg: dict, steps: int, warmup: int, hbm_gbs: float, check_tokens: int,
                  check_new: int) -> dict:
    """The integer decoder forward (runtime/src/model.rs forward_token,
    generate.rs greedy) on one GPU: random-init int8 weights of the named
    Qwen2.5 architecture (myelith_b200.synthetic.synthetic_model), uniform
    random prompt token ids. Per batch size B: prefill of B x prompt tokens
    (myl_forward, device time), then `new` greedy decode steps
    (myl_decode_greedy, one CUDA graph per step, device time), and the whole
    generate call from host prompt to host tokens (wall clock, e2e).

    Parity, in the same run: the CPU oracle's generate (tokens and the
    SHA-256 logits digest of dekodieren_mit_digest) on sequence 0, with the
    full workload when check_tokens >= prompt, else a shortened prompt of
    check_tokens and check_new steps on the same model; the timed decode's
    tokens must equal the checked run's, and sequence 0's tokens must not
    depend on the batch size."""
    import oracle as O
    from myelith_b200 import model as MD
    from myelith_b200 import synthetic as SY

    t0 = time.perf_counter()
    spec = SY.synthetic_model(cfg["variant"], seed=2)
    gm = MD.IntegerModel(ctx, spec)
    build_s = time.perf_counter() - t0
    P, N = cfg["prompt"], cfg["new"]
    prompts = {b: SY.prompt_tokens(spec.vocab, P, seed=100 + b) for b in range(max(cfg["batch"]))}
    # ---- parity against the oracle (sequence 0) ----
    cP, cN = (P, N) if check_tokens >= P else (check_tokens, check_new)
    t0 = time.perf_counter()
    om = O.OracleModel(spec, cP + cN)
    otok, olg = om.generate(prompts[0][:cP], cN)
    o_digest = MD.digest(olg, otok)
    oracle_s = time.perf_counter() - t0
    del om, olg
    gtok, gdig, _ = gm.generate(prompts[0][:cP], cN, digest=True)
    parity = bool(np.array_equal(gtok[0], otok)) and gdig[0] == o_digest
    out = {"workload": f"{cfg['variant']} architecture, random-init int8 weights, {P} random prompt "
                       f"tokens then {N} greedy decode steps",
           "weight_bytes_per_token": int(spec.weight_bytes_per_token()),
           "model_build_s": round(build_s, 1),
           "parity": parity,
           "parity_check": {"sequence": 0, "prompt": cP, "new": cN, "oracle_s": round(oracle_s, 1),
                            "tokens_equal": bool(np.array_equal(gtok[0], otok)),
                            "digest": o_digest, "digest_equal": gdig[0] == o_digest,
                            "cores": O.num_threads()},
           "batches": []}
    seq0 = None
    for B in cfg["batch"]:
        pr = np.stack([prompts[b] for b in range(B)])
        sess = gm.session(B, P + N)
        pre, dec, e2e, toks = [], [], [], None
        for it in range(warmup + steps):
            sess.reset()
            sess.forward(pr, want_logits=False)
            tk, _, _ = sess.decode(N)
            pms, dms = sess.timing()
            if it >= warmup:
                pre.append(pms)
                dec.append(dms)
            toks = tk if toks is None else toks
            if not np.array_equal(tk, toks):
                parity = False
        for it in range(max(1, steps // 2)):
            w0 = time.perf_counter()
            tk, _, _ = gm.generate(pr, N, session=sess)
            e2e.append(time.perf_counter() - w0)
            if not np.array_equal(tk, toks):
                parity = False
        if seq0 is None:
            seq0 = toks[0].copy()
        elif not np.array_equal(toks[0], seq0):
            parity = False
        if cP == P and cN == N and not np.array_equal(toks[0], otok):
            parity = False
        if cP == P and cN < N and not np.array_equal(toks[0][:cN], otok):
            parity = False
        sess.release()
        pms, dms = statistics.median(pre), statistics.median(dec)
        wb = spec.weight_bytes_per_token()
        out["batches"].append({
            "batch": B, "prefill_tok_s": round(B * P / (pms * 1e-3), 1), "prefill_ms": round(pms, 3),
            "decode_tok_s": round(B * N / (dms * 1e-3), 1), "decode_ms_per_step": round(dms / N, 4),
            "decode_weight_gbs": round(wb * N / (dms * 1e-3) / 1e9, 1),
            "decode_frac_of_hbm": round(wb * N / (dms * 1e-3) / 1e9 / hbm_gbs, 3),
            "e2e_generate_tok_s": round(B * N / statistics.median(e2e), 1),
            "e2e_generate_s": round(statistics.median(e2e), 4)})
    out["parity"] = parity
    gm.release()
    return out


def bench_forward_tp(ctx, cfg: dict, steps: int, warmup: int, rank: int, world: int, max_over_ranks,
                     check_tokens: int, check_new: int) -> dict:
    """The integer forward tensor-parallel over the job's GPUs (one process per
    GPU, myl_model_create_tp): every rank holds an even share of the query
    heads (and the KV heads they read), of the MLP channels and of the LM
    head's vocabulary rows; row-parallel partial sums go to every rank over
    peer memory and are summed and requantised once, so tokens are
    bit-identical to one GPU. Per batch size: prefill and decode device time
    (max over ranks). Parity: a shortened generate (check_tokens prompt
    tokens, check_new steps) on the same model against the CPU oracle (rank 0),
    and sequence 0's tokens independent of the batch size."""
    import torch
    import torch.distributed as dist

    import oracle as O
    from myelith_b200 import model as MD
    from myelith_b200 import synthetic as SY

    t0 = time.perf_counter()
    spec = SY.synthetic_model(cfg["variant"], seed=2)
    gm = MD.IntegerModel(ctx, spec, world, rank)
    build_s = time.perf_counter() - t0
    P, N = cfg["prompt"], cfg["new"]
    prompts = {b: SY.prompt_tokens(spec.vocab, P, seed=100 + b) for b in range(max(cfg["batch"]))}
    cP, cN = check_tokens, check_new
    s = gm.session(1, cP + cN)
    s.setup_tp()
    gtok, _, _ = gm.generate(prompts[0][:cP], cN, session=s)
    s.release()
    ok = 1
    oracle_s = None
    if rank == 0:
        t0 = time.perf_counter()
        om = O.OracleModel(spec, cP + cN)
        otok, _ = om.generate(prompts[0][:cP], cN, keep_logits=False)
        oracle_s = time.perf_counter() - t0
        ok = int(np.array_equal(gtok[0], otok))
        del om
    wb = spec.weight_bytes_per_token()
    del spec
    out = {"workload": f"{cfg['variant']} architecture, random-init int8 weights, {P} random prompt "
                       f"tokens then {N} greedy decode steps, tensor-parallel over {world} GPUs",
           "parallelism": f"tp{world}: heads, MLP channels and vocabulary rows split; row-parallel "
                          "int64 partials over peer memory",
           "weight_bytes_per_token": int(wb), "model_build_s": round(build_s, 1),
           "parity_check": {"sequence": 0, "prompt": cP, "new": cN, "against": "CPU oracle",
                            "oracle_s": None if oracle_s is None else round(oracle_s, 1)},
           "shard": gm.shard, "batches": []}
    seq0 = None
    for B in cfg["batch"]:
        pr = np.stack([prompts[b] for b in range(B)])
        sess = gm.session(B, P + N)
        sess.setup_tp()
        pre, dec, toks = [], [], None
        for it in range(warmup + steps):
            dist.barrier()
            sess.reset()
            sess.forward(pr, want_logits=False)
            tk, _, _ = sess.decode(N)
            pms, dms = sess.timing()
            if it >= warmup:
                pre.append(max_over_ranks(pms))
                dec.append(max_over_ranks(dms))
            toks = tk if toks is None else toks
            if not np.array_equal(tk, toks):
                ok = 0
        if seq0 is None:
            seq0 = toks[0].copy()
        elif not np.array_equal(toks[0], seq0):
            ok = 0
        if not np.array_equal(toks[0][:cN], gtok[0]) and cP == P:
            ok = 0
        sess.release()
        pms, dms = statistics.median(pre), statistics.median(dec)
        out["batches"].append({
            "batch": B, "prefill_tok_s": round(B * P / (pms * 1e-3), 1), "prefill_ms": round(pms, 3),
            "decode_tok_s": round(B * N / (dms * 1e-3), 1), "decode_ms_per_step": round(dms / N, 4)})
    t = torch.tensor([ok], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    out["parity"] = bool(t.item())
    out["parity_check"]["tokens_equal"] = out["parity"]
    gm.release()
    return out


def bench_moe(ctx, dev, stream, rank: int, world: int, local: int, steps: int, warmup: int,
              max_over_ranks, barrier, peer: bool = True) -> dict:
    """The MoE layer at config 4: 4096 tokens per step in total. One GPU: the
    fused layer (myl_moe_dev). N GPUs: expert parallelism, each rank holds
    E/N experts and 4096/N tokens, NCCL all_to_all dispatch and return."""
    import torch

    import myelith_b200 as myl
    from myelith_b200 import ep

    H, I, E, k, Is, T = (MOE[n] for n in ("H", "I", "E", "k", "shared_I", "T"))
    first, last = ep.shard_range(E, rank, world)
    moe, shared = moe_layer(ctx, H, I, E, k, Is, first, last - first, attach_shared=world == 1)
    Tr = T // world
    xr = np.random.default_rng(4100 + rank)
    x_h = np.clip(np.rint(xr.normal(0, 1024, size=(Tr, H))), -32767, 32767).astype(np.int16)
    with torch.cuda.stream(stream):
        x = torch.from_numpy(x_h).to(dev)
        out = torch.empty_like(x)
        idx = torch.empty((Tr, k), dtype=torch.int32, device=dev)
        prob = torch.empty_like(idx)
    stream.synchronize()
    if world == 1:
        def layer():
            moe.dev(x, out, idx, prob, stream)
    else:
        if peer:  # dispatch and return through peer memory
            epl = ep.PeerExpertParallelMoe(ctx, ep.LibMoeLocal(moe, shared), E, k, H, rank, world,
                                           max_tokens=Tr)
        else:
            epl = ep.ExpertParallelMoe(ep.LibMoeLocal(moe, shared), E, k, H, rank, world)

        def layer():
            out.copy_(epl(x))

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            layer()
        stream.synchronize()
        barrier()
        l0 = ctx.launch_count
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            layer()
        b.record(stream)
        stream.synchronize()
        launches = ctx.launch_count - l0
    ctx.synchronize()
    ms = max_over_ranks(a.elapsed_time(b) / steps)
    if world > 1:  # the expert-parallel layer routes internally: route once more for the load
        with torch.cuda.stream(stream):
            idx, _ = epl.local.route(x)
        stream.synchronize()
    load = torch.bincount(idx.reshape(-1).long(), minlength=E).cpu().numpy()
    res = {"workload": "config4: MoE layer, hidden 2048, 64 experts x MLP 1408, top-4, shared "
                       "expert 5632, 4096 tokens per step",
           "parallelism": "single GPU (myl_moe_dev)" if world == 1 else
           f"ep{world} ({'peer-memory dispatch and return' if peer else 'NCCL all_to_all'})",
           "tokens_per_rank": Tr, "ms_per_layer": round(ms, 4),
           "tops": round(moe_ops(T) / (ms * 1e-3) / 1e12, 2),
           "tokens_per_s": round(T / (ms * 1e-3), 1),
           "ops_per_layer": moe_ops(T), "gpu_launches_per_layer": launches / steps,
           "expert_rows_min_max_rank0": [int(load.min()), int(load.max())]}
    if world == 1:
        # end to end through the host-pointer entry point (myl_moe_forward)
        xp = torch.from_numpy(x_h).pin_memory().numpy()
        yp = torch.empty((Tr, H), dtype=torch.int16).pin_memory().numpy()
        L = myl.load_library()
        for _ in range(warmup):
            myl._check("myl_moe_forward", L.myl_moe_forward(ctx.handle, moe.handle, xp.ctypes.data, Tr,
                                                            yp.ctypes.data))
        t0 = time.perf_counter()
        for _ in range(steps):
            myl._check("myl_moe_forward", L.myl_moe_forward(ctx.handle, moe.handle, xp.ctypes.data, Tr,
                                                            yp.ctypes.data))
        e2e_s = (time.perf_counter() - t0) / steps
        res["e2e"] = {"ms_per_layer": round(e2e_s * 1e3, 4),
                      "tops": round(moe_ops(T) / e2e_s / 1e12, 2),
                      "h2d_bytes_per_step": int(x_h.nbytes), "d2h_bytes_per_step": int(yp.nbytes)}
    moe.release()
    shared.release()
    if world > 1 and peer:
        epl.close()
    return res


# ---------------------------------------------------------------------------------------
# GPU arm


_JSON_FD = None


def emit(line: dict) -> None:
    """Prints the one JSON line on the process's real stdout (everything else
    that reaches file descriptor 1, e.g. NCCL's version banner, goes to
    stderr; see main)."""
    s = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(s.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, s)


def mlp_decode_gemv(ctx, stream, peaks) -> dict:
    """The decode MLP as the forward runs it (M=1, 7B shapes): the gate/up
    GEMV over the interleaved [2I][H] weight with the SiLU pair epilogue, then
    the down GEMV; two MLPs (407 MB) rotate so the weights stream from HBM."""
    import torch

    import myelith_b200 as myl
    from myelith_b200.synthetic import kbits, silu_lut_spec
    H, I = SHAPES[0][0], SHAPES[0][1]
    rng = np.random.default_rng(11)
    mlps = []
    for _ in range(2):
        mlps.append(myl.Mlp(
            ctx, rng.integers(-127, 128, size=(I, H), dtype=np.int8),
            rng.integers(-127, 128, size=(I, H), dtype=np.int8),
            rng.integers(-127, 128, size=(H, I), dtype=np.int8), H, I,
            np.full(I, kbits(H), np.uint8), np.full(I, kbits(H), np.uint8), np.full(H, kbits(I), np.uint8),
            silu_lut_spec(), 8, 7, 7, 7, 6, 8192, 8, np.full(H, 6, np.uint8)))
    x = torch.from_numpy(np.clip(np.rint(rng.normal(0, 1024, size=(1, H))), -32767, 32767)
                         .astype(np.int16)).to("cuda")
    y = torch.empty((1, H), dtype=torch.int16, device="cuda")
    iters = 20
    with torch.cuda.stream(stream):
        for i in range(3):
            mlps[i % 2].dev(x, y, stream)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(iters):
            mlps[i % 2].dev(x, y, stream)
        b.record(stream)
        stream.synchronize()
    us = a.elapsed_time(b) / iters * 1e3
    wbytes = 3 * H * I
    for m in mlps:
        m.release()
    return {"us": round(us, 2), "weight_gbs": round(wbytes / (us * 1e-6) / 1e9, 1),
            "frac": round(wbytes / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 3),
            "launches": 2, "bytes": "gate/up + down weights (3 * H * I) per call"}


def main() -> None:
    global _JSON_FD
    # Native libraries print to file descriptor 1 (NCCL's banner on rank 0):
    # point it at stderr and keep the real stdout for the JSON line alone.
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--m", type=int, default=M_HEAD)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-moe", action="store_true")
    ap.add_argument("--no-forward", action="store_true")
    ap.add_argument("--sm-reserve", type=int, default=16,
                    help="N>1 with --exchange nccl: SMs left free for the overlapped collectives")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="N>1: row-parallel exchange through peer memory from the GEMM epilogue "
                         "(p2p) or NCCL reduce-scatter + all-gather overlapped with the gate/up GEMM")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    import myelith_b200 as myl

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # the exchanges are tens of MB: NCCL's bandwidth protocol, not the
        # low-latency one it picks otherwise for these int64 buffers
        os.environ.setdefault("NCCL_PROTO", "Simple")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    tp, r = world, rank
    ctx = myl.Context(local)
    stream = torch.cuda.Stream(device=dev)
    M = args.m
    peaks = load_peaks()

    # ---- weights: TP shards, NSETS rotating sets ----
    rng = np.random.default_rng(1000 + r)
    K1, N1 = SHAPES[0]
    K2, N2 = SHAPES[1]
    assert N1 % tp == 0 and K2 % tp == 0
    n1, k2 = N1 // tp, K2 // tp
    per_set = n1 * K1 + N2 * k2
    nsets = max(2, math.ceil(4 * L2_BYTES / per_set))
    # per-channel shifts belong to the full weight: the same on every rank
    srng = np.random.default_rng(999)
    s1 = srng.integers(kbits(K1) - 1, kbits(K1) + 2, size=N1).astype(np.uint8)[r * n1:(r + 1) * n1]
    s2 = srng.integers(kbits(K2) - 1, kbits(K2) + 2, size=N2).astype(np.uint8)
    W1s, W2s, R1s, R2s, host_w = [], [], [], [], []
    for _ in range(nsets):
        h1 = rng.integers(-127, 128, size=(n1, K1), dtype=np.int8)
        h2 = rng.integers(-127, 128, size=(N2, k2), dtype=np.int8)
        host_w.append((h1, h2))  # kept for the parity check of the timed step
        w1 = ctx.weight(h1, K1, s1)
        w2 = ctx.weight(h2, k2, s2)
        W1s.append(w1)
        W2s.append(w2)
        R1s.append(w1.requant(myl.RQ_SHIFT_I16, ACT_FRAC, OUT_FRAC))
        R2s.append(w2.requant(myl.RQ_SHIFT_I16, ACT_FRAC, OUT_FRAC))

    def act(shape):
        return np.clip(np.rint(rng.normal(0, 1024, size=shape)), -32767, 32767).astype(np.int16)

    x1_h, x2_h = act((M, K1)), act((M, k2))
    with torch.cuda.stream(stream):
        x1 = torch.from_numpy(x1_h).to(dev)
        x2 = torch.from_numpy(x2_h).to(dev)
        ldp1, ldp2 = (K1 + 15) // 16 * 16, (k2 + 15) // 16 * 16
        p1h = torch.empty((M, ldp1), dtype=torch.uint8, device=dev)
        p1l = torch.empty((M, ldp1), dtype=torch.uint8, device=dev)
        p2h = torch.empty((M, ldp2), dtype=torch.uint8, device=dev)
        p2l = torch.empty((M, ldp2), dtype=torch.uint8, device=dev)
        y1 = torch.empty((M, n1), dtype=torch.int16, device=dev)
        y2 = torch.empty((M, N2), dtype=torch.int16, device=dev)
        acc2 = torch.empty((M, N2), dtype=torch.int64, device=dev) if tp > 1 else None
    stream.synchronize()

    gemm_events: list = []

    def step(i: int, record: bool) -> None:
        s = i % nsets
        ctx.split_hilo_dev(x1, p1h, p1l, stream)
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        W1s[s].linear_planes_dev(R1s[s], p1h, p1l, M, y1, stream)
        if record:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(stream)
        ctx.split_hilo_dev(x2, p2h, p2l, stream)
        if record:
            e2 = torch.cuda.Event(enable_timing=True)
            e2.record(stream)
        if tp == 1:
            W2s[s].linear_planes_dev(R2s[s], p2h, p2l, M, y2, stream)
        else:
            W2s[s].linear_planes_dev(None, p2h, p2l, M, acc2, stream)
        if record:
            e3 = torch.cuda.Event(enable_timing=True)
            e3.record(stream)
            gemm_events.append((e0, e1))
            gemm_events.append((e2, e3))
        if tp > 1:
            dist.all_reduce(acc2, op=dist.ReduceOp.SUM)
            R2s[s].apply_acc_dev(acc2, y2, stream)

    # Tensor-parallel step with the exchange overlapped: the row-parallel down
    # projection runs first and its int64 partials go to a reduce-scatter
    # (NCCL, async) while the column-parallel gate/up projection computes on
    # the SMs the collective leaves free (myl_set_sm_limit); each rank
    # requantises its share of the rows and an all-gather of the int16 rows
    # gives every rank the full output, bit-identical to the all-reduce form.
    from myelith_b200.tp import overlapped_row_parallel

    def step_tp(i: int, record: bool) -> None:
        s = i % nsets
        ctx.split_hilo_dev(x2, p2h, p2l, stream)
        if record:
            e2 = torch.cuda.Event(enable_timing=True)
            e2.record(stream)

        def compute_acc(r0, r1, out):  # alone on the GPU: all SMs
            ctx.set_sm_limit(0)
            W2s[s].linear_planes_dev(None, p2h[r0:r1], p2l[r0:r1], r1 - r0, out, stream)
            ctx.set_sm_limit(max(1, ctx.num_sms - args.sm_reserve))

        def requant(acc, y):
            R2s[s].apply_acc_dev(acc, y, stream)

        ev = {}

        def gate_up():  # column-parallel, no exchange: overlaps the reduce-scatters
            if record:
                ev["e3"] = torch.cuda.Event(enable_timing=True)
                ev["e3"].record(stream)
            ctx.split_hilo_dev(x1, p1h, p1l, stream)
            if record:
                ev["e0"] = torch.cuda.Event(enable_timing=True)
                ev["e0"].record(stream)
            W1s[s].linear_planes_dev(R1s[s], p1h, p1l, M, y1, stream)
            if record:
                ev["e1"] = torch.cuda.Event(enable_timing=True)
                ev["e1"].record(stream)

        # one chunk: the down projection at full M keeps its tiles dense; its
        # reduce-scatter overlaps the gate/up projection instead
        y2.copy_(overlapped_row_parallel(compute_acc, requant, M, N2, tp, None, 1, dev, gate_up))
        if record:
            gemm_events.append((ev["e0"], ev["e1"]))
            gemm_events.append((e2, ev["e3"]))

    # Tensor-parallel step with the peer-memory exchange: the down projection's
    # GEMM stores its int64 partial rows into the owning ranks' receive
    # buffers (NVLink) from its epilogue; gate/up computes before the ranks
    # synchronise; then each rank sums and requantises its rows and writes
    # them into every rank's output (tp.PeerExchange).
    xchg = None
    p2p_out: dict = {}
    if tp > 1 and args.exchange == "p2p":
        from myelith_b200.tp import PeerExchange

        with torch.cuda.stream(stream):
            xchg = PeerExchange(ctx, M, N2, rank, world)

    def step_p2p(i: int, record: bool) -> None:
        s = i % nsets
        ev = {}

        def gate_up():
            ctx.split_hilo_dev(x1, p1h, p1l, stream)
            if record:
                ev["e0"] = torch.cuda.Event(enable_timing=True)
                ev["e0"].record(stream)
            W1s[s].linear_planes_dev(R1s[s], p1h, p1l, M, y1, stream)
            if record:
                ev["e1"] = torch.cuda.Event(enable_timing=True)
                ev["e1"].record(stream)

        p2p_out["y2"] = xchg(W2s[s], R2s[s], x2, stream, between=gate_up)  # a view, no copy
        if record:  # the gate/up GEMM carries the same work per rank as the down GEMM
            gemm_events.append((ev["e0"], ev["e1"]))

    tp_check = None
    if tp > 1:
        # the tensor-parallel step must equal the all-reduce step bit for bit
        step_x = step_p2p if xchg is not None else step_tp
        if xchg is not None:
            ctx.set_sm_limit(0)
        with torch.cuda.stream(stream):
            step(0, False)
            ref_y2 = y2.clone()
            y2.zero_()
            step_x(0, False)
            got = p2p_out.get("y2", y2)
            same = torch.tensor([int(torch.equal(ref_y2, got))], dtype=torch.int32, device=dev)
        stream.synchronize()
        if not bool(same.item()):
            bad = (ref_y2 != got).any(dim=1).nonzero().flatten().tolist()
            print(f"rank {rank}: overlapped step differs in {len(bad)} rows, first {bad[:8]}",
                  file=sys.stderr, flush=True)
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        tp_check = bool(same.item())
        del ref_y2
        if xchg is None:
            ctx.set_sm_limit(max(1, ctx.num_sms - args.sm_reserve))
        step = step_x

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if os.environ.get("MYL_BENCH_TRACE") and world > 1:  # one traced step per rank (diagnostics)
        from torch.profiler import ProfilerActivity, profile

        with torch.cuda.stream(stream):
            for i in range(3):
                step(i, False)
            stream.synchronize()
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                step(3, False)
                stream.synchronize()
        evs = sorted([e for e in prof.events() if e.device_type.name == "CUDA"],
                     key=lambda e: e.time_range.start)
        t0 = evs[0].time_range.start if evs else 0
        with open(os.path.join(os.environ["MYL_BENCH_TRACE"], f"trace_rank{rank}.txt"), "w") as f:
            for e in evs:
                f.write(f"{(e.time_range.start - t0) / 1e3:9.3f} ms +{(e.time_range.end - e.time_range.start) / 1e3:8.3f}"
                        f"  {e.name[:90]}\n")
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i, False)
        stream.synchronize()
        barrier()
        torch.cuda.synchronize()
        sampler = ClockSampler(local)
        sampler.start()
        if sampler.handle is None:
            time.sleep(0.3)  # nvidia-smi needs a moment to start
        launches0 = ctx.launch_count
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        w0 = time.perf_counter()
        for i in range(args.steps):
            step(args.warmup + i, True)
        t_end.record(stream)
        stream.synchronize()
        wall = time.perf_counter() - w0
        launches = ctx.launch_count - launches0
        clocks = sampler.stop()
        barrier()
        torch.cuda.synchronize()
    ctx.synchronize()
    dev_ms = t_start.elapsed_time(t_end)
    dev_ms = max_over_ranks(dev_ms)

    # ---- parity of the last timed step: every output element against the oracle ----
    import oracle as O

    O.set_num_threads(max(1, (os.cpu_count() or 1) // world))
    t0 = time.perf_counter()
    s_last = (args.warmup + args.steps - 1) % nsets
    h1, h2 = host_w[s_last]
    want1 = O.linear_w8a16_fast(x1_h, h1.reshape(-1), K1, s1, ACT_FRAC, OUT_FRAC)
    got1 = y1.cpu().numpy()
    if tp == 1:
        want2 = O.linear_w8a16_fast(x2_h, h2.reshape(-1), k2, s2, ACT_FRAC, OUT_FRAC)
    else:  # row-parallel: the ranks' exact partials, summed, requantised once
        acc = torch.from_numpy(O.linear_acc_fast(x2_h, h2.reshape(-1), k2, N2)).to(dev)
        dist.all_reduce(acc, op=dist.ReduceOp.SUM)
        want2 = O.requant_acc(acc.cpu().numpy(), s2, ACT_FRAC, OUT_FRAC)
    got2 = p2p_out.get("y2", y2).cpu().numpy()
    ok = int(np.array_equal(got1, want1) and np.array_equal(got2, want2))
    if world > 1:
        t = torch.tensor([ok], dtype=torch.int32, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = int(t.item())
    parity = {"ok": bool(ok), "elements": int(want1.size + want2.size) * (world if tp > 1 else 1),
              "checked": "every output of the last timed step, both shapes, against the CPU oracle"
                         + (" (row-parallel: the ranks' int64 partials summed)" if tp > 1 else ""),
              "oracle_s": round(time.perf_counter() - t0, 1)}
    del want1, want2, got1, got2
    ops_step = 2.0 * M * sum(K * N for K, N in SHAPES)
    value = ops_step * args.steps / (dev_ms * 1e-3) / 1e12
    gemm_ms = [a.elapsed_time(b) for a, b in gemm_events]
    gemm_avg_ms = statistics.mean(gemm_ms)
    gemm_ops = 2.0 * M * (n1 * K1)  # per launch; both shapes carry the same work per rank
    achieved = gemm_ops / (gemm_avg_ms * 1e-3) / 1e12
    long_step = dev_ms > 1000.0
    int8_dense = 2.0 * (peaks["bf16_tflops_sustained"] if long_step else peaks["bf16_tflops"])
    eff_peak = int8_dense / 2.0
    traffic = load_traffic().get(f"gemm_tc_M{M}_tp{tp}")

    # ---- e2e: host buffers through the reference-facing call ----
    e2e = None
    if tp == 1:
        x1_pin = torch.from_numpy(x1_h).pin_memory().numpy()
        x2_pin = torch.from_numpy(x2_h).pin_memory().numpy()
        y1_pin = torch.empty((M, n1), dtype=torch.int16).pin_memory().numpy()
        y2_pin = torch.empty((M, N2), dtype=torch.int16).pin_memory().numpy()
        L = myl.load_library()

        def e2e_step(i):
            s = i % nsets
            myl._check("myl_linear_w8a16", L.myl_linear_w8a16(
                ctx.handle, W1s[s].handle, x1_pin.ctypes.data, M, ACT_FRAC, OUT_FRAC, y1_pin.ctypes.data))
            myl._check("myl_linear_w8a16", L.myl_linear_w8a16(
                ctx.handle, W2s[s].handle, x2_pin.ctypes.data, M, ACT_FRAC, OUT_FRAC, y2_pin.ctypes.data))

        for i in range(args.warmup):
            e2e_step(i)
        t0 = time.perf_counter()
        for i in range(args.steps):
            e2e_step(i)
        e2e_s = time.perf_counter() - t0
        # pageable host memory, as a Rust caller's Vec<i16> (linear.rs:43) is
        y1_pg = np.empty((M, n1), np.int16)
        y2_pg = np.empty((M, N2), np.int16)

        def e2e_pageable(i):
            s = i % nsets
            myl._check("myl_linear_w8a16", L.myl_linear_w8a16(
                ctx.handle, W1s[s].handle, x1_h.ctypes.data, M, ACT_FRAC, OUT_FRAC, y1_pg.ctypes.data))
            myl._check("myl_linear_w8a16", L.myl_linear_w8a16(
                ctx.handle, W2s[s].handle, x2_h.ctypes.data, M, ACT_FRAC, OUT_FRAC, y2_pg.ctypes.data))

        for i in range(args.warmup):
            e2e_pageable(i)
        t0 = time.perf_counter()
        for i in range(args.steps):
            e2e_pageable(i)
        pg_s = time.perf_counter() - t0
        e2e = {"value": ops_step * args.steps / e2e_s / 1e12, "unit": "TOPS",
               "h2d_bytes_per_step": int(x1_h.nbytes + x2_h.nbytes),
               "d2h_bytes_per_step": int(y1_pin.nbytes + y2_pin.nbytes),
               "path": "myl_linear_w8a16 (host pointers, pinned), both shapes",
               "pageable": {"value": round(ops_step * args.steps / pg_s / 1e12, 3), "unit": "TOPS",
                            "path": "myl_linear_w8a16 on pageable numpy buffers (a Vec<i16>)"}}
    else:
        x1_pin = torch.from_numpy(x1_h).pin_memory()
        x2_pin = torch.from_numpy(x2_h).pin_memory()
        y2_pin = torch.empty((M, N2), dtype=torch.int16).pin_memory()
        y1_pin = torch.empty((M, n1), dtype=torch.int16).pin_memory()

        def e2e_step(i):
            x1.copy_(x1_pin, non_blocking=True)
            x2.copy_(x2_pin, non_blocking=True)
            step(i, False)
            y1_pin.copy_(y1, non_blocking=True)
            y2_pin.copy_(y2, non_blocking=True)
            stream.synchronize()

        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                e2e_step(i)
            barrier()
            t0 = time.perf_counter()
            for i in range(args.steps):
                e2e_step(i)
            e2e_s = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": ops_step * args.steps / e2e_s / 1e12, "unit": "TOPS",
               "h2d_bytes_per_step": int(x1_h.nbytes + x2_h.nbytes),
               "d2h_bytes_per_step": int(y1_pin.numel() * 2 + y2_pin.numel() * 2),
               "path": "host copies + tensor-parallel device step per rank"}

    # ---- M sweep and decode GEMV (N=1 only) ----
    sweep, gemv = None, None
    if tp == 1 and not args.no_sweep:
        sweep = []
        gemv_gbs = []
        for Ms in SWEEP_M:
            xs = {K: torch.from_numpy(act((Ms, K))).to(dev) for K, _ in SHAPES}
            ys = {N: torch.empty((Ms, N), dtype=torch.int16, device=dev) for _, N in SHAPES}
            res = {}
            for j, (K, N) in enumerate(SHAPES):
                Ws, Rs = (W1s, R1s) if j == 0 else (W2s, R2s)
                iters = 20 if Ms <= 128 else 8
                with torch.cuda.stream(stream):
                    for i in range(3):
                        Ws[i % nsets].linear_dev(Rs[i % nsets], xs[K], ys[N], stream)
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    for i in range(iters):
                        Ws[i % nsets].linear_dev(Rs[i % nsets], xs[K], ys[N], stream)
                    b.record(stream)
                    stream.synchronize()
                ms = a.elapsed_time(b) / iters
                tops = 2.0 * Ms * K * N / (ms * 1e-3) / 1e12
                bytes_ = N * K + 2 * Ms * K + 2 * Ms * N + N
                gbs = bytes_ / (ms * 1e-3) / 1e9
                res[f"{K}x{N}"] = {"us": round(ms * 1e3, 2), "tops": round(tops, 2), "gbs": round(gbs, 1)}
                if Ms == 1:
                    gemv_gbs.append(gbs)
            sweep.append({"M": Ms, **res})
        ctx.synchronize()
        gemv = {"gbs": round(statistics.mean(gemv_gbs), 1), "peak_gbs": peaks["hbm_gbs"],
                "frac": round(statistics.mean(gemv_gbs) / peaks["hbm_gbs"], 3),
                "per_shape_gbs": [round(g, 1) for g in gemv_gbs],
                "bytes": "N*K weights + 2K act + 2N out + N shift bytes per launch",
                "mlp_decode": None}
        try:
            gemv["mlp_decode"] = mlp_decode_gemv(ctx, stream, peaks)
        except myl.MylError as e:  # a measurement side leg: report, do not abort the bench
            gemv["mlp_decode"] = {"error": str(e)}

    # ---- the integer forward, configs 2 and 3 (N=1), config 3 tensor-parallel (N>1) ----
    forward = None
    if tp > 1 and not args.no_forward:
        forward = {"config3": bench_forward_tp(
            ctx, FWD_CFG3, max(1, min(args.steps, 3)), 1, rank, world, max_over_ranks,
            int(os.environ.get("MYL_CFG3_CHECK_PROMPT", "64")),
            int(os.environ.get("MYL_CFG3_CHECK_NEW", "16")))}
    if tp == 1 and not args.no_forward:
        fs, fw = max(1, min(args.steps, 3)), 1
        forward = {
            "config2": bench_forward(ctx, FWD_CFG2, fs, fw, peaks["hbm_gbs"], 1 << 30, 0),
            "config3": bench_forward(ctx, FWD_CFG3, fs, fw, peaks["hbm_gbs"],
                                     int(os.environ.get("MYL_CFG3_CHECK_PROMPT", "64")),
                                     int(os.environ.get("MYL_CFG3_CHECK_NEW", "16"))),
        }

    # ---- MoE layer (config 4): every rank takes part (all_to_all at N > 1) ----
    moe = None
    if not args.no_moe:
        moe = bench_moe(ctx, dev, stream, rank, world, local, max(3, args.steps // 2), args.warmup,
                        max_over_ranks, barrier, peer=args.exchange == "p2p")

    # ---- CPU baseline (rank 0, N=1) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample_tops(float(os.environ.get("MYL_CPU_SAMPLE_S", "8.0")),
                              np.random.default_rng(77))
        cpu.pop("seconds", None)

    if world > 1:
        barrier()
    all_parity = parity["ok"] and (forward is None or all(f["parity"] for f in forward.values()))
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3) if all_parity else None, "unit": "TOPS",
            "n_gpus": world, "parity": bool(all_parity), "parity_config1": parity,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8xint16->int64", "data": "synthetic",
            "config": config1(tp, "p2p" if xchg is not None else "nccl") if M == M_HEAD else
            dict(config1(tp, "p2p" if xchg is not None else "nccl"), M=M),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(eff_peak, 1),
                         "unit": "TFLOP/s", "frac": round(achieved / eff_peak, 4),
                         "traffic": traffic,
                         "kernel": "gemm_w8a16_tc_kernel", "launches": len(gemm_ms),
                         "avg_us": round(gemm_avg_ms * 1e3, 2),
                         "peak_basis": ("effective split-byte peak = int8 dense / 2; int8 dense = 2 x "
                                        f"cuBLAS bf16 {'sustained' if long_step else 'burst'} "
                                        f"({peaks['source']} MEASURED_PEAKS)"),
                         "ops": "integer ops, 2 per algorithmic MAC; the tensor pipe runs 2x these"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "wall_s_timed": round(wall, 4),
            "gemv": gemv,
            "sweep": sweep,
            "moe": moe,
            "forward": forward,
            "tp_check": tp_check,
        }
        emit(line)
    if xchg is not None:
        xchg.close()
    if world > 1:
        dist.destroy_process_group()
    if not all_parity:
        sys.exit(1)  # no number without a passing parity check in the same run


if __name__ == "__main__":
    main()
