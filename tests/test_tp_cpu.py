"""Tensor-parallel host logic on CPU (gloo, world size 2 and 3).

The layers of myelith_b200.tp shard a linear by output rows (column-parallel)
or input columns (row-parallel, int64 partial sums all-reduced, one requant
after the sum) and the MLP by intermediate channels. Here every rank computes
its shard with the CPU oracle (OracleLocal, test-only) and the exchange runs
over gloo; the gathered / reduced outputs must equal the unsharded oracle
result bit for bit, including uneven shards.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import gen
import oracle as O
from make_golden import silu_lut_spec
from myelith_b200 import selection_key, tp


def rne_shift_np(acc, s):
    """Vectorised rescale_i64 (fixed_point.rs:57-71, :184-191)."""
    acc = acc.astype(np.int64)
    s = np.broadcast_to(np.asarray(s, np.int64), acc.shape)
    pos = np.maximum(s, 1)
    q = acc >> pos
    r = acc & ((np.int64(1) << pos) - 1)
    h = np.int64(1) << (pos - 1)
    right = q + ((r > h) | ((r == h) & ((q & 1) == 1))).astype(np.int64)
    return np.where(s > 0, right, np.where(s == 0, acc, acc << np.maximum(-s, 0)))


class OracleLocal(tp.Local):
    """Per-rank arithmetic on the CPU oracle (test infrastructure)."""

    def __init__(self):
        self.lin, self.mlps = {}, {}

    def add_linear(self, key, W, in_features, w_shifts, act_frac, out_frac):
        self.lin[key] = (np.asarray(W, np.int8), in_features, np.asarray(w_shifts, np.uint8), act_frac,
                         out_frac)

    def add_mlp(self, key, a):
        self.mlps[key] = a

    def linear(self, key, x):
        W, K, ws, af, of = self.lin[key]
        fn = O.linear_w8a16 if np.ndim(of) == 0 else O.linear_w8a16_pc
        return torch.from_numpy(fn(x.numpy(), W.reshape(-1), K, ws, af, of))

    def acc(self, key, x):
        if key in self.mlps:
            a = self.mlps[key]
            h = O.mlp_hidden(x.numpy(), a["W_gate"], a["W_up"], a["hidden"], a["intermediate"],
                             a["gate_w_shifts"], a["up_w_shifts"], a["silu_lut"], a["in_frac"],
                             a["gate_out_frac"], a["up_out_frac"], a["down_in_frac"], a["silu_in_frac"],
                             a["silu_lut_offset"], a["silu_out_frac"])
            return torch.from_numpy(O.linear_acc_i64(h, a["W_down"].reshape(-1), a["intermediate"],
                                                     a["hidden"]))
        W, K, ws, af, of = self.lin[key]
        return torch.from_numpy(O.linear_acc_i64(x.numpy(), W.reshape(-1), K, W.shape[0]))

    def requant(self, key, acc):
        if key in self.mlps:
            a = self.mlps[key]
            s = a["down_w_shifts"].astype(np.int64) + a["down_in_frac"] - a["out_frac"].astype(np.int64)
        else:
            W, K, ws, af, of = self.lin[key]
            s = ws.astype(np.int64) + af - np.asarray(of, np.int64)
        return torch.from_numpy(np.clip(rne_shift_np(acc.numpy(), s[None, :]), -32768, 32767)
                                .astype(np.int16))

    def add_lm_head(self, key, W, in_features, w_shifts, final_norm_frac, logit_frac):
        self.lin[key] = (np.asarray(W, np.int8), in_features, np.asarray(w_shifts, np.uint8),
                         final_norm_frac, logit_frac)

    def lm_head_logits(self, key, x):
        W, K, ws, nf, lf = self.lin[key]
        return torch.from_numpy(O.lm_head_w8a16_i32(x.numpy(), W.reshape(-1), K, ws, nf, lf))

    def lm_head_keys(self, key, x, index_base):
        logits = self.lm_head_logits(key, x).numpy()
        if logits.shape[1] == 0:
            return torch.full((logits.shape[0],), -(2**63), dtype=torch.int64)
        keys = [selection_key(int(r.max()), index_base + O.argmax_int(r)) for r in logits]
        return torch.tensor(keys, dtype=torch.int64)


def _problem(seed=3):
    rng = np.random.default_rng(seed)
    M, K, N = 5, 37, 33  # uneven: 37 and 33 do not split evenly over 2 or 3 ranks
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    ws = rng.integers(6, 10, size=N).astype(np.uint8)
    of = rng.integers(2, 6, size=N).astype(np.uint8)
    x = rng.integers(-4000, 4000, size=(M, K), dtype=np.int16)
    H, I = 24, 29
    mlp = dict(W_gate=rng.integers(-127, 128, size=(I, H), dtype=np.int8),
               W_up=rng.integers(-127, 128, size=(I, H), dtype=np.int8),
               W_down=rng.integers(-127, 128, size=(H, I), dtype=np.int8),
               hidden=H, intermediate=I,
               gate_w_shifts=rng.integers(7, 10, size=I).astype(np.uint8),
               up_w_shifts=rng.integers(7, 10, size=I).astype(np.uint8),
               down_w_shifts=rng.integers(7, 10, size=H).astype(np.uint8),
               silu_lut=silu_lut_spec(), in_frac=6, gate_out_frac=6, up_out_frac=6, down_in_frac=6,
               silu_in_frac=6, silu_lut_offset=8192, silu_out_frac=8,
               out_frac=rng.integers(3, 7, size=H).astype(np.uint8))
    xm = rng.integers(-3000, 3000, size=(M, H), dtype=np.int16)
    return W, ws, of, x, mlp, xm


def _lm_head_problem(seed=4):
    """Vocab 41 (uneven shards) whose second half repeats rows of the first, so
    the maximum of a token often sits in two shards: the lower index wins."""
    rng = np.random.default_rng(seed)
    V, K, M = 41, 19, 6
    W = rng.integers(-8, 8, size=(V, K), dtype=np.int8)
    W[21:] = W[:20]
    ws = np.full(V, 3, np.uint8)
    x = rng.integers(-40, 40, size=(M, K), dtype=np.int16)
    return W, ws, x


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W, ws, of, x, mlp, xm = _problem()
        K = W.shape[1]
        local = OracleLocal()
        xt = torch.from_numpy(x)
        col = tp.ColumnParallelLinear(local, "col", tp.LinearSpec(W, ws, 6, of), rank, world)
        y_col = col.gather(xt).numpy()
        row = tp.RowParallelLinear(local, "row", tp.LinearSpec(W, ws, 6, of), rank, world)
        y_row = row(row.x_shard(xt)).numpy()
        # the overlapped exchange (reduce-scatter, requant, all-gather) in row chunks
        x8 = torch.from_numpy(np.concatenate([x, x[::-1], x, x[::-1]])[: 4 * world * 2])
        y_ov = row.overlapped(row.x_shard(x8), chunks=2).numpy()
        ref_ov = O.linear_w8a16_pc(x8.numpy(), W.reshape(-1), K, ws, 6, of)
        ov_ok = bool(np.array_equal(y_ov, ref_ov))
        pm = tp.ParallelMlp(local, "mlp", **{k: v for k, v in mlp.items() if k not in ("hidden", "intermediate")},
                            hidden=mlp["hidden"], intermediate=mlp["intermediate"], rank=rank, world=world)
        y_mlp = pm(torch.from_numpy(xm)).numpy()
        ref = O.linear_w8a16_pc(x, W.reshape(-1), K, ws, 6, of)
        ref_mlp = O.mlp_int(xm, mlp["W_gate"], mlp["W_up"], mlp["W_down"], mlp["hidden"],
                            mlp["intermediate"], mlp["gate_w_shifts"], mlp["up_w_shifts"],
                            mlp["down_w_shifts"], mlp["silu_lut"], mlp["in_frac"], mlp["gate_out_frac"],
                            mlp["up_out_frac"], mlp["down_in_frac"], mlp["silu_in_frac"],
                            mlp["silu_lut_offset"], mlp["silu_out_frac"], mlp["out_frac"])
        # vocab-parallel greedy selection: one int64 MAX all-reduce
        Wl, wsl, xl = _lm_head_problem()
        head = tp.VocabParallelLMHead(local, "head", Wl, wsl, 2, 1, rank, world)
        tok, best = head.greedy(torch.from_numpy(xl))
        full = O.lm_head_w8a16_i32(xl, Wl.reshape(-1), Wl.shape[1], wsl, 2, 1)
        ref_tok = [O.argmax_int(r) for r in full]
        head_ok = tok.tolist() == ref_tok and best.tolist() == [int(r.max()) for r in full]
        results[rank] = (bool(np.array_equal(y_col, ref)), bool(np.array_equal(y_row, ref) and ov_ok),
                         bool(np.array_equal(y_mlp, ref_mlp) and head_ok), (col.lo, col.hi),
                         (row.lo, row.hi))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_tensor_parallel_layers_gloo(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world,
                           start_method="spawn", join=True)
        res = dict(results)
    assert sorted(res) == list(range(world))
    for rank, (col_ok, row_ok, mlp_ok, _, _) in res.items():
        assert col_ok, f"rank {rank}: column-parallel output differs"
        assert row_ok, f"rank {rank}: row-parallel output differs"
        assert mlp_ok, f"rank {rank}: parallel MLP or vocab-parallel greedy output differs"
    # shards tile the dimension exactly
    cols = sorted(r[3] for r in res.values())
    assert cols[0][0] == 0 and cols[-1][1] == 33 and all(a[1] == b[0] for a, b in zip(cols, cols[1:]))


def test_shard_range():
    for n in (0, 1, 7, 33, 18944):
        for world in (1, 2, 3, 8):
            parts = [tp.shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        tp.shard_range(4, 2, 2)
