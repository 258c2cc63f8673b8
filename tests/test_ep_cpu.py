"""Expert-parallel MoE host logic on CPU (gloo, world size 2 and 3).

myelith_b200.ep routes each rank's tokens, sends every (token, choice) pair
to the rank owning its expert (all_to_all of counts, rows and ids), runs the
experts there and sends the results back for the combine. Here each rank's
arithmetic is the CPU oracle (OracleMoeLocal, test-only) and the exchange
runs over gloo; every rank's output must equal the single-device oracle layer
on its tokens bit for bit, with uneven expert shares and ranks that receive
no rows.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import moe_ref as R
import oracle as O
from myelith_b200 import ep


class OracleMoeLocal(ep.MoeLocal):
    """Per-rank MoE arithmetic on the CPU oracle, holding experts [first, last)."""

    def __init__(self, p, s, first, last):
        self.p, self.s, self.first, self.last = p, s, first, last
        self.rows_seen = 0

    def route(self, x):
        idx, prob = R.route(self.p, x.numpy())
        return torch.from_numpy(idx), torch.from_numpy(prob)

    def experts(self, rows, ids):
        ids_np = ids.numpy()
        assert ((ids_np >= self.first) & (ids_np < self.last)).all(), "row sent to the wrong rank"
        self.rows_seen += len(ids_np)
        return torch.from_numpy(R.experts(self.p, rows.numpy(), ids_np))

    def shared(self, x):
        return None if self.s is None else torch.from_numpy(R.shared_mlp(self.s, x.numpy()))

    def combine(self, y, prob, shared):
        T, k = prob.shape
        sh = shared.numpy() if shared is not None else np.zeros((T, self.p["hidden"]), np.int16)
        return torch.from_numpy(O.moe_combine(y.numpy().reshape(T, k, -1), prob.numpy(), sh,
                                              self.p["prob_frac"]))


def _tokens(rank, T0=23):
    return R.activations(np.random.default_rng(100 + rank), T0 + 5 * rank, 64)


def _worker(rank, world, port, E, k, skew, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p, s = R.problem(H=64, I=48, E=E, k=k, shared_I=40, seed=21)
        if skew:
            # experts 0..k-1 win every token: the other ranks receive no rows
            p["W_router"][:] = 0
            p["W_router"][:k] = 0
            p["router_w_shifts"][:] = 0
            p["W_router"][:k, 0] = 127
        first, last = ep.shard_range(E, rank, world)
        local = OracleMoeLocal(p, s, first, last)
        layer = ep.ExpertParallelMoe(local, E, k, 64, rank, world)
        x = _tokens(rank)
        if skew:
            x[:, 0] = 1000
        out = layer(torch.from_numpy(x)).numpy()
        ref = R.forward(p, s, x)[0]
        results[rank] = (bool(np.array_equal(out, ref)), local.rows_seen, (first, last))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, E, k, skew=False):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), E, k, skew, results), nprocs=world,
                           start_method="spawn", join=True)
        return dict(results)


@pytest.mark.parametrize("world,E,k", [(2, 8, 2), (3, 5, 2), (3, 7, 3)])
def test_expert_parallel_gloo(world, E, k):
    res = _run(world, E, k)
    assert sorted(res) == list(range(world))
    for rank, (ok, _, _) in res.items():
        assert ok, f"rank {rank}: expert-parallel output differs from the single-device layer"
    # every pair is computed exactly once somewhere
    total_pairs = sum((23 + 5 * r) * k for r in range(world))
    assert sum(v[1] for v in res.values()) == total_pairs
    spans = sorted(v[2] for v in res.values())
    assert spans[0][0] == 0 and spans[-1][1] == E


def test_expert_parallel_ranks_without_rows():
    res = _run(2, 8, 2, skew=True)
    assert all(v[0] for v in res.values())
    assert res[1][1] == 0  # rank 1 holds experts 4..7, which no token chooses


def test_expert_owner():
    assert ep.expert_owner(8, 2).tolist() == [0, 0, 0, 0, 1, 1, 1, 1]
    assert ep.expert_owner(5, 3).tolist() == [0, 0, 1, 1, 2]


def test_device_owner_formula_matches_shard_ranges():
    """ep_dispatch_kernel finds the rank owning expert e without a table:
    with base, extra = divmod(E, world), experts below extra * (base + 1)
    belong to rank e // (base + 1), the rest to extra + (e - that) // base.
    The same integer steps here against the shard ranges of expert_owner."""
    from myelith_b200.ep import expert_owner

    for E in (1, 2, 3, 7, 8, 63, 64, 65, 100, 256):
        for world in range(1, 9):
            if E < world:
                continue
            base, extra = divmod(E, world)
            big = extra * (base + 1)
            own = [e // (base + 1) if e < big else extra + (e - big) // max(base, 1) for e in range(E)]
            assert own == expert_owner(E, world).tolist(), (E, world)
