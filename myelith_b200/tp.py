"""Megatron-style tensor parallelism for the W8A16 path (one process per GPU).

The reference distributes only by layer ranges over TCP
(INTEGER_LLM/pipeline/src/stage.rs:94); inside a layer everything is one
dot product per output element (kernels/src/linear.rs:61-68). Splitting a
layer across GPUs keeps the result bit-identical because the accumulator is an
exact integer:

  column-parallel  rank r owns output rows [lo_r, hi_r): its outputs are final
                   (same requant per row), no exchange;
  row-parallel     rank r owns input columns [lo_r, hi_r): it produces exact
                   int64 partial sums, the ranks add them (all-reduce, int64,
                   SUM; integer addition is associative) and the requant and
                   clamp run once, after the sum, as the reference's clamp at
                   the very end requires (fixed_point.rs:184-191);
  MLP              gate/up column-parallel and down row-parallel over the same
                   intermediate channels, so h never leaves its rank.
  LM head          vocab-parallel (column-parallel over vocab rows); greedy
                   selection needs no logits exchange: each rank reduces its
                   logits to one int64 key per token (logit, then lowest
                   index; argmax_int, sampling.rs:8-18) and one int64 MAX
                   all-reduce gives the global token.

int32 is not wide enough for the partial sums (up to ~1e10 for 7B shapes).

Row-parallel exchange without a collective library in the data path
(PeerExchange): the down/o projection's GEMM stores each exact int64 partial
row straight into the receive buffer of the rank that owns the row (peer
memory over NVLink, buffers shared through CUDA IPC), a one-element
barrier orders the ranks (flag words in peer memory, written and polled by a
one-block kernel on the stream), each rank sums its rows' slabs, requantises
and writes the int16 rows into every rank's output buffer, and a second
barrier orders the ranks again. The transfers ride inside the GEMM's epilogue
instead of a separate reduce-scatter and all-gather, and no collective
library is on the data path.

The per-rank arithmetic is behind ``Local``: ``LibLocal`` calls the sm_100a
kernels (torch CUDA tensors, NCCL); tests can supply another implementation
of the same three methods to run the sharding and exchange logic with gloo on
CPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of rank's share of n items: equal parts, the first n % world
    ranks take one more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class Local:
    """Per-rank arithmetic used by the tensor-parallel layers. The layers hand
    their shards over with add_linear / add_mlp and then call linear / acc /
    requant with the same key."""

    def add_linear(self, key, W, in_features, w_shifts, act_frac, out_frac):
        raise NotImplementedError

    def add_mlp(self, key, args: dict):  # ParallelMlp.args of this rank's slice
        raise NotImplementedError

    def linear(self, key, x):  # requantised output of a weight shard
        raise NotImplementedError

    def acc(self, key, x):  # exact int64 partial sums of a weight shard
        raise NotImplementedError

    def requant(self, key, acc):  # requant of summed int64 accumulators
        raise NotImplementedError

    def add_lm_head(self, key, W, in_features, w_shifts, final_norm_frac, logit_frac):
        raise NotImplementedError

    def lm_head_logits(self, key, x):  # int32 logits of a vocab shard
        raise NotImplementedError

    def lm_head_keys(self, key, x, index_base):  # int64 selection key per token
        raise NotImplementedError


@dataclass
class LinearSpec:
    """One W8A16 linear: W [N][K] int8 (host), one shift per row, scales."""

    W: np.ndarray
    w_shifts: np.ndarray
    act_frac: int
    out_frac: object  # int, or per-channel array (linear_w8a16_pc)


class LibLocal(Local):
    """The sm_100a kernels through libmyl_w8a16 (torch CUDA tensors)."""

    def __init__(self, ctx):
        import torch

        self.ctx = ctx
        self.torch = torch
        self.weights = {}
        self.plans = {}
        self.mlps = {}

    def add_linear(self, key, W, in_features, w_shifts, act_frac, out_frac):
        import myelith_b200 as myl

        w = myl.Weight(self.ctx, W, in_features, w_shifts)
        self.weights[key] = w
        self.plans[key] = w.requant(myl.RQ_SHIFT_I16, act_frac, out_frac)

    def add_mlp(self, key, a: dict):
        import myelith_b200 as myl

        self.mlps[key] = myl.Mlp(self.ctx, a["W_gate"], a["W_up"], a["W_down"], a["hidden"],
                                 a["intermediate"], a["gate_w_shifts"], a["up_w_shifts"],
                                 a["down_w_shifts"], a["silu_lut"], a["in_frac"], a["gate_out_frac"],
                                 a["up_out_frac"], a["down_in_frac"], a["silu_in_frac"],
                                 a["silu_lut_offset"], a["silu_out_frac"], a["out_frac"])

    def linear(self, key, x):
        w = self.weights[key]
        y = self.torch.empty((x.shape[0], w.out_features), dtype=self.torch.int16, device=x.device)
        w.linear_dev(self.plans[key], x, y)
        return y

    def acc(self, key, x):
        if key in self.mlps:
            m = self.mlps[key]
            acc = self.torch.empty((x.shape[0], m.hidden), dtype=self.torch.int64, device=x.device)
            m.partial_dev(x, acc)
            return acc
        w = self.weights[key]
        acc = self.torch.empty((x.shape[0], w.out_features), dtype=self.torch.int64, device=x.device)
        w.linear_acc_dev(x, acc)
        return acc

    def requant(self, key, acc):
        y = self.torch.empty(acc.shape, dtype=self.torch.int16, device=acc.device)
        if key in self.mlps:
            self.mlps[key].requant_dev(acc, y)
        else:
            self.plans[key].apply_acc_dev(acc, y)
        return y

    def add_lm_head(self, key, W, in_features, w_shifts, final_norm_frac, logit_frac):
        import myelith_b200 as myl

        w = myl.Weight(self.ctx, W, in_features, w_shifts)
        self.weights[key] = w
        self.plans[key] = w.requant(myl.RQ_SHIFT_I32, final_norm_frac, logit_frac)

    def lm_head_logits(self, key, x):
        w = self.weights[key]
        y = self.torch.empty((x.shape[0], w.out_features), dtype=self.torch.int32, device=x.device)
        w.linear_dev(self.plans[key], x, y)
        return y

    def lm_head_keys(self, key, x, index_base):
        logits = self.lm_head_logits(key, x)
        keys = self.torch.empty((x.shape[0],), dtype=self.torch.int64, device=x.device)
        self.ctx.argmax_keys_dev(logits, keys, index_base)
        return keys


class ColumnParallelLinear:
    """Rank owns output rows [lo, hi) of W; y shard = linear of those rows."""

    def __init__(self, local: Local, key, spec: LinearSpec, rank: int, world: int, group=None):
        N, K = spec.W.shape
        self.lo, self.hi = shard_range(N, rank, world)
        self.local, self.key, self.group, self.world = local, key, group, world
        self.N = N
        of = spec.out_frac
        of_shard = of if np.ndim(of) == 0 else np.asarray(of)[self.lo:self.hi]
        local.add_linear(key, np.ascontiguousarray(spec.W[self.lo:self.hi]), K,
                         np.asarray(spec.w_shifts)[self.lo:self.hi], spec.act_frac, of_shard)

    def __call__(self, x):
        return self.local.linear(self.key, x)

    def gather(self, x):
        """Full output [M][N] on every rank (all-gather of the shards)."""
        import torch
        import torch.distributed as dist

        y = self(x)
        if self.world == 1:
            return y
        # all_gather wants equal sizes: pad every shard to the widest one.
        ranges = [shard_range(self.N, r, self.world) for r in range(self.world)]
        width = max(b - a for a, b in ranges)
        mine = torch.zeros((x.shape[0], width), dtype=y.dtype, device=y.device)
        mine[:, : y.shape[1]] = y
        # NCCL and gloo have no int16 type: move the shards as bytes.
        raw = mine.view(torch.uint8)
        parts = [torch.empty_like(raw) for _ in range(self.world)]
        dist.all_gather(parts, raw, group=self.group)
        return torch.cat([p.view(y.dtype)[:, : b - a] for p, (a, b) in zip(parts, ranges)], dim=1)


class RowParallelLinear:
    """Rank owns input columns [lo, hi) of W; all ranks get the full output:
    int64 partials -> all-reduce (SUM) -> one requant."""

    def __init__(self, local: Local, key, spec: LinearSpec, rank: int, world: int, group=None):
        N, K = spec.W.shape
        self.lo, self.hi = shard_range(K, rank, world)
        self.local, self.key, self.group, self.world = local, key, group, world
        self.N = N
        # The column slice keeps every row, so the per-row shifts and the
        # requant plan are those of the full weight.
        local.add_linear(key, np.ascontiguousarray(spec.W[:, self.lo:self.hi]), self.hi - self.lo,
                         spec.w_shifts, spec.act_frac, spec.out_frac)

    def x_shard(self, x):
        return x[:, self.lo:self.hi].contiguous()

    def overlapped(self, x_shard, chunks: int = 4):
        """As __call__, with the exchange overlapped (overlapped_row_parallel)."""
        M = x_shard.shape[0]
        if self.world == 1:
            return self(x_shard)

        def compute_acc(r0, r1, out):
            out.copy_(self.local.acc(self.key, x_shard[r0:r1]))

        def requant(acc, y):
            y.copy_(self.local.requant(self.key, acc))

        return overlapped_row_parallel(compute_acc, requant, M, self.N, self.world, self.group,
                                       chunks, x_shard.device)

    def exchanged(self, x_shard, xchg: "PeerExchange", stream=None, between=None):
        """As __call__, through a PeerExchange (LibLocal only)."""
        return xchg(self.local.weights[self.key], self.local.plans[self.key], x_shard, stream, between)

    def __call__(self, x_shard):
        import torch.distributed as dist

        acc = self.local.acc(self.key, x_shard)
        if self.world > 1:
            dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.group)
        return self.local.requant(self.key, acc)


class VocabParallelLMHead:
    """LM head path B (runtime/src/model.rs:297-307) with the vocab rows
    sharded over the ranks; greedy() returns the global argmax_int token of
    every row of x (and its logit) from one int64 MAX all-reduce."""

    def __init__(self, local: Local, key, W, w_shifts, final_norm_frac: int, logit_frac: int,
                 rank: int, world: int, group=None):
        V, K = W.shape
        self.lo, self.hi = shard_range(V, rank, world)
        self.local, self.key, self.group, self.world = local, key, group, world
        local.add_lm_head(key, np.ascontiguousarray(W[self.lo:self.hi]), K,
                          np.asarray(w_shifts)[self.lo:self.hi], final_norm_frac, logit_frac)

    def logits(self, x):
        """int32 logits of this rank's vocab rows [lo, hi)."""
        return self.local.lm_head_logits(self.key, x)

    def greedy(self, x):
        """(tokens int64 [M], logits int64 [M]) of the whole vocab."""
        import torch.distributed as dist

        keys = self.local.lm_head_keys(self.key, x, self.lo)
        if self.world > 1:
            dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=self.group)
        return (0xFFFFFFFF - (keys & 0xFFFFFFFF)), keys >> 32


class _CudaBuffer:
    """__cuda_array_interface__ of a library buffer, for a torch view."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerExchange:
    """Buffers of one row-parallel layer shape (M tokens, N output channels)
    shared by the ranks of a node, and the exchange step (see the module
    notes). Rank o owns output rows [o R, min((o + 1) R, M)), R = ceil(M /
    world) rounded up to 16. Collective: every rank constructs it, calls it
    and closes it in the same order."""

    def __init__(self, ctx, M: int, N: int, rank: int, world: int, group=None, out_i32: bool = False):
        import torch
        import torch.distributed as dist

        from myelith_b200 import IPC_HANDLE_BYTES

        self.ctx, self.M, self.N, self.rank, self.world, self.group = ctx, M, N, rank, world, group
        self.R = ((M + world - 1) // world + 15) // 16 * 16
        esize = 4 if out_i32 else 2
        dev = torch.device("cuda", torch.cuda.current_device())
        recv_bytes = world * self.R * N * 8
        # the barrier's flag words (one per sender) follow the receive slabs
        self.recv_ptr, h_recv = ctx.ipc_alloc(recv_bytes + 256)
        self.out_ptr, h_out = ctx.ipc_alloc(world * self.R * N * esize)
        mine = torch.tensor(list(h_recv + h_out), dtype=torch.uint8, device=dev)
        allh = torch.empty((world, 2 * IPC_HANDLE_BYTES), dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(allh, mine, group=group)
        allh = allh.cpu().numpy()
        self.recv_ptrs, self.out_ptrs, self._opened = [], [], []
        for o in range(world):
            if o == rank:
                self.recv_ptrs.append(self.recv_ptr)
                self.out_ptrs.append(self.out_ptr)
                continue
            rp = ctx.ipc_open(bytes(allh[o, :IPC_HANDLE_BYTES]))
            op = ctx.ipc_open(bytes(allh[o, IPC_HANDLE_BYTES:]))
            self._opened += [rp, op]
            self.recv_ptrs.append(rp)
            self.out_ptrs.append(op)
        self.flag_ptrs = [p + recv_bytes for p in self.recv_ptrs]
        self.epoch = 0
        self.out = torch.as_tensor(_CudaBuffer(self.out_ptr, (world * self.R, N),
                                               "<i4" if out_i32 else "<i2"), device=dev)[:M]
        self._flag = torch.zeros(1, dtype=torch.int32, device=dev)
        self._host_barrier()

    def _host_barrier(self):
        """Set-up and tear-down: a one-element all-reduce on the current stream."""
        import torch.distributed as dist

        dist.all_reduce(self._flag, group=self.group)

    def barrier(self, stream=None):
        """Orders the ranks' work on the stream (flag words in peer memory)."""
        self.epoch += 1
        self.ctx.exchange_barrier_dev(self.flag_ptrs, self.rank, self.epoch, stream)

    def __call__(self, weight, requant, x_shard, stream=None, between=None):
        """Row-parallel output [M, N] (a view of this rank's output buffer,
        valid until the next call) of weight shard x x_shard; `between` runs
        after this rank's GEMM, before the ranks synchronise."""
        M = x_shard.shape[0]
        if M > self.M:
            raise ValueError(f"{M} rows, the exchange holds {self.M}")
        weight.acc_exchange_dev(x_shard, self.recv_ptrs, self.rank, self.R, stream)
        if between is not None:
            between()
        self.barrier(stream)
        requant.exchange_reduce_dev(self.recv_ptr, self.world, self.rank, self.R, M, self.out_ptrs,
                                    self.N, stream)
        self.barrier(stream)
        return self.out[:M]

    def close(self):
        import torch

        torch.cuda.synchronize()
        self._host_barrier()  # no rank still writes into another's buffers
        torch.cuda.synchronize()
        for p in self._opened:
            self.ctx.ipc_close(p)
        self._opened = []
        self._host_barrier()  # every peer mapping is gone before the memory is freed
        torch.cuda.synchronize()
        self.ctx.ipc_free(self.recv_ptr)
        self.ctx.ipc_free(self.out_ptr)


def overlapped_row_parallel(compute_acc, requant, M: int, N: int, world: int, group=None,
                            chunks: int = 4, device=None, between=None):
    """Row-parallel exchange overlapped with the computation of later rows.

    compute_acc(r0, r1, out) writes this rank's exact int64 partial sums of
    rows [r0, r1) into out [r1 - r0, N]; requant(acc, y) requantises summed
    rows into int16 y. The rows run in `chunks` groups; each group's partials
    go to a reduce-scatter (async) while the next group computes, each rank
    requantises its share of the summed rows, and an all-gather of the int16
    rows gives every rank the full [M, N] output. Integer sums, one requant
    after the sum: the result equals the all-reduce form bit for bit.
    between(), if given, runs after the last reduce-scatter is issued (other
    work that overlaps the exchange).
    """
    import torch
    import torch.distributed as dist

    if chunks < 1 or M % (chunks * world) != 0:
        chunks = 1 if M % world == 0 else 0
    if chunks == 0:  # rows do not split evenly: all-reduce form
        acc = torch.empty((M, N), dtype=torch.int64, device=device)
        compute_acc(0, M, acc)
        work = dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=group, async_op=True)
        if between is not None:
            between()
        work.wait()
        y = torch.empty((M, N), dtype=torch.int16, device=device)
        requant(acc, y)
        return y
    mc = M // chunks
    acc = torch.empty((M, N), dtype=torch.int64, device=device)
    part = torch.empty((chunks, mc // world, N), dtype=torch.int64, device=device)
    own = torch.empty((chunks, mc // world, N), dtype=torch.int16, device=device)
    y = torch.empty((M, N), dtype=torch.int16, device=device)
    works = []
    for c in range(chunks):
        r0, r1 = c * mc, (c + 1) * mc
        compute_acc(r0, r1, acc[r0:r1])
        works.append(dist.reduce_scatter_tensor(part[c], acc[r0:r1], op=dist.ReduceOp.SUM,
                                                group=group, async_op=True))
    if between is not None:
        between()
    gathers = []
    for c in range(chunks):
        works[c].wait()
        requant(part[c], own[c])
        # NCCL and gloo have no int16: the rows move as bytes
        gathers.append(dist.all_gather_into_tensor(y[c * mc:(c + 1) * mc].view(torch.uint8),
                                                   own[c].view(torch.uint8), group=group,
                                                   async_op=True))
    for g in gathers:
        g.wait()
    return y


class ParallelMlp:
    """mlp_int (kernels/src/mlp.rs:28-74) over intermediate channels [lo, hi):
    gate/up rows and down columns of the same channels stay on one rank, the
    down projection's int64 partials are all-reduced, the requant runs once."""

    def __init__(self, local: Local, key, W_gate, W_up, W_down, hidden, intermediate,
                 gate_w_shifts, up_w_shifts, down_w_shifts, silu_lut, in_frac, gate_out_frac,
                 up_out_frac, down_in_frac, silu_in_frac, silu_lut_offset, silu_out_frac, out_frac,
                 rank: int, world: int, group=None):
        self.lo, self.hi = shard_range(intermediate, rank, world)
        self.local, self.key, self.group, self.world = local, key, group, world
        lo, hi = self.lo, self.hi
        self.args = dict(
            W_gate=np.ascontiguousarray(np.asarray(W_gate).reshape(intermediate, hidden)[lo:hi]),
            W_up=np.ascontiguousarray(np.asarray(W_up).reshape(intermediate, hidden)[lo:hi]),
            W_down=np.ascontiguousarray(np.asarray(W_down).reshape(hidden, intermediate)[:, lo:hi]),
            hidden=hidden, intermediate=hi - lo,
            gate_w_shifts=np.asarray(gate_w_shifts)[lo:hi], up_w_shifts=np.asarray(up_w_shifts)[lo:hi],
            down_w_shifts=np.asarray(down_w_shifts), silu_lut=silu_lut, in_frac=in_frac,
            gate_out_frac=gate_out_frac, up_out_frac=up_out_frac, down_in_frac=down_in_frac,
            silu_in_frac=silu_in_frac, silu_lut_offset=silu_lut_offset, silu_out_frac=silu_out_frac,
            out_frac=np.asarray(out_frac))
        local.add_mlp(key, self.args)

    def __call__(self, x):
        import torch.distributed as dist

        acc = self.local.acc(self.key, x)
        if self.world > 1:
            dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.group)
        return self.local.requant(self.key, acc)
