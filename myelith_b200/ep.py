"""Expert parallelism for the MoE layer (one process per GPU).

Each rank owns a contiguous block of experts ([first, first + n) of E, equal
shares) and its own tokens. A layer step:

  1. route       every rank routes its tokens (the router covers all experts);
  2. dispatch    the (token, choice) pairs are sorted by the rank owning their
                 expert; the counts are exchanged (all_to_all of int64), then
                 the rows (int16, moved as bytes) and their expert ids;
  3. experts     each rank runs its experts on the rows it received
                 (grouped tensor-core GEMMs);
  4. return      the expert outputs travel back by the inverse all_to_all and
                 are put back in (token, choice) order;
  5. combine     the home rank sums p * y over its tokens' choices in the fixed
                 order j = 0..k-1, adds the shared expert and requantises.

Every row is computed by the same integer arithmetic on whichever rank holds
its expert, and the combine order is fixed, so the output is bit-identical to
the single-GPU layer at every rank count.

The per-rank arithmetic sits behind ``MoeLocal``; ``LibMoeLocal`` runs the
sm_100a kernels on torch CUDA tensors, tests can run the exchange logic on CPU
(gloo) with another implementation.
"""
from __future__ import annotations

import numpy as np

from .tp import shard_range


class MoeLocal:
    """Per-rank MoE arithmetic. Tensors are torch tensors on the rank's device."""

    def route(self, x):  # -> (topk_idx [T, k] int32, topk_prob [T, k] int32)
        raise NotImplementedError

    def experts(self, rows, ids):  # rows [P, H] int16, global ids [P] -> [P, H] int16
        raise NotImplementedError

    def shared(self, x):  # shared expert output [T, H] int16, or None
        raise NotImplementedError

    def combine(self, y, prob, shared):  # y [T * k, H] in (token, choice) order -> [T, H]
        raise NotImplementedError


class LibMoeLocal(MoeLocal):
    """libmyl_w8a16 MoE stages (myelith_b200.Moe holding this rank's experts)."""

    def __init__(self, moe, shared_mlp=None):
        import torch

        self.moe, self.shared_mlp, self.torch = moe, shared_mlp, torch

    def route(self, x):
        T, k = x.shape[0], self.moe.top_k
        idx = self.torch.empty((T, k), dtype=self.torch.int32, device=x.device)
        prob = self.torch.empty_like(idx)
        self.moe.route_dev(x, idx, prob)
        return idx, prob

    def experts(self, rows, ids):
        y = self.torch.empty_like(rows)
        if rows.shape[0]:
            self.moe.experts_dev(rows, ids, y)
        return y

    def shared(self, x):
        if self.shared_mlp is None:
            return None
        y = self.torch.empty_like(x)
        self.shared_mlp.dev(x, y)
        return y

    def combine(self, y, prob, shared):
        out = self.torch.empty((prob.shape[0], self.moe.hidden), dtype=self.torch.int16,
                               device=prob.device)
        self.moe.combine_dev(y, prob, shared, out)
        return out


def _as_bytes(t):
    """Flat uint8 view of a tensor (NCCL and gloo have no int16)."""
    import torch

    t = t.contiguous().reshape(-1)
    if t.numel() == 0:
        return torch.empty(0, dtype=torch.uint8, device=t.device)
    return t.view(torch.uint8)


def expert_owner(num_experts: int, world: int) -> np.ndarray:
    """owner[e] = the rank holding expert e (shard_range blocks)."""
    owner = np.empty(num_experts, np.int64)
    for r in range(world):
        lo, hi = shard_range(num_experts, r, world)
        owner[lo:hi] = r
    return owner


class ExpertParallelMoe:
    """One MoE layer over ``world`` ranks; call with this rank's tokens."""

    def __init__(self, local: MoeLocal, num_experts: int, top_k: int, hidden: int, rank: int,
                 world: int, group=None):
        self.local, self.E, self.k, self.H = local, num_experts, top_k, hidden
        self.rank, self.world, self.group = rank, world, group
        self.first, self.last = shard_range(num_experts, rank, world)
        self._owner = expert_owner(num_experts, world)

    def _a2a(self, out, inp, out_splits, in_splits):
        import torch.distributed as dist

        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def dispatch(self, x, idx):
        """Sorts this rank's (token, choice) pairs by owner rank and exchanges
        them. Returns (received rows, their expert ids, order, send counts,
        receive counts); order[i] is the pair index of the i-th sent row."""
        import torch

        dev = x.device
        owner = torch.from_numpy(self._owner).to(dev)
        flat = idx.reshape(-1).to(torch.int64)
        dest = owner[flat]
        # stable sort by destination: pairs keep their (token, choice) order per rank
        order = torch.sort(dest, stable=True).indices
        send = torch.bincount(dest, minlength=self.world)
        recv = torch.empty_like(send)
        self._a2a(recv, send, [1] * self.world, [1] * self.world)
        send_l, recv_l = send.tolist(), recv.tolist()
        rows = x[order // self.k]
        ids = flat[order].to(torch.int32)
        H = x.shape[1]
        rx = torch.empty((sum(recv_l), H), dtype=x.dtype, device=dev)
        self._a2a(_as_bytes(rx), _as_bytes(rows), [c * H * 2 for c in recv_l],
                  [c * H * 2 for c in send_l])
        rid = torch.empty(sum(recv_l), dtype=torch.int32, device=dev)
        self._a2a(rid, ids, recv_l, send_l)
        return rx, rid, order, send_l, recv_l

    def gather_back(self, y_recv, order, send_l, recv_l, pairs):
        """Inverse exchange: results return to the pairs' home rank and are
        put back in (token, choice) order."""
        import torch

        H = y_recv.shape[1]
        back = torch.empty((pairs, H), dtype=y_recv.dtype, device=y_recv.device)
        self._a2a(_as_bytes(back), _as_bytes(y_recv), [c * H * 2 for c in send_l],
                  [c * H * 2 for c in recv_l])
        y = torch.empty_like(back)
        y[order] = back
        return y

    def __call__(self, x):
        idx, prob = self.local.route(x)
        rx, rid, order, send_l, recv_l = self.dispatch(x, idx)
        y_recv = self.local.experts(rx, rid)
        y = self.gather_back(y_recv, order, send_l, recv_l, idx.numel())
        return self.local.combine(y, prob, self.local.shared(x))


class PeerExpertParallelMoe:
    """The expert-parallel layer without a collective library on the data
    path: dispatch and return through peer memory (myl_ep_dispatch_dev /
    myl_ep_return_dev), device-side barriers between them, one host read of
    the received row count per layer. Same arithmetic and combine order as
    ExpertParallelMoe, so the output is bit-identical. Collective: every rank
    constructs, calls and closes it in the same order."""

    def __init__(self, ctx, local: "LibMoeLocal", num_experts: int, top_k: int, hidden: int,
                 rank: int, world: int, max_tokens: int, group=None):
        import torch
        import torch.distributed as dist

        from myelith_b200 import IPC_HANDLE_BYTES
        from myelith_b200.tp import _CudaBuffer

        self.ctx, self.local, self.E, self.k, self.H = ctx, local, num_experts, top_k, hidden
        self.rank, self.world, self.group, self.max_tokens = rank, world, group, max_tokens
        self.capacity = world * max_tokens * top_k  # every pair of every rank, worst case

        def up(n):
            return (n + 255) // 256 * 256

        cap, H = self.capacity, hidden
        off_rows, off_ids = 0, up(cap * H * 2)
        off_src = off_ids + up(cap * 4)
        off_cnt = off_src + up(cap * 4)
        off_flag = off_cnt + 256
        total = off_flag + 256
        dev = torch.device("cuda", torch.cuda.current_device())
        self.buf, h1 = ctx.ipc_alloc(total)
        self.back, h2 = ctx.ipc_alloc(max(1, max_tokens * top_k) * H * 2)
        mine = torch.tensor(list(h1 + h2), dtype=torch.uint8, device=dev)
        allh = torch.empty((world, 2 * IPC_HANDLE_BYTES), dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(allh, mine, group=group)
        allh = allh.cpu().numpy()
        bases, backs, self._opened = [], [], []
        for o in range(world):
            if o == rank:
                bases.append(self.buf)
                backs.append(self.back)
                continue
            b = ctx.ipc_open(bytes(allh[o, :IPC_HANDLE_BYTES]))
            bk = ctx.ipc_open(bytes(allh[o, IPC_HANDLE_BYTES:]))
            self._opened += [b, bk]
            bases.append(b)
            backs.append(bk)
        self.rows_p = [b + off_rows for b in bases]
        self.ids_p = [b + off_ids for b in bases]
        self.src_p = [b + off_src for b in bases]
        self.cnt_p = [b + off_cnt for b in bases]
        self.flag_p = [b + off_flag for b in bases]
        self.back_p = backs
        self.epoch = 0
        view = lambda ptr, shape, t: torch.as_tensor(_CudaBuffer(ptr, shape, t), device=dev)  # noqa: E731
        self.rows_t = view(self.buf + off_rows, (cap, H), "<i2")
        self.ids_t = view(self.buf + off_ids, (cap,), "<i4")
        self.src_t = view(self.buf + off_src, (cap,), "<i4")
        self.cnt_t = view(self.buf + off_cnt, (1,), "<i4")
        self.back_t = view(self.back, (max(1, max_tokens * top_k), H), "<i2")
        self._flag = torch.zeros(1, dtype=torch.int32, device=dev)
        dist.all_reduce(self._flag, group=group)

    def barrier(self):
        self.epoch += 1
        self.ctx.exchange_barrier_dev(self.flag_p, self.rank, self.epoch)

    def __call__(self, x):
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens, the layer holds {self.max_tokens}")
        idx, prob = self.local.route(x)
        self.ctx.ep_dispatch_dev(x, idx, self.E, self.rank, self.rows_p, self.ids_p, self.src_p,
                                 self.cnt_p, self.capacity)
        shared = self.local.shared(x)  # this rank's shared expert while the peers dispatch
        self.barrier()
        n = int(self.cnt_t.item())
        self.cnt_t.zero_()  # peers dispatch again only after the closing barrier
        y = self.local.experts(self.rows_t[:n], self.ids_t[:n])
        self.ctx.ep_return_dev(y, n, self.src_t, self.back_p)
        self.barrier()
        return self.local.combine(self.back_t[: T * self.k], prob, shared)

    def close(self):
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.all_reduce(self._flag, group=self.group)
        torch.cuda.synchronize()
        for p in self._opened:
            self.ctx.ipc_close(p)
        self._opened = []
        dist.all_reduce(self._flag, group=self.group)
        torch.cuda.synchronize()
        self.ctx.ipc_free(self.buf)
        self.ctx.ipc_free(self.back)
