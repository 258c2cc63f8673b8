"""The tensor-core GEMM's tail split: when the output tiles fill some waves of
the SMs and leave a small last wave, the last wave's tiles run as K slices
whose exact int64 partials a second kernel adds before the epilogue. Results
must equal the CPU oracle bit for bit, for every epilogue mode (shift, LM-head
i32, multiplier, int64 partials, bias, and the MLP's SiLU pair epilogue).

Every case is also computed with the tail split switched off
(force_split_k = 1: one K slice, no tail), on all rows; the oracle checks a
sample of rows.
"""
import numpy as np
import pytest

import oracle as O
from make_golden import silu_lut_spec

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import myelith_b200 as myl  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = myl.Context(0)
    yield c
    c.close()


def _x(rng, M, K, sigma=1500.0):
    return np.clip(np.rint(rng.normal(0, sigma, size=(M, K))), -32767, 32767).astype(np.int16)


def _both(ctx, fn):
    ctx.set_dispatch(gemv_max_m=0)
    try:
        tail = fn()
        ctx.set_dispatch(gemv_max_m=0, force_split_k=1)
        plain = fn()
    finally:
        ctx.set_dispatch()
    return tail, plain


# (M, K, N): tiles = ceil(N/128) * ceil(M/128) > 148 SMs with a short last wave
SHAPES = [(520, 1024, 4864), (700, 2048, 3584), (2048, 18944, 3584)]


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_tail_split_shift(ctx, M, K, N):
    rng = np.random.default_rng(M + K + N)
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    sh = int(round(np.log2(73.6 * np.sqrt(K))))
    ws = rng.integers(sh - 1, sh + 2, size=N).astype(np.uint8)
    of = rng.integers(5, 10, size=N).astype(np.uint8)
    x = _x(rng, M, K)
    w = ctx.weight(W, K, ws)
    tail, plain = _both(ctx, lambda: w.linear(x, 8, of))
    assert np.array_equal(tail, plain)
    rows = np.random.default_rng(1).choice(M, size=12, replace=False)
    assert np.array_equal(tail[rows], O.linear_w8a16_pc(x[rows], W.reshape(-1), K, ws, 8, of))


def test_tail_split_other_modes(ctx):
    M, K, N = 520, 1024, 4864
    rng = np.random.default_rng(3)
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    ws = rng.integers(10, 13, size=N).astype(np.uint8)
    x = _x(rng, M, K, sigma=9000.0)
    w = ctx.weight(W, K, ws)
    rows = np.random.default_rng(2).choice(M, size=10, replace=False)
    # LM head (i32 clamp)
    tail, plain = _both(ctx, lambda: w.lm_head(x, 8, 10))
    assert np.array_equal(tail, plain)
    assert np.array_equal(tail[rows], O.lm_head_w8a16_i32(x[rows], W.reshape(-1), K, ws, 8, 10))
    # multiplier requant
    mult = rng.integers(2**30, 2**31 - 1, size=N).astype(np.int32)
    shift = rng.integers(40, 46, size=N).astype(np.uint8)
    tail, plain = _both(ctx, lambda: w.linear_mult(x, mult, shift))
    assert np.array_equal(tail, plain)
    assert np.array_equal(tail[rows], O.linear_w8a16_mult(x[rows], W.reshape(-1), K, mult, shift))
    # bias
    bias = rng.integers(-3000, 3000, size=N).astype(np.int16)
    bsh = rng.integers(0, 8, size=N).astype(np.uint8)
    tail, plain = _both(ctx, lambda: w.linear_bias(x, 8, 6, bias, bsh))
    assert np.array_equal(tail, plain)
    lin = O.linear_w8a16(x[rows], W.reshape(-1), K, ws, 8, 6)
    assert np.array_equal(tail[rows], np.stack([O.add_bias_i16(r, bias, bsh, 6) for r in lin]))
    # int64 partial sums (row-parallel tensor parallelism)
    xd = torch.from_numpy(x).cuda()

    def acc():
        a = torch.empty((M, N), dtype=torch.int64, device="cuda")
        w.linear_acc_dev(xd, a)
        torch.cuda.synchronize()
        return a.cpu().numpy()

    tail, plain = _both(ctx, acc)
    assert np.array_equal(tail, plain)
    assert np.array_equal(tail[rows], O.linear_acc_i64(x[rows], W.reshape(-1), K, N))


def test_tail_split_silu_pairs(ctx):
    """MLP gate/up with 2I = 19200 rows (150 channel tiles): the SiLU pair
    epilogue runs in the tail reduction."""
    H, I, M = 2048, 9600, 100
    rng = np.random.default_rng(9)
    Wg = rng.integers(-127, 128, size=(I, H), dtype=np.int8)
    Wu = rng.integers(-127, 128, size=(I, H), dtype=np.int8)
    Wd = rng.integers(-127, 128, size=(H, I), dtype=np.int8)
    gs = rng.integers(11, 14, size=I).astype(np.uint8)
    us = rng.integers(11, 14, size=I).astype(np.uint8)
    ds = rng.integers(13, 15, size=H).astype(np.uint8)
    of = rng.integers(3, 8, size=H).astype(np.uint8)
    lut = silu_lut_spec()
    args = (Wg, Wu, Wd, H, I, gs, us, ds, lut, 8, 7, 7, 7, 6, 8192, 8, of)
    m = myl.Mlp(ctx, *args)
    x = _x(rng, M, H)
    tail, plain = _both(ctx, lambda: m(x))
    assert np.array_equal(tail, plain)
    rows = np.arange(0, M, 9)
    assert np.array_equal(tail[rows], O.mlp_int(x[rows], *args))
