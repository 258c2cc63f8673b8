"""The CTA-pair tensor-core GEMM (one M = 256 MMA over two SMs, each SM
loading its 128 weight rows and one activation byte plane) against the
one-CTA kernel and the CPU oracle, bit for bit.

Shapes cover channel counts that are a multiple of 256, an odd multiple of
128 (the odd CTA of the last pair reads rows past the weight) and neither;
token counts with a partial last tile (the MMA's N trimmed to the valid
tokens); the tail split of the last wave; the K split of small grids; every
epilogue mode; the MLP's SiLU pair epilogue; and the bounded-wait failure
path of a pair.
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


def _pair_and_single(ctx, fn):
    ctx.set_dispatch(gemv_max_m=0, force_token_tile=128)
    try:
        ctx.set_tc_options(pair=True)
        pair = fn()
        ctx.set_tc_options(pair=False)
        single = fn()
    finally:
        ctx.set_tc_options(pair=True)
        ctx.set_dispatch()
    return pair, single


# (M, K, N): N % 256 in {0, 128, other}; M % 128 in {0, small, large}
SHAPES = [(256, 512, 256), (300, 1024, 4736), (130, 2048, 1000), (2048, 3584, 4864),
          (700, 18944, 3584), (129, 640, 384), (1000, 4096, 18944)]


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_pair_linear_shift(ctx, M, K, N):
    rng = np.random.default_rng(M * 7 + K + N)
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    sh = int(round(np.log2(73.6 * np.sqrt(K))))
    ws = rng.integers(sh - 1, sh + 2, size=N).astype(np.uint8)
    of = rng.integers(5, 10, size=N).astype(np.uint8)
    x = _x(rng, M, K)
    w = ctx.weight(W, K, ws)
    pair, single = _pair_and_single(ctx, lambda: w.linear(x, 8, of))
    assert np.array_equal(pair, single)
    rows = np.unique(np.r_[0, M - 1, np.random.default_rng(1).choice(M, size=min(M, 10), replace=False)])
    assert np.array_equal(pair[rows], O.linear_w8a16_pc(x[rows], W.reshape(-1), K, ws, 8, of))


def test_pair_other_modes(ctx):
    M, K, N = 333, 1024, 4736
    rng = np.random.default_rng(3)
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    ws = rng.integers(10, 13, size=N).astype(np.uint8)
    x = _x(rng, M, K, sigma=9000.0)
    w = ctx.weight(W, K, ws)
    rows = np.r_[0, 5, 128, 200, M - 1]
    pair, single = _pair_and_single(ctx, lambda: w.lm_head(x, 8, 10))
    assert np.array_equal(pair, single)
    assert np.array_equal(pair[rows], O.lm_head_w8a16_i32(x[rows], W.reshape(-1), K, ws, 8, 10))
    mult = rng.integers(2**30, 2**31 - 1, size=N).astype(np.int32)
    shift = rng.integers(40, 46, size=N).astype(np.uint8)
    pair, single = _pair_and_single(ctx, lambda: w.linear_mult(x, mult, shift))
    assert np.array_equal(pair, single)
    assert np.array_equal(pair[rows], O.linear_w8a16_mult(x[rows], W.reshape(-1), K, mult, shift))
    bias = rng.integers(-3000, 3000, size=N).astype(np.int16)
    bsh = rng.integers(0, 8, size=N).astype(np.uint8)
    pair, single = _pair_and_single(ctx, lambda: w.linear_bias(x, 8, 6, bias, bsh))
    assert np.array_equal(pair, single)
    xd = torch.from_numpy(x).cuda()

    def acc():
        a = torch.empty((M, N), dtype=torch.int64, device="cuda")
        w.linear_acc_dev(xd, a)
        torch.cuda.synchronize()
        return a.cpu().numpy()

    pair, single = _pair_and_single(ctx, acc)
    assert np.array_equal(pair, single)
    assert np.array_equal(pair[rows], O.linear_acc_i64(x[rows], W.reshape(-1), K, N))


def test_pair_noalloc_entry(ctx):
    import ctypes as C

    M, K, N = 400, 2048, 4736
    rng = np.random.default_rng(8)
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    ws = np.full(N, 13, np.uint8)
    x = _x(rng, M, K)
    w = ctx.weight(W, K, ws)
    rq = w.requant(myl.RQ_SHIFT_I16, act_frac=8, out_frac=np.full(N, 8, np.uint8))
    f = myl.load_library().myl_linear_noalloc_dev
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                  C.c_void_p, C.c_int64, C.c_void_p]
    f.restype = C.c_int
    xd = torch.from_numpy(x).cuda()

    def run():
        y = torch.empty((M, N), dtype=torch.int16, device="cuda")
        torch.cuda.synchronize()
        rc = f(ctx.handle, w.handle, rq.handle, xd.data_ptr(), M, xd.stride(0), y.data_ptr(),
               y.stride(0), None)
        assert rc == 0, myl.load_library().myl_last_error()
        ctx.synchronize()
        return y.cpu().numpy()

    pair, single = _pair_and_single(ctx, run)
    assert np.array_equal(pair, single)
    rows = np.r_[0, 127, 128, 399]
    assert np.array_equal(pair[rows], O.linear_w8a16(x[rows], W.reshape(-1), K, ws, 8, 8))


@pytest.mark.parametrize("M", [200, 1024])
def test_pair_mlp_silu(ctx, M):
    """gate/up 2I = 2 * 1216 rows (9.5 pairs of 256): the SiLU pair epilogue in
    both CTAs of a pair writes the down projection's byte planes."""
    H, I = 1024, 1216
    rng = np.random.default_rng(M)
    Wg = rng.integers(-127, 128, size=(I, H), dtype=np.int8)
    Wu = rng.integers(-127, 128, size=(I, H), dtype=np.int8)
    Wd = rng.integers(-127, 128, size=(H, I), dtype=np.int8)
    gs = rng.integers(11, 14, size=I).astype(np.uint8)
    us = rng.integers(11, 14, size=I).astype(np.uint8)
    ds = rng.integers(13, 15, size=H).astype(np.uint8)
    of = rng.integers(3, 8, size=H).astype(np.uint8)
    args = (Wg, Wu, Wd, H, I, gs, us, ds, silu_lut_spec(), 8, 7, 7, 7, 6, 8192, 8, of)
    m = myl.Mlp(ctx, *args)
    x = _x(rng, M, H)
    pair, single = _pair_and_single(ctx, lambda: m(x))
    assert np.array_equal(pair, single)
    rows = np.r_[0, 131, M - 1]
    assert np.array_equal(pair[rows], O.mlp_int(x[rows], *args))


def test_pair_bounded_wait_reports_error_and_context_survives(ctx):
    rng = np.random.default_rng(41)
    K, N, M = 512, 512, 256
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    x = _x(rng, M, K)
    ws = np.full(N, 10, np.uint8)
    w = ctx.weight(W, K, ws)
    ctx.set_dispatch(gemv_max_m=0, force_token_tile=128)
    ctx.set_wait_timeout_ns(50_000_000)  # 50 ms
    ctx.inject_wait_fault(True)
    try:
        with pytest.raises(myl.MylError) as e:
            w.linear(x, 8, 8)
        assert e.value.code == myl.MYL_ERR_DEVICE
    finally:
        ctx.inject_wait_fault(False)
        ctx.set_wait_timeout_ns(2_000_000_000)
    try:
        assert np.array_equal(w.linear(x, 8, 8), O.linear_w8a16(x, W.reshape(-1), K, ws, 8, 8))
    finally:
        ctx.set_dispatch()


def test_tc_options_rejects(ctx):
    with pytest.raises(myl.MylError):
        ctx.set_tc_options(pair=True, xbox_rows=48)
