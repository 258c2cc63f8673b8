"""GPU parity of the LM head's path A (runtime/src/model.rs:285-296): int16
weights with one shift per row, i64 dot, rescale to logit_frac, i32 clamp.

The library stores each int16 row as two int8 rows (high byte, low byte - 128)
and runs the ordinary GEMV / tensor-core kernels with a pair epilogue
(256 * a_hi + a_lo + 128 * sum(x)); every logit must equal the oracle's.
"""
import numpy as np
import pytest

import oracle as O

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


def _case(rng, M, K, N, w_sigma=8000.0, x_sigma=3000.0):
    W = np.clip(np.rint(rng.normal(0, w_sigma, size=(N, K))), -32768, 32767).astype(np.int16)
    W[0, :4] = [-32768, 32767, -32768, 32767]
    sh = rng.integers(10, 16, size=N).astype(np.uint8)
    x = np.clip(np.rint(rng.normal(0, x_sigma, size=(M, K))), -32768, 32767).astype(np.int16)
    return W, sh, x


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 40, 300])
@pytest.mark.parametrize("K,N", [(896, 1000), (100, 77), (64, 1)])
def test_lm_head16(ctx, M, K, N):
    rng = np.random.default_rng(M * 1000 + K + N)
    W, sh, x = _case(rng, M, K, N)
    w = ctx.weight16(W, K, sh)
    y = w.lm_head(x, 8, 6)
    assert np.array_equal(y, O.lm_head_w16a16_i32(x, W, K, sh, 8, 6))


@pytest.mark.parametrize("mode,split", [("gemv", 3), ("tc", 2), ("tc", 0)])
def test_lm_head16_split_and_saturation(ctx, mode, split):
    """Forced K splits (int64 partials reduced in the pair mode) and outputs
    that saturate at the i32 bounds."""
    rng = np.random.default_rng(split + 7)
    M = 3 if mode == "gemv" else 70
    W, sh, x = _case(rng, M, 2048, 500, w_sigma=20000.0, x_sigma=20000.0)
    sh[:] = 0
    ctx.set_dispatch(gemv_max_m=4 if mode == "gemv" else 0, force_split_k=split)
    try:
        y = ctx.weight16(W, 2048, sh).lm_head(x, 0, 2)
    finally:
        ctx.set_dispatch()
    ref = O.lm_head_w16a16_i32(x, W, 2048, sh, 0, 2)
    assert np.isin(ref, [2**31 - 1, -(2**31)]).any()
    assert np.array_equal(y, ref)


def test_lm_head16_tail_split(ctx):
    """9600 rows = 19200 int8 rows = 150 channel tiles: the last wave runs
    as K slices (tail reduction in the pair mode)."""
    rng = np.random.default_rng(11)
    W, sh, x = _case(rng, 100, 2048, 9600)
    ctx.set_dispatch(gemv_max_m=0)
    try:
        y = ctx.weight16(W, 2048, sh).lm_head(x, 8, 6)
    finally:
        ctx.set_dispatch()
    rows = np.arange(0, 100, 7)
    assert np.array_equal(y[rows], O.lm_head_w16a16_i32(x[rows], W, 2048, sh, 8, 6))


def test_lm_head16_device_path_qwen05b_vocab(ctx):
    """Qwen2.5-0.5B LM head shape (vocab 151936, hidden 896) through
    myl_linear_dev with an i32 plan, decode and a small prefill."""
    rng = np.random.default_rng(5)
    K, N = 896, 151936
    W, sh, _ = _case(rng, 1, K, N)
    w = ctx.weight16(W, K, sh)
    rq = w.requant(myl.RQ_SHIFT_I32, act_frac=8, out_frac=6)
    for M in (1, 16):
        x = np.clip(np.rint(rng.normal(0, 3000, size=(M, K))), -32768, 32767).astype(np.int16)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((M, N), dtype=torch.int32, device="cuda")
        w.linear_dev(rq, xd, yd)
        torch.cuda.synchronize()
        ctx.synchronize()
        cols = np.random.default_rng(M).choice(N, size=4000, replace=False)
        ref = O.lm_head_w16a16_i32(x, W[cols], K, sh[cols], 8, 6)
        assert np.array_equal(yd.cpu().numpy()[:, cols], ref.reshape(M, -1))


def test_lm_head16_rejects_other_entry_points(ctx):
    rng = np.random.default_rng(1)
    W, sh, x = _case(rng, 2, 64, 10)
    w = ctx.weight16(W, 64, sh)
    with pytest.raises(myl.MylError) as ei:
        w.linear(x, 8, 8)
    assert ei.value.code == myl.MYL_ERR_ARG
    with pytest.raises(myl.MylError) as ei:
        w.requant(myl.RQ_SHIFT_I16, act_frac=8, out_frac=6)
    assert ei.value.code == myl.MYL_ERR_ARG
