"""GPU parity of linear_backward (kernels/src/backward.rs:147-211) against the
CPU oracle, bit-exact: gx with the summands aligned to the largest shift and
rounded once (i128), and the outer product gw.
"""
import numpy as np
import pytest

import fixtures
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


def test_backward_golden_vector(ctx):  # conformance/vectors/op/backward_linear.golden.json
    for c in fixtures.backward_cases():
        W = np.asarray(c["W"], np.int8).reshape(len(c["w_shifts"]), c["in_features"])
        w = ctx.weight(W, c["in_features"], c["w_shifts"])
        gx, gw = w.backward(c["g"], c["x"], c["g_frac"], c["gx_frac"])
        assert gx.reshape(-1).tolist() == c["gx"]
        assert gw.reshape(-1).tolist() == c["gW"]


@pytest.mark.parametrize("M,N,K", [(1, 37, 29), (5, 300, 130), (9, 896, 1000), (2, 4864, 896)])
def test_backward_random(ctx, M, N, K):
    rng = np.random.default_rng(M + N + K)
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    shifts = rng.integers(0, 21, size=N).astype(np.uint8)
    g = rng.integers(-(2**31), 2**31, size=(M, N), dtype=np.int64).astype(np.int32)
    g[:, ::4] = rng.integers(-100, 100, size=g[:, ::4].shape)
    x = rng.integers(-32768, 32768, size=(M, K), dtype=np.int16)
    w = ctx.weight(W, K, shifts)
    for g_frac, gx_frac in ((6, 6), (10, 3), (2, 9)):
        gx, gw = w.backward(g, x, g_frac, gx_frac, want_gw=(g_frac == 6))
        rgx, rgw = O.linear_backward(g, x, W, K, shifts, g_frac, gx_frac, want_gw=(g_frac == 6))
        assert np.array_equal(gx, rgx), (g_frac, gx_frac)
        if rgw is not None:
            assert np.array_equal(gw, rgw)


def test_backward_device_path_and_rounding(ctx):
    """Summands that round to 0 one by one but not together (backward.rs:167-178),
    through the device entry point."""
    N, K = 6, 16
    W = np.ones((N, K), np.int8)
    w = ctx.weight(W, K, np.full(N, 4, np.uint8))
    g = torch.full((3, N), -6, dtype=torch.int32, device="cuda")
    x = torch.zeros((3, K), dtype=torch.int16, device="cuda")
    gx = torch.empty((3, K), dtype=torch.int32, device="cuda")
    w.backward_dev(g, x, 6, 6, gx)
    torch.cuda.synchronize()
    assert (gx.cpu().numpy() == -2).all()


def test_backward_rejects(ctx):
    w = ctx.weight(np.ones((2, 4), np.int8), 4, [65, 1])
    with pytest.raises(myl.MylError) as ei:
        w.backward(np.ones((1, 2), np.int32), np.ones((1, 4), np.int16), 0, 0)
    assert ei.value.code == myl.MYL_ERR_UNSUPPORTED
    w = ctx.weight(np.ones((2, 4), np.int8), 4, [1, 1])
    with pytest.raises(myl.MylError) as ei:  # i8 difference 100 - (-56) overflows
        w.backward(np.ones((1, 2), np.int32), np.ones((1, 4), np.int16), 100, 200)
    assert ei.value.code == myl.MYL_ERR_OVERFLOW
