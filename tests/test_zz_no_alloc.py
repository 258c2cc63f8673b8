"""The allocation-free linear, myl_linear_noalloc_dev, against the regular path.

Callers that reserve their whole device budget up front, or that cannot take
the device-wide stall of cudaMalloc/cudaFree, use this entry point: it keeps
its activation byte planes in a fixed array inside the library instead of a
workspace grown on demand. These tests call it through the C ABI, twice in a
row with different inputs, and require every output element to equal the
regular entry point's (myl_linear_dev; integer results, so the tolerance is
zero). They also check that its calls leave the device's free memory
unchanged, and that a call beyond the fixed array's size is refused.

This file sorts last so that a run stopping at the first failure has run
every other test first; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import myelith_b200 as myl  # noqa: E402

SCRATCH_BYTES = 16 * 1024 * 1024  # MYL_NOALLOC_SCRATCH_BYTES in include/myl_w8a16.h


def noalloc_fn():
    f = myl.load_library().myl_linear_noalloc_dev
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                  C.c_void_p, C.c_int64, C.c_void_p]
    f.restype = C.c_int
    return f


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = myl.Context(0)
    yield c
    c.close()


def _inputs(rng, M, K):
    return np.clip(np.rint(rng.normal(0, 1024, size=(M, K))), -32767, 32767).astype(np.int16)


@pytest.mark.parametrize("M,K,N", [(37, 896, 4864), (300, 3584, 1024), (5, 3584, 2048)])
def test_noalloc_matches_regular_path_twice(ctx, M, K, N):
    rng = np.random.default_rng(M * 7 + K + N)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = rng.integers(11, 14, size=N).astype(np.uint8)
    of = rng.integers(6, 10, size=N).astype(np.uint8)
    w = ctx.weight(W, K, ws)
    rq = w.requant(myl.RQ_SHIFT_I16, act_frac=8, out_frac=of)
    f = noalloc_fn()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream or None
    y_ref = torch.empty((M, N), dtype=torch.int16, device="cuda")
    y_na = torch.empty((M, N), dtype=torch.int16, device="cuda")
    xs = [torch.from_numpy(_inputs(rng, M, K)).cuda() for _ in range(2)]
    torch.cuda.synchronize()
    for call, x in enumerate(xs):  # two calls in a row, different inputs
        w.linear_dev(rq, x, y_ref, stream)
        rc = f(ctx.handle, w.handle, rq.handle, x.data_ptr(), M, x.stride(0), y_na.data_ptr(),
               y_na.stride(0), sp)
        assert rc == 0, myl.load_library().myl_last_error()
        torch.cuda.synchronize()
        ctx.synchronize()
        assert torch.equal(y_na, y_ref), f"call {call}: outputs differ from myl_linear_dev"
    # and both equal the CPU oracle on the last input
    ref = O.linear_w8a16_pc(xs[1].cpu().numpy(), W.reshape(-1), K, ws, 8, of)
    assert np.array_equal(y_na.cpu().numpy(), ref)


@pytest.mark.parametrize("M,mode", [(1, "shift16"), (4, "shift16"), (19, "mult16"), (7, "shift32"),
                                    (SCRATCH_BYTES // (2 * 3584), "shift16")])
def test_noalloc_every_requant_mode_and_size(ctx, M, mode):
    """M = 1 and 4 (where the regular path takes the GEMV), the multiplier and
    i32 requants, and a call that fills the fixed array exactly."""
    rng = np.random.default_rng(M * 13 + len(mode))
    K, N = 3584, 640
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    if mode == "mult16":
        w = ctx.weight(W, K, np.zeros(N, np.uint8))
        mult = rng.integers(1 << 30, (1 << 31) - 1, size=N, endpoint=True).astype(np.int32)
        rq = w.requant(myl.RQ_MULT_I16, mult=mult, shift=rng.integers(20, 28, size=N).astype(np.uint8))
        dt = torch.int16
    else:
        w = ctx.weight(W, K, rng.integers(11, 14, size=N).astype(np.uint8))
        rq = w.requant(myl.RQ_SHIFT_I32 if mode == "shift32" else myl.RQ_SHIFT_I16, act_frac=8,
                       out_frac=rng.integers(6, 10, size=N).astype(np.uint8))
        dt = torch.int32 if mode == "shift32" else torch.int16
    assert 2 * M * K <= SCRATCH_BYTES
    x = torch.from_numpy(_inputs(rng, M, K)).cuda()
    y_ref = torch.empty((M, N), dtype=dt, device="cuda")
    y_na = torch.empty((M, N), dtype=dt, device="cuda")
    stream = torch.cuda.current_stream()
    w.linear_dev(rq, x, y_ref, stream)
    rc = noalloc_fn()(ctx.handle, w.handle, rq.handle, x.data_ptr(), M, x.stride(0), y_na.data_ptr(),
                      y_na.stride(0), stream.cuda_stream or None)
    assert rc == 0, myl.load_library().myl_last_error()
    torch.cuda.synchronize()
    ctx.synchronize()
    assert torch.equal(y_na, y_ref)


def test_noalloc_leaves_free_memory_unchanged(ctx):
    rng = np.random.default_rng(3)
    M, K, N = 128, 3584, 4096
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    w = ctx.weight(W, K, np.full(N, 12, np.uint8))
    rq = w.requant(myl.RQ_SHIFT_I16, act_frac=8, out_frac=8)
    f = noalloc_fn()
    x = torch.from_numpy(_inputs(rng, M, K)).cuda()
    y = torch.empty((M, N), dtype=torch.int16, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream or None
    assert f(ctx.handle, w.handle, rq.handle, x.data_ptr(), M, K, y.data_ptr(), N, sp) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        assert f(ctx.handle, w.handle, rq.handle, x.data_ptr(), M, K, y.data_ptr(), N, sp) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_rejects_calls_beyond_the_fixed_scratch(ctx):
    K, N = 3584, 256
    w = ctx.weight(np.ones((N, K), np.int8), K, np.zeros(N, np.uint8))
    rq = w.requant(myl.RQ_SHIFT_I16, act_frac=0, out_frac=0)
    M = SCRATCH_BYTES // (2 * K) + 1  # one row more than fits
    x = torch.zeros((M, K), dtype=torch.int16, device="cuda")
    y = torch.empty((M, N), dtype=torch.int16, device="cuda")
    rc = noalloc_fn()(ctx.handle, w.handle, rq.handle, x.data_ptr(), M, K, y.data_ptr(), N, None)
    assert rc == myl.MYL_ERR_UNSUPPORTED
    assert b"scratch" in myl.load_library().myl_last_error()
