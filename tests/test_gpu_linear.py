"""GPU parity of the W8A16 linear path against the CPU oracle (bit-exact).

Everything here goes through the C ABI of libmyl_w8a16.so (ctypes), on cuda:0.
Integer work: the bar is equality of every output element. Both kernels are
covered (CUDA-core decode GEMV and the tcgen05 split-byte GEMM, forced through
the dispatch thresholds), with split-K, the weight-as-A (swap) and
activation-as-A tile shapes, ragged K, negative shifts, saturation, the
multiplier requant and the LM-head i32 clamp. At the full config-1 sizes, where
the oracle is too slow for every element, exact checksums cover every
accumulator: sum_n acc[m, n] = x[m] . colsum(W) and sum_m acc[m, n] =
W[n] . sum_m x[m], plus the requant of every element and a sampled set of
rows against the oracle.
"""
import numpy as np
import pytest

import fixtures
import gen
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


def normal_x(rng, M, K, sigma=1024.0):
    return np.clip(np.rint(rng.normal(0.0, sigma, size=(M, K))), -32767, 32767).astype(np.int16)


def rne_shift_np(acc: np.ndarray, s: np.ndarray) -> np.ndarray:
    """Vectorised rescale_i64 (fixed_point.rs:57-71, :184-191) for the
    full-size checks; pinned against the oracle in test_numpy_requant_matches_oracle."""
    acc = acc.astype(np.int64)
    s = np.broadcast_to(s.astype(np.int64), acc.shape)
    pos = np.maximum(s, 1)
    q = acc >> pos
    r = acc & ((np.int64(1) << pos) - 1)
    h = np.int64(1) << (pos - 1)
    up = (r > h) | ((r == h) & ((q & 1) == 1))
    right = q + up.astype(np.int64)
    left = acc << np.maximum(-s, 0)
    return np.where(s > 0, right, np.where(s == 0, acc, left))


MODES = {"gemv": dict(gemv_max_m=4), "tc": dict(gemv_max_m=0)}


def set_mode(ctx, mode, **kw):
    ctx.set_dispatch(**{**MODES[mode], **kw})


# ---- golden fixtures -------------------------------------------------------------

@pytest.mark.parametrize("mode", ["gemv", "tc"])
@pytest.mark.parametrize("case", fixtures.linear_cases(), ids=lambda c: c["name"])
def test_linear_fixtures(ctx, case, mode):
    set_mode(ctx, mode)
    c = case
    w = ctx.weight(c["W"], c["K"], c["w_shifts"])
    if c["kind"] == "lm_head":
        y = w.lm_head(c["x"], c["act_frac"], c["out_frac"])
    else:
        y = w.linear(c["x"], c["act_frac"], c["out_frac"])
    assert np.array_equal(y, c["y"])


def test_op_golden_vector(ctx):
    set_mode(ctx, "gemv")
    for v in fixtures.op_vectors():
        W = np.array(v["W"], np.int8)
        y = myl.Weight(ctx, W, W.shape[1], v["w_shifts"]).linear(np.array(v["x"]), v["act_frac"],
                                                                  v["out_frac"])
        assert y.tolist() == v["y"]


def test_backend_parity_fixture(ctx):
    lin, _ = fixtures.backend_parity()
    be = myl.CudaBackend.init(0)
    out = np.zeros(lin["N"], np.int16)
    be.linear_w8a16(lin["x"], lin["W"], out, lin["K"], lin["N"], lin["w_shifts"], lin["act_frac"],
                    lin["out_frac"])
    assert out.tolist() == lin["y"]


# ---- random shapes vs the oracle ----------------------------------------------------

SHAPES = [
    # M, K, N
    (1, 896, 4864), (2, 896, 4864), (3, 896, 1000), (4, 3584, 2048),
    (5, 896, 4864), (16, 3584, 1024), (33, 1000, 700), (64, 896, 4864),
    (128, 3584, 512), (129, 896, 300), (200, 512, 640), (256, 3584, 256),
    (257, 896, 1024), (512, 896, 4864), (300, 136, 520),
]


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_random_vs_oracle(ctx, M, K, N):
    rng = np.random.default_rng(M * 1000003 + K * 31 + N)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    x = normal_x(rng, M, K)
    ks = gen.nominal_shift(K, 12)
    w_shifts = rng.integers(ks - 1, ks + 2, size=N).astype(np.uint8)
    out_frac = rng.integers(6, 11, size=N).astype(np.uint8)
    ctx.set_dispatch()  # automatic selection
    w = ctx.weight(W, K, w_shifts)
    ref = O.linear_w8a16_pc(x, W.reshape(-1), K, w_shifts, 8, out_frac)
    assert np.array_equal(w.linear(x, 8, out_frac), ref)
    ref_s = O.linear_w8a16(x, W.reshape(-1), K, w_shifts, 8, 8)
    assert np.array_equal(w.linear(x, 8, 8), ref_s)


@pytest.mark.parametrize("split", [2, 3, 7])
@pytest.mark.parametrize("mode,M", [("gemv", 1), ("gemv", 3), ("tc", 8), ("tc", 300)])
def test_forced_split_k(ctx, split, mode, M):
    rng = np.random.default_rng(split * 7 + M)
    K, N = 3584, 777
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    x = normal_x(rng, M, K, 4000.0)
    w_shifts = rng.integers(12, 16, size=N).astype(np.uint8)
    set_mode(ctx, mode, force_split_k=split)
    try:
        y = ctx.weight(W, K, w_shifts).linear(x, 6, 6)
    finally:
        ctx.set_dispatch()
    assert np.array_equal(y, O.linear_w8a16(x, W.reshape(-1), K, w_shifts, 6, 6))


@pytest.mark.parametrize("tile", [32, 64, 128])
@pytest.mark.parametrize("M", [5, 40, 130, 256, 400])
def test_tile_shapes(ctx, tile, M):
    rng = np.random.default_rng(M + 17 * tile)
    K, N = 1152, 640
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    x = rng.integers(-32768, 32768, size=(M, K), dtype=np.int16)  # full int16 range
    w_shifts = rng.integers(16, 20, size=N).astype(np.uint8)
    set_mode(ctx, "tc", force_token_tile=tile)
    try:
        y = ctx.weight(W, K, w_shifts).linear(x, 4, 4)
    finally:
        ctx.set_dispatch()
    assert np.array_equal(y, O.linear_w8a16(x, W.reshape(-1), K, w_shifts, 4, 4))


# ---- edge cases -----------------------------------------------------------------------

@pytest.mark.parametrize("mode", ["gemv", "tc"])
def test_extreme_values_exact(ctx, mode):
    """All products at their largest magnitude (dot.rs:641-656, linear.rs:178)."""
    set_mode(ctx, mode)
    for K in (896, 4864, 18944):
        for wv, xv in ((127, 32767), (-128, 32767), (-128, -32768), (-128, -32513)):
            W = np.full((8, K), wv, np.int8)
            x = np.full((2 if mode == "gemv" else 9, K), xv, np.int16)
            w = ctx.weight(W, K, np.zeros(8, np.uint8))
            acc = O.linear_acc_i64(x, W.reshape(-1), K, 8)
            assert acc[0, 0] == K * wv * xv
            # LM-head path keeps 31 bits: shift down so the value survives the clamp.
            y = w.lm_head(x, 0, 0)
            assert np.array_equal(y, O.lm_head_w8a16_i32(x, W.reshape(-1), K, np.zeros(8), 0, 0))
            y16 = w.linear(x, 20, 0)
            assert np.array_equal(y16, O.linear_w8a16(x, W.reshape(-1), K, np.zeros(8), 20, 0))


def test_k_beyond_int32_slice_limit(ctx):
    """K > 65536 is split into int32-exact slices whose partials add in int64."""
    K, N, M = 70000, 64, 9
    W = np.full((N, K), -128, np.int8)
    x = np.full((M, K), -32513, np.int16)  # hi = -128, lo = 255: both MMAs at their bound
    set_mode(ctx, "tc")
    y = ctx.weight(W, K, np.full(N, 20, np.uint8)).lm_head(x, 0, 0)
    ctx.set_dispatch()
    assert np.array_equal(y, O.lm_head_w8a16_i32(x, W.reshape(-1), K, np.full(N, 20), 0, 0))


@pytest.mark.parametrize("M", [1, 2, 3, 4])
@pytest.mark.parametrize("K,N", [(18944, 64), (18944, 3584), (4096, 2048), (3584, 18944),
                                 (8192, 200), (1000, 777)])
def test_gemv_variants(ctx, M, K, N):
    """Shapes that select each GEMV variant: rows per warp, chunks in flight and
    warps per row group (K split inside a block)."""
    rng = np.random.default_rng(M * 7 + K + N)
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    x = normal_x(rng, M, K, 3000.0)
    ks = gen.nominal_shift(K, 13)
    ws = rng.integers(ks - 1, ks + 2, size=N).astype(np.uint8)
    set_mode(ctx, "gemv")
    y = ctx.weight(W, K, ws).linear(x, 8, 8)
    ctx.set_dispatch()
    assert np.array_equal(y, O.linear_w8a16(x, W.reshape(-1), K, ws, 8, 8))


@pytest.mark.parametrize("M", [1, 3])
def test_gemv_k_split_across_blocks(ctx, M):
    """x rows too long for one block's shared memory: the GEMV splits K
    across blocks and adds the exact int64 partials."""
    rng = np.random.default_rng(70 + M)
    K, N = 70000, 64
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    x = rng.integers(-32768, 32768, size=(M, K), dtype=np.int16)
    set_mode(ctx, "gemv")
    y = ctx.weight(W, K, np.full(N, 22, np.uint8)).linear(x, 0, 0)
    ctx.set_dispatch()
    assert np.array_equal(y, O.linear_w8a16(x, W.reshape(-1), K, np.full(N, 22), 0, 0))


def test_negative_shift_and_saturation(ctx):
    rng = np.random.default_rng(3)
    K, N = 640, 256
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    for M in (1, 77):
        x = rng.integers(-64, 64, size=(M, K), dtype=np.int16)
        w = ctx.weight(W, K, np.zeros(N, np.uint8))
        of = rng.integers(0, 12, size=N).astype(np.uint8)  # left shifts up to 12
        ctx.set_dispatch()
        y = w.linear(x, 0, of)
        ref = O.linear_w8a16_pc(x, W.reshape(-1), K, np.zeros(N, np.uint8), 0, of)
        assert np.array_equal(y, ref)
        assert (np.abs(ref.astype(np.int32)) == 32767).any() or (ref == -32768).any()


def test_ragged_and_tiny(ctx):
    rng = np.random.default_rng(11)
    for K in (1, 2, 3, 15, 17, 31, 129, 255):
        for M in (1, 4, 5, 19):
            N = 33
            W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
            x = rng.integers(-32768, 32768, size=(M, K), dtype=np.int16)
            ws = rng.integers(0, 9, size=N).astype(np.uint8)
            y = ctx.weight(W, K, ws).linear(x, 3, 5)
            assert np.array_equal(y, O.linear_w8a16(x, W.reshape(-1), K, ws, 3, 5)), (K, M)


def test_empty_inputs(ctx):
    W = np.ones((4, 8), np.int8)
    w = ctx.weight(W, 8, np.zeros(4, np.uint8))
    assert w.linear(np.zeros((0, 8), np.int16), 0, 0).shape == (0, 4)
    w0 = ctx.weight(np.zeros((0, 8), np.int8), 8, np.zeros(0, np.uint8))
    assert w0.linear(np.ones((3, 8), np.int16), 0, 0).shape == (3, 0)


def test_shape_and_overflow_errors(ctx):
    W = np.ones((4, 8), np.int8)
    with pytest.raises(myl.MylError) as e:
        myl.Weight(ctx, W.reshape(-1)[:30], 8, np.zeros(4, np.uint8))
    assert e.value.code == myl.MYL_ERR_SHAPE
    w = ctx.weight(W, 8, np.full(4, 200, np.uint8))
    with pytest.raises(myl.MylError) as e:
        w.linear(np.ones(8, np.int16), 100, 0)  # 200 + 100 overflows u8 (linear.rs:66)
    assert e.value.code == myl.MYL_ERR_OVERFLOW
    w = ctx.weight(W, 8, np.full(4, 63, np.uint8))
    with pytest.raises(myl.MylError) as e:
        w.linear(np.ones(8, np.int16), 0, 0)  # right shift 63: (1 << 63) - 1 overflows
    assert e.value.code == myl.MYL_ERR_OVERFLOW
    with pytest.raises(myl.MylError):
        myl.linear_w8a16(np.ones(3, np.int16), np.ones(7, np.int8), 3, [0, 0], 0, 0)


# ---- requant variants ------------------------------------------------------------------

@pytest.mark.parametrize("mode", ["gemv", "tc"])
def test_multiplier_requant(ctx, mode):
    rng = np.random.default_rng(5)
    K, N, M = 896, 4864, (1 if mode == "gemv" else 48)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    x = normal_x(rng, M, K)
    mult = rng.integers(1 << 30, (1 << 31) - 1, size=N, endpoint=True).astype(np.int32)
    set_mode(ctx, mode)
    w = ctx.weight(W, K, np.zeros(N, np.uint8))
    for lo, hi in ((51, 59), (20, 28)):  # Q31 multiplier, and the literal right shift
        shift = rng.integers(lo, hi + 1, size=N).astype(np.uint8)
        y = w.linear_mult(x, mult, shift)
        assert np.array_equal(y, O.linear_w8a16_mult(x, W.reshape(-1), K, mult, shift))
    # pow2 multiplier == reference shift (fixed_point.rs:365-379)
    ws = rng.integers(10, 13, size=N).astype(np.uint8)
    y = w.linear_mult(x, np.full(N, 1 << 12, np.int32), (ws + 12).astype(np.uint8))
    assert np.array_equal(y, O.linear_w8a16(x, W.reshape(-1), K, ws, 0, 0))


def _tie_tokens(rng):
    """Activations x = [a, b] with 127*a + b equal to exact RNE ties (2k+1)*2^(s-1)
    for s = 1..22, both signs, plus random values."""
    accs = []
    for s in range(1, 23):
        for k in (0, 1, 2, 5):
            v = (2 * k + 1) << (s - 1)
            if v <= 127 * 32000:
                accs += [v, -v, v + 1, -v - 1]
    accs += rng.integers(-127 * 32000, 127 * 32000, size=200).tolist()
    x = []
    for acc in accs:
        a = int(np.floor(acc / 127.0))
        b = acc - 127 * a
        if b > 100:
            a, b = a + 1, b - 127
        x.append([a, b])
    return np.array(x, np.int16)


@pytest.mark.parametrize("mode", ["gemv", "tc"])
def test_requant_every_shift_with_ties(ctx, mode):
    """Channel r uses the signed total shift s = r - 5 (s in [-5, 45]); the
    tensor-core epilogue's 32-bit fast path covers s in [8, 38], the rest runs
    in 64-bit. Ties are constructed exactly (K = 2, row [127, 1])."""
    rng = np.random.default_rng(123)
    N = 51
    ws = np.arange(N, dtype=np.uint8)
    of = np.full(N, 5, np.uint8)
    W2 = np.tile(np.array([127, 1], np.int8), (N, 1))
    x = _tie_tokens(rng)
    xs = [x[:2], x[:4]] if mode == "gemv" else [x]
    set_mode(ctx, mode)
    w = ctx.weight(W2, 2, ws)
    for xx in xs:
        assert np.array_equal(w.linear(xx, 0, of), O.linear_w8a16_pc(xx, W2.reshape(-1), 2, ws, 0, of))
        assert np.array_equal(w.lm_head(xx, 0, 5), O.lm_head_w8a16_i32(xx, W2.reshape(-1), 2, ws, 0, 5))
    # large accumulators (~2^35) for the upper shifts
    K = 4096
    Wb = rng.integers(64, 128, size=(N, K), dtype=np.int8)
    xb = rng.integers(16384, 32768, size=(2 if mode == "gemv" else 40, K), dtype=np.int16)
    xb[1::2] *= -1
    wb = ctx.weight(Wb, K, ws)
    assert np.array_equal(wb.linear(xb, 0, of), O.linear_w8a16_pc(xb, Wb.reshape(-1), K, ws, 0, of))
    assert np.array_equal(wb.lm_head(xb, 0, 5), O.lm_head_w8a16_i32(xb, Wb.reshape(-1), K, ws, 0, 5))
    ctx.set_dispatch()


def test_numpy_requant_matches_oracle():
    rng = np.random.default_rng(9)
    acc = rng.integers(-(1 << 40), 1 << 40, size=4000).astype(np.int64)
    acc[:50] = np.arange(-25, 25)
    for s in range(-20, 63):
        got = rne_shift_np(acc, np.full(acc.shape, s))
        want = [O.rescale_i64(int(a), max(s, 0), max(-s, 0)) for a in acc[:300]]
        assert got[:300].tolist() == want


# ---- backend trait mirror and the reference free functions -------------------------

def test_cuda_backend_trait(ctx):
    rng = np.random.default_rng(21)
    K, N = 896, 896
    W = rng.integers(-127, 128, size=N * K, dtype=np.int8)
    ws = rng.integers(10, 13, size=N).astype(np.uint8)
    be = myl.CudaBackend.init(0)
    assert be.name() == "cuda" and be.sm_version() >= 100
    for _ in range(3):
        x = normal_x(rng, 1, K)[0]
        out = np.zeros(N, np.int16)
        be.linear_w8a16(x, W, out, K, N, ws, 8, 8)
        assert np.array_equal(out, O.linear_w8a16(x, W, K, ws, 8, 8))
    ws2 = (ws + 1).astype(np.uint8)  # new shift table: the cached upload must not be reused
    out = np.zeros(N, np.int16)
    be.linear_w8a16(x, W, out, K, N, ws2, 8, 8)
    assert np.array_equal(out, O.linear_w8a16(x, W, K, ws2, 8, 8))
    # new weight bytes at the same address and the same shift table: re-uploaded
    W[:] = rng.integers(-127, 128, size=N * K, dtype=np.int8)
    W[7] = np.int8(-128)
    out = np.zeros(N, np.int16)
    be.linear_w8a16(x, W, out, K, N, ws2, 8, 8)
    assert np.array_equal(out, O.linear_w8a16(x, W, K, ws2, 8, 8))


def test_free_functions(ctx):
    rng = np.random.default_rng(22)
    K, N = 300, 129
    W = rng.integers(-127, 128, size=N * K, dtype=np.int8)
    ws = rng.integers(9, 12, size=N).astype(np.uint8)
    x = normal_x(rng, 3, K)
    of = rng.integers(5, 9, size=N).astype(np.uint8)
    assert np.array_equal(myl.linear_w8a16(x, W, K, ws, 8, 7), O.linear_w8a16(x, W, K, ws, 8, 7))
    assert np.array_equal(myl.linear_w8a16_pc(x, W, K, ws, 8, of), O.linear_w8a16_pc(x, W, K, ws, 8, of))
    assert np.array_equal(myl.lm_head_w8a16_i32(x, W, K, ws, 8, 6),
                          O.lm_head_w8a16_i32(x, W, K, ws, 8, 6))


# ---- device path, tensor-parallel partial sums -----------------------------------------

def test_device_path_and_partial_sums(ctx):
    rng = np.random.default_rng(31)
    K, N, M = 3584, 2048, 96
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    x = normal_x(rng, M, K)
    ws = rng.integers(11, 14, size=N).astype(np.uint8)
    of = rng.integers(6, 10, size=N).astype(np.uint8)
    ref = O.linear_w8a16_pc(x, W.reshape(-1), K, ws, 8, of)
    ctx.set_dispatch()
    w = ctx.weight(W, K, ws)
    rq = w.requant(myl.RQ_SHIFT_I16, act_frac=8, out_frac=of)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((M, N), dtype=torch.int16, device="cuda")
    w.linear_dev(rq, xd, yd)
    torch.cuda.synchronize()
    ctx.synchronize()
    assert np.array_equal(yd.cpu().numpy(), ref)
    # acc + separate requant == fused epilogue
    acc = torch.empty((M, N), dtype=torch.int64, device="cuda")
    w.linear_acc_dev(xd, acc)
    y2 = torch.empty_like(yd)
    rq.apply_acc_dev(acc, y2)
    torch.cuda.synchronize()
    assert np.array_equal(y2.cpu().numpy(), ref)
    # row-parallel shards (K split over 2/4/8 "ranks"): int64 partials add up exactly
    for tp in (2, 4, 8):
        kk = K // tp
        tot = torch.zeros((M, N), dtype=torch.int64, device="cuda")
        for r in range(tp):
            wr = myl.Weight(ctx, W[:, r * kk:(r + 1) * kk].copy(), kk, ws)
            part = torch.empty((M, N), dtype=torch.int64, device="cuda")
            wr.linear_acc_dev(xd[:, r * kk:(r + 1) * kk].contiguous(), part)
            tot += part
        y3 = torch.empty_like(yd)
        rq.apply_acc_dev(tot, y3)
        torch.cuda.synchronize()
        assert np.array_equal(y3.cpu().numpy(), ref), tp


# ---- full config-1 sizes ---------------------------------------------------------------

@pytest.mark.parametrize("K,N", [(3584, 18944), (18944, 3584)])
@pytest.mark.parametrize("M", [1, 16, 128, 2048])
def test_config1_full_size(ctx, K, N, M):
    rng = np.random.default_rng(K + N + M)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    x = normal_x(rng, M, K)
    ks = gen.nominal_shift(K, 12)
    ws = rng.integers(ks - 1, ks + 2, size=N).astype(np.uint8)
    ctx.set_dispatch()
    w = ctx.weight(W, K, ws)
    xd = torch.from_numpy(x).cuda()
    acc = torch.empty((M, N), dtype=torch.int64, device="cuda")
    w.linear_acc_dev(xd, acc)
    rq = w.requant(myl.RQ_SHIFT_I16, act_frac=8, out_frac=8)
    y = torch.empty((M, N), dtype=torch.int16, device="cuda")
    w.linear_dev(rq, xd, y)
    torch.cuda.synchronize()
    ctx.synchronize()
    acc_h = acc.cpu().numpy()
    y_h = y.cpu().numpy()
    # exact checksums over every accumulator
    colsum = W.astype(np.int64).sum(axis=0)
    assert np.array_equal(acc_h.sum(axis=1), x.astype(np.int64) @ colsum)
    xsum = x.astype(np.int64).sum(axis=0)
    assert np.array_equal(acc_h.sum(axis=0), W.astype(np.int64) @ xsum)
    # requant of every element
    s = (ws.astype(np.int64) + 8 - 8)[None, :]
    assert np.array_equal(y_h, np.clip(rne_shift_np(acc_h, s), -32768, 32767).astype(np.int16))
    # every element against the oracle (and every int64 accumulator)
    assert np.array_equal(acc_h, O.linear_acc_fast(x, W.reshape(-1), K, N))
    ref = O.linear_w8a16_fast(x, W.reshape(-1), K, ws, 8, 8)
    assert np.array_equal(y_h, ref)


# ---- failure detection without a GPU fault -------------------------------------------------

def test_bounded_wait_reports_error_and_context_survives(ctx):
    rng = np.random.default_rng(41)
    K, N, M = 512, 256, 64
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    x = normal_x(rng, M, K)
    ws = np.full(N, 10, np.uint8)
    w = ctx.weight(W, K, ws)
    set_mode(ctx, "tc")
    ctx.set_wait_timeout_ns(50_000_000)  # 50 ms
    ctx.inject_wait_fault(True)
    try:
        with pytest.raises(myl.MylError) as e:
            w.linear(x, 8, 8)
        assert e.value.code == myl.MYL_ERR_DEVICE
    finally:
        ctx.inject_wait_fault(False)
        ctx.set_wait_timeout_ns(2_000_000_000)
        ctx.set_dispatch()
    # the context is still usable and correct
    assert np.array_equal(w.linear(x, 8, 8), O.linear_w8a16(x, W.reshape(-1), K, ws, 8, 8))


def test_launch_count_increases(ctx):
    n0 = ctx.launch_count
    w = ctx.weight(np.ones((16, 32), np.int8), 32, np.zeros(16, np.uint8))
    w.linear(np.ones((2, 32), np.int16), 0, 0)
    assert ctx.launch_count > n0


@pytest.mark.parametrize("M", [256, 1000, 2048])
def test_host_call_pinned_pipeline(ctx, M):
    """Page-locked x and y: myl_linear_w8a16 runs the rows in chunks with the
    copies overlapping the kernels; equal to the one-pass (pageable) call and
    to the oracle."""
    rng = np.random.default_rng(M)
    K, N = 896, 4864
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = rng.integers(11, 14, size=N).astype(np.uint8)
    x = normal_x(rng, M, K)
    w = ctx.weight(W, K, ws)
    L = myl.load_library()
    xp = torch.from_numpy(x).pin_memory()
    yp = torch.zeros((M, N), dtype=torch.int16).pin_memory()
    myl._check("myl_linear_w8a16", L.myl_linear_w8a16(ctx.handle, w.handle, xp.data_ptr(), M, 8, 8,
                                                      yp.data_ptr()))
    plain = w.linear(x, 8, 8)
    assert np.array_equal(yp.numpy(), plain)
    rows = np.random.default_rng(1).choice(M, size=8, replace=False)
    assert np.array_equal(plain[rows], O.linear_w8a16(x[rows], W.reshape(-1), K, ws, 8, 8))
