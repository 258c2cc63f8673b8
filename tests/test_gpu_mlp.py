"""GPU parity of mlp_int (kernels/src/mlp.rs:28-74) and of the fused q/k/v
bias (linear.rs:132-145) against the CPU oracle, bit-exact.

The GPU computes gate and up in one kernel over interleaved weights, applies
the SiLU-LUT product in the epilogue (for M > 4 straight into the down
projection's byte planes) and then the down projection; the oracle runs the
reference's three steps.
"""
import numpy as np
import pytest

import fixtures
import gen
import oracle as O
from make_golden import silu_lut_spec

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import myelith_b200 as myl  # noqa: E402

MODES = {"gemv": dict(gemv_max_m=4), "tc": dict(gemv_max_m=0)}


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = myl.Context(0)
    yield c
    c.close()


def _mlp(ctx, c, p):
    return myl.Mlp(ctx, c["W_gate"], c["W_up"], c["W_down"], c["H"], c["I"], c["gate_w_shifts"],
                   c["up_w_shifts"], c["down_w_shifts"], c["silu_lut"], p["in_frac"], p["gate_out"],
                   p["up_out"], p["down_in"], p["silu_in"], p["offset"], p["silu_out"], c["out_frac"])


@pytest.mark.parametrize("mode", ["gemv", "tc"])
@pytest.mark.parametrize("case", fixtures.mlp_cases(), ids=lambda c: c["name"])
def test_mlp_fixtures(ctx, case, mode):
    ctx.set_dispatch(**MODES[mode])
    try:
        y = _mlp(ctx, case, case["params"])(case["x"])
    finally:
        ctx.set_dispatch()
    assert np.array_equal(y, case["y"])


def test_backend_trait_mlp(ctx):
    _, m = fixtures.backend_parity()
    p = m["params"]
    be = myl.CudaBackend.init(0)
    out = np.zeros(m["H"], np.int16)
    be.mlp(m["x"], m["W_gate"], m["W_up"], m["W_down"], out, m["gate_w_shifts"], m["up_w_shifts"],
           m["down_w_shifts"], m["silu_lut"], p["in_frac"], p["gate_out"], p["up_out"], p["down_in"],
           p["silu_in"], p["offset"], p["silu_out"], m["out_frac"])
    assert out.tolist() == m["y"]


def _random_case(rng, H, I, gate_out=7, silu_in=6):
    lut = silu_lut_spec()
    nh = gen.nominal_shift(H, 12)
    ni = gen.nominal_shift(I, 12)
    return dict(
        H=H, I=I, silu_lut=lut,
        W_gate=rng.integers(-127, 128, size=(I, H), dtype=np.int8),
        W_up=rng.integers(-127, 128, size=(I, H), dtype=np.int8),
        W_down=rng.integers(-127, 128, size=(H, I), dtype=np.int8),
        gate_w_shifts=rng.integers(nh - 1, nh + 2, size=I).astype(np.uint8),
        up_w_shifts=rng.integers(nh - 1, nh + 2, size=I).astype(np.uint8),
        down_w_shifts=rng.integers(ni - 1, ni + 2, size=H).astype(np.uint8),
        out_frac=rng.integers(3, 8, size=H).astype(np.uint8),
    ), dict(in_frac=8, gate_out=gate_out, up_out=7, down_in=7, silu_in=silu_in, offset=8192,
            silu_out=8)


def _oracle(c, p, x):
    return O.mlp_int(x, c["W_gate"], c["W_up"], c["W_down"], c["H"], c["I"], c["gate_w_shifts"],
                     c["up_w_shifts"], c["down_w_shifts"], c["silu_lut"], p["in_frac"], p["gate_out"],
                     p["up_out"], p["down_in"], p["silu_in"], p["offset"], p["silu_out"], c["out_frac"],
                     return_wraps=True)


@pytest.mark.parametrize("H,I", [(896, 4864), (128, 300), (100, 77)])
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 33, 200, 300])
def test_mlp_random(ctx, H, I, M):
    rng = np.random.default_rng(H + I + M)
    c, p = _random_case(rng, H, I)
    x = np.clip(np.rint(rng.normal(0, 2000, size=(M, H))), -32767, 32767).astype(np.int16)
    ctx.set_dispatch()
    y = _mlp(ctx, c, p)(x)
    ref, _ = _oracle(c, p, x)
    assert np.array_equal(y, ref)


def test_mlp_gate_left_shift_wraps_i16(ctx):
    """gate_out_frac < silu_in_frac: the gate is shifted left into the LUT
    domain and `as i16` truncates (mlp.rs:56-57, Rust release wrapping)."""
    rng = np.random.default_rng(5)
    c, p = _random_case(rng, 256, 512, gate_out=4, silu_in=6)
    x = np.clip(np.rint(rng.normal(0, 6000, size=(70, 256))), -32767, 32767).astype(np.int16)
    ref, wraps = _oracle(c, p, x)
    assert wraps > 0
    m = _mlp(ctx, c, p)
    for mode in ("gemv", "tc"):
        ctx.set_dispatch(**MODES[mode])
        try:
            xs = x[:3] if mode == "gemv" else x
            assert np.array_equal(m(xs), ref[: len(xs)]), mode
        finally:
            ctx.set_dispatch()


@pytest.mark.parametrize("split", [2, 5])
@pytest.mark.parametrize("M", [2, 40])
def test_mlp_split_k(ctx, split, M):
    """The SiLU pair epilogue also runs in the split-K reduction."""
    rng = np.random.default_rng(split * 10 + M)
    c, p = _random_case(rng, 2048, 384)
    x = np.clip(np.rint(rng.normal(0, 1500, size=(M, 2048))), -32767, 32767).astype(np.int16)
    ctx.set_dispatch(gemv_max_m=4, force_split_k=split)
    try:
        y = _mlp(ctx, c, p)(x)
    finally:
        ctx.set_dispatch()
    assert np.array_equal(y, _oracle(c, p, x)[0])


def test_mlp_qwen7b_shape(ctx):
    rng = np.random.default_rng(7)
    c, p = _random_case(rng, 3584, 18944)
    m = _mlp(ctx, c, p)
    for M in (1, 64):
        x = np.clip(np.rint(rng.normal(0, 1024, size=(M, 3584))), -32767, 32767).astype(np.int16)
        assert np.array_equal(m(x), _oracle(c, p, x)[0]), M


def test_mlp_device_path(ctx):
    rng = np.random.default_rng(11)
    c, p = _random_case(rng, 896, 4864)
    m = _mlp(ctx, c, p)
    x = np.clip(np.rint(rng.normal(0, 1500, size=(130, 896))), -32767, 32767).astype(np.int16)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((130, 896), dtype=torch.int16, device="cuda")
    m.dev(xd, yd)
    torch.cuda.synchronize()
    ctx.synchronize()
    assert np.array_equal(yd.cpu().numpy(), _oracle(c, p, x)[0])


# ---- q/k/v bias ------------------------------------------------------------------------

@pytest.mark.parametrize("mode,M", [("gemv", 1), ("gemv", 4), ("tc", 9), ("tc", 300)])
def test_linear_bias(ctx, mode, M):
    rng = np.random.default_rng(M + 3)
    K, N = 896, 640
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = rng.integers(10, 13, size=N).astype(np.uint8)
    bias = rng.integers(-32768, 32768, size=N).astype(np.int16)
    bias[:8] = [32767, -32768, 1, -1, 3, -3, 5, -5]
    bsh = rng.integers(0, 12, size=N).astype(np.uint8)
    x = np.clip(np.rint(rng.normal(0, 3000, size=(M, K))), -32767, 32767).astype(np.int16)
    ctx.set_dispatch(**MODES[mode])
    try:
        y = ctx.weight(W, K, ws).linear_bias(x, 8, 6, bias, bsh)
    finally:
        ctx.set_dispatch()
    lin = O.linear_w8a16(x, W.reshape(-1), K, ws, 8, 6)
    ref = np.stack([O.add_bias_i16(row, bias, bsh, 6) for row in lin])
    assert np.array_equal(y, ref)


def test_requant_plan_bias_device(ctx):
    rng = np.random.default_rng(13)
    K, N, M = 512, 384, 70
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = np.full(N, 11, np.uint8)
    bias = rng.integers(-2000, 2000, size=N).astype(np.int16)
    bsh = rng.integers(2, 9, size=N).astype(np.uint8)
    w = ctx.weight(W, K, ws)
    rq = w.requant(myl.RQ_SHIFT_I16, act_frac=6, out_frac=5)
    rq.set_bias(bias, bsh, 5)
    x = rng.integers(-4000, 4000, size=(M, K), dtype=np.int16)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((M, N), dtype=torch.int16, device="cuda")
    w.linear_dev(rq, xd, yd)
    torch.cuda.synchronize()
    lin = O.linear_w8a16(x, W.reshape(-1), K, ws, 6, 5)
    ref = np.stack([O.add_bias_i16(row, bias, bsh, 5) for row in lin])
    assert np.array_equal(yd.cpu().numpy(), ref)


@pytest.mark.parametrize("silu_out,up_out,down_in", [(8, 7, 7), (8, 7, 15), (16, 16, 1), (15, 16, 0),
                                                     (2, 2, 8), (8, 7, 0), (4, 4, 12)])
def test_mlp_product_rescale_range(ctx, silu_out, up_out, down_in):
    """The SiLU product rescale s2 = silu_out + up_out - down_in across the
    32-bit epilogue's cases: s2 in [1, 30], s2 >= 31 (always 0), s2 = 0 and
    s2 < 0 (left shift, clamped)."""
    rng = np.random.default_rng(silu_out * 100 + up_out * 10 + down_in)
    c, p = _random_case(rng, 256, 320)
    p = dict(p, silu_out=silu_out, up_out=up_out, down_in=down_in)
    m = _mlp(ctx, c, p)
    x = np.clip(np.rint(rng.normal(0, 3000, size=(70, 256))), -32767, 32767).astype(np.int16)
    ref = _oracle(c, p, x)[0]
    for mode in ("gemv", "tc"):
        ctx.set_dispatch(**MODES[mode])
        try:
            xs = x[:3] if mode == "gemv" else x
            assert np.array_equal(m(xs), ref[: len(xs)]), mode
        finally:
            ctx.set_dispatch()
