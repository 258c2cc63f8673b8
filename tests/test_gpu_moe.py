"""GPU parity of the MoE layer (router linear, integer top-k + softmax_int,
grouped tensor-core expert GEMMs, combine) against the composition of the
CPU oracle's primitives, bit-exact.

The GPU sorts the (token, choice) pairs by expert and runs every expert's
rows as one segment of a grouped GEMM (gate/up with the SiLU epilogue, then
down); the oracle calls mlp_int per expert on the same rows.
"""
import numpy as np
import pytest

import moe_ref as R

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


def _run_dev(m, x):
    T, k = len(x), m.top_k
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    prob = torch.empty((T, k), dtype=torch.int32, device="cuda")
    m.dev(xd, out, idx, prob)
    torch.cuda.synchronize()
    m.ctx.synchronize()
    return out.cpu().numpy(), idx.cpu().numpy(), prob.cpu().numpy()


@pytest.mark.parametrize("tile", [0, 32, 64, 128])
@pytest.mark.parametrize("shared", [0, 72])
def test_moe_small(ctx, tile, shared):
    # 2I = 192: channel tiles straddle two experts' rows of the stacked weight
    p, s = R.problem(H=128, I=96, E=8, k=2, shared_I=shared, seed=5)
    x = R.activations(np.random.default_rng(1), 37, 128)
    m = R.lib_moe(ctx, p, s)
    ref, ridx, rprob = R.forward(p, s, x)
    ctx.set_dispatch(force_token_tile=tile)
    try:
        out, idx, prob = _run_dev(m, x)
        host = m(x)
    finally:
        ctx.set_dispatch()
    assert np.array_equal(idx, ridx)
    assert np.array_equal(prob, rprob)
    assert np.array_equal(out, ref)
    assert np.array_equal(host, ref)


@pytest.mark.parametrize("T", [1, 2, 3, 4, 5, 130])
def test_moe_token_counts(ctx, T):
    """T <= 4 routes through the GEMV router; the experts always run grouped."""
    p, s = R.problem(H=96, I=80, E=16, k=4, shared_I=64, seed=T)
    x = R.activations(np.random.default_rng(T), T, 96, sigma=2000.0)
    m = R.lib_moe(ctx, p, s)
    assert np.array_equal(m(x), R.forward(p, s, x)[0])


def test_moe_router_ties_lowest_index(ctx):
    """Experts 2/6 and 3/4 have equal router rows: every token sees ties, the
    lower index must come first (sampling.rs:8-18), with equal probabilities."""
    p, s = R.problem(H=64, I=64, E=8, k=3, seed=9, tie_pairs=((2, 6), (3, 4)))
    x = R.activations(np.random.default_rng(2), 50, 64)
    m = R.lib_moe(ctx, p, None)
    out, idx, prob = _run_dev(m, x)
    ref, ridx, rprob = R.forward(p, None, x)
    assert np.array_equal(idx, ridx) and np.array_equal(prob, rprob)
    assert np.array_equal(out, ref)
    pairs = 0
    for t in range(len(x)):
        for a, b in ((2, 6), (3, 4)):
            if a in idx[t] and b in idx[t]:
                ja, jb = list(idx[t]).index(a), list(idx[t]).index(b)
                assert ja < jb and prob[t][ja] == prob[t][jb]
                pairs += 1
    assert pairs > 0


def test_moe_all_experts_chosen_and_k1(ctx):
    for E, k in ((4, 4), (6, 1)):
        p, s = R.problem(H=64, I=48, E=E, k=k, shared_I=32, seed=E * 10 + k)
        x = R.activations(np.random.default_rng(3), 21, 64)
        assert np.array_equal(R.lib_moe(ctx, p, s)(x), R.forward(p, s, x)[0]), (E, k)


def test_moe_saturating_combine(ctx):
    """Large activations: expert outputs and the combine saturate at +-32767."""
    p, s = R.problem(H=128, I=128, E=8, k=2, shared_I=64, seed=4)
    for e in range(8):
        p["out_frac"][e][:] = 7
    x = R.activations(np.random.default_rng(4), 40, 128, sigma=12000.0)
    ref = R.forward(p, s, x)[0]
    assert (np.abs(ref.astype(np.int32)) == 32767).any() or (ref == -32768).any()
    assert np.array_equal(R.lib_moe(ctx, p, s)(x), ref)


def test_moe_stages_expert_parallel_slice(ctx):
    """route / experts / combine as separate calls on an object holding
    experts [4, 10) of 16 (one expert-parallel rank's share)."""
    p, s = R.problem(H=128, I=96, E=16, k=2, shared_I=48, seed=12)
    x = R.activations(np.random.default_rng(5), 60, 128)
    full = R.lib_moe(ctx, p, s)
    part = R.lib_moe(ctx, p, None, first_expert=4, num_local=6)
    xd = torch.from_numpy(x).cuda()
    idx = torch.empty((60, 2), dtype=torch.int32, device="cuda")
    prob = torch.empty_like(idx)
    part.route_dev(xd, idx, prob)
    ridx, rprob = R.route(p, x)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), ridx) and np.array_equal(prob.cpu().numpy(), rprob)
    # rows for the slice's experts only, in arbitrary order
    rng = np.random.default_rng(6)
    ids = rng.integers(4, 10, size=90).astype(np.int32)
    rows = R.activations(rng, 90, 128)
    y = torch.empty((90, 128), dtype=torch.int16, device="cuda")
    part.experts_dev(torch.from_numpy(rows).cuda(), torch.from_numpy(ids).cuda(), y)
    torch.cuda.synchronize()
    ctx.synchronize()
    assert np.array_equal(y.cpu().numpy(), R.experts(p, rows, ids))
    # combine of oracle expert rows + shared output
    ys = R.experts(p, np.repeat(x, 2, axis=0), ridx)
    sh = R.shared_mlp(s, x)
    out = torch.empty((60, 128), dtype=torch.int16, device="cuda")
    full.combine_dev(torch.from_numpy(ys).cuda(), torch.from_numpy(rprob).cuda(),
                     torch.from_numpy(sh).cuda(), out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), R.forward(p, s, x)[0])


def test_moe_bad_expert_id_reports(ctx):
    """An id outside the object's experts gives a zero row and MYL_ERR_DEVICE
    at the next synchronising call; the context stays usable."""
    p, _ = R.problem(H=64, I=32, E=8, k=2, seed=13)
    part = R.lib_moe(ctx, p, None, first_expert=0, num_local=4)
    ids = np.array([0, 1, 7, 3], np.int32)
    rows = R.activations(np.random.default_rng(7), 4, 64)
    y = torch.full((4, 64), 5, dtype=torch.int16, device="cuda")
    part.experts_dev(torch.from_numpy(rows).cuda(), torch.from_numpy(ids).cuda(), y)
    torch.cuda.synchronize()
    with pytest.raises(myl.MylError) as ei:
        ctx.synchronize()
    assert ei.value.code == myl.MYL_ERR_DEVICE
    yy = y.cpu().numpy()
    assert (yy[2] == 0).all()
    good = [0, 1, 3]
    assert np.array_equal(yy[good], R.experts(p, rows[good], ids[good]))
    ctx.synchronize()  # cleared


def test_moe_register_rejects(ctx):
    p, _ = R.problem(H=64, I=32, E=8, k=2, seed=14)
    with pytest.raises(myl.MylError) as ei:
        p2 = dict(p, top_k=9)
        R.lib_moe(ctx, p2, None)
    assert ei.value.code == myl.MYL_ERR_UNSUPPORTED
    with pytest.raises(myl.MylError) as ei:
        R.lib_moe(ctx, dict(p, prob_frac=17), None)  # 16384 * 2^17 overflows i32
    assert ei.value.code == myl.MYL_ERR_OVERFLOW


def test_moe_deterministic(ctx):
    p, s = R.problem(H=256, I=128, E=32, k=4, shared_I=64, seed=15)
    x = R.activations(np.random.default_rng(8), 300, 256)
    m = R.lib_moe(ctx, p, s)
    a = _run_dev(m, x)[0]
    b = _run_dev(m, x)[0]
    assert np.array_equal(a, b)
    assert np.array_equal(a, R.forward(p, s, x)[0])


def test_moe_config4_shape(ctx):
    """hidden 2048, 64 experts x MLP 1408, top-4, shared expert 5632, 4096
    tokens: the routing and the output of every token against the oracle."""
    p, s = R.problem(H=2048, I=1408, E=64, k=4, shared_I=5632, seed=4)
    T = 4096
    x = R.activations(np.random.default_rng(40), T, 2048)
    m = R.lib_moe(ctx, p, s)
    out, idx, prob = _run_dev(m, x)
    ridx, rprob = R.route(p, x)
    assert np.array_equal(idx, ridx) and np.array_equal(prob, rprob)
    ref = R.forward(p, s, x)[0]
    assert np.array_equal(out, ref)


@pytest.mark.parametrize("H,I,T", [(100, 72, 45), (136, 40, 9)])
def test_moe_ragged_hidden(ctx, H, I, T):
    """hidden not a multiple of 8: the gather and combine take their
    element-by-element paths; I not a multiple of 16 pads the h planes."""
    p, s = R.problem(H=H, I=I, E=6, k=2, shared_I=24, seed=H + I)
    x = R.activations(np.random.default_rng(H), T, H)
    m = R.lib_moe(ctx, p, s)
    out, idx, prob = _run_dev(m, x)
    ref, ridx, rprob = R.forward(p, s, x)
    assert np.array_equal(idx, ridx) and np.array_equal(prob, rprob)
    assert np.array_equal(out, ref)
