"""Pins the CPU oracle to the reference.

Every known-answer test of the reference that touches the W8A16 path is
replayed here against the oracle (oracle/myl_oracle.c):
  fixed_point.rs:210-228 (RNE basics), :248-295 (division_semantics_vector),
  :303-333 (overflow_saturation_vector), :365-379 (pow2 multiplier identity);
  linear.rs:152-261 (linear and bias KATs); dot.rs:528-664 (reduction order,
  overflow bound, extremes, hand computation, zip semantics); prng.rs:57.
Then the fixtures of tests/golden (computed by the reference's own Python
restatement, generate.py:37-106) and the op golden vector
linear_w8a16_identity.
"""
import numpy as np
import pytest

import fixtures
import gen
import oracle as O


# ---- fixed_point.rs ---------------------------------------------------------

def test_rshift_round_basic():  # fixed_point.rs:210-222
    assert [O.rshift_round(v, 1) for v in (4, 3, 5, 7)] == [2, 2, 2, 4]
    assert [O.rshift_round(v, 1) for v in (-5, -4, -3)] == [-2, -2, -2]


def test_rescale_kat():  # fixed_point.rs:225-228
    assert O.rescale(127 * 127, 13, 6) == 126


DIVISION_VECTOR = [  # fixed_point.rs:251-275 (value, shift, expected)
    (0, 3, 0), (1, 1, 0), (2, 1, 1), (3, 1, 2), (4, 1, 2), (5, 1, 2), (6, 1, 3), (7, 1, 4),
    (8, 3, 1), (12, 3, 2), (1_000_000, 8, 3906),
    (-1, 1, 0), (-2, 1, -1), (-3, 1, -2), (-4, 1, -2), (-5, 1, -2), (-6, 1, -3), (-7, 1, -4),
    (-8, 3, -1), (-12, 3, -2), (-1_000_000, 8, -3906),
]


@pytest.mark.parametrize("value,shift,expected", DIVISION_VECTOR)
def test_division_semantics_vector(value, shift, expected):
    assert O.rshift_round(value, shift) == expected
    assert O.rshift_round_i64(value, shift) == expected


def test_overflow_saturation_vector():  # fixed_point.rs:303-333
    i32max, i32min = 2**31 - 1, -(2**31)
    i64max, i64min = 2**63 - 1, -(2**63)
    assert O.clamp_i8(i32max) == 127 and O.clamp_i8(i32min) == -128
    assert [O.clamp_i8(v) for v in (127, 128, -128, -129)] == [127, 127, -128, -128]
    assert O.clamp_i16(i32max) == 32767 and O.clamp_i16(i32min) == -32768
    assert [O.clamp_i16(v) for v in (32767, 32768, -32768, -32769)] == [32767, 32767, -32768, -32768]
    assert O.clamp_i16_from_i64(i64max) == 32767 and O.clamp_i16_from_i64(i64min) == -32768
    assert O.clamp_i16_from_i64(32768) == 32767 and O.clamp_i16_from_i64(-32769) == -32768
    assert O.clamp_i32(i64max) == i32max and O.clamp_i32(i64min) == i32min
    assert O.clamp_i32(i32max + 1) == i32max and O.clamp_i32(i32min - 1) == i32min


def test_pow2_multiplier_equals_shift():  # fixed_point.rs:365-379
    m = 12
    for x in (-100_003, -8, -7, -1, 0, 1, 7, 8, 9, 100_003, 1 << 30):
        for n in (1, 3, 5, 8, 16):
            assert O.rshift_round_i64(x, n) == O.rshift_round_i64(x * (1 << m), n + m)


def test_pow2_multiplier_mode_matches_reference_mode():
    """The multiplier epilogue with mult = 2^m and shift = s + m is the
    reference's pure shift (the identity above, on whole linear layers)."""
    K, N = 256, 64
    W = gen.int8_tensor(5, N * K)
    x = gen.int16_tensor(6, 3 * K).reshape(3, K)
    w_shifts = gen.uint8_tensor(7, N, 8, 14)
    ref = O.linear_w8a16(x, W, K, w_shifts, 6, 6)
    for m in (0, 1, 12, 30):
        mult = np.full(N, 1 << m, np.int64).astype(np.int32) if m < 31 else None
        shift = (w_shifts.astype(int) + m).astype(np.uint8)
        assert np.array_equal(O.linear_w8a16_mult(x, W, K, mult, shift), ref)


def test_rescale_overflow_is_an_error():
    # w_shift + act_frac overflowing u8, i8 subtraction overflow, shift >= width.
    with pytest.raises(O.OracleError):
        O.linear_w8a16([1], [1], 1, [200], 100, 0)
    with pytest.raises(O.OracleError):
        O.rescale_i64(1, 63, 0)          # mask (1 << 63) - 1 overflows i64
    with pytest.raises(O.OracleError):
        O.rescale(1, 0, 32)              # 1 << 32 on i32
    assert O.rescale_i64(1, 62, 0) == 0  # largest valid right shift
    assert O.rescale_i64(-1, 0, 63) == -(1 << 63)  # left shift by 63 wraps bits away


# ---- linear.rs:152-261 ---------------------------------------------------------

def test_linear_identity():  # linear.rs:152-162
    assert O.linear_w8a16([64, -64], [127, 0, 0, 127], 2, [7, 7], 6, 6).tolist() == [64, -64]


def test_linear_per_channel_shifts():  # linear.rs:165-175
    assert O.linear_w8a16([64], [64, 64], 1, [7, 6], 6, 6).tolist() == [32, 64]


def test_linear_large_accumulator():  # linear.rs:178-190
    n = 896
    out = O.linear_w8a16(np.full(n, 32767, np.int16), np.full(n, 127, np.int8), n, [7], 5, 3)
    assert out[0] == 32767


def test_linear_pc_uniform_matches_scalar():  # linear.rs:193-204
    x, W, s = [100, -50, 25], [64, -32, 16, 10, 20, -30], [6, 5]
    assert np.array_equal(O.linear_w8a16(x, W, 3, s, 4, 6), O.linear_w8a16_pc(x, W, 3, s, 4, [6, 6]))


def test_linear_pc_different_targets():  # linear.rs:207-222
    out = O.linear_w8a16_pc([100, 100], [64] * 4, 2, [6, 6], 0, [6, 3])
    assert out.tolist() == [12800, 1600]


def test_linear_shape_mismatch_is_an_error():  # linear.rs:51-58
    with pytest.raises(O.OracleError):
        O.linear_w8a16([1, 2], [1, 2, 3], 2, [0, 0], 0, 0)
    with pytest.raises(O.OracleError):
        O.linear_w8a16_pc([1, 2], [1, 2, 3, 4], 2, [0, 0], 0, [0])


def test_add_bias_kats():  # linear.rs:225-254
    assert O.add_bias_i16([10, -10], [1, 1], [2, 2], 4).tolist() == [14, -6]
    assert O.add_bias_i16([0, 0], [3, -3], [3, 3], 1).tolist() == [1, -1]
    assert O.add_bias_i16([0, 0], [4, 4], [1, 0], 0).tolist() == [2, 4]
    assert O.add_bias_i16([32766, -32767, 0], [4, -4, 0], [1, 1, 1], 0).tolist() == [32767, -32768, 0]
    with pytest.raises(O.OracleError):  # linear.rs:256-261
        O.add_bias_i16([0, 0, 0], [1, 1], [0, 0], 0)


# ---- dot.rs ----------------------------------------------------------------------

def _tree(p):
    p = list(p)
    while len(p) > 1:
        p = [sum(p[i:i + 2]) for i in range(0, len(p), 2)]
    return p[0] if p else 0


@pytest.mark.parametrize("n", [1, 2, 3, 7, 64, 255, 896, 4864, 18944, 20000])
def test_every_reduction_order_is_equal(n):  # dot.rs:528-558
    i = np.arange(n, dtype=np.int64)
    w = (((i * 37) % 255).astype(np.int64) - 127).astype(np.int8)
    x = (((i * 8191) % 65535) - 32767).astype(np.int16)
    fwd = O.dot_scalar(w, x)
    assert O.dot_scalar(w[::-1], x[::-1]) == fwd
    prods = w.astype(np.int64) * x.astype(np.int64)
    assert _tree(prods.tolist()) == fwd
    for block in (32, 64, 256, 1024):
        assert sum(O.dot_scalar(w[b:b + block], x[b:b + block]) for b in range(0, n, block)) == fwd


def test_accumulation_cannot_overflow():  # dot.rs:568-589
    worst = 128 * 32768 * (1 << 16)
    assert worst < (2**63 - 1) // 1000
    n = 4096
    assert O.dot_scalar(np.full(n, -128, np.int8), np.full(n, -32768, np.int16)) == n * 128 * 32768


def test_dot_hand_and_extremes():  # dot.rs:613-656
    assert O.dot_scalar([1, 2, 3], [10, 20, 30]) == 140
    assert O.dot_scalar([-1, 2], [100, -50]) == -200
    assert O.dot_scalar([], []) == 0
    n = 4864
    assert O.dot_scalar(np.full(n, 127, np.int8), np.full(n, 32767, np.int16)) == 127 * 32767 * n
    assert O.dot_scalar(np.full(n, -128, np.int8), np.full(n, 32767, np.int16)) == -128 * 32767 * n


def test_dot_zip_semantics():  # dot.rs:659-664
    assert O.dot_scalar([1, 2, 3, 4, 5], [10, 20, 30]) == 140
    assert O.dot_scalar([1, 2], [10, 20, 30]) == 50


# ---- prng.rs / sampling.rs -----------------------------------------------------

def test_splitmix64_matches_reference_outputs():
    kat = fixtures.splitmix_kat()
    state = kat["seed"]
    for s, z in kat["steps"]:
        state, out = O.splitmix64(state)
        assert (state, out) == (s, z)
    # gen.stream is the same sequence, evaluated counter-style.
    zs = gen.stream(kat["seed"], len(kat["steps"]))
    assert [int(v) for v in zs] == [z for _, z in kat["steps"]]


def test_argmax_lowest_index_on_ties():  # sampling.rs:8-18, spec.json tie_breaking
    assert O.argmax_int([1, 9, 3]) == 1
    assert O.argmax_int([5, 7, 7, 2, 7]) == 1


# ---- golden fixtures ---------------------------------------------------------------

def test_op_golden_vector_identity():
    for v in fixtures.op_vectors():
        W = np.array(v["W"], np.int8).reshape(-1)
        y = O.linear_w8a16(v["x"], W, len(v["W"][0]), v["w_shifts"], v["act_frac"], v["out_frac"])
        assert y.tolist() == v["y"]
        import hashlib
        assert hashlib.sha256(y.astype("<i2").tobytes()).hexdigest() == v["y_sha256_le_i16"]


@pytest.mark.parametrize("case", fixtures.linear_cases(), ids=lambda c: c["name"])
def test_linear_fixture(case):
    c = case
    if c["kind"] == "scalar":
        y = O.linear_w8a16(c["x"], c["W"], c["K"], c["w_shifts"], c["act_frac"], c["out_frac"])
    elif c["kind"] == "pc":
        y = O.linear_w8a16_pc(c["x"], c["W"], c["K"], c["w_shifts"], c["act_frac"], c["out_frac"])
    else:
        y = O.lm_head_w8a16_i32(c["x"], c["W"], c["K"], c["w_shifts"], c["act_frac"], c["out_frac"])
    assert np.array_equal(y, c["y"])


def test_lm_head_fixture_saturates():
    c = [c for c in fixtures.linear_cases() if c["name"] == "lmhead_k64_n50_sat"][0]
    sat = np.isin(c["y"], [2**31 - 1, -(2**31)]).mean()
    assert 0.3 < sat < 1.0  # the case exercises the i32 clamp


def test_lm_head_w16a16_known_answers():
    """model.rs:285-296 (path A): int16 x int16 products in i64, no i32 overflow."""
    W = np.array([[32767, -32768], [1, -1]], np.int16)
    x = np.array([32767, 1], np.int16)
    y = O.lm_head_w16a16_i32(x, W, 2, [0, 0], 0, 0)
    assert y.tolist() == [32767 * 32767 - 32768, 32766]
    # logit_frac above the row's fraction: a left shift, then the i32 clamp
    y = O.lm_head_w16a16_i32(x, W, 2, [0, 0], 0, 2)
    assert y.tolist() == [2**31 - 1, 32766 * 4]
    # round half to even on the rescale: acc = 6 -> 6 / 4 = 1.5 -> 2; acc = 10 -> 2.5 -> 2
    y = O.lm_head_w16a16_i32(np.array([[3, 0], [5, 0]], np.int16), np.array([[2, 0]], np.int16), 2,
                             [1], 1, 0)
    assert y.tolist() == [[2], [2]]
    # u8 overflow of shifts[row] + final_norm_frac panics in a debug build
    with pytest.raises(O.OracleError):
        O.lm_head_w16a16_i32(x, W, 2, [250, 0], 10, 0)


@pytest.mark.parametrize("case", [c for c in fixtures.linear_cases() if c["kind"] == "lm_head"],
                         ids=lambda c: c["name"])
def test_lm_head_w16a16_equals_path_b_on_int8_range(case):
    """With weights inside the int8 range both LM-head paths compute the same
    i64 dot, so path A reproduces the path-B fixtures."""
    c = case
    W16 = np.asarray(c["W"], np.int8).astype(np.int16)
    y = O.lm_head_w16a16_i32(c["x"], W16, c["K"], c["w_shifts"], c["act_frac"], c["out_frac"])
    assert np.array_equal(y, c["y"])


def test_linear_backward_golden_vector():  # conformance/vectors/op/backward_linear.golden.json
    for c in fixtures.backward_cases():
        gx, gw = O.linear_backward(c["g"], c["x"], c["W"], c["in_features"], c["w_shifts"],
                                   c["g_frac"], c["gx_frac"])
        assert gx.tolist() == c["gx"]
        assert gw.reshape(-1).tolist() == c["gW"]


def test_linear_backward_outer_product():  # backward.rs:678-685
    _, gw = O.linear_backward([5, -2], [3, -7, 11], np.zeros(6, np.int8), 3, [0, 0], 0, 0)
    assert gw.reshape(-1).tolist() == [15, -35, 55, -6, 14, -22]


def test_linear_backward_aligns_before_one_shift():
    """backward.rs:167-178: the summands are aligned to the largest shift and
    rounded once. Six summands of -6 at shift 4 round to 0 one by one but to
    round(-36 / 16) = -2 together; mixed shifts divide by each row's own scale."""
    gx, _ = O.linear_backward([-6] * 6, [1], np.ones(6, np.int8), 1, [4] * 6, 6, 6, want_gw=False)
    assert gx.tolist() == [-2]
    gx, _ = O.linear_backward([1, 1], [0], np.array([8, 16], np.int8), 1, [2, 4], 0, 0, want_gw=False)
    assert gx.tolist() == [3]  # 8 / 2^2 + 16 / 2^4
    with pytest.raises(O.OracleError):  # empty w_shifts: .max().expect(...) panics
        O.linear_backward(np.zeros((1, 0), np.int32), [1], np.zeros(0, np.int8), 1, [], 0, 0)


def _linear_backward_py(g, W, shifts, g_frac, gx_frac):
    """Python big-int restatement of backward.rs:180-199 for one token."""
    ref = int(max(shifts))
    acc = [0] * W.shape[1]
    for i, gi in enumerate(g):
        for j in range(W.shape[1]):
            acc[j] += (int(gi) * int(W[i, j])) << (ref - int(shifts[i]))
    out = []
    for a in acc:
        q = a >> ref
        r = a - (q << ref)
        h = (1 << (ref - 1)) if ref > 0 else 0
        if ref > 0 and (r > h or (r == h and q & 1)):
            q += 1
        q = max(-(2**63), min(2**63 - 1, q))
        s = g_frac - gx_frac
        if s > 0:
            qq = q >> s
            rr = q - (qq << s)
            hh = 1 << (s - 1)
            if rr > hh or (rr == hh and qq & 1):
                qq += 1
            v = qq
        else:
            v = q << (-s)
        out.append(max(-(2**31), min(2**31 - 1, v)))
    return out


def test_linear_backward_random_against_bigint():
    rng = np.random.default_rng(77)
    for trial in range(6):
        N, K = int(rng.integers(1, 40)), int(rng.integers(1, 30))
        W = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
        shifts = rng.integers(0, 21, size=N).astype(np.uint8)
        g = rng.integers(-(2**31), 2**31, size=N, dtype=np.int64).astype(np.int32)
        g[::3] = rng.integers(-50, 50, size=g[::3].size)
        x = rng.integers(-32768, 32768, size=K, dtype=np.int16)
        g_frac, gx_frac = int(rng.integers(0, 12)), int(rng.integers(0, 12))
        gx, gw = O.linear_backward(g, x, W, K, shifts, g_frac, gx_frac)
        assert gx.tolist() == _linear_backward_py(g, W, shifts, g_frac, gx_frac), trial
        assert np.array_equal(gw, g.astype(np.int64)[:, None] * x.astype(np.int64)[None, :])


@pytest.mark.parametrize("case", fixtures.mlp_cases(), ids=lambda c: c["name"])
def test_mlp_fixture(case):
    c, p = case, case["params"]
    y = O.mlp_int(c["x"], c["W_gate"], c["W_up"], c["W_down"], c["H"], c["I"], c["gate_w_shifts"],
                  c["up_w_shifts"], c["down_w_shifts"], c["silu_lut"], p["in_frac"], p["gate_out"],
                  p["up_out"], p["down_in"], p["silu_in"], p["offset"], p["silu_out"], c["out_frac"])
    assert np.array_equal(y, c["y"])


def test_backend_parity_fixtures():  # test_backend_parity.rs:160-255
    lin, mlp = fixtures.backend_parity()
    y = O.linear_w8a16(lin["x"], lin["W"], lin["K"], lin["w_shifts"], lin["act_frac"], lin["out_frac"])
    assert y.tolist() == lin["y"]
    p = mlp["params"]
    y = O.mlp_int(mlp["x"], mlp["W_gate"], mlp["W_up"], mlp["W_down"], mlp["H"], mlp["I"],
                  mlp["gate_w_shifts"], mlp["up_w_shifts"], mlp["down_w_shifts"], mlp["silu_lut"],
                  p["in_frac"], p["gate_out"], p["up_out"], p["down_in"], p["silu_in"], p["offset"],
                  p["silu_out"], mlp["out_frac"])
    assert y.tolist() == mlp["y"]


@pytest.mark.parametrize("case", fixtures.softmax_cases(), ids=lambda c: c["name"])
def test_softmax_int_fixture(case):  # softmax.rs:24-64, golden vector softmax_basic
    out = O.softmax_int(case["logits"], case["exp_lut"], case["lut_shift"], case["frac_bits"])
    assert out.tolist() == case["probs"]


def test_moe_route_ties_go_to_lowest_index():
    lut = [int(round(np.exp(-i / 256.0) * (1 << 14))) for i in range(16384)]
    logits = np.array([[5, 9, 9, 1, 9, 3], [0, 0, 0, 0, 0, 0]], np.int32)
    idx, prob = O.moe_route(logits, 3, lut, 0, 14)
    assert idx.tolist() == [[1, 2, 4], [0, 1, 2]]
    assert prob[1].tolist() == O.softmax_int([0, 0, 0], lut, 0, 14).tolist()


def test_thread_count_does_not_change_results():
    K, N, M = 896, 300, 4
    W = gen.int8_tensor(91, N * K)
    x = gen.int16_tensor(92, M * K).reshape(M, K)
    s = gen.uint8_tensor(93, N, 10, 14)
    n0 = O.num_threads()
    try:
        O.set_num_threads(1)
        a = O.linear_w8a16(x, W, K, s, 6, 6)
        O.set_num_threads(max(2, n0))
        b = O.linear_w8a16(x, W, K, s, 6, 6)
    finally:
        O.set_num_threads(n0)
    assert np.array_equal(a, b)


def test_fast_oracle_paths_equal_the_scalar_restatement():
    """The blocked-dot helpers used by the full-size checks (linear_w8a16_fast,
    linear_acc_fast, requant_acc, mlp_int_fast) give the scalar restatement's
    outputs, extremes included."""
    import numpy as np

    import oracle as O
    from make_golden import silu_lut_spec

    rng = np.random.default_rng(12)
    for M, K, N in ((3, 1000, 40), (2, 18944, 24), (4, 257, 33), (1, 7, 5)):
        x = rng.integers(-32768, 32768, size=(M, K)).astype(np.int16)
        x[0] = -32768
        W = rng.integers(-128, 128, size=N * K, dtype=np.int8)
        W[:K] = -128
        s = rng.integers(8, 16, size=N).astype(np.uint8)
        of = rng.integers(0, 12, size=N).astype(np.uint8)
        ref = O.linear_w8a16_pc(x, W, K, s, 8, of)
        assert np.array_equal(O.linear_w8a16_fast(x, W, K, s, 8, of), ref)
        acc = O.linear_acc_fast(x, W, K, N)
        assert np.array_equal(acc, O.linear_acc_i64(x, W, K, N))
        assert np.array_equal(O.requant_acc(acc, s, 8, of), ref)
    H, I = 64, 96
    args = (rng.integers(-127, 128, size=(I, H), dtype=np.int8), rng.integers(-127, 128, size=(I, H), dtype=np.int8),
            rng.integers(-127, 128, size=(H, I), dtype=np.int8), H, I,
            rng.integers(9, 12, size=I).astype(np.uint8), rng.integers(9, 12, size=I).astype(np.uint8),
            rng.integers(9, 12, size=H).astype(np.uint8), silu_lut_spec(), 8, 7, 7, 7, 6, 8192, 8,
            rng.integers(3, 8, size=H).astype(np.uint8))
    x = rng.integers(-20000, 20000, size=(5, H)).astype(np.int16)
    assert np.array_equal(O.mlp_int_fast(x, *args), O.mlp_int(x, *args))
