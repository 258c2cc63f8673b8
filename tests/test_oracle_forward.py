"""Pins the CPU oracle of the integer forward pass (oracle/myl_forward.c).

Known answers transcribed from the reference's unit tests (rmsnorm.rs:155-377,
rope.rs:58-123, attention.rs:96-141, fixed_point.rs:336-395,
generate.rs:236-290), the op golden vector rmsnorm_basic, seeded cases computed
by the reference's own Python restatement generate.py:66 rmsnorm_i16_ref
(tests/golden/forward_cases.json, written by tests/golden/make_golden.py), the
hashes of the LUT files the reference ships in scale_packs/, and the exactness
of the oracle's evaluation-order freedoms (layer-major prefill, blocked dots).
"""
from __future__ import annotations

import hashlib
import json
import math
import os

import numpy as np
import pytest

import oracle
from myelith_b200 import synthetic as S
from myelith_b200.model import digest
from model_fixtures import loader_fixture_model

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "forward_cases.json")


@pytest.fixture(scope="module")
def cases():
    with open(GOLDEN) as f:
        return json.load(f)


def spec_lut(n):
    """rmsnorm.rs:159-171: round(4096 / sqrt(x)) (f64::round, half away from zero), lut[0] = 256."""
    return np.array([256] + [math.floor(4096.0 / math.sqrt(x) + 0.5) for x in range(1, n)], np.int16)


def rms(x, xs, g, gs, lut, out_frac):
    n = len(x)
    return oracle.rmsnorm_i16(np.array(x), np.array(xs), np.array(g), np.array(gs), lut, 8, 8,
                              oracle.inv_n_q20(n), out_frac)


# ---- fixed_point.rs / rmsnorm.rs constants ---------------------------------------

def test_inv_n_q20_and_isqrt_kats():
    assert oracle.inv_n_q20(896) == 1170 and oracle.inv_n_q20(1) == 1 << 20
    for n, r in ((0, 0), (1, 1), (2, 1), (3, 2), (4, 2), (8_388_608, 2896), (16_777_216, 4096)):
        assert oracle.isqrt_round(n) == r
    for n in (5, 99, 1000, 123_456, 1 << 40):
        assert oracle.isqrt_round(n) == round(math.sqrt(n))
    assert [oracle.inv_sqrt_q15(d) for d in (4, 16, 64, 256)] == [1 << 14, 1 << 13, 1 << 12, 1 << 11]
    assert [oracle.inv_sqrt_q15(d) for d in (128, 512, 2)] == [2896, 1448, 23170]


# ---- rmsnorm_i16 ------------------------------------------------------------------

def test_rmsnorm_reference_unit_tests():
    lut1k, lut = spec_lut(1024), spec_lut(32768)
    assert rms([0, 0, 0], [0] * 3, [64] * 3, [6] * 3, lut1k, 6).tolist() == [0, 0, 0]
    assert rms([16, 16], [0, 0], [64, 64], [6, 6], lut, 6).tolist() == [64, 64]
    assert rms([-16, -16], [0, 0], [64, 64], [6, 6], lut, 6).tolist() == [-64, -64]
    big = rms([12000, 12000], [0, 0], [32, 32], [5, 5], lut, 3)
    assert abs(int(big[0]) - 8) <= 1 and abs(int(big[1]) - 8) <= 1
    two = rms([16, 0], [0, 0], [32, 32], [5, 5], lut, 6)
    assert int(two[0]) in (90, 91) and two[1] == 0
    assert rms([16, 16], [0, 0], [32, 32], [5, 5], lut, 6).tolist() == [64, 64]
    assert rms([16, 16], [0, 0], [64, 64], [5, 5], lut, 6).tolist() == [128, 128]
    assert rms([16, 16], [0, 0], [32, 32], [5, 4], lut, 6).tolist() == [64, 128]
    ref = rms([3000, -500, 7, 12000], [0] * 4, [32, 40, 20, 8], [5] * 4, lut, 6)
    for s in (1, 5, 9, 14):
        assert np.array_equal(rms([3000, -500, 7, 12000], [s] * 4, [32, 40, 20, 8], [5] * 4, lut, 6), ref)
    outl = rms([9600, 1024, -2048, 3072], [1, 12, 12, 12], [64] * 4, [6] * 4, lut, 8)
    assert abs(abs(int(outl[0]) / 256.0) - 2.0) < 0.1
    a = rms([9600, 1024, -2048, 3072], [1, 12, 12, 12], [64] * 4, [6] * 4, lut, 8)
    b = rms([19200, 256, -512, 768], [2, 10, 10, 10], [64] * 4, [6] * 4, lut, 8)
    assert np.array_equal(a, b)
    w = rms([9600, 1024, 4800, 4], [2, 10, 1, 2], [64] * 4, [6] * 4, lut, 8)
    assert w[1] == w[3] and w[0] == w[2]
    ext = rms([32767, 32767, 1, 1], [0, 20, 0, 20], [127] * 4, [20] * 4, lut, 0)
    assert (ext >= 0).all()


def test_rmsnorm_golden_vector_and_generate_py_cases(cases):
    spec_rsqrt = S.rsqrt_lut()
    for c in cases["rmsnorm"]:
        if c["lut"] == "spec_rsqrt_32768":
            lut = spec_rsqrt
            assert hashlib.sha256(lut.astype("<i2").tobytes()).hexdigest() == c["lut_sha256"]
        else:
            lut = np.array(c["lut"], np.int16)
        n = len(c["x"])
        assert c["inv_n_q20"] == oracle.inv_n_q20(n)
        y = oracle.rmsnorm_i16(np.array(c["x"]), np.full(n, c["x_shift"]), np.array(c["gamma"]),
                               np.full(n, c["gamma_shift"]), lut, c["lut_input_shift"],
                               c["lut_output_frac"], c["inv_n_q20"], c["out_frac"])
        assert y.tolist() == c["y"], c["name"]


def test_lut_generators_match_the_reference_scale_packs(cases):
    for pack, hd in (("qwen2.5-0.5b", 64), ("qwen2.5-7b", 128)):
        luts = S.spec_luts(hd)
        for name, e in cases["scale_pack_luts"][pack].items():
            assert len(luts[name]) == e["length"], (pack, name)
            assert hashlib.sha256(luts[name].astype("<i2").tobytes()).hexdigest() == e["sha256"], (pack, name)


# ---- rope.rs --------------------------------------------------------------------

def test_rope_reference_unit_tests():
    v = [100, -200, 32000, -32000]
    assert oracle.rotate_half_split_i16(v, [256, 256], [0, 0], 8).tolist() == v
    assert oracle.rotate_half_split_i16([100, 200, 300, 400], [0, 0], [256, 256], 8).tolist() == \
        [-300, -400, 100, 200]
    assert oracle.rotate_half_split_i16([4096, 0, 0, 0], [256, 256], [0, 0], 8).tolist() == [4096, 0, 0, 0]
    # rounding and saturation of the i32 path
    out = oracle.rotate_half_split_i16([32767, 32767], [181], [181], 8)
    assert out.tolist() == [0, 32767]


# ---- attention.rs ------------------------------------------------------------------

def _exp_lut_129():
    return np.array([round(math.exp(-i / 256.0) * 256.0) for i in range(129)], np.int16)


def test_attention_reference_unit_tests():
    lut = _exp_lut_129()
    q = [[64, 0], [64, 0]]
    k = [[64, 0], [64, 0]]
    v = [[100, -50], [100, -50]]
    mask = [[1, 0], [1, 1]]
    out = oracle.attention_int(q, k, v, mask, 1 << 15, 4 + 15, lut, 0, 8)
    assert abs(int(out[0][0]) - 100) <= 1 and abs(int(out[0][1]) + 50) <= 1
    assert abs(int(out[1][0]) - 100) <= 1
    out = oracle.attention_int([[64, 0]], [[64, 0]] * 3, [[100, 0], [200, 0], [300, 0]], None,
                               1 << 15, 4 + 15, lut, 0, 8)
    assert abs(int(out[0][0]) - 200) <= 2 and abs(int(out[0][1])) <= 1


def test_attention_row_matches_softmax_and_weighted_sum():
    """attention_int restated from its parts: scores = rne(dot * mult, shift) as
    i32, softmax_int, sum_j p_j * v_j rounded by prob_frac and clamped."""
    rng = np.random.default_rng(3)
    lut = S.exp_lut()
    for kv in (1, 7, 300):
        q = rng.integers(-4000, 4000, size=(1, 64)).astype(np.int16)
        k = rng.integers(-4000, 4000, size=(kv, 64)).astype(np.int16)
        v = rng.integers(-32768, 32768, size=(kv, 64)).astype(np.int16)
        out = oracle.attention_int(q, k, v, None, 4096, 23, lut, 6, 14)
        sc = [oracle.rshift_round_i64(int(np.dot(q[0].astype(np.int64), k[j].astype(np.int64))) * 4096, 23)
              for j in range(kv)]
        sc = [((s + 2**31) % 2**32) - 2**31 for s in sc]
        p = oracle.softmax_int(np.array(sc, np.int32), lut, 6, 14).astype(np.int64)
        row = (p[:, None] * v.astype(np.int64)).sum(0)
        exp = [oracle.clamp_i16_from_i64(oracle.rshift_round_i64(int(r), 14)) for r in row]
        assert out[0].tolist() == exp


# ---- generate.rs: digest byte order ----------------------------------------------

def test_digest_byte_order():
    steps = [([7, -3, 1], 0), ([2, 9, -1], 1)]
    raw = b"".join(np.array(l, "<i4").tobytes() + np.array([t], "<u4").tobytes() for l, t in steps)
    assert raw[:4] == (7).to_bytes(4, "little", signed=True)
    assert raw[12:16] == (0).to_bytes(4, "little") and len(raw) == 2 * (3 + 1) * 4
    assert digest(np.array([s[0] for s in steps]), [s[1] for s in steps]) == hashlib.sha256(raw).hexdigest()
    assert len(digest(np.array([s[0] for s in steps]), [0, 1])) == 64


# ---- the forward oracle's own exactness ---------------------------------------------

def test_layer_major_prefill_equals_token_by_token():
    spec = S.synthetic_model("qwen2.5-0.5b", seed=11, num_layers=2, vocab=512,
                             dims=(2, 128, 4, 2, 32, 256, 512, True))
    p = S.prompt_tokens(spec.vocab, 20, seed=1)
    a = oracle.OracleModel(spec, 32)
    la = a.forward(p, 0)
    b = oracle.OracleModel(spec, 32)
    for i, t in enumerate(p):
        lb = b.forward([t], i)
    c = oracle.OracleModel(spec, 32)
    c.forward(p[:7], 0, want_logits=False)
    lc = c.forward(p[7:], 7)
    assert np.array_equal(la, lb) and np.array_equal(la, lc)
    assert np.array_equal(a.k_cache, b.k_cache) and np.array_equal(a.v_cache, b.v_cache)


def test_forward_linears_match_the_scalar_linear():
    """The forward's blocked dot equals dot_scalar: the key the forward caches
    for a token at position 0 (RoPE row 0 is cos 1, sin 0: the identity) is
    the scalar linear_w8a16 of the normed embedding plus the k bias."""
    spec = S.synthetic_model("qwen2.5-7b", seed=3, num_layers=1, vocab=64,
                             dims=(1, 1024, 8, 2, 128, 512, 64, False))
    L, H = spec.layers[0], spec.hidden
    tok = 17
    om = oracle.OracleModel(spec, 4)
    om.forward([tok], 0, want_logits=False)
    emb = np.array([oracle.clamp_i16(oracle.rescale(int(v), int(spec.embed_shifts[tok]),
                                                    int(L.residual_in_frac[i])))
                    for i, v in enumerate(spec.embed[tok])], np.int16)
    xn = oracle.rmsnorm_i16(emb, L.residual_in_frac, L.ln1_gamma, L.ln1_gamma_shifts,
                            spec.rsqrt_lut, 8, 8, oracle.inv_n_q20(H), L.norm_attn_frac)
    k = oracle.linear_w8a16(xn.reshape(1, -1), L.wk.reshape(-1), H, L.sk, L.norm_attn_frac, L.k_frac).reshape(-1)
    k = oracle.add_bias_i16(k, L.bk, L.bk_shifts, L.k_frac)
    v = oracle.linear_w8a16(xn.reshape(1, -1), L.wv.reshape(-1), H, L.sv, L.norm_attn_frac, L.v_frac).reshape(-1)
    v = oracle.add_bias_i16(v, L.bv, L.bv_shifts, L.v_frac)
    assert np.array_equal(om.k_cache[0, :, 0].reshape(-1), k)
    assert np.array_equal(om.v_cache[0, :, 0].reshape(-1), v)


def test_rope_wraps_past_the_table():
    """model.rs:469-471: position p uses LUT row p % n_pos. A 4-row table gives
    the same cache as the same 4 rows tiled to cover every position."""
    spec = S.synthetic_model("qwen2.5-0.5b", seed=5, num_layers=1, vocab=64,
                             dims=(1, 64, 2, 1, 32, 128, 64, True))
    half = 16
    rows_c, rows_s = spec.cos_lut[1 * half: 5 * half].copy(), spec.sin_lut[1 * half: 5 * half].copy()
    p = S.prompt_tokens(64, 11, seed=2)
    spec.cos_lut, spec.sin_lut = rows_c, rows_s
    a = oracle.OracleModel(spec, 12)
    la = a.forward(p, 0)
    spec.cos_lut, spec.sin_lut = np.tile(rows_c, 3), np.tile(rows_s, 3)
    b = oracle.OracleModel(spec, 12)
    lb = b.forward(p, 0)
    assert np.array_equal(a.k_cache, b.k_cache) and np.array_equal(la, lb)
    spec.cos_lut, spec.sin_lut = np.roll(np.tile(rows_c, 3), half), np.roll(np.tile(rows_s, 3), half)
    c = oracle.OracleModel(spec, 12)
    c.forward(p, 0, want_logits=False)
    assert not np.array_equal(a.k_cache, c.k_cache)


def test_loader_fixture_forward_runs():
    """loader.rs:1582-1600: forward_token(0, 0) on the synthetic artifact gives
    vocab_size logits (tied and untied, with and without biases)."""
    for tied in (True, False):
        for bias in (True, False):
            spec = loader_fixture_model(tied, bias)
            om = oracle.OracleModel(spec, 8)
            lg = om.forward([0], 0)
            assert lg.shape == (3,)
            toks, steps = oracle.OracleModel(spec, 8).generate([0, 2, 1], 5)
            assert toks.shape == (5,) and steps.shape == (5, 3)


def test_generate_is_deterministic_and_records_its_inputs():
    spec = S.synthetic_model("qwen2.5-0.5b", seed=9, num_layers=2, vocab=1000,
                             dims=(2, 128, 4, 2, 32, 256, 1000, True))
    p = S.prompt_tokens(spec.vocab, 12, seed=4)
    t1, l1 = oracle.OracleModel(spec, 32).generate(p, 8)
    t2, l2 = oracle.OracleModel(spec, 32).generate(p, 8)
    assert np.array_equal(t1, t2) and np.array_equal(l1, l2)
    for s in range(8):
        assert t1[s] == oracle.argmax_int(l1[s])
    # step s's logits are the forward of the prompt plus tokens[:s]
    om = oracle.OracleModel(spec, 32)
    lg = om.forward(np.r_[p, t1[:3]], 0)
    assert np.array_equal(lg, l1[3])


def test_softmax_division_by_reciprocal_is_exact():
    """The prefill and decode PV kernels divide num = e * one (< 2^31) by the
    row's exponential sum S (< 2^31) as floor(2 * num * R / 2^64) with
    R = ceil(2^63 / S), then apply softmax.rs:41-62's round-half-even step.
    Checked here against exact integer division on random and edge values
    (u64 / u32 arithmetic emulated with Python integers)."""
    def exact(num, S):
        q, r = divmod(num, S)
        return q + (1 if (2 * r > S or (2 * r == S and q & 1)) else 0)

    def recip(num, S):
        R = ((1 << 63) + S - 1) // S
        q = (((num << 1) * R) >> 64) & 0xFFFFFFFF
        twice = (2 * ((num - q * S) & 0xFFFFFFFF)) & 0xFFFFFFFF
        return q + (1 if (twice > S or (twice == S and q & 1)) else 0)

    rng = np.random.default_rng(2024)
    for _ in range(200000):
        frac = int(rng.integers(0, 31))
        one = 1 << frac
        e = int(rng.integers(0, (2**31 - 1) // one + 1))
        S = int(rng.integers(1, 2**31)) if rng.random() < 0.5 else int(rng.integers(1, 70000))
        assert recip(e * one, S) == exact(e * one, S), (e, S, one)
    for S in (1, 2, 3, 5, 16384, 2**30, 2**31 - 1):
        for num in (0, 1, S - 1, S, S // 2, (S // 2) * 3, 2**31 - 1):
            if 0 <= num < 2**31:
                assert recip(num, S) == exact(num, S), (num, S)
