"""GPU parity of the integer decoder forward (myl_model_*, myl_rmsnorm_i16,
myl_attention_int) against the CPU oracle (oracle/myl_forward.c), through
the C ABI. Every comparison is element for element: logits, generated token
ids and the SHA-256 digests of dekodieren_mit_digest (generate.rs:161-200).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

import oracle
from myelith_b200 import synthetic as S
from myelith_b200 import model as M
from model_fixtures import loader_fixture_model

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "forward_cases.json")


@pytest.fixture(scope="module")
def ctx():
    import myelith_b200 as myl

    c = myl.Context(0)
    yield c
    c.close()


# ---- rmsnorm_i16 -----------------------------------------------------------------

def test_rmsnorm_golden_cases(ctx):
    with open(GOLDEN) as f:
        cases = json.load(f)["rmsnorm"]
    for c in cases:
        lut = S.rsqrt_lut() if c["lut"] == "spec_rsqrt_32768" else np.array(c["lut"], np.int16)
        n = len(c["x"])
        y = M.rmsnorm_i16(ctx, np.array(c["x"]), np.full(n, c["x_shift"]), np.array(c["gamma"]),
                          np.full(n, c["gamma_shift"]), lut, c["lut_input_shift"],
                          c["lut_output_frac"], c["inv_n_q20"], c["out_frac"])
        assert y.tolist() == c["y"], c["name"]


@pytest.mark.parametrize("n,sigma,span,out_frac", [
    (896, 3000, 0, 10), (896, 3000, 6, 10), (3584, 900, 15, 12), (7, 30000, 3, 4),
    (64, 1, 20, 14), (4, 32767, 30, 0), (1000, 200, 10, 20)])
def test_rmsnorm_random_vs_oracle(ctx, n, sigma, span, out_frac):
    rng = np.random.default_rng(n + span)
    lut = S.rsqrt_lut()
    M_ = 9
    x = np.clip(np.rint(rng.normal(0, sigma, size=(M_, n))), -32768, 32767).astype(np.int16)
    x[3] = 0                      # the all-zero row (rmsnorm.rs:99-101)
    x[4, :] = -32768              # extreme values
    xs = rng.integers(10, 11 + span, size=n).astype(np.uint8) if span else np.full(n, 9, np.uint8)
    g = rng.integers(-128, 128, size=n).astype(np.int8)
    gs = rng.integers(3, 9, size=n).astype(np.uint8)
    inv = oracle.inv_n_q20(n)
    want = oracle.rmsnorm_i16(x, xs, g, gs, lut, 8, 8, inv, out_frac)
    got = M.rmsnorm_i16(ctx, x, xs, g, gs, lut, 8, 8, inv, out_frac)
    assert np.array_equal(got, want)


def test_rmsnorm_small_lut_and_reference_kats(ctx):
    lut = np.array([256] + [int(4096.0 / np.sqrt(x) + 0.5) for x in range(1, 32768)], np.int16)
    for x, xs, g, gs, of in (
            ([16, 16], [0, 0], [64, 64], [6, 6], 6), ([9600, 1024, -2048, 3072], [1, 12, 12, 12], [64] * 4, [6] * 4, 8),
            ([32767, 32767, 1, 1], [0, 20, 0, 20], [127] * 4, [20] * 4, 0),
            ([9600, 1024, 4800, 4], [2, 10, 1, 2], [64] * 4, [6] * 4, 8)):
        n = len(x)
        want = oracle.rmsnorm_i16(np.array(x), np.array(xs), np.array(g), np.array(gs), lut, 8, 8,
                                  oracle.inv_n_q20(n), of)
        got = M.rmsnorm_i16(ctx, np.array(x), np.array(xs), np.array(g), np.array(gs), lut, 8, 8,
                            oracle.inv_n_q20(n), of)
        assert np.array_equal(got, want), x
    tiny = np.array([256, 181, 148], np.int16)
    x = np.array([[100, -7, 3, 2000], [0, 0, 0, 0]], np.int16)
    args = (np.full(4, 5, np.uint8), np.array([1, 2, 3, 4], np.int8), np.zeros(4, np.uint8), tiny, 8,
            8, oracle.inv_n_q20(4), 3)
    assert np.array_equal(M.rmsnorm_i16(ctx, x, *args), oracle.rmsnorm_i16(x, *args))


# ---- attention_int ----------------------------------------------------------------

@pytest.mark.parametrize("hd,kv,q_len,sigma,shift", [
    (64, 1, 1, 2000, 23), (64, 255, 2, 2000, 23), (64, 256, 1, 3000, 23), (64, 257, 3, 3000, 22),
    (128, 700, 2, 1500, 24), (128, 2304, 1, 2000, 25), (2, 5, 4, 300, 11), (6, 33, 2, 30000, 30),
    (128, 40, 2, 32767, 40)])
def test_attention_random_vs_oracle(ctx, hd, kv, q_len, sigma, shift):
    rng = np.random.default_rng(hd * 1000 + kv)
    lut = S.exp_lut()
    q = np.clip(np.rint(rng.normal(0, sigma, size=(q_len, hd))), -32768, 32767).astype(np.int16)
    k = np.clip(np.rint(rng.normal(0, sigma, size=(kv, hd))), -32768, 32767).astype(np.int16)
    v = rng.integers(-32768, 32768, size=(kv, hd)).astype(np.int16)
    mult = oracle.inv_sqrt_q15(hd)
    want = oracle.attention_int(q, k, v, None, mult, shift, lut, 6, 14)
    got = M.attention_int(ctx, q, k, v, None, mult, shift, lut, 6, 14)
    assert np.array_equal(got, want)


def test_attention_masks_extremes_and_uniform_fallback(ctx):
    rng = np.random.default_rng(1)
    lut = S.exp_lut()
    hd, kv = 64, 300
    q = rng.integers(-32768, 32768, size=(4, hd)).astype(np.int16)
    k = rng.integers(-32768, 32768, size=(kv, hd)).astype(np.int16)
    v = rng.integers(-32768, 32768, size=(kv, hd)).astype(np.int16)
    q[0] = -32768
    k[:5] = -32768                  # (-32768)^2 products: the int16 extremes of the split dot
    mask = rng.random((4, kv)) < 0.7
    mask[2] = False                 # an all-masked row: every score i32::MIN
    mask[3, :] = False
    mask[3, 17] = True
    for shift in (0, 20, 45):
        want = oracle.attention_int(q, k, v, mask, 4096, shift, lut, 6, 14)
        got = M.attention_int(ctx, q, k, v, mask, 4096, shift, lut, 6, 14)
        assert np.array_equal(got, want), shift
    # exp table whose exp(0) is 0: the sum is 0 and softmax_int returns the
    # uniform distribution (softmax.rs:47-53)
    zero_lut = np.zeros(16, np.int16)
    want = oracle.attention_int(q[:2], k[:9], v[:9], None, 4096, 20, zero_lut, 0, 14)
    got = M.attention_int(ctx, q[:2], k[:9], v[:9], None, 4096, 20, zero_lut, 0, 14)
    assert np.array_equal(got, want)
    # the reference's own cases (attention.rs:96-141)
    small = np.array([round(np.exp(-i / 256.0) * 256.0) for i in range(129)], np.int16)
    args = ([[64, 0], [64, 0]], [[64, 0], [64, 0]], [[100, -50], [100, -50]], [[1, 0], [1, 1]],
            1 << 15, 19, small, 0, 8)
    assert np.array_equal(M.attention_int(ctx, *args), oracle.attention_int(*args))


# ---- the model -------------------------------------------------------------------

def _small(seed=3, L=2, V=1000, dims=None, tied=True):
    d = dims or (L, 128, 4, 2, 32, 256, V, tied)
    return S.synthetic_model("qwen2.5-0.5b", seed=seed, num_layers=d[0], vocab=d[6], dims=d)


@pytest.mark.parametrize("tied,bias", [(True, True), (False, True), (True, False), (False, False)])
def test_loader_fixture_model(ctx, tied, bias):
    """The reference loader's synthetic artifact (loader.rs:1361-1504): hidden
    4, head_dim 2, vocab 3, LUTs of 3-4 entries."""
    spec = loader_fixture_model(tied, bias)
    gm = M.IntegerModel(ctx, spec)
    s = gm.session(1, 8)
    got = s.forward([[0]])
    want = oracle.OracleModel(spec, 8).forward([0], 0)
    assert np.array_equal(got[0], want)
    toks, dg, lg = gm.generate([0, 2, 1], 5, keep_logits=True, digest=True)
    wt, wl = oracle.OracleModel(spec, 8).generate([0, 2, 1], 5)
    assert np.array_equal(toks[0], wt) and np.array_equal(lg[0], wl)
    assert dg[0] == M.digest(wl, wt)


def test_forward_chunks_and_single_tokens_match_oracle(ctx):
    spec = _small()
    gm = M.IntegerModel(ctx, spec)
    p = S.prompt_tokens(spec.vocab, 40, seed=2)
    om = oracle.OracleModel(spec, 64)
    want = om.forward(p, 0)
    s = gm.session(1, 64)
    assert np.array_equal(s.forward(p[None])[0], want)
    s.reset()
    s.forward(p[None, :13], want_logits=False)
    lg = s.forward(p[None, 13:39])
    assert np.array_equal(lg[0], oracle.OracleModel(spec, 64).forward(p[:39], 0))
    lg = s.forward(p[None, 39:40])
    assert np.array_equal(lg[0], want) and s.position == 40


def test_generate_digest_matches_oracle(ctx):
    spec = _small(seed=4, L=3, V=5000)
    gm = M.IntegerModel(ctx, spec)
    p = S.prompt_tokens(spec.vocab, 33, seed=7)
    toks, dg, lg = gm.generate(p, 20, digest=True, keep_logits=True)
    wt, wl = oracle.OracleModel(spec, 60).generate(p, 20)
    assert np.array_equal(toks[0], wt)
    assert np.array_equal(lg[0], wl)
    assert dg[0] == M.digest(wl, wt)
    # the graph-replayed decode (no host step) gives the same tokens
    toks2, _, _ = gm.generate(p, 20)
    assert np.array_equal(toks2[0], wt)


def test_batch_of_sequences_matches_each_alone(ctx):
    spec = _small(seed=5, L=2, V=3000, dims=(2, 256, 8, 2, 32, 512, 3000, False))
    gm = M.IntegerModel(ctx, spec)
    B, P, N = 5, 21, 12
    prompts = np.stack([S.prompt_tokens(spec.vocab, P, seed=10 + b) for b in range(B)])
    toks, dg, lg = gm.generate(prompts, N, digest=True, keep_logits=True)
    for b in range(B):
        wt, wl = oracle.OracleModel(spec, P + N).generate(prompts[b], N)
        assert np.array_equal(toks[b], wt), b
        assert dg[b] == M.digest(wl, wt), b
    toks_g, _, _ = gm.generate(prompts, N)
    assert np.array_equal(toks_g, toks)


def test_gqa_groups_beyond_eight_heads_and_rope_wrap(ctx):
    """16 query heads per KV head (two sub-groups of the scores kernel) and a
    RoPE table of 8 positions for 30 positions (model.rs:470-471)."""
    spec = _small(seed=8, L=1, V=700, dims=(1, 512, 16, 1, 32, 256, 700, True))
    half = 16
    spec.cos_lut = spec.cos_lut[: 8 * half].copy()
    spec.sin_lut = spec.sin_lut[: 8 * half].copy()
    gm = M.IntegerModel(ctx, spec)
    p = S.prompt_tokens(spec.vocab, 18, seed=3)
    toks, dg, lg = gm.generate(p, 12, digest=True, keep_logits=True)
    wt, wl = oracle.OracleModel(spec, 30).generate(p, 12)
    assert np.array_equal(toks[0], wt) and dg[0] == M.digest(wl, wt)


def test_model_rejects_what_the_reference_panics_on(ctx):
    import myelith_b200 as myl

    spec = _small(seed=9, L=1, V=100)
    spec.layers[0].attn_out_frac = spec.layers[0].v_frac + 40   # i32 rescale shift out of range
    with pytest.raises(myl.MylError):
        M.IntegerModel(ctx, spec)
    spec = _small(seed=9, L=1, V=100)
    gm = M.IntegerModel(ctx, spec)
    s = gm.session(1, 8)
    with pytest.raises(myl.MylError):
        s.forward([[5, 100]])           # token id outside the vocabulary
    with pytest.raises(myl.MylError):
        s.forward(np.zeros((1, 9), np.int32))   # beyond max_positions


def test_config2_full_generate_matches_oracle(ctx):
    """Qwen2.5-0.5B architecture (24 layers, hidden 896,
    14/2 heads of 64, MLP 4864, vocab 151936, tied), 512 random prompt tokens
    and 128 greedy steps: token ids and the logits digest equal the oracle's."""
    spec = S.synthetic_model("qwen2.5-0.5b", seed=2)
    gm = M.IntegerModel(ctx, spec)
    p = S.prompt_tokens(spec.vocab, 512, seed=5)
    toks, dg, _ = gm.generate(p, 128, digest=True)
    wt, wl = oracle.OracleModel(spec, 640).generate(p, 128)
    assert np.array_equal(toks[0], wt)
    assert dg[0] == M.digest(wl, wt)
    toks2, _, _ = gm.generate(p, 128)   # graph-replayed decode
    assert np.array_equal(toks2[0], wt)


def test_config3_full_generate_matches_oracle(ctx):
    """BASELINE config 3 at batch 1: Qwen2.5-7B architecture (28 layers, hidden
    3584, 28/4 heads of 128, MLP 18944, vocab 152064, untied LM head), 2048
    random prompt tokens and 256 greedy steps; positions 2048..2303 wrap the
    2048-row RoPE table (model.rs:470-471). Tokens and digest equal the
    oracle's; at batch 8 the same prompt in sequence 0 gives the same tokens."""
    spec = S.synthetic_model("qwen2.5-7b", seed=2)
    gm = M.IntegerModel(ctx, spec)
    p = S.prompt_tokens(spec.vocab, 2048, seed=100)
    toks, dg, _ = gm.generate(p, 256, digest=True)
    om = oracle.OracleModel(spec, 2304)
    wt, wl = om.generate(p, 256)
    assert np.array_equal(toks[0], wt)
    assert dg[0] == M.digest(wl, wt)
    del om, wl
    prompts = np.stack([p] + [S.prompt_tokens(spec.vocab, 2048, seed=101 + b) for b in range(7)])
    tb, _, _ = gm.generate(prompts, 256)
    assert np.array_equal(tb[0], wt)
