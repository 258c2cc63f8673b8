"""Seeded random-init layers at the benchmark shapes (no checkpoints exist
here): int8 weights uniform in [-127, 127], per-row power-of-two shifts that
keep outputs mostly unsaturated, int16 activations rounded N(0, 1024^2).
"""
from __future__ import annotations

import math

import numpy as np

# BASELINE config 4
MOE_CONFIG4 = dict(H=2048, I=1408, E=64, k=4, shared_I=5632, T=4096)


def kbits(K: int) -> int:
    """Per-row weight shift that keeps outputs unsaturated: round(log2(73.6*sqrt(K)))."""
    return int(round(math.log2(73.6 * math.sqrt(K))))


def activations(rng, shape, sigma: float = 1024.0) -> np.ndarray:
    return np.clip(np.rint(rng.normal(0, sigma, size=shape)), -32767, 32767).astype(np.int16)


def exp_lut14() -> np.ndarray:
    """exp(-i / 256) at 14 fractional bits, 16384 entries."""
    return np.array([int(round(math.exp(-i / 256.0) * (1 << 14))) for i in range(16384)], np.int16)


def silu_lut() -> np.ndarray:
    """SiLU over [-128, 128) at 6 fractional input bits, 8 output bits; offset 8192."""
    xs = (np.arange(16384) - 8192) / 64.0
    return np.clip(np.round(xs / (1.0 + np.exp(-xs)) * 256), -32768, 32767).astype(np.int16)


def moe_layer(ctx, H: int, I: int, E: int, k: int, shared_I: int, first: int = 0,
              num_local: int | None = None, attach_shared: bool = True, seed: int = 4000):
    """(Moe, shared Mlp or None) with experts [first, first + num_local).
    Every rank that uses the same seed gets the same weights. The router
    shifts are equal across experts, so the expected load is balanced."""
    import myelith_b200 as myl

    nl = E - first if num_local is None else num_local
    rng = np.random.default_rng(seed)
    sh = kbits(H)

    def ints(shape):
        return rng.integers(-127, 128, size=shape, dtype=np.int8)

    Wr = ints((E, H))
    rs = np.full(E, sh + 4, np.uint8)
    Wg, Wu, Wd = ints((E, I, H)), ints((E, I, H)), ints((E, H, I))
    gs = rng.integers(sh - 1, sh + 2, size=(E, I)).astype(np.uint8)
    us = rng.integers(sh - 1, sh + 2, size=(E, I)).astype(np.uint8)
    ds = rng.integers(kbits(I) - 1, kbits(I) + 2, size=(E, H)).astype(np.uint8)
    of = rng.integers(3, 8, size=(E, H)).astype(np.uint8)
    silu = silu_lut()
    shared = None
    if shared_I:
        shared = myl.Mlp(ctx, ints((shared_I, H)), ints((shared_I, H)), ints((H, shared_I)), H, shared_I,
                         rng.integers(sh - 1, sh + 2, size=shared_I).astype(np.uint8),
                         rng.integers(sh - 1, sh + 2, size=shared_I).astype(np.uint8),
                         rng.integers(kbits(shared_I) - 1, kbits(shared_I) + 2, size=H).astype(np.uint8),
                         silu, 8, 7, 7, 7, 6, 8192, 8, rng.integers(3, 8, size=H).astype(np.uint8))
    sl = slice(first, first + nl)
    moe = myl.Moe(ctx, H, I, E, k, Wr, rs, 8, 12, exp_lut14(), 4, 14, Wg[sl], Wu[sl], Wd[sl], gs[sl],
                  us[sl], ds[sl], of[sl], silu, 8, 7, 7, 7, 6, 8192, 8,
                  shared=shared if attach_shared else None, first_expert=first, num_local=nl)
    return moe, shared


# ---- lookup tables of theta_v/spec.json "nonlinear" ----------------------------
# Restated from the reference's LUT generators (calibrate/src/luts.py:32-150):
# every entry is round-half-even(f(real) * 2^out_frac) of Python floats, the
# real input being index * 2^-in_frac. Pinned against the hashes of the LUT
# files the reference ships in scale_packs/ (tests/golden/lut_hashes.json).

def _round(v: float) -> int:
    return int(round(v))


def rsqrt_lut(max_input: int = 32767, input_shift: int = 8, frac_bits: int = 8) -> np.ndarray:
    """luts.py:32-49: index 0 is the sentinel 1.0."""
    scale = 1 << frac_bits
    out = [scale] + [_round(1.0 / math.sqrt(x / (1 << input_shift)) * scale)
                     for x in range(1, max_input + 1)]
    return np.array(out, np.int16)


def silu_lut_spec(input_min: int = -8192, input_max: int = 8191, input_frac_bits: int = 6,
                  output_frac_bits: int = 8) -> np.ndarray:
    """luts.py:52-69: silu(x * 2^-in) at 2^out, x in [input_min, input_max]."""
    ins, outs = 1 << input_frac_bits, 1 << output_frac_bits
    vals = []
    for x in range(input_min, input_max + 1):
        xf = x / ins
        vals.append(_round(xf * (1.0 / (1.0 + math.exp(-xf))) * outs))
    return np.array(vals, np.int16)


def exp_lut(exp_range: int = 16384, input_frac_bits: int = 8, output_frac_bits: int = 14) -> np.ndarray:
    """luts.py:106-123: exp(-i * 2^-in) at 2^out, i in [0, exp_range]."""
    ins, outs = 1 << input_frac_bits, 1 << output_frac_bits
    return np.array([_round(math.exp(-(i / ins)) * outs) for i in range(exp_range + 1)], np.int16)


def rope_luts(head_dim: int, max_seq_len: int = 2048, rope_theta: float = 1000000.0,
              frac_bits: int = 8):
    """luts.py:126-150: (sin, cos), flat [max_seq_len][head_dim/2], pair j has
    theta_j = rope_theta^-(j / half), angle p * theta_j."""
    scale, half = 1 << frac_bits, head_dim // 2
    sin_l, cos_l = [], []
    for p in range(max_seq_len):
        for j in range(half):
            angle = p * (1.0 / (rope_theta ** (j / half)))
            cos_l.append(_round(math.cos(angle) * scale))
            sin_l.append(_round(math.sin(angle) * scale))
    return np.array(sin_l, np.int16), np.array(cos_l, np.int16)


def spec_luts(head_dim: int) -> dict:
    """The five tables of an artifact for a model with this head_dim."""
    sin_l, cos_l = rope_luts(head_dim)
    return dict(rsqrt=rsqrt_lut(), silu=silu_lut_spec(), exp=exp_lut(), sin=sin_l, cos=cos_l)


# ---- random-init integer models (BASELINE configs 2 and 3) ----------------------

QWEN_DIMS = {
    # num_layers, hidden, heads, kv_heads, head_dim, intermediate, vocab, tied
    "qwen2.5-0.5b": (24, 896, 14, 2, 64, 4864, 151936, True),
    "qwen2.5-7b": (28, 3584, 28, 4, 128, 18944, 152064, False),
}


def synthetic_model(variant: str = "qwen2.5-0.5b", seed: int = 2, num_layers: int | None = None,
                    vocab: int | None = None, dims: tuple | None = None):
    """A ModelSpec of the Qwen2.5 architecture with random-init int8 weights
    (uniform in [-127, 127]) and power-of-two scales chosen so that every stage
    stays mostly unsaturated:
      - weight rows: shift kbits(K) + {-1, 0, +1} (output RMS ~ input RMS);
      - residual stream: per-channel shifts around a per-layer base (10..11),
        1 % of the channels four bits coarser (the wide spans the reference's
        per-channel residual scales carry, rmsnorm.rs:87-106);
      - norm outputs at 12 fractional bits, q/k/v/gate/up at 11, the attention
        output rescaled from 11 to 12, gamma 48..80 at shift 6;
      - int16 q/k/v biases (|b| <= 2048 at shifts 11..13), embedding rows at
        shift 7; the LM head tied to the embedding (0.5B) or its own int8
        matrix (7B) at kbits(H) - 4;
      - the spec's lookup tables (spec_luts).
    `num_layers`/`vocab`/`dims` shrink the model for tests."""
    from .model import LayerSpec, ModelSpec

    L, H, nq, nkv, hd, I, V, tied = QWEN_DIMS[variant] if dims is None else dims
    L = num_layers if num_layers is not None else L
    V = vocab if vocab is not None else V
    QD, KD = nq * hd, nkv * hd
    rng = np.random.default_rng(seed)

    def w(rows, cols):
        return rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)

    def wshift(rows, K):
        return (kbits(K) + rng.integers(-1, 2, size=rows)).astype(np.uint8)

    def residual(base):
        s = base + rng.choice([-1, 0, 0, 1], size=H)
        out = rng.random(H) < 0.01
        s[out] = base - 4
        return s.astype(np.uint8)

    def gamma():
        return rng.integers(48, 81, size=H, dtype=np.int8), np.full(H, 6, np.uint8)

    def bias(n):
        return (rng.integers(-2048, 2049, size=n).astype(np.int16),
                rng.integers(11, 14, size=n).astype(np.uint8))

    bases = [11 - (2 * l) // max(L, 1) for l in range(L + 1)]
    res_in = [residual(bases[l]) for l in range(L + 1)]
    layers = []
    for l in range(L):
        g1, g1s = gamma()
        g2, g2s = gamma()
        bq, bqs = bias(QD)
        bk, bks = bias(KD)
        bv, bvs = bias(KD)
        layers.append(LayerSpec(
            ln1_gamma=g1, ln1_gamma_shifts=g1s, ln2_gamma=g2, ln2_gamma_shifts=g2s,
            wq=w(QD, H), sq=wshift(QD, H), wk=w(KD, H), sk=wshift(KD, H),
            wv=w(KD, H), sv=wshift(KD, H), wo=w(H, QD), so=wshift(H, QD),
            wg=w(I, H), sg=wshift(I, H), wu=w(I, H), su=wshift(I, H),
            wd=w(H, I), sd=wshift(H, I),
            norm_attn_frac=12, q_frac=11, k_frac=11, v_frac=11, attn_out_frac=12,
            norm_mlp_frac=12, gate_frac=11, up_frac=11, down_in_frac=12,
            residual_in_frac=res_in[l], residual_mid_frac=residual(bases[l]),
            bq=bq, bq_shifts=bqs, bk=bk, bk_shifts=bks, bv=bv, bv_shifts=bvs))
    embed = w(V, H)
    fg, fgs = gamma()
    luts = spec_luts(hd)
    spec = ModelSpec(
        vocab=V, hidden=H, num_layers=L, num_heads=nq, num_kv_heads=nkv, head_dim=hd,
        intermediate=I, embed=embed, embed_shifts=np.full(V, 7, np.uint8),
        final_gamma=fg, final_gamma_shifts=fgs, final_norm_frac=10,
        final_residual_frac=res_in[L], layers=layers,
        cos_lut=luts["cos"], sin_lut=luts["sin"], exp_lut=luts["exp"], silu_lut=luts["silu"],
        rsqrt_lut=luts["rsqrt"])
    if not tied:
        spec.lm_head = w(V, H)
        spec.lm_head_shifts = np.full(V, kbits(H) - 4, np.uint8)
    return spec


def prompt_tokens(vocab: int, n: int, seed: int = 5) -> np.ndarray:
    """n uniform-random token ids (BASELINE configs 2/3: random prompts)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.int32)
