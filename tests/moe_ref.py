"""MoE layer problems and their oracle result (test infrastructure).

The reference has no MoE; the layer is composed of its primitives, and the
oracle result is that composition on the CPU oracle:
  logits = lm_head_w8a16_i32(x, W_router, router_w_shifts, router_in_frac, router_frac)
           (runtime/src/model.rs:297-307)
  topk, p = moe_route(logits, k, exp_lut, lut_shift, prob_frac)
           (k x argmax with the lowest index on ties, sampling.rs:8-18; softmax_int,
           softmax.rs:24-64)
  y[t][j] = mlp_int(x[t], expert topk[t][j])               (mlp.rs:28-74; the oracle's
           blocked-dot composition mlp_int_fast, equal to mlp_int, test_oracle_kat.py)
  out     = moe_combine(y, p, mlp_int(x, shared expert) or 0, prob_frac)
"""
from __future__ import annotations

import numpy as np

import gen
import oracle as O
from make_golden import silu_lut_spec

# exp(-i / 256) at 14 fractional bits (the table of softmax_cases.json).
EXP_LUT14 = np.array([int(round(np.exp(-i / 256.0) * (1 << 14))) for i in range(16384)], np.int16)

FRACS = dict(in_frac=8, gate_out_frac=7, up_out_frac=7, down_in_frac=7, silu_in_frac=6,
             silu_lut_offset=8192, silu_out_frac=8)


def activations(rng, T, H, sigma=1024.0):
    """int16 = clamp(round(N(0, sigma^2)), +-32767)."""
    return np.clip(np.rint(rng.normal(0, sigma, size=(T, H))), -32767, 32767).astype(np.int16)


def problem(H, I, E, k, shared_I=0, seed=1, tie_pairs=(), prob_frac=14):
    """Seeded MoE parameters. tie_pairs: (a, b) expert pairs whose router rows
    and shifts are equal, so their logits tie for every token."""
    rng = np.random.default_rng(seed)
    nh = gen.nominal_shift(H, 12)
    ni = gen.nominal_shift(I, 12)
    Wr = rng.integers(-127, 128, size=(E, H), dtype=np.int8)
    # router scales 2^4 above the nominal shift: logits of a few units, so the
    # top-k probabilities are mixed rather than one-hot
    rs = rng.integers(nh + 3, nh + 6, size=E).astype(np.uint8)
    for a, b in tie_pairs:
        Wr[b] = Wr[a]
        rs[b] = rs[a]
    p = dict(
        hidden=H, intermediate=I, num_experts=E, top_k=k,
        W_router=Wr, router_w_shifts=rs, router_in_frac=8, router_frac=12,
        exp_lut=EXP_LUT14, exp_lut_shift=4, prob_frac=prob_frac,
        W_gate=rng.integers(-127, 128, size=(E, I, H), dtype=np.int8),
        W_up=rng.integers(-127, 128, size=(E, I, H), dtype=np.int8),
        W_down=rng.integers(-127, 128, size=(E, H, I), dtype=np.int8),
        gate_w_shifts=rng.integers(nh - 1, nh + 2, size=(E, I)).astype(np.uint8),
        up_w_shifts=rng.integers(nh - 1, nh + 2, size=(E, I)).astype(np.uint8),
        down_w_shifts=rng.integers(ni - 1, ni + 2, size=(E, H)).astype(np.uint8),
        out_frac=rng.integers(3, 8, size=(E, H)).astype(np.uint8),
        silu_lut=silu_lut_spec(), **FRACS)
    shared = None
    if shared_I:
        ns = gen.nominal_shift(shared_I, 12)
        shared = dict(
            W_gate=rng.integers(-127, 128, size=(shared_I, H), dtype=np.int8),
            W_up=rng.integers(-127, 128, size=(shared_I, H), dtype=np.int8),
            W_down=rng.integers(-127, 128, size=(H, shared_I), dtype=np.int8),
            hidden_size=H, intermediate_size=shared_I,
            gate_w_shifts=rng.integers(nh - 1, nh + 2, size=shared_I).astype(np.uint8),
            up_w_shifts=rng.integers(nh - 1, nh + 2, size=shared_I).astype(np.uint8),
            down_w_shifts=rng.integers(ns - 1, ns + 2, size=H).astype(np.uint8),
            silu_lut=silu_lut_spec(), in_frac_bits=8, gate_out_frac=7, up_out_frac=7,
            down_in_frac=7, silu_in_frac=6, silu_lut_offset=8192, silu_out_frac=8,
            out_frac_bits=rng.integers(3, 8, size=H).astype(np.uint8))
    return p, shared


def expert_mlp(p, e, x):
    H, I = p["hidden"], p["intermediate"]
    return O.mlp_int_fast(x, p["W_gate"][e], p["W_up"][e], p["W_down"][e], H, I, p["gate_w_shifts"][e],
                     p["up_w_shifts"][e], p["down_w_shifts"][e], p["silu_lut"], p["in_frac"],
                     p["gate_out_frac"], p["up_out_frac"], p["down_in_frac"], p["silu_in_frac"],
                     p["silu_lut_offset"], p["silu_out_frac"], p["out_frac"][e])


def shared_mlp(s, x):
    return O.mlp_int_fast(x, s["W_gate"], s["W_up"], s["W_down"], s["hidden_size"], s["intermediate_size"],
                     s["gate_w_shifts"], s["up_w_shifts"], s["down_w_shifts"], s["silu_lut"],
                     s["in_frac_bits"], s["gate_out_frac"], s["up_out_frac"], s["down_in_frac"],
                     s["silu_in_frac"], s["silu_lut_offset"], s["silu_out_frac"], s["out_frac_bits"])


def router_logits(p, x):
    return O.lm_head_w8a16_i32(x, p["W_router"].reshape(-1), p["hidden"], p["router_w_shifts"],
                               p["router_in_frac"], p["router_frac"]).reshape(len(x), -1)


def route(p, x):
    return O.moe_route(router_logits(p, x), p["top_k"], p["exp_lut"], p["exp_lut_shift"],
                       p["prob_frac"])


def experts(p, x, ids):
    """y[q] = mlp_int(x[q], expert ids[q]), one oracle call per expert."""
    ids = np.asarray(ids).reshape(-1)
    y = np.zeros((len(ids), p["hidden"]), np.int16)
    for e in np.unique(ids):
        rows = np.nonzero(ids == e)[0]
        y[rows] = expert_mlp(p, int(e), x[rows])
    return y


def forward(p, s, x):
    """Oracle MoE layer output of the tokens x [T, H] (and the routing)."""
    T = len(x)
    idx, prob = route(p, x)
    xs = np.repeat(x, p["top_k"], axis=0)
    y = experts(p, xs, idx)
    sh = shared_mlp(s, x) if s is not None else np.zeros_like(x)
    return O.moe_combine(y.reshape(T, p["top_k"], -1), prob, sh, p["prob_frac"]), idx, prob


def lib_moe(ctx, p, s, first_expert=0, num_local=None):
    """The GPU layer (myelith_b200.Moe) of a problem, optionally a slice of
    the experts."""
    import myelith_b200 as myl

    E = p["num_experts"]
    n = E if num_local is None else num_local
    sl = slice(first_expert, first_expert + n)
    shared = myl.Mlp(ctx, **s) if s is not None else None
    return myl.Moe(ctx, p["hidden"], p["intermediate"], E, p["top_k"], p["W_router"],
                   p["router_w_shifts"], p["router_in_frac"], p["router_frac"], p["exp_lut"],
                   p["exp_lut_shift"], p["prob_frac"], p["W_gate"][sl], p["W_up"][sl],
                   p["W_down"][sl], p["gate_w_shifts"][sl], p["up_w_shifts"][sl],
                   p["down_w_shifts"][sl], p["out_frac"][sl], p["silu_lut"], p["in_frac"],
                   p["gate_out_frac"], p["up_out_frac"], p["down_in_frac"], p["silu_in_frac"],
                   p["silu_lut_offset"], p["silu_out_frac"], shared=shared,
                   first_expert=first_expert, num_local=n)
