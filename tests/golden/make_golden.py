"""Generates the golden fixtures in this directory from the reference project.

Run it where a Myelith checkout is available (it is not needed afterwards):

    python tests/golden/make_golden.py --reference <path to the Myelith checkout>

It imports the reference's own Python restatement of the linear op,
``INTEGER_LLM/tests/golden/generate.py`` (functions ``rshift_round``,
``rescale``, ``clamp_i16``, ``linear_w8a16_ref``, ``splitmix64``,
``deterministic_tensor``; generate.py:37-106, 147-165), and uses it to compute
the expected outputs of seeded cases. Weights and activations are not stored:
the fixtures keep the seeds and the tests regenerate the tensors with
``gen.py`` (whose int8 stream is checked here against ``deterministic_tensor``).

Outputs written:
  linear_cases.json   linear_w8a16 / linear_w8a16_pc / LM-head cases; the
                      expected outputs come from generate.py applied row by
                      row (per-row shifts, per-channel out_frac).
  mlp_cases.json      mlp.rs:28-74 composed from generate.py's rescale,
                      rshift_round and linear_w8a16_ref.
  op_vectors.json     the reference's op golden vector linear_w8a16_identity
                      (conformance/vectors/op/linear_w8a16_identity.golden.json)
  forward_cases.json  rmsnorm_i16: the op golden vector rmsnorm_basic and seeded
                      rows computed by generate.py:66 rmsnorm_i16_ref (the
                      uniform-shift form of rmsnorm.rs:61); the SHA-256 of the
                      LUT files shipped in scale_packs/qwen2.5-{0.5b,7b}/
                      (luts.json), which the LUT generators are checked against.
  backward_cases.json the op golden vector backward_linear
                      (conformance/vectors/op/backward_linear.golden.json)
                      re-emitted in this repo's fixture format.
  splitmix_kat.json   the first outputs of the reference's splitmix64.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import gen  # noqa: E402


def load_reference_generate(ref_root: str):
    path = os.path.join(ref_root, "INTEGER_LLM", "tests", "golden", "generate.py")
    spec = importlib.util.spec_from_file_location("myelith_generate", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_linear(G, x_rows, W, K, w_shifts, act_frac, out_frac, clamp_i32=False):
    """generate.py:98 linear_w8a16_ref applied one output row at a time, so that
    each row carries its own weight shift and out_frac (linear.rs:61-68,
    :110-117). For the LM head the i16 clamp is replaced by the i32 clamp of
    runtime/src/model.rs:305."""
    N = len(w_shifts)
    out = np.zeros((len(x_rows), N), np.int64)
    for m, x in enumerate(x_rows):
        xl = [int(v) for v in x]
        for r in range(N):
            row = [int(v) for v in W[r * K:(r + 1) * K]]
            of = int(out_frac[r]) if hasattr(out_frac, "__len__") else int(out_frac)
            if clamp_i32:
                acc = sum(w * v for w, v in zip(row, xl))
                y = G.rescale(acc, int(w_shifts[r]) + act_frac, of)
                y = max(-(1 << 31), min((1 << 31) - 1, y))
            else:
                y = G.linear_w8a16_ref(xl, [row], act_frac, int(w_shifts[r]), of)[0]
            out[m, r] = y
    return out


LINEAR_CASES = [
    # name, M, K, N, x_bits, kind, shift jitter, seed
    ("k1_n1", 1, 1, 1, 16, "scalar", 0, 11),
    ("k2_n5", 2, 2, 5, 16, "scalar", 2, 12),
    ("k3_n7_ragged", 3, 3, 7, 16, "pc", 3, 13),
    ("k16_n32", 1, 16, 32, 12, "scalar", 2, 14),
    ("k17_n33_ragged", 2, 17, 33, 12, "pc", 3, 15),
    ("k64_n32", 1, 64, 32, 11, "scalar", 2, 16),
    ("k100_n48_pc", 3, 100, 48, 16, "pc", 4, 17),
    ("k128_n128", 2, 128, 128, 11, "scalar", 1, 18),
    ("k896_n64", 2, 896, 64, 11, "scalar", 1, 19),
    ("k896_n64_pc", 1, 896, 64, 16, "pc", 2, 20),
    ("k1000_n40_neg_shift", 1, 1000, 40, 6, "pc", 0, 21),
    ("k4864_n16", 1, 4864, 16, 11, "scalar", 1, 22),
    ("lmhead_k896_n96", 2, 896, 96, 11, "lm_head", 2, 23),
    ("lmhead_k64_n50_sat", 1, 64, 50, 16, "lm_head", 0, 24),
]


def make_linear(G):
    cases = []
    for name, M, K, N, x_bits, kind, jitter, seed in LINEAR_CASES:
        W = gen.int8_tensor(seed * 1000 + 1, N * K)
        x = gen.int16_tensor(seed * 1000 + 2, M * K, x_bits).reshape(M, K)
        nominal = gen.nominal_shift(K, x_bits)
        act_frac = 6
        if kind == "lm_head":
            logit_frac = 6
            if name.endswith("_sat"):
                # Left shift by 8: about half of the logits leave the i32 range and clamp.
                w_shifts = np.zeros(N, np.uint8)
                act_frac, logit_frac = 0, 8
            else:
                w_shifts = gen.uint8_tensor(seed * 1000 + 3, N, 0, 2 * jitter) + max(
                    0, nominal - jitter - 6)
            out_frac = logit_frac
        else:
            lo = max(0, nominal - jitter)
            w_shifts = gen.uint8_tensor(seed * 1000 + 3, N, lo, nominal + jitter)
            if kind == "pc":
                out_frac = gen.uint8_tensor(seed * 1000 + 4, N, 4, 10)
                if name.endswith("_neg_shift"):
                    # out_frac above w_shift + act_frac: negative total shift (left shift).
                    w_shifts = np.zeros(N, np.uint8)
                    act_frac = 0
                    out_frac = gen.uint8_tensor(seed * 1000 + 4, N, 0, 3)
            else:
                out_frac = 6
        y = ref_linear(G, x, W, K, w_shifts, act_frac, out_frac, clamp_i32=(kind == "lm_head"))
        dtype = np.int32 if kind == "lm_head" else np.int16
        y = y.astype(dtype)
        case = {
            "name": name, "kind": kind, "M": M, "K": K, "N": N, "x_bits": x_bits,
            "w_seed": seed * 1000 + 1, "x_seed": seed * 1000 + 2,
            "w_shifts": [int(v) for v in w_shifts], "act_frac": act_frac,
            "out_frac": [int(v) for v in out_frac] if hasattr(out_frac, "__len__") else int(out_frac),
            "y": y.reshape(-1).tolist(), "y_sha256": sha(y),
        }
        cases.append(case)
        print(f"linear {name}: {M}x{K}->{N} kind={kind}")
    return cases


def ref_mlp(G, x_rows, Wg, Wu, Wd, H, I, gs, us, ds, lut, in_frac, gate_out, up_out, down_in,
            silu_in, offset, silu_out, out_frac):
    """mlp.rs:28-74 written with generate.py's primitives (rescale,
    linear_w8a16_ref, clamp_i16). The SiLU index follows mlp.rs:56-57 and
    integer_math.rs:166-170 with Rust release i16 wrapping."""
    def wrap16(v):
        return ((int(v) + 32768) & 0xFFFF) - 32768

    outs = []
    for x in x_rows:
        gate = ref_linear(G, [x], Wg, H, gs, in_frac, gate_out)[0]
        up = ref_linear(G, [x], Wu, H, us, in_frac, up_out)[0]
        h = []
        for g, u in zip(gate, up):
            g_dom = G.rescale(int(g), gate_out, silu_in)
            idx = wrap16(wrap16(g_dom) + offset)
            idx = max(0, min(len(lut) - 1, idx))
            prod = int(lut[idx]) * int(u)
            h.append(G.clamp_i16(G.rescale(prod, silu_out + up_out, down_in)))
        outs.append(ref_linear(G, [h], Wd, I, ds, down_in, out_frac)[0])
    return np.array(outs, np.int16)


def silu_lut_spec(n=16384, in_frac=6, out_frac=8):
    """A SiLU table in the theta_v layout (spec.json 'silu': input [-8192, 8191]
    at input_frac 6, output_frac 8); offset = 8192."""
    xs = (np.arange(n) - n // 2) / float(1 << in_frac)
    vals = xs / (1.0 + np.exp(-xs)) * (1 << out_frac)
    return np.clip(np.round(vals), -32768, 32767).astype(np.int16)


MLP_CASES = [
    # name, M, H, I, x_bits, seed
    ("h32_i64", 1, 32, 64, 11, 31),
    ("h64_i96_m3", 3, 64, 96, 11, 32),
    ("h128_i256", 2, 128, 256, 12, 33),
]


def make_mlp(G):
    lut = silu_lut_spec()
    cases = []
    for name, M, H, I, x_bits, seed in MLP_CASES:
        Wg = gen.int8_tensor(seed * 1000 + 1, I * H)
        Wu = gen.int8_tensor(seed * 1000 + 2, I * H)
        Wd = gen.int8_tensor(seed * 1000 + 3, H * I)
        x = gen.int16_tensor(seed * 1000 + 4, M * H, x_bits).reshape(M, H)
        nh = gen.nominal_shift(H, x_bits)
        ni = gen.nominal_shift(I, 12)
        gs = gen.uint8_tensor(seed * 1000 + 5, I, max(0, nh - 1), nh + 1)
        us = gen.uint8_tensor(seed * 1000 + 6, I, max(0, nh - 1), nh + 1)
        ds = gen.uint8_tensor(seed * 1000 + 7, H, max(0, ni - 1), ni + 1)
        of = gen.uint8_tensor(seed * 1000 + 8, H, 3, 7)
        params = dict(in_frac=6, gate_out=6, up_out=6, down_in=6, silu_in=6, offset=8192,
                      silu_out=8)
        y = ref_mlp(G, x, Wg, Wu, Wd, H, I, gs, us, ds, lut, params["in_frac"], params["gate_out"],
                    params["up_out"], params["down_in"], params["silu_in"], params["offset"],
                    params["silu_out"], of)
        cases.append({
            "name": name, "M": M, "H": H, "I": I, "x_bits": x_bits,
            "wg_seed": seed * 1000 + 1, "wu_seed": seed * 1000 + 2, "wd_seed": seed * 1000 + 3,
            "x_seed": seed * 1000 + 4,
            "gate_w_shifts": gs.tolist(), "up_w_shifts": us.tolist(), "down_w_shifts": ds.tolist(),
            "out_frac": of.tolist(), "params": params,
            "y": y.reshape(-1).tolist(), "y_sha256": sha(y),
        })
        print(f"mlp {name}: M={M} H={H} I={I}")
    return cases


def make_backend_parity(G):
    """The inputs of kernels/tests/test_backend_parity.rs: linear 64->32
    (:160-183) and MLP hidden 32 / intermediate 64 (:218-255), with the SiLU
    table of :35-42. The Rust test compares two backends; here the expected
    outputs come from generate.py's restatement."""
    K, N = 64, 32
    x = [i * 7 - 200 for i in range(K)]
    W = [(i % 120) - 60 for i in range(N * K)]
    w_shifts = [(i % 8) + 4 for i in range(N)]
    y = ref_linear(G, [x], np.array(W, np.int8), K, w_shifts, 6, 6)[0]
    lin = {"name": "backend_parity_linear", "M": 1, "K": K, "N": N, "x": x, "W": W,
           "w_shifts": w_shifts, "act_frac": 6, "out_frac": 6, "y": y.astype(int).tolist()}

    H, I = 32, 64
    lut = []
    for i in range(2048):
        xf = (i - 1024.0) / 8.0
        lut.append(int(round(xf * (1.0 / (1.0 + np.exp(-xf))) * 64.0)))
    x = [i * 5 - 80 for i in range(H)]
    Wg = [(i % 120) - 60 for i in range(I * H)]
    Wu = [(i % 100) - 50 for i in range(I * H)]
    Wd = [(i % 80) - 40 for i in range(H * I)]
    gs = [4 + (i % 6) for i in range(I)]
    us = [5 + (i % 5) for i in range(I)]
    ds = [4 + (i % 7) for i in range(H)]
    of = [2 + (i % 6) for i in range(H)]
    y = ref_mlp(G, [x], np.array(Wg, np.int8), np.array(Wu, np.int8), np.array(Wd, np.int8), H, I,
                gs, us, ds, lut, 6, 8, 8, 8, 3, 1024, 6, of)[0]
    mlp = {"name": "backend_parity_mlp", "M": 1, "H": H, "I": I, "x": x, "W_gate": Wg, "W_up": Wu,
           "W_down": Wd, "gate_w_shifts": gs, "up_w_shifts": us, "down_w_shifts": ds,
           "out_frac": of, "silu_lut": lut,
           "params": dict(in_frac=6, gate_out=8, up_out=8, down_in=8, silu_in=3, offset=1024,
                          silu_out=6),
           "y": y.astype(int).tolist()}
    return [lin, mlp]


def make_forward(G, ref_root: str):
    """RMSNorm cases and the scale packs' LUT hashes (see the module docstring)."""
    vp = os.path.join(ref_root, "INTEGER_LLM", "conformance", "vectors", "op",
                      "rmsnorm_basic.golden.json")
    with open(vp) as f:
        v = json.load(f)
    md = v["metadata"]
    cases = [{
        "name": v["name"], "x": v["inputs"]["x"]["data"], "gamma": v["inputs"]["gamma"]["data"],
        "x_shift": 0, "gamma_shift": md["gamma_shift"], "lut": md["rsqrt_lut"],
        "lut_input_shift": md["lut_input_shift"], "lut_output_frac": md["lut_output_frac"],
        "inv_n_q20": md["inv_n_q20"], "out_frac": md["out_frac"], "y": v["outputs"]["y"]["data"]}]
    lut = G.spec_rsqrt_lut(32768)
    rng = np.random.default_rng(7)
    for i, (n, sigma, out_frac, gshift) in enumerate(
            ((896, 3000, 10, 6), (896, 40, 12, 6), (64, 30000, 8, 5), (3584, 800, 11, 7),
             (7, 1, 14, 6), (128, 12000, 6, 4), (896, 0, 10, 6))):
        x = np.clip(np.rint(rng.normal(0, sigma, size=n)), -32768, 32767).astype(int).tolist()
        gamma = rng.integers(-128, 128, size=n).astype(int).tolist()
        y = G.rmsnorm_i16_ref(x, gamma, gshift, lut, 8, 8, G.inv_n_q20(n), out_frac)
        cases.append({"name": f"rmsnorm_ref_{i}", "x": x, "gamma": gamma,
                      "x_shift": int(rng.integers(0, 16)), "gamma_shift": gshift,
                      "lut": "spec_rsqrt_32768", "lut_sha256": sha(np.array(lut, "<i2")),
                      "lut_input_shift": 8, "lut_output_frac": 8, "inv_n_q20": G.inv_n_q20(n),
                      "out_frac": out_frac, "y": [int(t) for t in y]})
    packs = {}
    for pack in ("qwen2.5-0.5b", "qwen2.5-7b"):
        with open(os.path.join(ref_root, "INTEGER_LLM", "scale_packs", pack, "luts.json")) as f:
            packs[pack] = {k: {"length": e["length"], "sha256": e["hash"]}
                           for k, e in json.load(f).items()}
    return {"rmsnorm": cases, "scale_pack_luts": packs}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the Myelith checkout")
    args = ap.parse_args()
    G = load_reference_generate(args.reference)

    # The int8 stream of gen.py must be the reference's deterministic_tensor.
    for seed in (0, 1, 42, 123456789):
        ref = np.array(G.deterministic_tensor(4, 8, seed), np.int8)
        assert np.array_equal(ref, gen.int8_tensor(seed, 32)), seed

    kat = []
    state = 42
    for _ in range(8):
        state, z = G.splitmix64(state)
        kat.append([state, z])
    with open(os.path.join(HERE, "splitmix_kat.json"), "w") as f:
        json.dump({"seed": 42, "steps": kat}, f, indent=1)

    vec_path = os.path.join(args.reference, "INTEGER_LLM", "conformance", "vectors", "op",
                            "linear_w8a16_identity.golden.json")
    with open(vec_path) as f:
        v = json.load(f)
    W = v["metadata"]["W"]
    op = [{
        "name": v["name"], "x": v["inputs"]["x"]["data"], "W": W,
        "w_shifts": [v["metadata"]["weight_frac"]] * len(W),
        "act_frac": v["metadata"]["act_frac"], "out_frac": v["metadata"]["out_frac"],
        "y": v["outputs"]["y"]["data"], "y_sha256_le_i16": v["outputs"]["y"]["hash"],
    }]
    # The reference's identity vector must agree with its own restatement.
    assert G.linear_w8a16_ref(op[0]["x"], W, op[0]["act_frac"], v["metadata"]["weight_frac"],
                              op[0]["out_frac"]) == op[0]["y"]
    with open(os.path.join(HERE, "op_vectors.json"), "w") as f:
        json.dump(op, f, indent=1)

    # linear_backward (kernels/src/backward.rs:147-211): the op golden vector
    # backward_linear, transcribed as inputs and expected outputs.
    bl_path = os.path.join(args.reference, "INTEGER_LLM", "conformance", "vectors", "op",
                           "backward_linear.golden.json")
    with open(bl_path) as f:
        bv = json.load(f)
    bwd = [{
        "name": bv["name"], "in_features": bv["metadata"]["in_features"],
        "w_shifts": bv["metadata"]["w_shifts"], "g_frac": bv["metadata"]["g_frac"],
        "gx_frac": bv["metadata"]["gx_frac"], "g": bv["inputs"]["g"]["data"],
        "x": bv["inputs"]["x"]["data"], "W": bv["inputs"]["W"]["data"],
        "gx": bv["outputs"]["gx"]["data"], "gW": bv["outputs"]["gW"]["data"],
    }]
    with open(os.path.join(HERE, "backward_cases.json"), "w") as f:
        json.dump(bwd, f, separators=(",", ":"))

    # softmax_int: the op golden vector softmax_basic plus cases computed by
    # generate.py:119 softmax_int_ref (its LUT's first entry equals 2^frac_bits,
    # where the reference's exp(0) lookup and `one` coincide).
    sm_path = os.path.join(args.reference, "INTEGER_LLM", "conformance", "vectors", "op",
                           "softmax_basic.golden.json")
    with open(sm_path) as f:
        sv = json.load(f)
    softmax = [{"name": sv["name"], "logits": sv["inputs"]["logits"]["data"],
                "exp_lut": sv["metadata"]["exp_lut"], "lut_shift": sv["metadata"]["lut_shift"],
                "frac_bits": sv["metadata"]["frac_bits"], "probs": sv["outputs"]["probs"]["data"]}]
    lut14 = [int(round(np.exp(-i / 256.0) * (1 << 14))) for i in range(16384)]
    rng = np.random.default_rng(99)
    for n, spread in ((4, 300), (4, 3000), (8, 50), (2, 0), (4, 40000)):
        lg = [int(v) for v in rng.integers(-spread - 1, spread + 1, size=n)]
        softmax.append({"name": f"softmax_n{n}_spread{spread}", "logits": lg, "exp_lut": lut14,
                        "lut_shift": 0, "frac_bits": 14,
                        "probs": [int(v) for v in G.softmax_int_ref(lg, lut14, 0, 14)]})
    with open(os.path.join(HERE, "softmax_cases.json"), "w") as f:
        json.dump(softmax, f, separators=(",", ":"))

    with open(os.path.join(HERE, "linear_cases.json"), "w") as f:
        json.dump(make_linear(G), f, separators=(",", ":"))
    with open(os.path.join(HERE, "mlp_cases.json"), "w") as f:
        json.dump(make_mlp(G), f, separators=(",", ":"))
    with open(os.path.join(HERE, "backend_parity.json"), "w") as f:
        json.dump(make_backend_parity(G), f, separators=(",", ":"))
    with open(os.path.join(HERE, "forward_cases.json"), "w") as f:
        json.dump(make_forward(G, args.reference), f, separators=(",", ":"))
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
