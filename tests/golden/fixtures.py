"""Loads the golden fixtures and regenerates their seeded tensors."""
from __future__ import annotations

import json
import os

import numpy as np

import gen

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(name):
    with open(os.path.join(HERE, name)) as f:
        return json.load(f)


def linear_cases():
    """Each case with W [N*K] int8, x [M, K] int16 and the expected y."""
    out = []
    for c in _load("linear_cases.json"):
        c = dict(c)
        c["W"] = gen.int8_tensor(c["w_seed"], c["N"] * c["K"])
        c["x"] = gen.int16_tensor(c["x_seed"], c["M"] * c["K"], c["x_bits"]).reshape(c["M"], c["K"])
        c["w_shifts"] = np.array(c["w_shifts"], np.uint8)
        if isinstance(c["out_frac"], list):
            c["out_frac"] = np.array(c["out_frac"], np.uint8)
        dt = np.int32 if c["kind"] == "lm_head" else np.int16
        c["y"] = np.array(c["y"], dt).reshape(c["M"], c["N"])
        out.append(c)
    return out


def mlp_cases():
    from make_golden import silu_lut_spec

    lut = silu_lut_spec()
    out = []
    for c in _load("mlp_cases.json"):
        c = dict(c)
        H, I, M = c["H"], c["I"], c["M"]
        c["W_gate"] = gen.int8_tensor(c["wg_seed"], I * H)
        c["W_up"] = gen.int8_tensor(c["wu_seed"], I * H)
        c["W_down"] = gen.int8_tensor(c["wd_seed"], H * I)
        c["x"] = gen.int16_tensor(c["x_seed"], M * H, c["x_bits"]).reshape(M, H)
        c["silu_lut"] = lut
        for k in ("gate_w_shifts", "up_w_shifts", "down_w_shifts", "out_frac"):
            c[k] = np.array(c[k], np.uint8)
        c["y"] = np.array(c["y"], np.int16).reshape(M, H)
        out.append(c)
    return out


def backend_parity():
    lin, mlp = _load("backend_parity.json")
    return lin, mlp


def op_vectors():
    return _load("op_vectors.json")


def backward_cases():
    return _load("backward_cases.json")


def softmax_cases():
    return _load("softmax_cases.json")


def splitmix_kat():
    return _load("splitmix_kat.json")
