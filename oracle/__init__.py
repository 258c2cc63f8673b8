"""CPU oracle for the W8A16 integer linear path (TEST INFRASTRUCTURE ONLY).

This package wraps ``oracle/_build/libmyl_oracle.so``, a plain-C restatement of
the reference Rust kernels (INTEGER_LLM/kernels/src/{fixed_point,dot,linear,
mlp,integer_math,sampling,prng}.rs and the LM head of runtime/src/model.rs).
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it, and only as the checker. The product library
(``myelith_b200``) never imports it.

Errors: where the reference panics (shape asserts, integer overflow in a
debug build) the C functions return a nonzero status; the wrappers raise
``OracleError`` with the same meaning.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libmyl_oracle.so")
_lib = None

ERR_SHAPE = 1
ERR_OVERFLOW = 2


class OracleError(RuntimeError):
    """Raised where the reference would panic (status 1 = shape, 2 = overflow)."""

    def __init__(self, fn: str, code: int):
        kind = {ERR_SHAPE: "shape mismatch", ERR_OVERFLOW: "integer overflow"}.get(code, "error")
        super().__init__(f"{fn}: {kind} (status {code})")
        self.code = code


def build() -> str:
    """Compiles the oracle with its Makefile (gcc, OpenMP) and returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        srcs = [os.path.join(_HERE, f)
                for f in ("myl_oracle.c", "myl_oracle.h", "myl_forward.c", "myl_forward.h")]
        if not os.path.exists(_LIB_PATH) or any(
                os.path.getmtime(f) > os.path.getmtime(_LIB_PATH) for f in srcs if os.path.exists(f)):
            build()
        L = C.CDLL(_LIB_PATH)
        i64, u8, i32 = C.c_int64, C.c_uint8, C.c_int32
        p = C.c_void_p
        L.mylo_rshift_round.argtypes = [i32, u8]
        L.mylo_rshift_round.restype = i32
        L.mylo_rshift_round_i64.argtypes = [i64, u8]
        L.mylo_rshift_round_i64.restype = i64
        L.mylo_rescale.argtypes = [i32, u8, u8, p]
        L.mylo_rescale_i64.argtypes = [i64, u8, u8, p]
        for name in ("mylo_clamp_i8", "mylo_clamp_i16"):
            getattr(L, name).argtypes = [i32]
            getattr(L, name).restype = C.c_int32
        L.mylo_clamp_i8.restype = C.c_int8
        L.mylo_clamp_i16.restype = C.c_int16
        L.mylo_clamp_i16_from_i64.argtypes = [i64]
        L.mylo_clamp_i16_from_i64.restype = C.c_int16
        L.mylo_clamp_i32.argtypes = [i64]
        L.mylo_clamp_i32.restype = i32
        L.mylo_dot_scalar.argtypes = [p, p, i64]
        L.mylo_dot_scalar.restype = i64
        L.mylo_linear_w8a16.argtypes = [p, i64, p, i64, i64, p, u8, u8, p]
        L.mylo_linear_w8a16_pc.argtypes = [p, i64, p, i64, i64, p, u8, p, p]
        L.mylo_lm_head_w8a16_i32.argtypes = [p, i64, p, i64, i64, p, u8, u8, p]
        L.mylo_lm_head_w16a16_i32.argtypes = [p, i64, p, i64, i64, p, u8, u8, p]
        L.mylo_linear_backward.argtypes = [p, p, i64, p, i64, i64, p, u8, u8, p, p]
        L.mylo_linear_w8a16_mult.argtypes = [p, i64, p, i64, i64, p, p, p]
        L.mylo_linear_acc_i64.argtypes = [p, i64, p, i64, i64, p]
        L.mylo_add_bias_i16.argtypes = [p, p, p, i64, u8]
        L.mylo_lut_lookup.argtypes = [C.c_int16, p, i64, u8, C.c_int16]
        L.mylo_lut_lookup.restype = C.c_int16
        L.mylo_mlp_int.argtypes = [p, i64, p, p, p, i64, i64, p, p, p, p, i64,
                                   u8, u8, u8, u8, u8, C.c_int16, u8, p, p, p]
        L.mylo_mlp_hidden.argtypes = [p, i64, p, p, i64, i64, p, p, p, i64,
                                      u8, u8, u8, u8, u8, C.c_int16, u8, p, p]
        L.mylo_softmax_int.argtypes = [p, i64, p, i64, u8, u8, p]
        L.mylo_silu_product.argtypes = [p, p, i64, p, i64, u8, u8, u8, u8, C.c_int16, u8, p, p]
        L.mylo_inv_n_q20.argtypes = [i64]
        L.mylo_inv_n_q20.restype = i64
        L.mylo_isqrt_round.argtypes = [C.c_uint64]
        L.mylo_isqrt_round.restype = C.c_uint64
        L.mylo_inv_sqrt_q15.argtypes = [i64]
        L.mylo_inv_sqrt_q15.restype = i64
        L.mylo_rmsnorm_i16.argtypes = [p, i64, p, p, p, p, i64, u8, u8, i64, u8, p]
        L.mylo_rotate_half_split_i16.argtypes = [p, i64, p, p, u8, p]
        L.mylo_attention_int.argtypes = [p, i64, p, p, i64, i64, p, i64, u8, p, i64, u8, u8, p]
        L.mylo_forward.argtypes = [p, p, p, i64, p, i64, i64, p]
        L.mylo_linear_w8a16_pc_fast.argtypes = [p, i64, p, i64, i64, p, u8, p, p]
        L.mylo_linear_acc_fast.argtypes = [p, i64, p, i64, i64, p]
        L.mylo_requant_acc.argtypes = [p, i64, i64, p, u8, p, p]
        L.mylo_generate.argtypes = [p, p, p, i64, p, i64, i64, p, p]
        L.mylo_moe_route.argtypes = [p, i64, i64, i64, p, i64, u8, u8, p, p]
        L.mylo_moe_combine.argtypes = [p, p, p, i64, i64, i64, u8, p]
        L.mylo_argmax_i32.argtypes = [p, i64]
        L.mylo_argmax_i32.restype = i64
        L.mylo_splitmix64.argtypes = [C.c_uint64, p]
        L.mylo_splitmix64.restype = C.c_uint64
        L.mylo_num_threads.restype = C.c_int
        L.mylo_set_num_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


def _check(fn: str, rc: int) -> None:
    if rc != 0:
        raise OracleError(fn, rc)


# ---- fixed_point.rs --------------------------------------------------------

def rshift_round(value: int, shift: int) -> int:
    return lib().mylo_rshift_round(value, shift)


def rshift_round_i64(value: int, shift: int) -> int:
    return lib().mylo_rshift_round_i64(value, shift)


def rescale(acc: int, in_frac: int, out_frac: int) -> int:
    out = np.zeros(1, np.int32)
    _check("rescale", lib().mylo_rescale(acc, in_frac, out_frac, _ptr(out)))
    return int(out[0])


def rescale_i64(acc: int, in_frac: int, out_frac: int) -> int:
    out = np.zeros(1, np.int64)
    _check("rescale_i64", lib().mylo_rescale_i64(acc, in_frac, out_frac, _ptr(out)))
    return int(out[0])


def clamp_i8(x: int) -> int:
    return lib().mylo_clamp_i8(x)


def clamp_i16(x: int) -> int:
    return lib().mylo_clamp_i16(x)


def clamp_i16_from_i64(x: int) -> int:
    return lib().mylo_clamp_i16_from_i64(x)


def clamp_i32(x: int) -> int:
    return lib().mylo_clamp_i32(x)


# ---- dot.rs / linear.rs ------------------------------------------------------

def dot_scalar(w, x) -> int:
    w = _c(w, np.int8)
    x = _c(x, np.int16)
    n = min(w.size, x.size)  # zip semantics, dot.rs:393-399
    return lib().mylo_dot_scalar(_ptr(w), _ptr(x), n)


def _rows(x, K):
    x = _c(x, np.int16)
    if x.ndim == 1:
        return x.reshape(1, -1), True
    return x.reshape(-1, K), False


def linear_w8a16(x, W, in_features: int, w_shifts, act_frac: int, out_frac: int) -> np.ndarray:
    """linear.rs:43 on one row ([K]) or a batch of rows ([M, K]); returns int16."""
    W = _c(W, np.int8).reshape(-1)
    w_shifts = _c(w_shifts, np.uint8)
    N = w_shifts.size
    if in_features <= 0 or W.size != in_features * N:
        raise OracleError("linear_w8a16", ERR_SHAPE)
    xs, single = _rows(x, in_features)
    y = np.zeros((xs.shape[0], N), np.int16)
    _check("linear_w8a16", lib().mylo_linear_w8a16(
        _ptr(xs), xs.shape[0], _ptr(W), in_features, N, _ptr(w_shifts), act_frac, out_frac, _ptr(y)))
    return y[0] if single else y


def linear_w8a16_pc(x, W, in_features: int, w_shifts, act_frac: int, out_frac) -> np.ndarray:
    """linear.rs:87: per-output-channel out_frac."""
    W = _c(W, np.int8).reshape(-1)
    w_shifts = _c(w_shifts, np.uint8)
    out_frac = _c(out_frac, np.uint8)
    N = w_shifts.size
    if in_features <= 0 or W.size != in_features * N or out_frac.size != N:
        raise OracleError("linear_w8a16_pc", ERR_SHAPE)
    xs, single = _rows(x, in_features)
    y = np.zeros((xs.shape[0], N), np.int16)
    _check("linear_w8a16_pc", lib().mylo_linear_w8a16_pc(
        _ptr(xs), xs.shape[0], _ptr(W), in_features, N, _ptr(w_shifts), act_frac, _ptr(out_frac),
        _ptr(y)))
    return y[0] if single else y


def lm_head_w8a16_i32(x, W, in_features: int, w_shifts, final_norm_frac: int,
                      logit_frac: int) -> np.ndarray:
    """runtime/src/model.rs:297-307: i64 dot, rescale_i64, clamp to i32."""
    W = _c(W, np.int8).reshape(-1)
    w_shifts = _c(w_shifts, np.uint8)
    N = w_shifts.size
    if in_features <= 0 or W.size != in_features * N:
        raise OracleError("lm_head_w8a16_i32", ERR_SHAPE)
    xs, single = _rows(x, in_features)
    y = np.zeros((xs.shape[0], N), np.int32)
    _check("lm_head_w8a16_i32", lib().mylo_lm_head_w8a16_i32(
        _ptr(xs), xs.shape[0], _ptr(W), in_features, N, _ptr(w_shifts), final_norm_frac, logit_frac,
        _ptr(y)))
    return y[0] if single else y


def lm_head_w16a16_i32(x, W, in_features: int, w_shifts, final_norm_frac: int,
                       logit_frac: int) -> np.ndarray:
    """runtime/src/model.rs:285-296 (path A): int16 weights, i64 dot, rescale_i64,
    clamp to i32."""
    W = _c(W, np.int16).reshape(-1)
    w_shifts = _c(w_shifts, np.uint8)
    N = w_shifts.size
    if in_features <= 0 or W.size != in_features * N:
        raise OracleError("lm_head_w16a16_i32", ERR_SHAPE)
    xs, single = _rows(x, in_features)
    y = np.zeros((xs.shape[0], N), np.int32)
    _check("lm_head_w16a16_i32", lib().mylo_lm_head_w16a16_i32(
        _ptr(xs), xs.shape[0], _ptr(W), in_features, N, _ptr(w_shifts), final_norm_frac, logit_frac,
        _ptr(y)))
    return y[0] if single else y


def linear_backward(g, x, W, in_features: int, w_shifts, g_frac: int, gx_frac: int,
                    want_gw: bool = True):
    """kernels/src/backward.rs:147-211 on M tokens: g [M, N] int32, x [M, K] int16
    -> (gx [M, K] int32, gw [M, N, K] int64 or None)."""
    W = _c(W, np.int8).reshape(-1)
    w_shifts = _c(w_shifts, np.uint8)
    N = w_shifts.size
    if N == 0 or in_features <= 0 or W.size != in_features * N:
        raise OracleError("linear_backward", ERR_SHAPE)  # .max().expect(...) / chunks_exact
    g = _c(g, np.int32)
    single = g.ndim == 1
    g = np.ascontiguousarray(g.reshape(-1, N))
    xs = np.ascontiguousarray(_c(x, np.int16).reshape(-1, in_features))
    if xs.shape[0] != g.shape[0]:
        raise OracleError("linear_backward", ERR_SHAPE)
    M = g.shape[0]
    gx = np.zeros((M, in_features), np.int32)
    gw = np.zeros((M, N, in_features), np.int64) if want_gw else None
    _check("linear_backward", lib().mylo_linear_backward(
        _ptr(g), _ptr(xs), M, _ptr(W), in_features, N, _ptr(w_shifts), g_frac, gx_frac, _ptr(gx),
        _ptr(gw) if gw is not None else None))
    if single:
        return gx[0], (gw[0] if gw is not None else None)
    return gx, gw


def linear_w8a16_mult(x, W, in_features: int, mult, shift) -> np.ndarray:
    """Multiplier requant: clamp_i16(rne_i128(dot * mult[r], shift[r]))."""
    W = _c(W, np.int8).reshape(-1)
    mult = _c(mult, np.int32)
    shift = _c(shift, np.uint8)
    N = mult.size
    if in_features <= 0 or W.size != in_features * N or shift.size != N:
        raise OracleError("linear_w8a16_mult", ERR_SHAPE)
    xs, single = _rows(x, in_features)
    y = np.zeros((xs.shape[0], N), np.int16)
    _check("linear_w8a16_mult", lib().mylo_linear_w8a16_mult(
        _ptr(xs), xs.shape[0], _ptr(W), in_features, N, _ptr(mult), _ptr(shift), _ptr(y)))
    return y[0] if single else y


def linear_acc_i64(x, W, in_features: int, out_features: int) -> np.ndarray:
    """Raw i64 accumulators [M, N] (before requant)."""
    W = _c(W, np.int8).reshape(-1)
    if in_features <= 0 or W.size != in_features * out_features:
        raise OracleError("linear_acc_i64", ERR_SHAPE)
    xs, single = _rows(x, in_features)
    acc = np.zeros((xs.shape[0], out_features), np.int64)
    _check("linear_acc_i64", lib().mylo_linear_acc_i64(
        _ptr(xs), xs.shape[0], _ptr(W), in_features, out_features, _ptr(acc)))
    return acc[0] if single else acc


def add_bias_i16(out, bias, bias_shifts, out_frac: int) -> np.ndarray:
    """linear.rs:132: returns a new array (the reference mutates in place)."""
    o = _c(out, np.int16).copy()
    bias = _c(bias, np.int16)
    bias_shifts = _c(bias_shifts, np.uint8)
    if o.size != bias.size or bias.size != bias_shifts.size:
        raise OracleError("add_bias_i16", ERR_SHAPE)
    _check("add_bias_i16", lib().mylo_add_bias_i16(_ptr(o), _ptr(bias), _ptr(bias_shifts), o.size,
                                                   out_frac))
    return o


def lut_lookup(x: int, lut, shift: int, offset: int) -> int:
    lut = _c(lut, np.int16)
    return lib().mylo_lut_lookup(x, _ptr(lut), lut.size, shift, offset)


def mlp_int(x, W_gate, W_up, W_down, hidden_size: int, intermediate_size: int,
            gate_w_shifts, up_w_shifts, down_w_shifts, silu_lut, in_frac_bits: int,
            gate_out_frac: int, up_out_frac: int, down_in_frac: int, silu_in_frac: int,
            silu_lut_offset: int, silu_out_frac: int, out_frac_bits, return_wraps: bool = False):
    """mlp.rs:28 on one row or a batch of rows."""
    H, I = hidden_size, intermediate_size
    Wg = _c(W_gate, np.int8).reshape(-1)
    Wu = _c(W_up, np.int8).reshape(-1)
    Wd = _c(W_down, np.int8).reshape(-1)
    gs, us, ds = (_c(a, np.uint8) for a in (gate_w_shifts, up_w_shifts, down_w_shifts))
    lut = _c(silu_lut, np.int16)
    of = _c(out_frac_bits, np.uint8)
    if (Wg.size != H * I or Wu.size != H * I or Wd.size != H * I or gs.size != I or us.size != I
            or ds.size != H or of.size != H):
        raise OracleError("mlp_int", ERR_SHAPE)
    xs, single = _rows(x, H)
    y = np.zeros((xs.shape[0], H), np.int16)
    wraps = np.zeros(1, np.int64)
    _check("mlp_int", lib().mylo_mlp_int(
        _ptr(xs), xs.shape[0], _ptr(Wg), _ptr(Wu), _ptr(Wd), H, I, _ptr(gs), _ptr(us), _ptr(ds),
        _ptr(lut), lut.size, in_frac_bits, gate_out_frac, up_out_frac, down_in_frac, silu_in_frac,
        silu_lut_offset, silu_out_frac, _ptr(of), _ptr(y), _ptr(wraps)))
    out = y[0] if single else y
    return (out, int(wraps[0])) if return_wraps else out


def mlp_hidden(x, W_gate, W_up, hidden_size: int, intermediate_size: int, gate_w_shifts,
               up_w_shifts, silu_lut, in_frac_bits: int, gate_out_frac: int, up_out_frac: int,
               down_in_frac: int, silu_in_frac: int, silu_lut_offset: int,
               silu_out_frac: int) -> np.ndarray:
    """mlp.rs:49-64: h [M, I], the input of the down projection."""
    H, I = hidden_size, intermediate_size
    Wg = _c(W_gate, np.int8).reshape(-1)
    Wu = _c(W_up, np.int8).reshape(-1)
    gs, us = _c(gate_w_shifts, np.uint8), _c(up_w_shifts, np.uint8)
    lut = _c(silu_lut, np.int16)
    if Wg.size != H * I or Wu.size != H * I or gs.size != I or us.size != I:
        raise OracleError("mlp_hidden", ERR_SHAPE)
    xs, single = _rows(x, H)
    h = np.zeros((xs.shape[0], I), np.int16)
    _check("mlp_hidden", lib().mylo_mlp_hidden(
        _ptr(xs), xs.shape[0], _ptr(Wg), _ptr(Wu), H, I, _ptr(gs), _ptr(us), _ptr(lut), lut.size,
        in_frac_bits, gate_out_frac, up_out_frac, down_in_frac, silu_in_frac, silu_lut_offset,
        silu_out_frac, _ptr(h), None))
    return h[0] if single else h


def softmax_int(logits, exp_lut, lut_shift: int, frac_bits: int) -> np.ndarray:
    """softmax.rs:24-64."""
    lg = _c(logits, np.int32)
    lut = _c(exp_lut, np.int16)
    out = np.zeros(lg.size, np.int32)
    _check("softmax_int", lib().mylo_softmax_int(_ptr(lg), lg.size, _ptr(lut), lut.size, lut_shift,
                                                 frac_bits, _ptr(out)))
    return out


def moe_route(logits, k: int, exp_lut, lut_shift: int, prob_frac: int):
    """Top-k experts per token (argmax_int repeated, lowest index on ties) and
    softmax_int of their logits. logits [T, E] int32 -> (idx [T, k], prob [T, k])."""
    lg = _c(logits, np.int32)
    T, E = lg.shape
    lut = _c(exp_lut, np.int16)
    idx = np.zeros((T, k), np.int32)
    prob = np.zeros((T, k), np.int32)
    _check("moe_route", lib().mylo_moe_route(_ptr(lg), T, E, k, _ptr(lut), lut.size, lut_shift,
                                             prob_frac, _ptr(idx), _ptr(prob)))
    return idx, prob


def moe_combine(y_experts, topk_prob, shared, prob_frac: int) -> np.ndarray:
    """y_experts [T, k, H] int16, topk_prob [T, k], shared [T, H] -> out [T, H]."""
    y = _c(y_experts, np.int16)
    p = _c(topk_prob, np.int32)
    sh = _c(shared, np.int16)
    T, k, H = y.shape
    out = np.zeros((T, H), np.int16)
    _check("moe_combine", lib().mylo_moe_combine(_ptr(y), _ptr(p), _ptr(sh), T, k, H, prob_frac,
                                                 _ptr(out)))
    return out


def argmax_int(values) -> int:
    v = _c(values, np.int32)
    return int(lib().mylo_argmax_i32(_ptr(v), v.size))


def splitmix64(state: int):
    out = np.zeros(1, np.uint64)
    new_state = lib().mylo_splitmix64(state, _ptr(out))
    return int(new_state), int(out[0])


def num_threads() -> int:
    return lib().mylo_num_threads()


def set_num_threads(n: int) -> None:
    lib().mylo_set_num_threads(n)


# ---- forward pass (myl_forward.c) ---------------------------------------------

def linear_w8a16_fast(x, W, in_features: int, w_shifts, act_frac: int, out_frac) -> np.ndarray:
    """linear_w8a16 / linear_w8a16_pc with the blocked exact dot (same outputs
    as linear_w8a16_pc; out_frac scalar or per channel)."""
    x = _c(x, np.int16).reshape(-1, in_features)
    W = _c(W, np.int8)
    ws = _c(w_shifts, np.uint8)
    N = len(ws)
    of = _c(np.broadcast_to(np.asarray(out_frac, np.uint8), (N,)), np.uint8)
    y = np.zeros((x.shape[0], N), np.int16)
    _check("linear_w8a16_pc_fast", lib().mylo_linear_w8a16_pc_fast(
        _ptr(x), x.shape[0], _ptr(W), in_features, N, _ptr(ws), act_frac, _ptr(of), _ptr(y)))
    return y


def mlp_int_fast(x, W_gate, W_up, W_down, hidden_size: int, intermediate_size: int,
                 gate_w_shifts, up_w_shifts, down_w_shifts, silu_lut, in_frac_bits: int,
                 gate_out_frac: int, up_out_frac: int, down_in_frac: int, silu_in_frac: int,
                 silu_lut_offset: int, silu_out_frac: int, out_frac_bits) -> np.ndarray:
    """mlp_int (mlp.rs:28-74) composed of the blocked-dot linears and the SiLU
    product: the same outputs as mlp_int, for full-size checks."""
    H, I = hidden_size, intermediate_size
    x = _c(x, np.int16).reshape(-1, H)
    gate = linear_w8a16_fast(x, np.asarray(W_gate).reshape(-1), H, gate_w_shifts, in_frac_bits,
                             gate_out_frac)
    up = linear_w8a16_fast(x, np.asarray(W_up).reshape(-1), H, up_w_shifts, in_frac_bits, up_out_frac)
    lut = _c(silu_lut, np.int16)
    h = np.zeros_like(gate)
    _check("silu_product", lib().mylo_silu_product(
        _ptr(gate), _ptr(up), gate.size, _ptr(lut), len(lut), gate_out_frac, up_out_frac,
        down_in_frac, silu_in_frac, silu_lut_offset, silu_out_frac, _ptr(h), None))
    return linear_w8a16_fast(h, np.asarray(W_down).reshape(-1), I, down_w_shifts, down_in_frac,
                             out_frac_bits)


def linear_acc_fast(x, W, in_features: int, out_features: int) -> np.ndarray:
    """Exact int64 accumulators [M][N] (blocked dot)."""
    x = _c(x, np.int16).reshape(-1, in_features)
    W = _c(W, np.int8)
    acc = np.zeros((x.shape[0], out_features), np.int64)
    _check("linear_acc_fast", lib().mylo_linear_acc_fast(
        _ptr(x), x.shape[0], _ptr(W), in_features, out_features, _ptr(acc)))
    return acc


def requant_acc(acc, w_shifts, act_frac: int, out_frac) -> np.ndarray:
    """clamp_i16(rescale_i64(acc, w_shift + act_frac, out_frac)) per channel."""
    acc = _c(acc, np.int64)
    ws = _c(w_shifts, np.uint8)
    N = len(ws)
    of = _c(np.broadcast_to(np.asarray(out_frac, np.uint8), (N,)), np.uint8)
    y = np.zeros(acc.shape, np.int16)
    _check("requant_acc", lib().mylo_requant_acc(_ptr(acc), acc.shape[0], N, _ptr(ws), act_frac,
                                                 _ptr(of), _ptr(y)))
    return y


def inv_n_q20(n: int) -> int:
    return lib().mylo_inv_n_q20(n)


def isqrt_round(n: int) -> int:
    return lib().mylo_isqrt_round(n)


def inv_sqrt_q15(head_dim: int) -> int:
    return lib().mylo_inv_sqrt_q15(head_dim)


def rmsnorm_i16(x, x_shifts, gamma, gamma_shifts, rsqrt_lut, lut_input_shift: int,
                lut_output_frac: int, inv_n: int, out_frac_bits: int) -> np.ndarray:
    """rmsnorm.rs:61-153 on one row [n] or on each row of [M, n]."""
    x = _c(x, np.int16)
    rows = x.reshape(-1, x.shape[-1])
    n = rows.shape[1]
    xs, g, gs = _c(x_shifts, np.uint8), _c(gamma, np.int8), _c(gamma_shifts, np.uint8)
    lut = _c(rsqrt_lut, np.int16)
    if len(xs) != n or len(g) != n or len(gs) != n:
        raise OracleError("rmsnorm_i16", ERR_SHAPE)
    out = np.zeros_like(rows)
    for r in range(rows.shape[0]):
        _check("rmsnorm_i16", lib().mylo_rmsnorm_i16(
            _ptr(rows[r]), n, _ptr(xs), _ptr(g), _ptr(gs), _ptr(lut), len(lut), lut_input_shift,
            lut_output_frac, inv_n, out_frac_bits, _ptr(out[r])))
    return out.reshape(x.shape)


def rotate_half_split_i16(vec, cos_row, sin_row, frac_bits: int) -> np.ndarray:
    """rope.rs:17-32."""
    v = _c(vec, np.int16)
    c, s = _c(cos_row, np.int16), _c(sin_row, np.int16)
    if len(c) != len(v) // 2 or len(s) != len(v) // 2:
        raise OracleError("rotate_half_split_i16", ERR_SHAPE)
    out = np.zeros_like(v)
    _check("rotate_half_split_i16", lib().mylo_rotate_half_split_i16(
        _ptr(v), len(v), _ptr(c), _ptr(s), frac_bits, _ptr(out)))
    return out


def attention_int(q, k, v, mask, score_mult: int, score_shift: int, exp_lut, lut_shift: int,
                  prob_frac_bits: int) -> np.ndarray:
    """attention.rs:42-94; q [q_len][d], k/v [kv_len][d], mask [q_len][kv_len] bools or None."""
    q, k, v = _c(q, np.int16), _c(k, np.int16), _c(v, np.int16)
    lut = _c(exp_lut, np.int16)
    mk = None if mask is None else _c(mask, np.uint8)
    out = np.zeros_like(q)
    _check("attention_int", lib().mylo_attention_int(
        _ptr(q), q.shape[0], _ptr(k), _ptr(v), k.shape[0], q.shape[1],
        None if mk is None else _ptr(mk), score_mult, score_shift, _ptr(lut), len(lut), lut_shift,
        prob_frac_bits, _ptr(out)))
    return out


class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "ln1_gamma", "ln1_gamma_shifts", "ln2_gamma", "ln2_gamma_shifts",
        "wq", "wk", "wv", "wo", "wg", "wu", "wd",
        "sq", "sk", "sv", "so", "sg", "su", "sd", "bq", "bk", "bv",
        "bq_shifts", "bk_shifts", "bv_shifts")] + [(n, C.c_uint8) for n in (
        "norm_attn_frac", "q_frac", "k_frac", "v_frac", "attn_out_frac", "norm_mlp_frac",
        "gate_frac", "up_frac", "down_in_frac")] + [
        ("residual_in_frac", C.c_void_p), ("residual_mid_frac", C.c_void_p)]


class _Model(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "vocab", "hidden", "num_layers", "num_heads", "num_kv_heads", "head_dim",
        "intermediate")] + [(n, C.c_void_p) for n in (
        "embed", "embed_shifts", "lm_head", "lm_head_shifts", "lm_head16", "lm_head16_shifts",
        "final_gamma", "final_gamma_shifts")] + [
        ("final_norm_frac", C.c_uint8), ("final_residual_frac", C.c_void_p),
        ("layers", C.c_void_p), ("cos_lut", C.c_void_p), ("sin_lut", C.c_void_p),
        ("rope_len", C.c_int64), ("exp_lut", C.c_void_p), ("exp_len", C.c_int64),
        ("silu_lut", C.c_void_p), ("silu_len", C.c_int64), ("rsqrt_lut", C.c_void_p),
        ("rsqrt_len", C.c_int64)] + [(n, C.c_uint8) for n in (
        "score_frac_bits", "exp_input_frac", "prob_frac_bits", "rope_frac_bits", "silu_in_frac",
        "silu_out_frac", "rsqrt_input_shift", "rsqrt_output_frac", "logit_frac_bits")] + [
        ("silu_lut_offset", C.c_int16)]


_LAYER_ARRAYS = {
    "ln1_gamma": np.int8, "ln1_gamma_shifts": np.uint8, "ln2_gamma": np.int8,
    "ln2_gamma_shifts": np.uint8, "wq": np.int8, "wk": np.int8, "wv": np.int8, "wo": np.int8,
    "wg": np.int8, "wu": np.int8, "wd": np.int8, "sq": np.uint8, "sk": np.uint8, "sv": np.uint8,
    "so": np.uint8, "sg": np.uint8, "su": np.uint8, "sd": np.uint8, "bq": np.int16,
    "bk": np.int16, "bv": np.int16, "bq_shifts": np.uint8, "bk_shifts": np.uint8,
    "bv_shifts": np.uint8, "residual_in_frac": np.uint8, "residual_mid_frac": np.uint8}


class OracleModel:
    """The reference IntegerModel (runtime/src/model.rs) on the CPU, built from
    any object with ModelSpec's attributes (vocab, hidden, ..., layers, luts,
    constants). Holds the KV cache of one sequence (kv_cache.rs)."""

    def __init__(self, spec, max_positions: int):
        self._keep = []
        H = spec.hidden

        def arr(a, dt):
            if a is None:
                return None
            a = _c(a, dt)
            self._keep.append(a)
            return _ptr(a)

        layers = (_Layer * spec.num_layers)()
        for i, Ls in enumerate(spec.layers):
            L = layers[i]
            for name, dt in _LAYER_ARRAYS.items():
                setattr(L, name, arr(getattr(Ls, name), dt))
            for name in ("norm_attn_frac", "q_frac", "k_frac", "v_frac", "attn_out_frac",
                         "norm_mlp_frac", "gate_frac", "up_frac", "down_in_frac"):
                setattr(L, name, int(getattr(Ls, name)))
        self._layers = layers
        m = _Model()
        for n in ("vocab", "hidden", "num_layers", "num_heads", "num_kv_heads", "head_dim",
                  "intermediate"):
            setattr(m, n, int(getattr(spec, n)))
        m.embed = arr(spec.embed, np.int8)
        m.embed_shifts = arr(spec.embed_shifts, np.uint8)
        if spec.lm_head is None:
            m.lm_head, m.lm_head_shifts = m.embed, m.embed_shifts
        else:
            m.lm_head = arr(spec.lm_head, np.int8)
            m.lm_head_shifts = arr(spec.lm_head_shifts, np.uint8)
        m.lm_head16 = arr(spec.lm_head16, np.int16)
        m.lm_head16_shifts = arr(spec.lm_head16_shifts, np.uint8)
        m.final_gamma = arr(spec.final_gamma, np.int8)
        m.final_gamma_shifts = arr(spec.final_gamma_shifts, np.uint8)
        m.final_norm_frac = int(spec.final_norm_frac)
        m.final_residual_frac = arr(spec.final_residual_frac, np.uint8)
        m.layers = C.cast(layers, C.c_void_p)
        for name in ("cos_lut", "sin_lut", "exp_lut", "silu_lut", "rsqrt_lut"):
            a = _c(getattr(spec, name), np.int16)
            self._keep.append(a)
            setattr(m, name, _ptr(a))
            setattr(m, {"cos_lut": "rope_len", "sin_lut": "rope_len", "exp_lut": "exp_len",
                        "silu_lut": "silu_len", "rsqrt_lut": "rsqrt_len"}[name], len(a))
        for n, v in spec.constants.items():
            setattr(m, n, int(v))
        self._m = m
        self.spec = spec
        self.max_positions = int(max_positions)
        shape = (spec.num_layers, spec.num_kv_heads, self.max_positions, spec.head_dim)
        self.k_cache = np.zeros(shape, np.int16)
        self.v_cache = np.zeros(shape, np.int16)
        self.vocab = spec.vocab
        self.hidden = H

    def forward(self, tokens, pos0: int, want_logits: bool = True):
        """forward_token for consecutive tokens at pos0.. (logits of the last)."""
        t = _c(tokens, np.int32).reshape(-1)
        logits = np.zeros(self.vocab, np.int32) if want_logits else None
        _check("forward", lib().mylo_forward(
            C.byref(self._m), _ptr(self.k_cache), _ptr(self.v_cache), self.max_positions, _ptr(t),
            len(t), pos0, None if logits is None else _ptr(logits)))
        return logits

    def generate(self, prompt, max_new: int, keep_logits: bool = True):
        """dekodieren_mit_digest, greedy: (tokens [max_new], step logits or None)."""
        p = _c(prompt, np.int32).reshape(-1)
        out = np.zeros(max_new, np.int32)
        lg = np.zeros((max_new, self.vocab), np.int32) if keep_logits else None
        _check("generate", lib().mylo_generate(
            C.byref(self._m), _ptr(self.k_cache), _ptr(self.v_cache), self.max_positions, _ptr(p),
            len(p), max_new, _ptr(out), None if lg is None else _ptr(lg)))
        return out, lg
