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
        srcs = [os.path.join(_HERE, f) for f in ("myl_oracle.c", "myl_oracle.h")]
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
