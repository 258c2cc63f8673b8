"""Integer decoder forward of the Qwen2.5 architecture on the B200.

Host-side mirror of the reference runtime's model API
(INTEGER_LLM/runtime/src/model.rs, generate.rs) over the C ABI of
libmyl_w8a16.so (``myl_model_*``, include/myl_w8a16.h):

  IntegerModel(ctx, spec)                  loader.rs:709-851 build_model
  Session(model, batch, max_positions)     kv_cache.rs:13-36 KVCache::new
  Session.forward(tokens)                  model.rs:229-311 forward_token (T tokens)
  Session.decode(n, digest=...)            generate.rs:101-113 / :181-196 (greedy)
  IntegerModel.generate(prompt, n,         generate.rs:76-116 generate (greedy) and,
                        digest=True)       :161-200 dekodieren_mit_digest

``ModelSpec`` / ``LayerSpec`` hold the tensors and calibrated scales the
reference's IntegerModel / TransformerLayer hold (model.rs:62-163), as numpy
arrays in the artifact layout: weights row-major [out][in] int8 with one
power-of-two shift per row, int16 attention biases with one shift per element,
per-channel residual-stream shifts, the five lookup tables, and the numeric
constants of theta_v/spec.json (loader.rs:654-682).

Every compute call runs on the GPU; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import hashlib
from dataclasses import dataclass, field

import numpy as np

# theta_v/spec.json "nonlinear" + loader.rs:669-681 (ModelConfig)
SPEC_CONSTANTS = dict(
    score_frac_bits=14,      # softmax.exp_lut_frac_bits
    exp_input_frac=8,        # softmax.exp_input_frac_bits
    prob_frac_bits=14,       # softmax.prob_frac_bits
    rope_frac_bits=8,        # rope.frac_bits
    silu_in_frac=6,          # silu.input_frac_bits
    silu_lut_offset=8192,    # -silu.input_range[0]
    silu_out_frac=8,         # silu.output_frac_bits
    rsqrt_input_shift=8,     # rsqrt.input_shift
    rsqrt_output_frac=8,     # rsqrt.output_frac_bits
    logit_frac_bits=6,       # loader.rs:680
)


@dataclass
class LayerSpec:
    """One TransformerLayer (model.rs:95-117) with its LayerScales (:62-92)."""
    ln1_gamma: np.ndarray            # input_layernorm gamma [H] int8
    ln1_gamma_shifts: np.ndarray     # [H] u8
    ln2_gamma: np.ndarray            # post_attention_layernorm
    ln2_gamma_shifts: np.ndarray
    wq: np.ndarray                   # [heads*head_dim][H] int8
    sq: np.ndarray                   # [heads*head_dim] u8
    wk: np.ndarray
    sk: np.ndarray
    wv: np.ndarray
    sv: np.ndarray
    wo: np.ndarray                   # [H][heads*head_dim]
    so: np.ndarray
    wg: np.ndarray                   # [I][H]
    sg: np.ndarray
    wu: np.ndarray
    su: np.ndarray
    wd: np.ndarray                   # [H][I]
    sd: np.ndarray
    norm_attn_frac: int
    q_frac: int
    k_frac: int
    v_frac: int
    attn_out_frac: int
    norm_mlp_frac: int
    gate_frac: int
    up_frac: int
    down_in_frac: int
    residual_in_frac: np.ndarray     # [H] u8 (per channel)
    residual_mid_frac: np.ndarray    # [H] u8
    bq: np.ndarray | None = None     # int16 biases + per-element shifts (loader.rs:145-148)
    bq_shifts: np.ndarray | None = None
    bk: np.ndarray | None = None
    bk_shifts: np.ndarray | None = None
    bv: np.ndarray | None = None
    bv_shifts: np.ndarray | None = None


@dataclass
class ModelSpec:
    """IntegerModel (model.rs:120-163) as host arrays."""
    vocab: int
    hidden: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    embed: np.ndarray                # [vocab][H] int8
    embed_shifts: np.ndarray         # [vocab] u8
    final_gamma: np.ndarray
    final_gamma_shifts: np.ndarray
    final_norm_frac: int
    final_residual_frac: np.ndarray  # [H] u8
    layers: list
    cos_lut: np.ndarray              # [n_pos * head_dim/2] int16
    sin_lut: np.ndarray
    exp_lut: np.ndarray
    silu_lut: np.ndarray
    rsqrt_lut: np.ndarray
    lm_head: np.ndarray | None = None        # path B int8 [vocab][H]; None: tied to embed
    lm_head_shifts: np.ndarray | None = None
    lm_head16: np.ndarray | None = None      # path A int16 [vocab][H] (loader.rs:119-128)
    lm_head16_shifts: np.ndarray | None = None
    constants: dict = field(default_factory=lambda: dict(SPEC_CONSTANTS))

    @property
    def tied(self) -> bool:
        return self.lm_head is None

    def head_weight(self):
        """(int8 weight, shifts) of LM-head path B (the embedding when tied)."""
        if self.lm_head is None:
            return self.embed, self.embed_shifts
        return self.lm_head, self.lm_head_shifts

    def weight_bytes_per_token(self) -> int:
        """Weight bytes one decode step streams (layers + LM head)."""
        H, I, QD = self.hidden, self.intermediate, self.num_heads * self.head_dim
        KD = self.num_kv_heads * self.head_dim
        per_layer = (QD + 2 * KD) * H + H * QD + 2 * I * H + H * I
        head = self.vocab * H * (2 if self.lm_head16 is not None else 1)
        return self.num_layers * per_layer + head


def digest(step_logits: np.ndarray, tokens: np.ndarray) -> str:
    """SHA-256 over, per decode step, the logits as i32 little-endian then the
    chosen token as u32 little-endian (generate.rs:177-198)."""
    h = hashlib.sha256()
    lg = np.ascontiguousarray(step_logits, dtype="<i4")
    tk = np.asarray(tokens, dtype="<u4")
    for s in range(len(tk)):
        h.update(lg[s].tobytes())
        h.update(tk[s:s + 1].tobytes())
    return h.hexdigest()


# ---- the C ABI of the forward (include/myl_w8a16.h, myl_model_*) --------------

class _LayerSpecC(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "ln1_gamma", "ln1_gamma_shifts", "ln2_gamma", "ln2_gamma_shifts",
        "wq", "wk", "wv", "wo", "wg", "wu", "wd",
        "sq", "sk", "sv", "so", "sg", "su", "sd", "bq", "bk", "bv",
        "bq_shifts", "bk_shifts", "bv_shifts")] + [(n, C.c_uint8) for n in (
        "norm_attn_frac", "q_frac", "k_frac", "v_frac", "attn_out_frac", "norm_mlp_frac",
        "gate_frac", "up_frac", "down_in_frac")] + [
        ("residual_in_frac", C.c_void_p), ("residual_mid_frac", C.c_void_p)]


class _ModelSpecC(C.Structure):
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


_LAYER_DTYPES = {
    "ln1_gamma": np.int8, "ln1_gamma_shifts": np.uint8, "ln2_gamma": np.int8,
    "ln2_gamma_shifts": np.uint8, "wq": np.int8, "wk": np.int8, "wv": np.int8, "wo": np.int8,
    "wg": np.int8, "wu": np.int8, "wd": np.int8, "sq": np.uint8, "sk": np.uint8, "sv": np.uint8,
    "so": np.uint8, "sg": np.uint8, "su": np.uint8, "sd": np.uint8, "bq": np.int16,
    "bk": np.int16, "bv": np.int16, "bq_shifts": np.uint8, "bk_shifts": np.uint8,
    "bv_shifts": np.uint8, "residual_in_frac": np.uint8, "residual_mid_frac": np.uint8}

_bound = False


def _lib():
    global _bound
    from . import load_library

    L = load_library()
    if not _bound:
        vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int
        for name, args, res in (
                ("myl_model_create", [vp, C.POINTER(_ModelSpecC), C.POINTER(vp)], i32),
                ("myl_model_release", [vp, vp], i32),
                ("myl_session_create", [vp, vp, i64, i64, C.POINTER(vp)], i32),
                ("myl_session_release", [vp, vp], i32),
                ("myl_session_reset", [vp, vp], i32),
                ("myl_session_position", [vp], i64),
                ("myl_forward", [vp, vp, vp, vp, i64, vp], i32),
                ("myl_generate", [vp, vp, vp, vp, i64, i64, vp, vp, vp], i32),
                ("myl_decode_greedy", [vp, vp, vp, i64, vp, vp, vp], i32),
                ("myl_model_create_tp", [vp, C.POINTER(_ModelSpecC), i32, i32, C.POINTER(vp)], i32),
                ("myl_model_shard", [vp, C.POINTER(i64)], i32),
                ("myl_session_tp_bytes", [vp], i64),
                ("myl_session_set_tp", [vp, vp, C.POINTER(vp)], i32),
                ("myl_session_timing", [vp, C.POINTER(C.c_float), C.POINTER(C.c_float)], i32),
                ("myl_rmsnorm_i16", [vp, vp, i64, i64, vp, vp, vp, vp, i64, C.c_uint8, C.c_uint8,
                                     i64, C.c_uint8, vp], i32),
                ("myl_attention_int", [vp, vp, i64, vp, vp, i64, i64, vp, i64, C.c_uint8, vp, i64,
                                       C.c_uint8, C.c_uint8, vp], i32)):
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _bound = True
    return L


def _check(fn, rc):
    from . import _check as chk

    chk(fn, rc)


class IntegerModel:
    """The reference's IntegerModel on one GPU (loader.rs:709-851 build_model,
    model.rs:229-311 forward_token, generate.rs greedy generation). Tensors are
    uploaded once; the numpy spec may be dropped afterwards."""

    def __init__(self, ctx, spec: ModelSpec, world: int = 1, rank: int = 0):
        L = _lib()
        keep = []

        def arr(a, dt):
            if a is None:
                return None
            a = np.ascontiguousarray(np.asarray(a, dtype=dt))
            keep.append(a)
            return a.ctypes.data

        layers = (_LayerSpecC * spec.num_layers)()
        for i, ls in enumerate(spec.layers):
            c = layers[i]
            for name, dt in _LAYER_DTYPES.items():
                setattr(c, name, arr(getattr(ls, name), dt))
            for name in ("norm_attn_frac", "q_frac", "k_frac", "v_frac", "attn_out_frac",
                         "norm_mlp_frac", "gate_frac", "up_frac", "down_in_frac"):
                setattr(c, name, int(getattr(ls, name)))
        ms = _ModelSpecC()
        for n in ("vocab", "hidden", "num_layers", "num_heads", "num_kv_heads", "head_dim",
                  "intermediate"):
            setattr(ms, n, int(getattr(spec, n)))
        ms.embed = arr(spec.embed, np.int8)
        ms.embed_shifts = arr(spec.embed_shifts, np.uint8)
        ms.lm_head = arr(spec.lm_head, np.int8)
        ms.lm_head_shifts = arr(spec.lm_head_shifts, np.uint8)
        ms.lm_head16 = arr(spec.lm_head16, np.int16)
        ms.lm_head16_shifts = arr(spec.lm_head16_shifts, np.uint8)
        ms.final_gamma = arr(spec.final_gamma, np.int8)
        ms.final_gamma_shifts = arr(spec.final_gamma_shifts, np.uint8)
        ms.final_norm_frac = int(spec.final_norm_frac)
        ms.final_residual_frac = arr(spec.final_residual_frac, np.uint8)
        ms.layers = C.cast(layers, C.c_void_p)
        for name, ln in (("cos_lut", "rope_len"), ("sin_lut", None), ("exp_lut", "exp_len"),
                         ("silu_lut", "silu_len"), ("rsqrt_lut", "rsqrt_len")):
            a = np.ascontiguousarray(np.asarray(getattr(spec, name), np.int16))
            keep.append(a)
            setattr(ms, name, a.ctypes.data)
            if ln:
                setattr(ms, ln, len(a))
        for n, v in spec.constants.items():
            setattr(ms, n, int(v))
        h = C.c_void_p()
        _check("myl_model_create_tp", L.myl_model_create_tp(ctx.handle, C.byref(ms), world, rank,
                                                            C.byref(h)))
        self._h = h
        self.ctx = ctx
        self.world, self.rank = world, rank
        info = (C.c_int64 * 10)()
        _check("myl_model_shard", L.myl_model_shard(h, info))
        # this rank's ranges: query heads, KV heads, MLP channels, vocabulary rows
        self.shard = dict(q=(info[2], info[3]), kv=(info[4], info[5]), mlp=(info[6], info[7]),
                          vocab=(info[8], info[9]))
        self.vocab_local = info[9] - info[8]
        self.vocab = spec.vocab
        self.hidden = spec.hidden
        self.num_layers = spec.num_layers
        self.weight_bytes_per_token = spec.weight_bytes_per_token()

    @property
    def handle(self):
        return self._h

    def release(self) -> None:
        if self._h:
            _lib().myl_model_release(self.ctx.handle, self._h)
            self._h = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def session(self, batch: int = 1, max_positions: int = 2048) -> "Session":
        return Session(self, batch, max_positions)

    def forward_token(self, token_ids, session: "Session") -> np.ndarray:
        """forward_token for each sequence's next token(s): token_ids [B] or
        [B][T]; returns the last token's logits [B][vocab] int32."""
        return session.forward(token_ids)

    def generate(self, prompt, max_new: int, session: "Session | None" = None,
                 digest: bool = False, keep_logits: bool = False):
        """Greedy generation (generate.rs:76-116 / dekodieren_mit_digest :161-200)
        from an empty cache. prompt [B][P] (or [P]). Returns (tokens [B][max_new],
        digests (hex strings) or None, step logits [B][max_new][vocab] or None)."""
        p = np.ascontiguousarray(np.asarray(prompt, np.int32))
        if p.ndim == 1:
            p = p[None]
        B, P = p.shape
        s = session or Session(self, B, P + max_new)
        out = np.zeros((B, max_new), np.int32)
        dg = np.zeros((B, 32), np.uint8) if digest else None
        lg = np.zeros((B, max_new, self.vocab), np.int32) if keep_logits else None
        _check("myl_generate", _lib().myl_generate(
            self.ctx.handle, self._h, s.handle, p.ctypes.data, P, max_new, out.ctypes.data,
            None if dg is None else dg.ctypes.data, None if lg is None else lg.ctypes.data))
        return out, (None if dg is None else [bytes(d).hex() for d in dg]), lg


class Session:
    """KV caches of `batch` sequences (kv_cache.rs:13-36) plus the forward's
    work buffers on the GPU."""

    def __init__(self, model: IntegerModel, batch: int, max_positions: int):
        h = C.c_void_p()
        _check("myl_session_create", _lib().myl_session_create(
            model.ctx.handle, model.handle, batch, max_positions, C.byref(h)))
        self._h = h
        self.model = model
        self.batch = batch
        self.max_positions = max_positions

    @property
    def handle(self):
        return self._h

    @property
    def position(self) -> int:
        return int(_lib().myl_session_position(self._h))

    def reset(self) -> None:
        _check("myl_session_reset", _lib().myl_session_reset(self.model.ctx.handle, self._h))

    def setup_tp(self, group=None) -> None:
        """Tensor parallelism: shares this rank's peer-memory region with the
        other ranks of the torch.distributed group (one process per GPU) and
        hands every rank's region to the session (myl_session_set_tp)."""
        import torch.distributed as dist

        L = _lib()
        world, rank = self.model.world, self.model.rank
        nbytes = int(L.myl_session_tp_bytes(self._h))
        ptr, handle = self.model.ctx.ipc_alloc(nbytes)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self._tp_ptrs = [ptr if o == rank else self.model.ctx.ipc_open(handles[o]) for o in range(world)]
        self._tp_own = ptr
        bases = (C.c_void_p * world)(*self._tp_ptrs)
        _check("myl_session_set_tp", L.myl_session_set_tp(self.model.ctx.handle, self._h, bases))
        dist.barrier(group=group)

    def forward(self, tokens, want_logits: bool = True):
        """The logits of this rank's vocabulary rows (all of them at world 1)."""
        t = np.ascontiguousarray(np.asarray(tokens, np.int32)).reshape(self.batch, -1)
        lg = np.zeros((self.batch, self.model.vocab_local), np.int32) if want_logits else None
        _check("myl_forward", _lib().myl_forward(
            self.model.ctx.handle, self.model.handle, self._h, t.ctypes.data, t.shape[1],
            None if lg is None else lg.ctypes.data))
        return lg

    def decode(self, max_new: int, digest: bool = False, keep_logits: bool = False):
        """The greedy decode loop (generate.rs:101-113) after forward() of the
        prompt: (tokens [B][max_new], digests or None, step logits or None)."""
        B, V = self.batch, self.model.vocab
        out = np.zeros((B, max_new), np.int32)
        dg = np.zeros((B, 32), np.uint8) if digest else None
        lg = np.zeros((B, max_new, V), np.int32) if keep_logits else None
        _check("myl_decode_greedy", _lib().myl_decode_greedy(
            self.model.ctx.handle, self.model.handle, self._h, max_new, out.ctypes.data,
            None if dg is None else dg.ctypes.data, None if lg is None else lg.ctypes.data))
        return out, (None if dg is None else [bytes(d).hex() for d in dg]), lg

    def timing(self) -> tuple[float, float]:
        """Device ms of the last prompt pass and of the last decode loop."""
        a, b = C.c_float(), C.c_float()
        _check("myl_session_timing", _lib().myl_session_timing(self._h, C.byref(a), C.byref(b)))
        return float(a.value), float(b.value)

    def release(self, _from_del: bool = False) -> None:
        if getattr(self, "_tp_ptrs", None) and not _from_del:
            # the other ranks' last kernels may still store into this rank's
            # region: every rank reaches this point before any region is freed
            import torch
            import torch.distributed as dist

            torch.cuda.synchronize()
            dist.barrier()
        if self._h:
            _lib().myl_session_release(self.model.ctx.handle, self._h)
            self._h = None
        ctx = self.model.ctx
        for o, ptr in enumerate(getattr(self, "_tp_ptrs", [])):
            if ptr != self._tp_own:
                ctx.ipc_close(ptr)
        if getattr(self, "_tp_own", None):
            ctx.ipc_free(self._tp_own)
        self._tp_ptrs, self._tp_own = [], None

    def __del__(self):
        try:
            if not getattr(self, "_tp_ptrs", None):  # shared regions need release() on every rank
                self.release(_from_del=True)
        except Exception:
            pass


def rmsnorm_i16(ctx, x, x_shifts, gamma, gamma_shifts, rsqrt_lut, lut_input_shift: int,
                lut_output_frac: int, inv_n_q20: int, out_frac_bits: int) -> np.ndarray:
    """rmsnorm_i16 (rmsnorm.rs:61-153) on the GPU, each row of x [M][n]."""
    x = np.ascontiguousarray(np.asarray(x, np.int16))
    rows = x.reshape(-1, x.shape[-1])
    out = np.zeros_like(rows)
    xs, g, gs = (np.ascontiguousarray(np.asarray(a, dt)) for a, dt in (
        (x_shifts, np.uint8), (gamma, np.int8), (gamma_shifts, np.uint8)))
    lut = np.ascontiguousarray(np.asarray(rsqrt_lut, np.int16))
    _check("myl_rmsnorm_i16", _lib().myl_rmsnorm_i16(
        ctx.handle, rows.ctypes.data, rows.shape[0], rows.shape[1], xs.ctypes.data, g.ctypes.data,
        gs.ctypes.data, lut.ctypes.data, len(lut), lut_input_shift, lut_output_frac, inv_n_q20,
        out_frac_bits, out.ctypes.data))
    return out.reshape(x.shape)


def attention_int(ctx, q, k, v, mask, score_mult: int, score_shift: int, exp_lut, lut_shift: int,
                  prob_frac_bits: int) -> np.ndarray:
    """attention_int (attention.rs:42-94) on the GPU."""
    q, k, v = (np.ascontiguousarray(np.asarray(a, np.int16)) for a in (q, k, v))
    lut = np.ascontiguousarray(np.asarray(exp_lut, np.int16))
    mk = None if mask is None else np.ascontiguousarray(np.asarray(mask, np.uint8))
    out = np.zeros_like(q)
    _check("myl_attention_int", _lib().myl_attention_int(
        ctx.handle, q.ctypes.data, q.shape[0], k.ctypes.data, v.ctypes.data, k.shape[0], q.shape[1],
        None if mk is None else mk.ctypes.data, score_mult, score_shift, lut.ctypes.data, len(lut),
        lut_shift, prob_frac_bits, out.ctypes.data))
    return out
