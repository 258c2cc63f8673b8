"""Integer decoder forward of the Qwen2.5 architecture on the B200.

Host-side mirror of the reference runtime's model API
(INTEGER_LLM/runtime/src/model.rs, generate.rs) over the C ABI of
libmyl_w8a16.so (``myl_model_*``, include/myl_w8a16.h):

  IntegerModel(ctx, spec)                  loader.rs:709-851 build_model
  IntegerModel.forward_token(tok, pos, s)  model.rs:229-311
  IntegerModel.generate(prompt, n)         generate.rs:13-67 (greedy)
  IntegerModel.generate_with_digest(...)   generate.rs:161-200 dekodieren_mit_digest
  Session(model, batch, max_positions)     kv_cache.rs:13-36 KVCache::new

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
