"""Model fixtures shared by the forward-pass tests.

loader_fixture_model(): the synthetic artifact of the reference's loader
tests (runtime/src/loader.rs:1361-1504 write_full_fixture: 1 layer, hidden 4,
2 query heads / 1 KV head of dim 2, intermediate 4, vocab 3; weights
(i % 7) as int8 with shift 0; int16 biases (i % 11) - 5 with shifts i % 3; the
scales of its scales.json; LUTs cos [256, 0, -256, 0], sin [0, 256, 0, -256],
exp [256, 128, 64], silu [-10, 0, 10, 20], rsqrt [256, 181, 148]) rebuilt as
a ModelSpec. The reference runs forward_token(0, 0) on it
(loader.rs:1582-1600); here it is the tiny-shape edge case of the forward.
"""
from __future__ import annotations

import numpy as np

from myelith_b200.model import LayerSpec, ModelSpec


def _w(rows, cols=None):
    n = rows * (cols or 1)
    a = (np.arange(n) % 7).astype(np.int8)
    return a.reshape(rows, cols) if cols else a


def _bias(n):
    return ((np.arange(n) % 11) - 5).astype(np.int16), (np.arange(n) % 3).astype(np.uint8)


def loader_fixture_model(tied: bool = True, attention_bias: bool = True) -> ModelSpec:
    hidden, heads, kv_heads, head_dim, inter, vocab = 4, 2, 1, 2, 4, 3
    QD, KD = heads * head_dim, kv_heads * head_dim
    z = lambda n: np.zeros(n, np.uint8)  # noqa: E731  (manifest "shift": 0, replicated per row)
    bq, bqs = _bias(QD)
    bk, bks = _bias(KD)
    bv, bvs = _bias(KD)
    layer = LayerSpec(
        ln1_gamma=_w(hidden), ln1_gamma_shifts=z(hidden),
        ln2_gamma=_w(hidden), ln2_gamma_shifts=z(hidden),
        wq=_w(QD, hidden), sq=z(QD), wk=_w(KD, hidden), sk=z(KD), wv=_w(KD, hidden), sv=z(KD),
        wo=_w(hidden, QD), so=z(hidden), wg=_w(inter, hidden), sg=z(inter),
        wu=_w(inter, hidden), su=z(inter), wd=_w(hidden, inter), sd=z(hidden),
        norm_attn_frac=4, q_frac=5, k_frac=5, v_frac=5, attn_out_frac=6, norm_mlp_frac=3,
        gate_frac=4, up_frac=3, down_in_frac=0,
        residual_in_frac=np.full(hidden, 12, np.uint8),
        residual_mid_frac=np.full(hidden, 5, np.uint8),
        bq=bq if attention_bias else None, bq_shifts=bqs if attention_bias else None,
        bk=bk if attention_bias else None, bk_shifts=bks if attention_bias else None,
        bv=bv if attention_bias else None, bv_shifts=bvs if attention_bias else None)
    spec = ModelSpec(
        vocab=vocab, hidden=hidden, num_layers=1, num_heads=heads, num_kv_heads=kv_heads,
        head_dim=head_dim, intermediate=inter, embed=_w(vocab, hidden), embed_shifts=z(vocab),
        final_gamma=_w(hidden), final_gamma_shifts=z(hidden), final_norm_frac=2,
        final_residual_frac=np.full(hidden, 4, np.uint8), layers=[layer],
        cos_lut=np.array([256, 0, -256, 0], np.int16), sin_lut=np.array([0, 256, 0, -256], np.int16),
        exp_lut=np.array([256, 128, 64], np.int16), silu_lut=np.array([-10, 0, 10, 20], np.int16),
        rsqrt_lut=np.array([256, 181, 148], np.int16))
    if not tied:
        spec.lm_head = _w(vocab, hidden)
        spec.lm_head_shifts = z(vocab)
    return spec
