"""An artifact written in the θ_v layout (the reference's loader fixture,
runtime/src/loader.rs:1355-1440: weights_manifest.json, raw .bin tensors,
per-row shift files, an int16 LM head, luts.json) is read, its tensors are
registered on the GPU straight from the artifact, and the projections and
the LM head computed from them equal the CPU oracle on the same bytes.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import oracle as O
from make_golden import silu_lut_spec

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import myelith_b200 as myl  # noqa: E402


def _write_artifact(d, rng, hidden=64, inter=96, vocab=200):
    manifest, luts = {}, {}

    def put(name, arr, shifts=None, dtype="int8"):
        safe = name.replace(".", "_")
        raw = arr.astype("<i2" if dtype == "int16" else np.int8).tobytes()
        (d / f"{safe}.bin").write_bytes(raw)
        e = {"original_name": name, "file": f"{safe}.bin", "shape": list(arr.shape), "scale": 1.0,
             "shift": 0, "dtype": dtype, "hash": hashlib.sha256(raw).hexdigest()}
        if shifts is not None:
            (d / f"{safe}_shifts.bin").write_bytes(shifts.tobytes())
            e.update(shift=-1, scale=-1.0, shifts_file=f"{safe}_shifts.bin",
                     shifts_hash=hashlib.sha256(shifts.tobytes()).hexdigest())
        manifest["lm_head" if name == "lm_head" else safe] = e

    W = {}
    for name, shape in [("model.layers.0.self_attn.q_proj.weight", (hidden, hidden)),
                        ("model.layers.0.mlp.gate_proj.weight", (inter, hidden)),
                        ("model.layers.0.mlp.down_proj.weight", (hidden, inter))]:
        W[name] = (rng.integers(-128, 128, size=shape, dtype=np.int8),
                   rng.integers(8, 12, size=shape[0]).astype(np.uint8))
        put(name, *W[name])
    put("model.norm.weight", rng.integers(-128, 128, size=hidden, dtype=np.int8))
    lm = np.clip(np.rint(rng.normal(0, 6000, size=(vocab, hidden))), -32768, 32767).astype(np.int16)
    lm_sh = rng.integers(10, 14, size=vocab).astype(np.uint8)
    put("lm_head", lm, lm_sh, dtype="int16")
    silu = silu_lut_spec()
    (d / "silu.bin").write_bytes(silu.astype("<i2").tobytes())
    luts["silu"] = {"file": "silu.bin", "hash": hashlib.sha256(silu.astype("<i2").tobytes()).hexdigest(),
                    "length": int(silu.size), "dtype": "int16"}
    (d / "weights_manifest.json").write_text(json.dumps(manifest))
    (d / "luts.json").write_text(json.dumps(luts))
    return W, lm, lm_sh, silu


def test_artifact_to_device(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = myl.Context(0)
    rng = np.random.default_rng(3)
    W, lm, lm_sh, silu = _write_artifact(tmp_path, rng)
    art = myl.Artifact(tmp_path)
    assert len(art) == 5 and np.array_equal(art.lut("silu"), silu)
    for name, (Wn, sh) in W.items():
        w = art.register(ctx, name)
        K = Wn.shape[1]
        for M in (1, 40):
            x = rng.integers(-3000, 3000, size=(M, K), dtype=np.int16)
            assert np.array_equal(w.linear(x, 8, 6), O.linear_w8a16(x, Wn.reshape(-1), K, sh, 8, 6)), name
    head = art.register(ctx, "lm_head")
    for M in (1, 9):
        x = rng.integers(-4000, 4000, size=(M, lm.shape[1]), dtype=np.int16)
        assert np.array_equal(head.lm_head(x, 8, 6), O.lm_head_w16a16_i32(x, lm, lm.shape[1], lm_sh, 8, 6))
    with pytest.raises(myl.MylError):  # 1-D tensors are not weights
        art.register(ctx, "model.norm.weight")
    ctx.close()
