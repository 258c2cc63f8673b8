"""θ_v artifact reader (runtime/src/loader.rs:322-560) on the CPU: the cases of
the reference's own loader tests (loader.rs:889-1100, 1341-1352): SHA-256
known answers, round trip with uniform and per-row shifts, rejected hashes,
sizes, dtypes and shift files, names with dots, LUT tables.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import myelith_b200 as myl


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def entry(file, shape, shift, h, dtype="int8", **kw):
    e = {"original_name": file.replace(".bin", "").replace("_", "."), "file": file, "shape": shape,
         "scale": 1.0, "shift": shift, "dtype": dtype, "hash": h}
    e.update(kw)
    return e


def write(d, manifest, luts=None):
    with open(os.path.join(d, "weights_manifest.json"), "w") as f:
        json.dump(manifest, f)
    if luts is not None:
        with open(os.path.join(d, "luts.json"), "w") as f:
            json.dump(luts, f)


def test_sha256_known_vectors():  # loader.rs:889-900 (FIPS 180-4)
    assert myl.sha256(b"abc").hex() == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    assert myl.sha256(b"").hex() == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"
    rng = np.random.default_rng(1)
    for n in (1, 55, 56, 63, 64, 65, 119, 1000, 100003):
        data = rng.integers(0, 256, size=n, dtype=np.uint8).tobytes()
        assert myl.sha256(data).hex() == sha(data), n


def test_roundtrip_uniform_shift(tmp_path):  # loader.rs:903-925
    raw = bytes([0x80, 0xFF, 0x00, 0x01, 0x7F, 0x40])
    (tmp_path / "t_a.bin").write_bytes(raw)
    write(tmp_path, {"t_a": entry("t_a.bin", [2, 3], 2, sha(raw))})
    a = myl.Artifact(tmp_path)
    assert len(a) == 1
    key, _, data, shifts = a.tensor("t_a")
    assert key == "t_a"
    assert data.tolist() == [[-128, -1, 0], [1, 127, 64]]
    assert shifts.tolist() == [2, 2]


def test_per_channel_shifts(tmp_path):  # loader.rs:927-946
    raw = bytes([1, 2, 3, 4, 5, 6])
    (tmp_path / "t_c.bin").write_bytes(raw)
    (tmp_path / "t_c_shifts.bin").write_bytes(bytes([7, 9]))
    write(tmp_path, {"t_c": entry("t_c.bin", [2, 3], -1, sha(raw), scale=-1.0,
                                  shifts_file="t_c_shifts.bin", shifts_hash=sha(bytes([7, 9])))})
    assert myl.Artifact(tmp_path).tensor("t_c")[3].tolist() == [7, 9]


@pytest.mark.parametrize("case", ["hash", "size", "dtype", "int16_name", "int16_no_shifts", "shift_range",
                                  "shifts_len", "shifts_hash"])
def test_rejections(tmp_path, case):  # loader.rs:948-975 and load_weights' checks
    raw = bytes([1, 2, 3, 4])
    (tmp_path / "t.bin").write_bytes(raw)
    (tmp_path / "s.bin").write_bytes(bytes([1, 2, 3]))
    e = {
        "hash": entry("t.bin", [4], 0, "0" * 64),
        "size": entry("t.bin", [2, 3], 0, sha(raw)),
        "dtype": entry("t.bin", [4], 0, sha(raw), dtype="float32"),
        "int16_name": entry("t.bin", [2], 0, sha(raw), dtype="int16", shifts_file="s.bin"),
        "int16_no_shifts": dict(entry("t.bin", [1, 2], 0, sha(raw), dtype="int16")),
        "shift_range": entry("t.bin", [4], 300, sha(raw)),
        "shifts_len": entry("t.bin", [2, 2], -1, sha(raw), shifts_file="s.bin"),
        "shifts_hash": entry("t.bin", [3, 1], -1, sha(raw)[:0] + sha(raw), shifts_file="s.bin",
                             shifts_hash="1" * 64),
    }[case]
    name = "lm_head" if case == "int16_no_shifts" else "t"
    if case == "shifts_hash":
        (tmp_path / "t.bin").write_bytes(raw[:3])
        e["hash"] = sha(raw[:3])
    write(tmp_path, {name: e})
    with pytest.raises(myl.MylError) as ei:
        myl.Artifact(tmp_path)
    assert ei.value.code == myl.MYL_ERR_CORRUPT, str(ei.value)


def test_missing_manifest(tmp_path):  # loader.rs:976-983
    with pytest.raises(myl.MylError) as ei:
        myl.Artifact(tmp_path)
    assert ei.value.code == myl.MYL_ERR_IO and "weights_manifest.json" in str(ei.value)


def test_int16_lm_head_and_bias(tmp_path):
    lm = np.array([[1, -2, 3], [32767, -32768, 5]], np.int16)
    bias = np.array([7, -8], np.int16)
    (tmp_path / "lm.bin").write_bytes(lm.astype("<i2").tobytes())
    (tmp_path / "lm_s.bin").write_bytes(bytes([4, 5]))
    (tmp_path / "b.bin").write_bytes(bias.astype("<i2").tobytes())
    (tmp_path / "b_s.bin").write_bytes(bytes([1, 2]))
    write(tmp_path, {
        "lm_head": entry("lm.bin", [2, 3], -1, sha(lm.astype("<i2").tobytes()), dtype="int16",
                         shifts_file="lm_s.bin"),
        "model_layers_0_self_attn_q_proj_bias": entry("b.bin", [2], -1, sha(bias.astype("<i2").tobytes()),
                                                      dtype="int16", shifts_file="b_s.bin"),
    })
    a = myl.Artifact(tmp_path)
    assert np.array_equal(a.tensor("lm_head")[2], lm)
    assert a.tensor("lm_head")[3].tolist() == [4, 5]
    assert np.array_equal(a.tensor("model.layers.0.self_attn.q_proj.bias")[2], bias)


def test_names_with_dots(tmp_path):  # loader.rs:1341-1352
    raw = bytes([1, 2])
    (tmp_path / "model_norm_weight.bin").write_bytes(raw)
    write(tmp_path, {"model_norm_weight": entry("model_norm_weight.bin", [2], 0, sha(raw))})
    a = myl.Artifact(tmp_path)
    assert a.tensor("model.norm.weight")[0] == "model_norm_weight"
    with pytest.raises(myl.MylError):
        a.index("does.not.exist")


def test_luts(tmp_path):  # loader.rs:1008-1100
    silu = np.arange(-5, 5, dtype=np.int16)
    exp = np.array([16384, 8000, 100], np.int16)
    (tmp_path / "silu.bin").write_bytes(silu.astype("<i2").tobytes())
    (tmp_path / "exp.bin").write_bytes(exp.astype("<i2").tobytes())
    write(tmp_path, {}, {
        "silu": {"file": "silu.bin", "hash": sha(silu.astype("<i2").tobytes()), "length": 10, "dtype": "int16"},
        "exp": {"file": "exp.bin", "hash": sha(exp.astype("<i2").tobytes()), "length": 3, "dtype": "int16"},
    })
    a = myl.Artifact(tmp_path)
    assert np.array_equal(a.lut("silu"), silu) and np.array_equal(a.lut("exp"), exp)
    write(tmp_path, {}, {"exp": {"file": "exp.bin", "hash": "0" * 64, "length": 3, "dtype": "int16"}})
    with pytest.raises(myl.MylError):
        myl.Artifact(tmp_path)
    write(tmp_path, {}, {"exp": {"file": "exp.bin", "hash": sha(exp.astype("<i2").tobytes()), "length": 4,
                                 "dtype": "int16"}})
    with pytest.raises(myl.MylError):
        myl.Artifact(tmp_path)
    write(tmp_path, {}, {"exp": {"file": "exp.bin", "hash": sha(exp.astype("<i2").tobytes()), "length": 3,
                                 "dtype": "int8"}})
    with pytest.raises(myl.MylError):
        myl.Artifact(tmp_path)
