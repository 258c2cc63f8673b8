"""The pipeline wire format through the library (host codec) against the CPU
restatement of codec.rs (oracle.wire) and the reference's own codec tests
(INTEGER_LLM/pipeline/src/codec.rs:181-339), restated here."""
import zlib

import numpy as np
import pytest

import myelith_b200 as myl
from oracle import wire as W

META = dict(version=1, theta_v_hash=0xDEAD_BEEF, request_id=7, sequence_id=3, stage_id=2,
            token_position=11, flags=0, reserved=0)


def _corrupt(fn):
    with pytest.raises(myl.MylError) as e:
        fn()
    assert e.value.code == myl.MYL_ERR_CORRUPT


def test_crc_check_value_and_zlib():
    assert myl.crc32(b"123456789") == 0xCBF43926  # the published CRC-32 check value
    assert myl.crc32(b"") == 0
    rng = np.random.default_rng(0)
    for n in (1, 7, 64, 1000, 65537):
        b = rng.integers(0, 256, size=n, dtype=np.uint8).tobytes()
        assert myl.crc32(b) == zlib.crc32(b)


def test_roundtrip_keeps_meta_and_tensor():  # codec.rs:197-211
    t = [-32768, -1, 0, 1, 32767]
    buf = myl.wire_encode(dict(META, payload_len=10), t)
    m, v = myl.wire_decode(buf)
    assert v.tolist() == t
    for k in ("request_id", "sequence_id", "stage_id", "token_position", "theta_v_hash"):
        assert m[k] == META[k]
    assert m["payload_len"] == 10


def test_bytes_equal_the_restatement():
    rng = np.random.default_rng(1)
    for n in (0, 1, 2, 3, 5, 8, 33, 1000):
        t = rng.integers(-32768, 32768, size=n).astype(np.int16)
        meta = dict(META, flags=n % 8, reserved=n * 3, payload_len=999)  # payload_len is recomputed
        lib = myl.wire_encode(meta, t)
        ref = W.encode_message(meta, t.tolist())
        assert lib == ref, n
        m, v = myl.wire_decode(ref)
        rm, rv = W.decode_message(ref)
        assert v.tolist() == rv and all(m[k] == rm[k] for k in rm)


def test_empty_tensor_is_valid():  # codec.rs:213-219
    m, v = myl.wire_decode(myl.wire_encode(dict(META, payload_len=0), []))
    assert v.size == 0 and m["payload_len"] == 0


def test_output_is_eight_byte_aligned():  # codec.rs:221-231
    for n in range(8):
        buf = myl.wire_encode(META, list(range(n)))
        assert len(buf) % 8 == 0
        assert len(buf) == myl.load_library().myl_wire_frame_bytes(n)


def test_encoding_is_deterministic():  # codec.rs:233-239
    assert myl.wire_encode(META, [5, -5, 100]) == myl.wire_encode(META, [5, -5, 100])


def test_wrong_magic_rejected():  # codec.rs:241-246
    buf = bytearray(myl.wire_encode(META, [1]))
    buf[0] = ord("X")
    _corrupt(lambda: myl.wire_decode(bytes(buf)))
    with pytest.raises(W.WireError):
        W.decode_message(bytes(buf))


def test_short_buffer_rejected():  # codec.rs:248-258
    buf = myl.wire_encode(META, [1])
    for n in range(W.HEADER_SIZE):
        _corrupt(lambda: myl.wire_decode(buf[:n]))


def test_every_payload_bit_flip_caught():  # codec.rs:260-279
    t = list(range(32))
    orig = myl.wire_encode(dict(META, payload_len=64), t)
    for byte in range(W.HEADER_SIZE, W.HEADER_SIZE + 64):
        for bit in range(8):
            b = bytearray(orig)
            b[byte] ^= 1 << bit
            _corrupt(lambda: myl.wire_decode(bytes(b)))


def test_overflowing_payload_length_rejected():  # codec.rs:281-288
    buf = bytearray(myl.wire_encode(META, [1]))
    off = 8 + 6 * 8
    buf[off:off + 8] = (2**64 - 1).to_bytes(8, "little")
    _corrupt(lambda: myl.wire_decode(bytes(buf)))
    buf[off:off + 8] = (2**64 - 84).to_bytes(8, "little")  # offset + length would wrap to 0
    _corrupt(lambda: myl.wire_decode(bytes(buf)))


def test_odd_payload_rejected_after_the_crc():
    # a frame whose payload length is odd but whose CRC matches
    payload = b"\x01\x02\x03"
    import struct
    head = [META.get(f, 0) for f in W.FIELDS]
    head[W.FIELDS.index("payload_len")] = 3
    buf = W.MAGIC + struct.pack("<9Q", *head) + struct.pack("<I", zlib.crc32(payload)) + payload + b"\0" * 5
    _corrupt(lambda: myl.wire_decode(buf))
    with pytest.raises(W.WireError, match="odd"):
        W.decode_message(buf)


def test_flags_survive_the_roundtrip():  # codec.rs:303-312
    m, _ = myl.wire_decode(myl.wire_encode(
        dict(META, flags=myl.WIRE_FLAG_STARTS_GENERATION | myl.WIRE_FLAG_TOKEN_INPUT), []))
    assert m["flags"] & myl.WIRE_FLAG_STARTS_GENERATION
    assert m["flags"] & myl.WIRE_FLAG_TOKEN_INPUT
    assert not m["flags"] & myl.WIRE_FLAG_ABORT


def test_tokens_roundtrip_over_the_u32_range():  # codec.rs:326-332
    tokens = [0, 1, 0x7FFF, 0x8000, 0xFFFF, 0x1_0000, 0x7FFF_FFFF, 2**32 - 1]
    packed = myl.pack_tokens(tokens)
    assert packed.tolist() == W.pack_tokens(tokens)
    assert myl.unpack_tokens(packed).tolist() == tokens


def test_odd_token_payload_rejected():  # codec.rs:334-338
    with pytest.raises(myl.MylError):
        myl.unpack_tokens([1, 2, 3])
    assert myl.unpack_tokens([]).size == 0


def test_capacity_errors():
    buf = myl.wire_encode(META, [1, 2, 3])
    L = myl.load_library()
    import ctypes as C
    m = myl.WireMeta()
    n = C.c_uint64()
    out = np.zeros(2, np.int16)
    b = np.frombuffer(buf, np.uint8)
    rc = L.myl_wire_decode(b.ctypes.data, b.size, C.byref(m), out.ctypes.data, 2, C.byref(n))
    assert rc == myl.MYL_ERR_SHAPE and n.value == 3
