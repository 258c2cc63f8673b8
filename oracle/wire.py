"""CPU restatement of the pipeline wire format (TEST INFRASTRUCTURE ONLY).

Follows INTEGER_LLM/pipeline/src/codec.rs: encode_message (:86-111),
decode_message (:113-178), pack_tokens / unpack_tokens (:38-63). The CRC is
the published CRC-32 that the reference takes from the crc32fast crate
(1.3, pipeline/Cargo.toml:24): reflected polynomial 0xEDB88320, initial value
and final XOR 0xFFFFFFFF; Python's zlib.crc32 computes the same function and
is used here as that algorithm's implementation. Only tests import this
module, as the checker of the library's codec.
"""
from __future__ import annotations

import struct
import zlib

MAGIC = b"IINTPIPE"
HEADER_SIZE = 8 + 8 * 9 + 4  # codec.rs:13
FIELDS = ("version", "theta_v_hash", "request_id", "sequence_id", "stage_id", "token_position",
          "payload_len", "flags", "reserved")


class WireError(ValueError):
    """decode_message's Err (codec.rs:113-178)."""


def encode_message(meta: dict, tensor) -> bytes:
    """codec.rs:86-111: payload_len is the payload's length, not meta's."""
    payload = b"".join(struct.pack("<h", int(v)) for v in tensor)
    crc = zlib.crc32(payload) & 0xFFFFFFFF
    head = [int(meta.get(f, 0)) for f in FIELDS]
    head[FIELDS.index("payload_len")] = len(payload)
    buf = MAGIC + struct.pack("<9Q", *head) + struct.pack("<I", crc) + payload
    return buf + b"\0" * ((8 - len(buf) % 8) % 8)


def decode_message(buf: bytes) -> tuple[dict, list[int]]:
    """codec.rs:113-178, same checks in the same order."""
    if len(buf) < HEADER_SIZE:
        raise WireError(f"buffer too small: {len(buf)} < {HEADER_SIZE}")
    if buf[:8] != MAGIC:
        raise WireError("bad magic")
    vals = struct.unpack("<9Q", buf[8:80])
    meta = dict(zip(FIELDS, vals))
    meta["crc"] = struct.unpack("<I", buf[80:84])[0]
    end = HEADER_SIZE + meta["payload_len"]  # Python ints do not wrap: the checked_add
    if end > len(buf):
        raise WireError(f"payload runs past the buffer: {end} > {len(buf)}")
    payload = buf[HEADER_SIZE:end]
    if zlib.crc32(payload) & 0xFFFFFFFF != meta["crc"]:
        raise WireError("CRC mismatch")
    if len(payload) % 2:
        raise WireError("odd payload length")
    return meta, [v[0] for v in struct.iter_unpack("<h", payload)]


def pack_tokens(tokens) -> list[int]:
    """codec.rs:38-47: low then high 16 bits of each u32 id, as i16."""
    out = []
    for t in tokens:
        lo, hi = t & 0xFFFF, (t >> 16) & 0xFFFF
        out += [lo - 65536 if lo >= 32768 else lo, hi - 65536 if hi >= 32768 else hi]
    return out


def unpack_tokens(payload) -> list[int]:
    """codec.rs:49-63."""
    if len(payload) % 2:
        raise WireError("token payload needs an even number of int16")
    return [(payload[i] & 0xFFFF) | ((payload[i + 1] & 0xFFFF) << 16)
            for i in range(0, len(payload), 2)]
