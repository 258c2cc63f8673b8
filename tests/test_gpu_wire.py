"""The wire format's device path: CRC-32 computed on the GPU (zlib is the
reference implementation of the same published CRC), frames decoded straight
into device memory and encoded from it, against the host codec and the CPU
restatement of codec.rs."""
import zlib

import numpy as np
import pytest

from oracle import wire as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import myelith_b200 as myl  # noqa: E402

META = dict(version=1, theta_v_hash=0x1234_5678_9ABC, request_id=42, sequence_id=1, stage_id=3,
            token_position=2048, flags=myl.WIRE_FLAG_STARTS_GENERATION, reserved=0)


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = myl.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("n", [0, 1, 15, 16, 17, 255, 256, 65535, 65536, 65537, 1_000_003,
                               2048 * 3584 * 2])
def test_crc32_dev_matches_zlib(ctx, n):
    rng = np.random.default_rng(n)
    data = rng.integers(0, 256, size=n + 3, dtype=np.uint8)
    d = torch.from_numpy(data).cuda()
    for off in (0, 1, 3):  # aligned and unaligned starts
        if off + n > data.size:
            continue
        assert ctx.crc32_dev(d[off:off + n]) == zlib.crc32(data[off:off + n].tobytes()), (n, off)


def test_decode_dev_prefill_hidden(ctx):
    """A prefill hidden state (2048 tokens x 3584) decoded into HBM."""
    rng = np.random.default_rng(5)
    h = rng.integers(-32768, 32768, size=(2048, 3584)).astype(np.int16)
    frame = myl.wire_encode(META, h)
    assert frame[80:84] == zlib.crc32(h.tobytes()).to_bytes(4, "little")
    dev = torch.empty(h.size, dtype=torch.int16, device="cuda")
    meta, n = ctx.wire_decode_dev(frame, dev)
    torch.cuda.synchronize()
    assert n == h.size
    assert np.array_equal(dev.cpu().numpy().reshape(h.shape), h)
    assert meta["token_position"] == 2048 and meta["payload_len"] == 2 * h.size
    # the encoder from device memory gives the host encoder's bytes
    assert ctx.wire_encode_dev(META, dev) == frame


def test_decode_dev_rejects_like_decode_message(ctx):
    t = np.arange(-300, 300, dtype=np.int16)
    frame = bytearray(myl.wire_encode(META, t))
    dev = torch.empty(t.size, dtype=torch.int16, device="cuda")
    rng = np.random.default_rng(2)
    for byte in rng.choice(np.arange(W.HEADER_SIZE, W.HEADER_SIZE + 2 * t.size), size=24, replace=False):
        b = bytearray(frame)
        b[byte] ^= 1 << int(rng.integers(0, 8))
        with pytest.raises(myl.MylError) as e:
            ctx.wire_decode_dev(bytes(b), dev)
        assert e.value.code == myl.MYL_ERR_CORRUPT
        with pytest.raises(W.WireError):
            W.decode_message(bytes(b))
    bad = bytearray(frame)
    bad[:8] = b"IINTPIPX"
    with pytest.raises(myl.MylError):
        ctx.wire_decode_dev(bytes(bad), dev)
    with pytest.raises(myl.MylError):  # too small a device buffer
        ctx.wire_decode_dev(bytes(frame), dev[:10])
    meta, n = ctx.wire_decode_dev(bytes(frame), dev)  # still decodes after the errors
    assert n == t.size and np.array_equal(dev.cpu().numpy(), t)
