"""Greedy selection keys on the GPU (myl_argmax_keys_dev) against argmax_int
of the CPU oracle (sampling.rs:8-18: the lowest index among the maxima),
including ties inside a block, across blocks and across rows, empty vocab
shards and a vocab offset."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import myelith_b200 as myl  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = myl.Context(0)
    yield c
    c.close()


def _keys(ctx, logits, base=0):
    d = torch.from_numpy(logits).cuda()
    k = torch.empty((logits.shape[0],), dtype=torch.int64, device="cuda")
    ctx.argmax_keys_dev(d, k, base)
    torch.cuda.synchronize()
    return k.cpu().numpy()


@pytest.mark.parametrize("M,V", [(1, 1), (3, 4095), (2, 4096), (5, 4097), (4, 19008), (1, 152064)])
def test_keys_match_argmax_int(ctx, M, V):
    rng = np.random.default_rng(M * 1000 + V)
    logits = rng.integers(-2**31, 2**31 - 1, size=(M, V), dtype=np.int64).astype(np.int32)
    if V > 8:  # plant ties: the same maximum at several positions, across blocks
        for m in range(M):
            pos = rng.choice(V, size=min(V, 5), replace=False)
            logits[m, pos] = 2**31 - 1
    logits[0, :] = logits[0, :] // 1024  # small range: many ties of the row maximum
    base = 7 if V < 2**20 else 0
    k = _keys(ctx, logits, base)
    tok, best = myl.keys_to_tokens(k)
    for m in range(M):
        assert tok[m] == base + O.argmax_int(logits[m]), m
        assert best[m] == logits[m].max(), m
        assert k[m] == myl.selection_key(int(logits[m].max()), base + O.argmax_int(logits[m]))


def test_keys_many_rows_and_negative(ctx):
    M, V = 70000, 9  # more rows than one grid dimension holds
    rng = np.random.default_rng(1)
    logits = rng.integers(-5, 0, size=(M, V), dtype=np.int32)
    k = _keys(ctx, logits)
    tok, best = myl.keys_to_tokens(k)
    ref_tok = np.argmax(logits, axis=1)  # numpy argmax also returns the first maximum
    assert np.array_equal(tok, ref_tok)
    assert np.array_equal(best, logits.max(axis=1))


def test_keys_empty_shard_and_rejects(ctx):
    k = torch.empty((3,), dtype=torch.int64, device="cuda")
    ctx.argmax_keys_dev(torch.empty((3, 0), dtype=torch.int32, device="cuda"), k, 5)
    torch.cuda.synchronize()
    assert (k.cpu().numpy() == np.iinfo(np.int64).min).all()
    with pytest.raises(myl.MylError):  # indices beyond 32 bits
        ctx.argmax_keys_dev(torch.zeros((1, 4), dtype=torch.int32, device="cuda"), k, 2**32 - 2)
