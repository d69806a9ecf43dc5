"""Input pipeline: the window order and batches of Spar's LMBatchIterator (src/data/
batch_iterator.cpp) over its WindowDataset, against the reference itself (oracle/_ref) on a
byte-level corpus, and the device gather on a GPU. Bitwise (integer data)."""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
import cpu_ref  # noqa: E402

DOCS = [bytes(np.random.default_rng(i).integers(0, 256, n, dtype=np.uint8))
        for i, n in enumerate([57, 0, 130, 3, 77, 1, 240])]


def _ours(tokens, seq, stride, batch, shuffle, seed, drop_last, epochs, world=1):
    """Our batches (host-only window order + host gather), rank shares concatenated."""
    from spar_b200.data import batch_windows

    out = []
    for e in range(epochs):
        cursor = 0
        while True:
            parts = []
            for r in range(world):
                starts, grows, nxt = batch_windows(len(tokens), seq, stride, batch, shuffle, seed,
                                                   drop_last, e, cursor, r, world)
                parts.append(np.stack([tokens[s:s + seq] for s in starts.astype(np.int64)])
                             if len(starts) else np.empty((0, seq), np.int32))
            if grows == 0:
                break
            out.append(np.concatenate(parts))
            cursor = nxt
    return out


@pytest.mark.skipif(not cpu_ref.available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("seq,stride,batch,shuffle,seed,drop_last", [
    (16, 16, 4, True, 7, False), (16, 5, 3, True, 123456789, True), (9, 1, 64, False, 0, False),
    (32, 32, 1, True, 2, False), (600, 600, 2, True, 1, False),  # corpus shorter than a window
])
def test_batches_match_reference_iterator(seq, stride, batch, shuffle, seed, drop_last):
    tokens, ref = cpu_ref.batches(DOCS, seq, stride, batch, shuffle, seed, drop_last, 3)
    got = _ours(tokens, seq, stride, batch, shuffle, seed, drop_last, 3)
    assert len(got) == len(ref)
    for a, b in zip(got, ref):
        assert np.array_equal(a, b)


@pytest.mark.skipif(not cpu_ref.available(), reason="oracle/_ref not built here")
def test_rank_shares_partition_each_batch():
    tokens, ref = cpu_ref.batches(DOCS, 8, 3, 10, True, 5, False, 2)
    for world in (2, 3, 4):
        got = _ours(tokens, 8, 3, 10, True, 5, False, 2, world)
        assert len(got) == len(ref) and all(np.array_equal(a, b) for a, b in zip(got, ref))


@pytest.mark.skipif(not cpu_ref.available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("count,validation,seed", [(10, 3, 1), (1, 0, 5), (0, 0, 9),
                                                   (1000, 100, 0x5EED), (7, 7, 2)])
def test_split_documents_matches_reference(count, validation, seed):
    from spar_b200.data import split_documents

    got = split_documents(count, validation, seed)
    ref = cpu_ref.split_documents(count, validation, seed)
    assert all(np.array_equal(a, b) for a, b in zip(got, ref))


@pytest.mark.gpu
def test_device_batches_match_host_order(cuda):
    """The device iterator (resident corpus, window gather kernel) gives the host-order batches,
    across epochs and after a state restore; rank shares tile the batch."""
    import torch

    from spar_b200.data import BatchIterator, batch_windows

    rng = np.random.default_rng(3)
    tokens = rng.integers(0, 32768, 200_000, dtype=np.int32)
    seq, stride, batch = 1024, 512, 16
    it = BatchIterator(tokens, seq, stride, batch, shuffle=True, seed=11)
    for epoch in range(2):
        cursor = 0
        while True:
            ids = it.next()
            starts, grows, nxt = batch_windows(len(tokens), seq, stride, batch, True, 11, False,
                                               epoch, cursor)
            if ids is None:
                assert grows == 0
                break
            torch.cuda.synchronize()
            want = np.stack([tokens[s:s + seq] for s in starts.astype(np.int64)])
            assert np.array_equal(ids.cpu().numpy(), want)
            cursor = nxt
        it.next_epoch()
    it.set_state(1, 48)
    ids = it.next()
    torch.cuda.synchronize()
    starts, _, _ = batch_windows(len(tokens), seq, stride, batch, True, 11, False, 1, 48)
    assert np.array_equal(ids.cpu().numpy(), np.stack([tokens[s:s + seq] for s in starts.astype(np.int64)]))
    it.close()
    parts = []
    for r in range(4):
        itr = BatchIterator(tokens, seq, stride, batch, shuffle=True, seed=11, rank=r, world=4)
        parts.append(itr.next().cpu().numpy())
        itr.close()
    first = BatchIterator(tokens, seq, stride, batch, shuffle=True, seed=11)
    assert np.array_equal(np.concatenate(parts), first.next().cpu().numpy())
    first.close()
