"""Synthetic token batches drawn from Spar's random stream.

Spar's Random is SplitMix64 (src/core/random.cpp:22-28) and its batch iterator samples indices
with bounded_index (src/data/batch_iterator.cpp:22-32: reject draws below (2^64 - bound) % bound,
then take value % bound). This module draws token ids the same way, vectorised, to feed the
training step with reproducible synthetic data of a workload's shape.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def _mix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def draws(seed: int, start: int, count: int) -> np.ndarray:
    """Draws start .. start+count-1 of a Random seeded with `seed`."""
    idx = np.arange(start + 1, start + count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix(np.uint64(seed & ((1 << 64) - 1)) + idx * _GOLDEN)


def token_ids(seed: int, count: int, vocab: int) -> np.ndarray:
    """`count` ids in [0, vocab) by bounded_index rejection sampling on one stream."""
    threshold = np.uint64(((1 << 64) - vocab) % vocab)
    out = np.empty(count, dtype=np.int64)
    filled, pos = 0, 0
    while filled < count:
        need = count - filled
        v = draws(seed, pos, need + need // 8 + 16)
        pos += len(v)
        keep = v[v >= threshold] if threshold else v
        take = min(need, len(keep))
        out[filled:filled + take] = (keep[:take] % np.uint64(vocab)).astype(np.int64)
        filled += take
        if take < len(keep):  # rewind the stream to just after the last accepted draw
            accepted = np.nonzero(v >= threshold)[0] if threshold else np.arange(len(v))
            pos = pos - len(v) + int(accepted[take - 1]) + 1
    return out


def rank_share(seed: int, global_seqs: int, accum: int, seq: int, vocab: int, rank: int,
               world: int) -> np.ndarray:
    """Data-parallel share of one optimiser step's global batch: `global_seqs` sequences of `seq`
    ids drawn from one stream, rank r taking the contiguous sequences [r*per, (r+1)*per) with
    per = global_seqs / world, as int32 [accum, per / accum, seq] micro-steps. Every rank draws
    the same global batch, so the shares partition it without any communication."""
    if global_seqs % world or (global_seqs // world) % accum:
        raise ValueError("global batch must split evenly over ranks and micro-steps")
    ids = token_ids(seed, global_seqs * seq, vocab).reshape(global_seqs, seq)
    per = global_seqs // world
    mine = ids[rank * per:(rank + 1) * per]
    return np.ascontiguousarray(mine.reshape(accum, per // accum, seq).astype(np.int32))
