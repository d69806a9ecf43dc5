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


def batch_windows(token_count: int, seq: int, stride: int, batch: int, shuffle: bool, seed: int,
                  drop_last: bool, epoch: int, cursor: int, rank: int = 0, world: int = 1):
    """Host-only (no GPU): this rank's window start offsets of the batch at (epoch, cursor) of
    Spar's LMBatchIterator order, the batch's row count and the cursor after it."""
    import ctypes

    from . import _lib

    lib = _lib.load()
    starts = np.empty(max(batch, 1), np.uint64)
    rows, grows, nxt = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
    _lib.check("spar_b200_batch_windows",
               lib.spar_b200_batch_windows(token_count, seq, stride, batch, int(shuffle), seed,
                                           int(drop_last), epoch, cursor, rank, world,
                                           starts.ctypes.data, ctypes.byref(rows),
                                           ctypes.byref(grows), ctypes.byref(nxt)))
    return starts[:rows.value].copy(), grows.value, nxt.value


def split_documents(document_count: int, validation_count: int, seed: int):
    """Spar's data::split_documents: (train indices, validation indices)."""
    from . import _lib

    order = np.empty(max(document_count, 1), np.uint64)
    _lib.check("spar_b200_split_documents",
               _lib.load().spar_b200_split_documents(document_count, validation_count, seed,
                                                     order.ctypes.data))
    order = order[:document_count].astype(np.int64)
    return order[validation_count:], order[:validation_count]


class BatchIterator:
    """Spar's LMBatchIterator over a packed token corpus held in device memory: each `next`
    gathers this rank's rows of the next batch as int32 ids [rows, seq] on the device."""

    def __init__(self, tokens, seq: int, stride: int, batch: int, shuffle: bool = True,
                 seed: int = 0, drop_last: bool = False, rank: int = 0, world: int = 1,
                 device: int = 0):
        import ctypes

        from . import _lib

        self.lib = _lib.load()
        self.seq, self.device, self._batch = seq, device, batch
        self.handle = None
        toks = np.ascontiguousarray(tokens, np.int32)
        h = ctypes.c_void_p()
        _lib.check("spar_b200_batches_create",
                   self.lib.spar_b200_batches_create(toks.ctypes.data, toks.size, seq, stride,
                                                     batch, int(shuffle), seed, int(drop_last),
                                                     rank, world, device, ctypes.byref(h)))
        self.handle = h

    def next(self, out=None):
        """(ids tensor [rows, seq] on the device, or None at the end of the epoch)."""
        import ctypes

        import torch

        from . import _lib

        rows, grows = ctypes.c_uint64(), ctypes.c_uint64()
        dev = torch.device("cuda", self.device)
        buf = out if out is not None else torch.empty(self._batch, self.seq, dtype=torch.int32,
                                                      device=dev)
        _lib.check("spar_b200_batches_next",
                   self.lib.spar_b200_batches_next(self.handle, buf.data_ptr(), ctypes.byref(rows),
                                                   ctypes.byref(grows),
                                                   torch.cuda.current_stream(dev).cuda_stream))
        if grows.value == 0:
            return None
        return buf[:rows.value]

    def next_epoch(self):
        from . import _lib

        _lib.check("spar_b200_batches_next_epoch", self.lib.spar_b200_batches_next_epoch(self.handle))

    def state(self):
        import ctypes

        from . import _lib

        e, c, w = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        _lib.check("spar_b200_batches_state", self.lib.spar_b200_batches_state(
            self.handle, ctypes.byref(e), ctypes.byref(c), ctypes.byref(w)))
        return e.value, c.value

    def set_state(self, epoch: int, cursor: int):
        from . import _lib

        _lib.check("spar_b200_batches_set_state",
                   self.lib.spar_b200_batches_set_state(self.handle, epoch, cursor))

    def close(self):
        if self.handle:
            self.lib.spar_b200_batches_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
