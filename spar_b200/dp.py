"""Data-parallel host logic of the training runtime.

One process per GPU. Every rank draws the same global batch and takes a contiguous share of its
sequences (`spar_b200.data.rank_share`); the loss gradient of each rank is scaled by
1 / (tokens per rank x micro-steps x world), so summing the ranks' gradients gives the gradient
of the mean loss over the global batch. The runtime sums them with one NCCL all-reduce per
bucket, issued during the last micro-step's backward in the order of `buckets()`: each block's
contiguous parameter range as soon as its backward finishes (last block first), then the tied
embedding and the final norm. With the sharded optimiser (the default at world > 1) each bucket
is reduce-scattered instead: rank r keeps the sum of piece r (`shards`), runs the norm pass and
AdamW on its pieces only (the sums of squares all-reduced), and the next step starts by
all-gathering the updated parameter pieces. This module exposes that plan, queried from the
runtime itself (host-only C-ABI calls, no GPU needed), and packs / unpacks per-tensor gradients
along it.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from .lm import LMConfig, native_config


@dataclass(frozen=True)
class TensorSlot:
    name: str
    offset: int  # floats into the parameter arena
    rows: int
    cols: int    # 0 for vectors
    ld: int      # row stride in the arena (3d for the fused q / k / v projections)

    @property
    def shape(self):
        return (self.rows,) if self.cols == 0 else (self.rows, self.cols)

    @property
    def extent(self):
        """[first, last + 1) arena indices the tensor touches."""
        if self.cols == 0:
            return self.offset, self.offset + self.rows
        return self.offset, self.offset + (self.rows - 1) * self.ld + self.cols


def layout(cfg: LMConfig):
    """(flat size, tensors in arena order, all-reduce buckets (offset, count) in issue order)."""
    lib = _lib.load()
    c = native_config(cfg)
    flat, nt, nb = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
    _lib.check("spar_b200_lm_layout", lib.spar_b200_lm_layout(ctypes.byref(c), ctypes.byref(flat),
                                                              ctypes.byref(nt), ctypes.byref(nb)))
    tensors = []
    buf = ctypes.create_string_buffer(256)
    vals = [ctypes.c_uint64() for _ in range(4)]
    for i in range(nt.value):
        _lib.check("spar_b200_lm_layout_tensor",
                   lib.spar_b200_lm_layout_tensor(ctypes.byref(c), i, buf, len(buf),
                                                  *[ctypes.byref(v) for v in vals]))
        tensors.append(TensorSlot(buf.value.decode(), *[v.value for v in vals]))
    buckets = []
    off, cnt = ctypes.c_uint64(), ctypes.c_uint64()
    for i in range(nb.value):
        _lib.check("spar_b200_lm_layout_bucket",
                   lib.spar_b200_lm_layout_bucket(ctypes.byref(c), i, ctypes.byref(off),
                                                  ctypes.byref(cnt)))
        buckets.append((off.value, cnt.value))
    return flat.value, tensors, buckets


@dataclass(frozen=True)
class BucketShard:
    """One rank's part of a bucket under the sharded optimiser: the reduce-scattered piece
    [own_offset, own_offset + shard) it updates, and the uneven tail [tail_offset, + tail_count)
    that is all-reduced and updated on every rank."""
    own_offset: int
    shard: int
    tail_offset: int
    tail_count: int


def shards(cfg: LMConfig, world: int, rank: int) -> list[BucketShard]:
    """The runtime's piece of every bucket (issue order) for `rank` of `world` (host-only query)."""
    lib = _lib.load()
    c = native_config(cfg)
    _, _, buckets = layout(cfg)
    vals = [ctypes.c_uint64() for _ in range(4)]
    out = []
    for i in range(len(buckets)):
        _lib.check("spar_b200_lm_layout_shard",
                   lib.spar_b200_lm_layout_shard(ctypes.byref(c), i, world, rank,
                                                 *[ctypes.byref(v) for v in vals]))
        out.append(BucketShard(*[v.value for v in vals]))
    return out


def to_arena(grads: dict, flat: int, tensors, dtype=np.float64) -> np.ndarray:
    """Places per-tensor arrays at their arena slots (padding stays zero)."""
    arena = np.zeros(flat, dtype)
    for t in tensors:
        g = np.asarray(grads[t.name], dtype)
        if t.cols == 0:
            arena[t.offset:t.offset + t.rows] = g
        else:
            view = np.lib.stride_tricks.as_strided(arena[t.offset:], shape=(t.rows, t.cols),
                                                   strides=(t.ld * arena.itemsize, arena.itemsize))
            view[...] = g
    return arena


def from_arena(arena: np.ndarray, tensors) -> dict:
    out = {}
    for t in tensors:
        if t.cols == 0:
            out[t.name] = arena[t.offset:t.offset + t.rows].copy()
        else:
            out[t.name] = np.lib.stride_tricks.as_strided(
                arena[t.offset:], shape=(t.rows, t.cols),
                strides=(t.ld * arena.itemsize, arena.itemsize)).copy()
    return out


def allreduce_sum(arena: np.ndarray, buckets, reduce_fn) -> np.ndarray:
    """Sums the arena across ranks bucket by bucket in the runtime's issue order;
    reduce_fn(view) reduces a contiguous slice in place (e.g. torch.distributed.all_reduce on a
    tensor sharing its memory)."""
    for off, cnt in buckets:
        reduce_fn(arena[off:off + cnt])
    return arena


class RankLost(RuntimeError):
    """A data-parallel peer did not reach the next step (it exited or stopped between steps)."""

    def __init__(self, step: int, missing: list[int], left: list[int]):
        self.step, self.missing, self.left = step, missing, left
        super().__init__(f"step {step}: ranks {missing} did not arrive"
                         + (f" (ranks {left} left)" if left else ""))


class Heartbeat:
    """Host-side liveness check between optimiser steps, through the process group's key-value
    store (no collective, no GPU work). Before launching step s every rank records that it reached
    s and waits, with a deadline, until every rank has; a rank that exited or stopped between
    steps is named in RankLost before any collective of step s is launched, so no rank blocks in
    a collective whose peer is gone. A rank leaving on purpose calls leave(), which lets the
    others fail at once instead of at the deadline. (Inside a step, a peer that dies is caught by
    the runtime's bounded wait: spar_b200_comm_wait, code 3.)"""

    def __init__(self, store, rank: int, world: int, timeout: float = 60.0, poll: float = 0.01,
                 prefix: str = "spar_b200/heartbeat"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout, self.poll, self.prefix = timeout, poll, prefix

    def leave(self) -> None:
        self.store.set(f"{self.prefix}/left/{self.rank}", "1")

    def arrive(self, step: int) -> None:
        """Records this rank at `step`, then waits for all ranks (RankLost at the deadline, or
        as soon as a missing rank has left)."""
        import time

        self.store.set(f"{self.prefix}/{step}/{self.rank}", "1")
        deadline = time.monotonic() + self.timeout
        while True:
            missing = [r for r in range(self.world)
                       if not self.store.check([f"{self.prefix}/{step}/{r}"])]
            if not missing:
                return
            left = [r for r in missing if self.store.check([f"{self.prefix}/left/{r}"])]
            if left or time.monotonic() > deadline:
                raise RankLost(step, missing, left)
            time.sleep(self.poll)
