"""Worker for tests/test_dp_gpu.py: one process per GPU under torchrun.

Two optimiser steps of the training runtime over a 64-sequence global batch, split across the
ranks (spar_b200.data.rank_share: rank r takes sequences [r*per, (r+1)*per) as micro-steps of 8
sequences), gradients reduced over NCCL by the runtime itself (bucket all-reduce, or
reduce-scatter + per-piece AdamW + parameter all-gather with the sharded optimiser). Afterwards
every arena is gathered (a collective) and rank 0 writes parameters, gradients and both moments
(and step 1's gradients and parameters), plus each step's mean loss over the global batch and
norm, to --out. Run with world
size 1 (no torchrun) it is the single-GPU run of the same global batch: the same 8-sequence
micro-steps (eight of them), so every micro-step computes exactly what the matching micro-step of
a rank computes, and the runs differ only in how the micro-steps' gradients are summed (in one
arena, or per rank and then across ranks) and in the data-parallel optimiser path.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GLOBAL_SEQS, MICRO = 64, 8


def accum(world: int) -> int:
    return GLOBAL_SEQS // world // MICRO


def config(world: int, precision: int, family: int = 0):
    """family 0: the LayerNorm / GELU block; 1: Spar's own block (RMSNorm, SwiGLU, grouped-query
    attention with two key / value heads, qk-norm)."""
    from spar_b200.lm import LMConfig

    extra = dict(family=1, kv_heads=2, qk_norm=True) if family else {}
    return LMConfig(vocab=1000, dim=256, hidden=1024, layers=2, heads=4, seq=128,
                    micro_batch=MICRO, precision=precision, **extra)


def run(out: str, precision: int, steps: int = 2, family: int = 0) -> None:
    import torch

    from spar_b200 import _lib
    from spar_b200.data import rank_share
    from spar_b200.lm import DecoderLM

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    cfg = config(world, precision, family)
    lm = DecoderLM(cfg, local)
    lm.init_normal(0x5EED0009, 0.02)
    lib = _lib.load()
    comm = None
    if world > 1:
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            _lib.check("spar_b200_comm_unique_id", lib.spar_b200_comm_unique_id(uid, 128))
        obj = [bytes(uid.raw)]
        dist.broadcast_object_list(obj, src=0)
        uid = ctypes.create_string_buffer(obj[0], 128)
        comm = ctypes.c_void_p()
        _lib.check("spar_b200_comm_init", lib.spar_b200_comm_init(uid, rank, world, local,
                                                                  ctypes.byref(comm)))
        lm.attach_comm(comm, world)
    losses, norms = [], []
    state = {}
    for step in range(1, steps + 1):
        ids = rank_share(0x5EED1009 + step, GLOBAL_SEQS, accum(world), cfg.seq, cfg.vocab, rank,
                         world)
        loss, norm, flags = lm.train_step(ids, 3e-4, step=step)
        if flags != (0, 0):
            raise RuntimeError(f"rank {rank} step {step}: flags {flags}")
        losses.append(loss)
        norms.append(norm)
        if step == 1:  # step 1's gradients and update, before they shape step 2's inputs
            if comm is not None:
                for which in ("param", "grad"):
                    lm.gather(which)
            state["param1"] = lm.state_dict("param")
            state["grad1"] = lm.state_dict("grad")
    if comm is not None:
        for which in ("param", "grad", "m", "v"):
            lm.gather(which)
    state.update({w: lm.state_dict(w) for w in ("param", "grad", "m", "v")})
    if world > 1:  # each rank reports the mean loss over its own (equal) share
        all_losses = [None] * world
        dist.all_gather_object(all_losses, losses)
        losses = list(np.mean(np.array(all_losses), axis=0))
    if rank == 0:
        np.savez(out, losses=np.array(losses), norms=np.array(norms), world=world,
                 **{f"{w}:{n}": v for w, d in state.items() for n, v in d.items()})
    lm.close()
    if comm is not None:
        lib.spar_b200_comm_destroy(comm, 0)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--precision", type=int, default=0)
    ap.add_argument("--family", type=int, default=0)
    a = ap.parse_args()
    run(a.out, a.precision, family=a.family)
