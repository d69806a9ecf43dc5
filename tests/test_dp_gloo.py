"""Data-parallel host logic on CPU: the batch sharding, the gradient all-reduce bucket plan the
runtime issues (queried from the C ABI without a GPU) and, across two gloo ranks, that summing the
rank-scaled share gradients bucket by bucket gives the full-batch gradient.

The gradients come from the float64 oracle, so the bar is float64 rounding (rel-L2 <= 1e-12).
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

from oracle import spar_oracle as O

TINY = dict(vocab=64, dim=64, hidden=128, layers=2, heads=2, seq=16)
GLOBAL_SEQS, ACCUM, SEED_W, SEED_IDS = 8, 2, 0x5EED0201, 0x5EED1201


def _cfg(world):
    from spar_b200.lm import LMConfig

    return LMConfig(micro_batch=GLOBAL_SEQS // world // ACCUM, **TINY)


def _share_grads(params, ids, cfg):
    """Mean over the share's micro-steps of the oracle gradient of each micro-step's mean loss."""
    total = None
    for micro in ids:
        _, g = O.lm_forward_backward(params, micro, cfg.oracle_dict())
        total = g if total is None else {k: total[k] + g[k] for k in g}
    return {k: v / len(ids) for k, v in total.items()}


def test_rank_shares_partition_the_global_batch():
    from spar_b200.data import rank_share

    full = rank_share(SEED_IDS, GLOBAL_SEQS, ACCUM, 16, 64, 0, 1).reshape(GLOBAL_SEQS, 16)
    for world in (2, 4):
        parts = [rank_share(SEED_IDS, GLOBAL_SEQS, ACCUM, 16, 64, r, world).reshape(-1, 16)
                 for r in range(world)]
        assert np.array_equal(np.concatenate(parts), full)
    with pytest.raises(ValueError):
        rank_share(SEED_IDS, GLOBAL_SEQS, ACCUM, 16, 64, 0, 3)


@pytest.mark.parametrize("which", ["tiny", "c5"])
def test_bucket_plan_tiles_the_arena(which):
    from spar_b200 import dp
    from spar_b200.lm import C5

    cfg = _cfg(1) if which == "tiny" else C5
    flat, tensors, buckets = dp.layout(cfg)
    assert len(buckets) == cfg.layers + 2
    spans = sorted(buckets)
    assert spans[0][0] == 0 and sum(c for _, c in spans) == flat
    for (o0, c0), (o1, _) in zip(spans, spans[1:]):
        assert o0 + c0 == o1  # contiguous, no overlap
    # Issue order: last block first, ..., block 0, then the tied embedding and the final norm.
    def holder(t):
        lo, hi = t.extent
        owners = [i for i, (o, c) in enumerate(buckets) if o <= lo and hi <= o + c]
        assert len(owners) == 1, t.name
        return owners[0]
    for t in tensors:
        i = holder(t)
        if t.name.startswith("blocks."):
            assert i == cfg.layers - 1 - int(t.name.split(".")[1]), t.name
        elif t.name == "token_embedding.weight":
            assert i == cfg.layers
        else:
            assert t.name.startswith("final_norm.") and i == cfg.layers + 1
    assert [t.name for t in tensors] == O.parameter_names(cfg.layers)


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    from spar_b200 import dp
    from spar_b200.data import rank_share

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    cfg = _cfg(world)
    params = O.init_parameters(cfg.oracle_dict(), SEED_W)
    ids = rank_share(SEED_IDS, GLOBAL_SEQS, ACCUM, cfg.seq, cfg.vocab, rank, world)
    grads = _share_grads(params, ids, cfg)
    flat, tensors, buckets = dp.layout(cfg)
    # The runtime folds 1 / world into the loss-gradient scale, then sums over ranks.
    arena = dp.to_arena({k: v / world for k, v in grads.items()}, flat, tensors)
    dp.allreduce_sum(arena, buckets, lambda view: dist.all_reduce(torch.from_numpy(view)))
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), arena)
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_sum_to_full_batch_gradient():
    import torch.multiprocessing as mp

    from spar_b200 import dp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_worker, args=(2, port, out), nprocs=2, join=True,
                           start_method="spawn")
        arenas = [np.load(os.path.join(out, f"rank{r}.npy")) for r in range(2)]
    assert np.array_equal(arenas[0], arenas[1])  # every rank holds the same summed gradient
    cfg1 = _cfg(1)
    params = O.init_parameters(cfg1.oracle_dict(), SEED_W)
    from spar_b200.data import rank_share

    full = _share_grads(params, rank_share(SEED_IDS, GLOBAL_SEQS, ACCUM, cfg1.seq, cfg1.vocab,
                                           0, 1), cfg1)
    flat, tensors, _ = dp.layout(_cfg(2))
    got = dp.from_arena(arenas[0], tensors)
    for name, ref in full.items():
        err = np.linalg.norm(got[name] - ref) / max(np.linalg.norm(ref), 1e-300)
        assert err <= 1e-12, (name, err)


@pytest.mark.parametrize("world", [1, 2, 3, 5, 8])
def test_shard_plan_tiles_every_bucket(world):
    """Sharded optimiser: the ranks' pieces of each bucket (equal, 64-float multiples, in rank
    order) and the all-reduced tail tile the bucket exactly."""
    from spar_b200 import dp
    from spar_b200.lm import C5

    for cfg in (_cfg(1), C5):
        _, _, buckets = dp.layout(cfg)
        plans = [dp.shards(cfg, world, r) for r in range(world)]
        for i, (off, cnt) in enumerate(buckets):
            pieces = [p[i] for p in plans]
            shard = pieces[0].shard
            assert shard % 64 == 0 and all(p.shard == shard for p in pieces)
            assert [p.own_offset for p in pieces] == [off + r * shard for r in range(world)]
            assert all(p.tail_offset == off + world * shard for p in pieces)
            assert pieces[0].tail_offset + pieces[0].tail_count == off + cnt
            assert pieces[0].tail_count < world * 64  # only what does not split evenly
    # C5's buckets split evenly over 2, 4 and 8 ranks: nothing is all-reduced there.
    if world in (2, 8):
        assert all(p.tail_count == 0 for p in dp.shards(C5, world, 0))


OPT = dict(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)


def _sharded_worker(rank, world, port, out_dir, max_norm):
    """One rank of the sharded optimiser step, restated on the host: reduce (all-reduce, then
    keep this rank's pieces: the reduce-scatter result), norm of the own pieces (+ the tails on
    rank 0) all-reduced, AdamW on the own pieces and the tails, all-gather of the parameters."""
    import torch
    import torch.distributed as dist

    from spar_b200 import dp

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    cfg = _cfg(1)
    flat, _, buckets = dp.layout(cfg)
    rng = np.random.default_rng(7)
    p = rng.normal(0, 0.02, flat).astype(np.float32)
    m = rng.normal(0, 1e-3, flat).astype(np.float32)
    v = np.abs(rng.normal(0, 1e-6, flat)).astype(np.float32)
    g = np.random.default_rng(100 + rank).normal(0, 1e-2, flat).astype(np.float32)
    t = torch.from_numpy(g)
    dist.all_reduce(t)
    g = t.numpy()
    plan = dp.shards(cfg, world, rank)
    own = [(b.own_offset, b.shard) for b in plan if b.shard]
    tails = [(b.tail_offset, b.tail_count) for b in plan if b.tail_count]
    counted = own + (tails if rank == 0 else [])
    ssq = torch.tensor([sum(float(np.dot(g[o:o + c].astype(np.float64), g[o:o + c].astype(np.float64)))
                            for o, c in counted)], dtype=torch.float64)
    dist.all_reduce(ssq)
    clip = O.clip_factor(float(np.sqrt(ssq.item())), max_norm)
    for o, c in own + tails:
        p[o:o + c], m[o:o + c], v[o:o + c] = O.adamw_update(p[o:o + c], g[o:o + c], m[o:o + c],
                                                            v[o:o + c], 3, clip=clip, **OPT)
    for b in plan:
        if b.shard:
            piece = torch.from_numpy(p[b.own_offset:b.own_offset + b.shard].copy())
            parts = [torch.empty_like(piece) for _ in range(world)]
            dist.all_gather(parts, piece)
            start = b.own_offset - rank * b.shard
            p[start:start + world * b.shard] = torch.cat(parts).numpy()
    np.save(os.path.join(out_dir, f"p{rank}.npy"), p)
    np.save(os.path.join(out_dir, f"g{rank}.npy"), g)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,max_norm", [(2, 1e30), (3, 1e30), (3, 1e-3)])
def test_gloo_sharded_optimizer_matches_replicated(world, max_norm):
    """The sharded optimiser step over `world` gloo ranks (3: uneven tails) gives every rank the
    parameters of the replicated step: bitwise without clipping, and to 1e-6 with clipping active
    (the norm's double sum runs in another order)."""
    import torch.multiprocessing as mp

    from spar_b200 import dp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_sharded_worker, args=(world, port, out, max_norm), nprocs=world,
                           join=True, start_method="spawn")
        ps = [np.load(os.path.join(out, f"p{r}.npy")) for r in range(world)]
        g = np.load(os.path.join(out, "g0.npy"))
    for r in range(1, world):
        assert np.array_equal(ps[0], ps[r])
    flat, _, _ = dp.layout(_cfg(1))
    rng = np.random.default_rng(7)
    p = rng.normal(0, 0.02, flat).astype(np.float32)
    m = rng.normal(0, 1e-3, flat).astype(np.float32)
    v = np.abs(rng.normal(0, 1e-6, flat)).astype(np.float32)
    clip = O.clip_factor(O.global_grad_norm([g]), max_norm)
    want, _, _ = O.adamw_update(p, g, m, v, 3, clip=clip, **OPT)
    if clip == 1.0:
        assert np.array_equal(ps[0], want)
    else:
        np.testing.assert_allclose(ps[0], want, rtol=1e-6, atol=1e-9)
