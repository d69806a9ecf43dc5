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
