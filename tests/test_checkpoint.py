"""SPARCKPT v1 training checkpoints (Spar's src/checkpoint/checkpoint.cpp format) written and read
by this library's host-side code, against the reference's own save_training_checkpoint /
load_training_checkpoint (oracle/_ref): a checkpoint from either side loads bitwise in the other.
CPU only (the format code needs no GPU); skipped where the reference library is not built.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
import cpu_ref  # noqa: E402

from oracle import spar_oracle as O  # noqa: E402

CFG = dict(vocab=64, dim=128, hidden=256, layers=2, heads=4, kv_heads=2, qk_norm=1)
OPT = {"beta1": 0.9, "beta2": 0.95, "eps": 1e-8, "weight_decay": 0.1}

pytestmark = pytest.mark.skipif(not cpu_ref.available(), reason="oracle/_ref not built here")


def _cfg(**kw):
    from spar_b200.lm import LMConfig

    c = dict(CFG, **kw)
    return LMConfig(vocab=c["vocab"], dim=c["dim"], hidden=c["hidden"], layers=c["layers"],
                    heads=c["heads"], seq=32, micro_batch=2, family=1, kv_heads=c["kv_heads"],
                    qk_norm=bool(c["qk_norm"]), beta1=OPT["beta1"], beta2=OPT["beta2"],
                    adam_eps=OPT["eps"], weight_decay=OPT["weight_decay"])


def _state(seed):
    params = O.spar_family_parameters(CFG, seed)
    names = list(params)
    r = np.random.default_rng(seed)
    vals = [np.ascontiguousarray(params[n], np.float32).ravel() for n in names]
    m = [(1e-3 * r.standard_normal(a.size)).astype(np.float32) for a in vals]
    v = [np.abs(1e-6 * r.standard_normal(a.size)).astype(np.float32) for a in vals]
    return names, vals, m, v


def test_checkpoint_written_here_loads_in_the_reference(tmp_path):
    from spar_b200.lm import write_checkpoint

    names, vals, m, v = _state(11)
    path = tmp_path / "ours.sparckpt"
    write_checkpoint(path, _cfg(), vals, m, v, global_step=7, tokens_seen=7 * 4096,
                     rng_state=0x1234567890ABCDEF, learning_rate=2.5e-4, adam_step=7)
    ps, ms, vs, step, gstep, tokens, rng, lr = cpu_ref.spar_ckpt_load(path, CFG)
    assert (step, gstep, tokens, rng, lr) == (7, 7, 7 * 4096, 0x1234567890ABCDEF, 2.5e-4)
    for a, b in zip(vals + m + v, ps + ms + vs):
        assert np.array_equal(a, b)


def test_reference_checkpoint_reads_here(tmp_path):
    from spar_b200.lm import read_checkpoint

    names, vals, m, v = _state(12)
    path = tmp_path / "ref.sparckpt"
    cpu_ref.spar_ckpt_save(path, CFG, vals, m, v, 3, 30, 3000, 42, 1e-4, OPT)
    rv, rm, rvv, meta = read_checkpoint(path, _cfg(), [a.size for a in vals])
    assert meta == {"global_step": 30, "tokens_seen": 3000, "rng_state": 42,
                    "learning_rate": 1e-4, "adam_step": 3}
    for a, b in zip(vals + m + v, rv + rm + rvv):
        assert np.array_equal(a, b)


def test_checkpoint_without_optimizer_state_and_rejections(tmp_path):
    from spar_b200._lib import SparError
    from spar_b200.lm import read_checkpoint, write_checkpoint

    names, vals, m, v = _state(13)
    sizes = [a.size for a in vals]
    path = tmp_path / "fresh.sparckpt"
    cpu_ref.spar_ckpt_save(path, CFG, vals, m, v, 0, 0, 0, 5, 3e-4, OPT)  # no AdamW state
    rv, rm, _, meta = read_checkpoint(path, _cfg(), sizes)
    assert meta["adam_step"] == 0 and all(not a.any() for a in rm)
    assert all(np.array_equal(a, b) for a, b in zip(vals, rv))
    # another model shape, other AdamW settings, a truncated file: refused
    with pytest.raises(SparError):
        read_checkpoint(path, _cfg(hidden=512), sizes)
    with pytest.raises(SparError):
        read_checkpoint(path, _cfg(qk_norm=0), sizes)
    bad = tmp_path / "short.sparckpt"
    bad.write_bytes(path.read_bytes()[:-100])
    with pytest.raises(SparError):
        read_checkpoint(bad, _cfg(), sizes)
    ours = tmp_path / "ours.sparckpt"
    write_checkpoint(ours, _cfg(), vals, None, None, rng_state=5, learning_rate=3e-4)
    assert ours.read_bytes() == path.read_bytes()  # byte-identical to the reference's file


@pytest.mark.parametrize("kv_heads,qk_norm", [(4, 0), (2, 1), (1, 1)])
def test_spar_family_layout_matches_reference_parameters(kv_heads, qk_norm):
    """The runtime's named tensors for Spar-family configs (host-only layout query) are the
    reference nn::DecoderLM's named_parameters: same names, order and element counts."""
    from spar_b200 import dp

    cfg = _cfg(kv_heads=kv_heads, qk_norm=qk_norm)
    _, tensors, buckets = dp.layout(cfg)
    ref = cpu_ref.spar_param_info(dict(CFG, kv_heads=kv_heads, qk_norm=qk_norm))
    assert [t.name for t in tensors] == [n for n, _ in ref]
    assert [t.rows * (t.cols or 1) for t in tensors] == [k for _, k in ref]
    assert len(buckets) == cfg.layers + 2
    spans = sorted(buckets)
    for (o0, c0), (o1, _) in zip(spans, spans[1:]):
        assert o0 + c0 == o1
    for world in (2, 4):  # the sharded optimiser's pieces tile every bucket of this family too
        plans = [dp.shards(cfg, world, r) for r in range(world)]
        for i, (off, cnt) in enumerate(buckets):
            p0 = plans[0][i]
            assert p0.tail_offset + p0.tail_count == off + cnt
            assert [p[i].own_offset for p in plans] == [off + r * p0.shard for r in range(world)]
