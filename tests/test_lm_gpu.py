"""One full training step of the decoder (forward, LM cross-entropy, backward, clip, AdamW)
through the C ABI, against the CPU oracle on identical seeded weights and ids.

Tolerances (gradient and parameter relative L2 error after one step): <= 1e-5 in 3xTF32 mode,
<= 2e-3 in TF32 mode; loss relative error at the same bars.
"""
import numpy as np
import pytest

from _util import rel_l2
from oracle import spar_oracle as O

pytestmark = pytest.mark.gpu

SEED_W, SEED_IDS = 0x5EED0001, 0x5EED1001


def _setup(cfg, micro_steps, seed_w=SEED_W):
    params = O.init_parameters(cfg.oracle_dict(), seed_w)
    rng = O.Random(SEED_IDS)
    ids = rng.bounded(micro_steps * cfg.micro_batch * cfg.seq, cfg.vocab)
    return params, ids.reshape(micro_steps, cfg.micro_batch, cfg.seq).astype(np.int32)


def _run(cfg, micro_steps, lr=3e-4):
    from spar_b200.lm import DecoderLM

    params, ids = _setup(cfg, micro_steps)
    lm = DecoderLM(cfg, 0)
    lm.load_state_dict(params)
    loss, norm, flags = lm.train_step(ids, lr, step=1)
    from spar_b200 import ops

    assert ops.gemm_error(0) == 0 and ops.attention_error(0) == 0
    grads = lm.state_dict("grad")
    new = lm.state_dict("param")
    lm.close()
    o_loss, o_grads, o_new, _ = O.lm_train_step(params, {}, list(ids), cfg.oracle_dict(), 1, lr,
                                                cfg.opt_dict())
    return (loss, norm, flags, grads, new), (o_loss, o_grads, o_new)


def _flat(d, names):
    return np.concatenate([np.asarray(d[n], np.float64).ravel() for n in names])


@pytest.mark.parametrize("precision,tol", [(1, 1e-5), (0, 2e-3)])
def test_c1_one_step_parity(cuda, precision, tol):
    from spar_b200.lm import C1
    from dataclasses import replace

    cfg = replace(C1, precision=precision)
    (loss, norm, flags, grads, new), (o_loss, o_grads, o_new) = _run(cfg, 1)
    names = list(o_grads)
    assert flags == (0, 0)
    assert abs(loss - o_loss) <= tol * abs(o_loss)
    assert abs(norm - O.global_grad_norm([o_grads[n] for n in names])) <= tol * norm
    assert rel_l2(_flat(grads, names), _flat(o_grads, names)) <= tol
    for n in names:  # every tensor, including biases and LayerNorm parameters
        assert rel_l2(grads[n], o_grads[n]) <= 10 * tol, n
    assert rel_l2(_flat(new, names), _flat(o_new, names)) <= tol


def test_gradient_accumulation_over_micro_steps(cuda):
    """Two micro-steps accumulate on the device to the gradient of the mean loss."""
    from spar_b200.lm import C1
    from dataclasses import replace

    cfg = replace(C1, precision=1, micro_batch=4)
    (loss, norm, flags, grads, new), (o_loss, o_grads, o_new) = _run(cfg, 2)
    names = list(o_grads)
    assert flags == (0, 0)
    assert abs(loss - o_loss) <= 1e-5 * abs(o_loss)
    assert rel_l2(_flat(grads, names), _flat(o_grads, names)) <= 1e-5


def test_device_init_matches_oracle_stream(cuda):
    from spar_b200.lm import C1, DecoderLM

    lm = DecoderLM(C1, 0)
    lm.init_normal(SEED_W, 0.02)
    got = lm.state_dict()
    lm.close()
    ref = O.init_parameters(C1.oracle_dict(), SEED_W)
    for n in ref:
        np.testing.assert_allclose(got[n], ref[n], rtol=1e-6, atol=1e-9, err_msg=n)


def test_steps_are_deterministic(cuda):
    from spar_b200.lm import C1, DecoderLM

    params, ids = _setup(C1, 1)
    outs = []
    for _ in range(2):
        lm = DecoderLM(C1, 0)
        lm.load_state_dict(params)
        for step in range(1, 3):
            lm.train_step(ids, 3e-4, step=step)
        outs.append(_flat(lm.state_dict(), lm.names))
        lm.close()
    assert np.array_equal(outs[0], outs[1])


def test_invalid_token_sets_flag(cuda):
    from spar_b200.lm import C1, DecoderLM

    params, ids = _setup(C1, 1)
    ids[0, 0, 5] = C1.vocab + 3
    lm = DecoderLM(C1, 0)
    lm.load_state_dict(params)
    _, _, flags = lm.train_step(ids, 3e-4, step=1)
    lm.close()
    assert flags[0] == 1


def test_nonfinite_gradient_skips_update(cuda):
    """clip_grad_norm throws on a non-finite norm before any parameter changes
    (src/training/gradients.cpp:181-183); the fused kernel reports it and updates nothing."""
    from spar_b200.lm import C1, DecoderLM

    params, ids = _setup(C1, 1)
    bad = dict(params)
    w = bad["blocks.0.mlp.up_proj.weight"].copy()
    w[3, 7] = np.nan
    bad["blocks.0.mlp.up_proj.weight"] = w
    lm = DecoderLM(C1, 0)
    lm.load_state_dict(bad)
    _, norm, flags = lm.train_step(ids, 3e-4, step=1)
    after = lm.state_dict()
    lm.close()
    assert flags[1] == 1 and not np.isfinite(norm)
    for n in params:
        np.testing.assert_array_equal(after[n], bad[n])


@pytest.mark.parametrize("kernel", [0, 1])
def test_wait_error_fails_the_step_and_skips_the_update(cuda, kernel):
    """A GEMM (0) or attention (1) kernel that gives up one of its bounded waits raises a device
    flag. The flag is set here from the host (no kernel is made to wait); the norm pass reads it,
    AdamW updates nothing, and the step returns {2, cudaErrorTimeout}, eagerly and in graph
    replay. Once the flag is cleared the next step updates as usual."""
    from spar_b200 import _lib, ops
    from spar_b200._lib import SparError
    from spar_b200.lm import C1, DecoderLM

    lib = _lib.load()
    params, ids = _setup(C1, 1)
    lm = DecoderLM(C1, 0)
    lm.load_state_dict(params)
    try:
        for step in (1, 2, 3):  # step 1 eager, 2 captured, 3 replayed
            if step > 1:
                before = _flat(lm.state_dict(), lm.names)
                assert lib.spar_b200_set_wait_error(0, kernel, 1) == 0
                with pytest.raises(SparError) as err:
                    lm.train_step(ids, 3e-4, step=step)
                assert (err.value.code, err.value.cuda_error) == (2, 909)
                assert np.array_equal(_flat(lm.state_dict(), lm.names), before)
                assert lib.spar_b200_set_wait_error(0, kernel, 0) == 0
            _, _, flags = lm.train_step(ids, 3e-4, step=step)
            assert flags == (0, 0)
    finally:
        lib.spar_b200_set_wait_error(0, kernel, 0)
        lm.close()
    assert ops.gemm_error(0) == 0 and ops.attention_error(0) == 0


def test_graph_replay_matches_eager_steps(cuda):
    """train_step runs its first step eagerly, captures the second into a CUDA graph and replays
    it afterwards (AdamW scalars refreshed from device memory): three steps must give the same
    parameters, bit for bit, as three eager steps (profiling keeps a runtime eager)."""
    from spar_b200.lm import C1, DecoderLM

    params, ids = _setup(C1, 2)
    outs, losses = [], []
    for eager in (False, True):
        lm = DecoderLM(C1, 0)
        lm.load_state_dict(params)
        if eager:
            lm.profile(True)
        ls = []
        for step in range(1, 4):
            loss, _, flags = lm.train_step(ids, 3e-4 * step, step=step)
            assert flags == (0, 0)
            ls.append(loss)
        outs.append(_flat(lm.state_dict(), lm.names))
        losses.append(ls)
        lm.close()
    assert losses[0] == losses[1]
    assert np.array_equal(outs[0], outs[1])


def _lanes_cfg():
    from dataclasses import replace

    from spar_b200.lm import C1

    return replace(C1, precision=0, micro_batch=2)  # small micro-batch: several lanes in flight


def test_lanes_match_oracle(cuda):
    """Micro-batch 2 runs its micro-steps side by side (lanes with their own buffers and gradient
    arenas, added in a fixed order): one step of 4 micro-steps against the oracle."""
    cfg = _lanes_cfg()
    (loss, _, flags, grads, new), (o_loss, o_grads, o_new) = _run(cfg, 4)
    assert flags == (0, 0)
    names = list(o_grads)
    assert abs(loss - o_loss) <= 2e-3 * abs(o_loss)
    assert rel_l2(_flat(grads, names), _flat(o_grads, names)) <= 2e-3
    assert rel_l2(_flat(new, names), _flat(o_new, names)) <= 2e-3


def test_lanes_match_one_lane_and_repeat(cuda, monkeypatch):
    """The same step with lanes switched off (SPAR_B200_LANES=0) differs only by the order of the
    gradient sums (fp32 rounding: the gradients within 1e-6); with lanes, repeated runs (eager
    first step, then graph replays) are bitwise equal. After the first update the two runs' weights
    differ in their last bits, and the TF32 rounding of the weights the GEMMs read turns some of
    those into TF32-ulp differences, so three steps are compared at 1e-4."""
    from spar_b200.lm import DecoderLM

    cfg = _lanes_cfg()
    params, ids = _setup(cfg, 4)

    def steps():
        lm = DecoderLM(cfg, 0)
        lm.load_state_dict(params)
        ls = [lm.train_step(ids, 3e-4, step=1)[0]]
        g1 = _flat(lm.state_dict("grad"), lm.names)
        ls += [lm.train_step(ids, 3e-4, step=s)[0] for s in range(2, 4)]
        out = _flat(lm.state_dict(), lm.names)
        lm.close()
        return ls, g1, out

    a_l, a_g, a = steps()
    b_l, b_g, b = steps()
    monkeypatch.setenv("SPAR_B200_LANES", "0")
    c_l, c_g, c = steps()
    assert a_l == b_l and np.array_equal(a_g, b_g) and np.array_equal(a, b)
    assert rel_l2(a_g, c_g) <= 1e-6 and abs(a_l[0] - c_l[0]) <= 1e-6 * abs(c_l[0])
    assert rel_l2(a, c) <= 1e-4
    np.testing.assert_allclose(a_l, c_l, rtol=1e-4)


def _one_rank_comm():
    import ctypes

    from spar_b200 import _lib

    lib = _lib.load()
    uid = ctypes.create_string_buffer(128)
    _lib.check("spar_b200_comm_unique_id", lib.spar_b200_comm_unique_id(uid, 128))
    comm = ctypes.c_void_p()
    _lib.check("spar_b200_comm_init", lib.spar_b200_comm_init(uid, 0, 1, 0, ctypes.byref(comm)))
    return lib, comm


@pytest.mark.parametrize("lanes", ["0", "2", "4"])
def test_one_rank_communicator_matches_no_communicator(cuda, monkeypatch, lanes):
    """A one-rank NCCL communicator drives the data-parallel path on one GPU: per-layer bucket
    reductions on the communication stream during the last micro-steps, with the lanes' gradients
    merged per bucket (lanes on) instead of once at step end. The all-reduce over one rank is an
    identity and the merge order is the same, so every step is bitwise equal to the same steps
    without a communicator (eager first step, then graph replays)."""
    from spar_b200.lm import DecoderLM

    monkeypatch.setenv("SPAR_B200_LANES", lanes)
    cfg = _lanes_cfg()
    params, ids = _setup(cfg, 4)

    def steps(with_comm):
        lm = DecoderLM(cfg, 0)
        lm.load_state_dict(params)
        lib = comm = None
        if with_comm:
            lib, comm = _one_rank_comm()
            lm.attach_comm(comm, 1)
        out = [lm.train_step(ids, 3e-4, step=s) for s in range(1, 4)]
        state = _flat(lm.state_dict(), lm.names)
        grads = _flat(lm.state_dict("grad"), lm.names)
        lm.close()
        if comm is not None:
            lib.spar_b200_comm_destroy(comm, 0)
        return out, state, grads

    a_out, a, a_g = steps(False)
    b_out, b, b_g = steps(True)
    assert [o[2] for o in b_out] == [(0, 0)] * 3
    assert [o[0] for o in a_out] == [o[0] for o in b_out]
    assert [o[1] for o in a_out] == [o[1] for o in b_out]
    assert np.array_equal(a_g, b_g) and np.array_equal(a, b)


@pytest.mark.parametrize("lanes", ["0", "2"])
def test_sharded_optimizer_one_rank_matches_replicated(cuda, monkeypatch, lanes):
    """The sharded optimiser path on one GPU (SPAR_B200_SHARD_OPT=1 with a one-rank communicator):
    reduce-scatter per bucket, norm pass and AdamW per bucket piece, parameter all-gather at the
    next step's start. Over one rank the collectives are identities, so three steps match the
    replicated steps without a communicator: losses and parameters bitwise, the norm to double
    rounding. Reads need the collective gather first."""
    from spar_b200._lib import SparError
    from spar_b200.lm import DecoderLM

    monkeypatch.setenv("SPAR_B200_LANES", lanes)
    monkeypatch.setenv("SPAR_B200_SHARD_OPT", "1")
    cfg = _lanes_cfg()
    params, ids = _setup(cfg, 4)

    def steps(with_comm):
        lm = DecoderLM(cfg, 0)
        lm.load_state_dict(params)
        lib = comm = None
        if with_comm:
            lib, comm = _one_rank_comm()
            lm.attach_comm(comm, 1)
        out = [lm.train_step(ids, 3e-4, step=s) for s in range(1, 4)]
        if with_comm:
            with pytest.raises(SparError):
                lm.get(lm.names[0])
            for which in ("param", "grad", "m", "v"):
                lm.gather(which)
        state = [_flat(lm.state_dict(w), lm.names) for w in ("param", "grad", "m", "v")]
        lm.close()
        if comm is not None:
            lib.spar_b200_comm_destroy(comm, 0)
        return out, state

    a_out, a = steps(False)
    b_out, b = steps(True)
    assert [o[2] for o in b_out] == [(0, 0)] * 3
    np.testing.assert_allclose([o[1] for o in a_out], [o[1] for o in b_out], rtol=1e-12)
    # A clip factor from a norm that differs in its last double bit can move a clipped fp32
    # gradient by one ulp (rarely); with identical norms the steps are bitwise equal.
    exact = [o[1] for o in a_out] == [o[1] for o in b_out]
    if exact:
        assert [o[0] for o in a_out] == [o[0] for o in b_out]
    else:
        np.testing.assert_allclose([o[0] for o in a_out], [o[0] for o in b_out], rtol=1e-6)
    for x, y in zip(a, b):
        assert np.array_equal(x, y) if exact else rel_l2(x, y) <= 1e-6


def test_spar_family_checkpoint_exact_resume(cuda, tmp_path):
    """Spar-family runtime: two steps, a SPARCKPT v1 checkpoint (parameters + AdamW moments), a new
    runtime that loads it, then the same third step on both: bitwise equal losses and weights."""
    from spar_b200.lm import DecoderLM, LMConfig

    c = dict(vocab=64, dim=128, hidden=256, layers=2, heads=4, kv_heads=2, qk_norm=1)
    cfg = LMConfig(vocab=64, dim=128, hidden=256, layers=2, heads=4, seq=32, micro_batch=2,
                   family=1, kv_heads=2, qk_norm=True)
    ids = O.Random(0x5EED1401).bounded(3 * 2 * 2 * 32, 64).reshape(3, 2, 2, 32).astype(np.int32)
    a = DecoderLM(cfg, 0)
    a.load_state_dict(O.spar_family_parameters(c, 0x5EED0401))
    for s in (1, 2):
        a.train_step(ids[s - 1], 3e-4, step=s)
    path = tmp_path / "step2.sparckpt"
    a.save_checkpoint(path, global_step=2, tokens_seen=2 * 128, rng_state=99, learning_rate=3e-4,
                      adam_step=2)
    b = DecoderLM(cfg, 0)
    meta = b.load_checkpoint(path)
    assert meta == {"global_step": 2, "tokens_seen": 256, "rng_state": 99,
                    "learning_rate": 3e-4, "adam_step": 2}
    la = a.train_step(ids[2], 3e-4, step=3)
    lb = b.train_step(ids[2], 3e-4, step=3)
    pa, pb = _flat(a.state_dict(), a.names), _flat(b.state_dict(), b.names)
    a.close()
    b.close()
    assert la == lb
    assert np.array_equal(pa, pb)


def test_spar_family_sharded_one_rank_matches_replicated(cuda, monkeypatch):
    """The data-parallel path (bucket reduce-scatter, per-piece AdamW, parameter all-gather) with
    the Spar-family runtime on a one-rank communicator: the same steps as without one."""
    from spar_b200.lm import DecoderLM, LMConfig

    monkeypatch.setenv("SPAR_B200_SHARD_OPT", "1")
    c = dict(vocab=64, dim=128, hidden=256, layers=2, heads=4, kv_heads=1, qk_norm=0)
    cfg = LMConfig(vocab=64, dim=128, hidden=256, layers=2, heads=4, seq=32, micro_batch=2,
                   family=1, kv_heads=1)
    ids = O.Random(0x5EED1501).bounded(4 * 2 * 32, 64).reshape(4, 2, 32).astype(np.int32)

    def steps(with_comm):
        lm = DecoderLM(cfg, 0)
        lm.load_state_dict(O.spar_family_parameters(c, 0x5EED0501))
        lib = comm = None
        if with_comm:
            lib, comm = _one_rank_comm()
            lm.attach_comm(comm, 1)
        out = [lm.train_step(ids, 3e-4, step=s) for s in range(1, 4)]
        if with_comm:
            lm.gather("param")
        state = _flat(lm.state_dict(), lm.names)
        lm.close()
        if comm is not None:
            lib.spar_b200_comm_destroy(comm, 0)
        return out, state

    a_out, a = steps(False)
    b_out, b = steps(True)
    assert [o[2] for o in b_out] == [(0, 0)] * 3
    np.testing.assert_allclose([o[1] for o in a_out], [o[1] for o in b_out], rtol=1e-12)
    if [o[1] for o in a_out] == [o[1] for o in b_out]:
        assert [o[0] for o in a_out] == [o[0] for o in b_out] and np.array_equal(a, b)
    else:
        assert rel_l2(a, b) <= 1e-6


@pytest.mark.parametrize("kv_heads,qk_norm,precision", [(2, True, 0), (4, False, 0), (1, True, 0),
                                                     (2, True, 1), (4, False, 1)])
def test_spar_family_grads_match_oracle(cuda, kv_heads, qk_norm, precision):
    """Every gradient of one Spar-family step (two micro-steps) against the float64
    restatement: relative L2 over all gradients <= 3e-3, per tensor <= 1e-2 (TF32 products; with
    one key/value head for four query heads each dK / dV entry sums four heads' TF32 products,
    which measured 2.03e-3 overall, just past the 2e-3 of the benchmark model's tests)."""
    from spar_b200.lm import DecoderLM, LMConfig

    c = dict(vocab=64, dim=128, hidden=256, layers=2, heads=4, kv_heads=kv_heads,
             qk_norm=int(qk_norm))
    cfg = LMConfig(vocab=64, dim=128, hidden=256, layers=2, heads=4, seq=64, micro_batch=2,
                   family=1, kv_heads=kv_heads, qk_norm=qk_norm, precision=precision)
    params = O.spar_family_parameters(c, 0x5EED0601 + kv_heads)
    ids = O.Random(0x5EED1601).bounded(2 * 2 * 64, 64).reshape(2, 2, 64).astype(np.int32)
    lm = DecoderLM(cfg, 0)
    lm.load_state_dict(params)
    loss, norm, flags = lm.train_step(ids, 3e-4, step=1)
    grads = lm.state_dict("grad")
    lm.close()
    total, o_loss = None, 0.0
    for m in ids:
        lo, g = O.spar_lm_forward_backward(params, m, c)
        o_loss += lo / len(ids)
        total = g if total is None else {k: total[k] + g[k] for k in g}
    o_grads = {k: v / len(ids) for k, v in total.items()}
    assert flags == (0, 0)
    # 3xTF32 (unfused attention, grouped heads expanded and summed back): the 1e-5 bar.
    tol_loss, tol_all, tol_each = (2e-3, 3e-3, 1e-2) if precision == 0 else (1e-5, 1e-5, 1e-5)
    assert abs(loss - o_loss) <= tol_loss * abs(o_loss)
    names = list(o_grads)
    assert rel_l2(_flat(grads, names), _flat(o_grads, names)) <= tol_all
    for n in names:
        assert rel_l2(grads[n], o_grads[n]) <= tol_each, n
