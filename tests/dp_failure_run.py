"""Worker for tests/test_dp_gpu.py::test_peer_missing_a_step_gets_code_3: one process per GPU
under torchrun, NVLS off. Both ranks run steps 1 and 2 of the training runtime with a NCCL
communicator (so every collective the step uses has made its connections: NCCL connects lazily,
inside the enqueue, on the host); then the last rank stays alive but does not join step 3 (it
waits on the host until rank 0 is done, so none of its memory goes away while rank 0's
collectives wait for it). Rank 0's step 3 (a graph replay, or eager with SPAR_B200_GRAPHS=0) must
end with status code 3 from the communicator's bounded wait (deadline 5 s) instead of hanging.
Rank 0 then runs a computation on a new stream (the step's own streams may still hold the aborted
work), writes what it saw to --out and exits without tearing the runtime down: after a failed
step the recovery is a new process resuming from a checkpoint.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def progress(out: str, line: str) -> None:
    """Appends a stage marker to out + '.progress' (the test shows it if the run fails)."""
    with open(out + ".progress", "a") as f:
        f.write(line + "\n")
    print(line, file=sys.stderr, flush=True)


def main(out: str) -> None:
    import torch
    import torch.distributed as dist

    from spar_b200 import _lib
    from spar_b200.data import rank_share
    from spar_b200.lm import DecoderLM, LMConfig

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    store = dist.distributed_c10d._get_default_store()
    cfg = LMConfig(vocab=256, dim=128, hidden=256, layers=1, heads=4, seq=64,
                   micro_batch=8 // world)
    lm = DecoderLM(cfg, local)
    lm.init_normal(7, 0.02)
    lib = _lib.load()
    uid = ctypes.create_string_buffer(128)
    if rank == 0:
        _lib.check("spar_b200_comm_unique_id", lib.spar_b200_comm_unique_id(uid, 128))
    obj = [bytes(uid.raw)]
    dist.broadcast_object_list(obj, src=0)
    uid = ctypes.create_string_buffer(obj[0], 128)
    comm = ctypes.c_void_p()
    _lib.check("spar_b200_comm_init", lib.spar_b200_comm_init(uid, rank, world, local,
                                                              ctypes.byref(comm)))
    _lib.check("spar_b200_comm_set_timeout", lib.spar_b200_comm_set_timeout(comm, 5.0))
    lm.attach_comm(comm, world)
    ids = [rank_share(11 + s, 8, 1, cfg.seq, cfg.vocab, rank, world) for s in (1, 2, 3)]
    lm.train_step(ids[0], 3e-4, step=1)
    lm.train_step(ids[1], 3e-4, step=2)
    torch.cuda.synchronize()
    dist.barrier()  # steps 1 and 2 done everywhere
    progress(out, f"rank {rank}: steps 1 and 2 done")
    if rank == world - 1:
        store.wait(["rank0_done"], datetime.timedelta(seconds=120))  # alive, but skips step 3
        # The trainer (its captured steps hold the communicator's collectives) goes first: an
        # NCCL abort with such graphs still alive did not return.
        lm.close()
        lib.spar_b200_comm_destroy(comm, 1)
        return
    start = time.monotonic()
    progress(out, "rank 0: step 3 starts")
    stream = torch.cuda.Stream()  # the step's streams, not torch's legacy default stream
    try:
        lm.train_step(ids[2], 3e-4, step=3, stream=stream.cuda_stream)
        seen = "step 3 completed"
    except _lib.SparError as e:
        seen = f"code {e.code} after {time.monotonic() - start:.1f}s (nccl {e.cuda_error})"
    progress(out, f"rank 0: step 3 returned: {seen}")
    # The context still works after the failure: a plain computation on a new stream.
    with torch.cuda.stream(torch.cuda.Stream()):
        x = torch.arange(4.0, device="cuda")
        seen += f"; device ok {float((x * 2).sum().item()):.0f}"
    progress(out, f"rank 0: {seen}")
    with open(out, "w") as f:
        f.write(seen)
    lib.spar_b200_comm_destroy(comm, 1)
    store.set("rank0_done", "1")
    os._exit(0)  # no teardown of a runtime whose step failed


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    main(ap.parse_args().out)
