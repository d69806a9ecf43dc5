"""Failure detection of the data-parallel host logic, on CPU with gloo ranks (no GPU is faulted,
trapped or hung; the failure is made on the host).

A rank leaves between steps (it stops after step 1). The others must learn of it before they
launch step 2's collectives: spar_b200.dp.Heartbeat names the missing rank (RankLost), at once
when the rank announced leaving and at the deadline when it just stopped. The survivors then
exit cleanly; nothing blocks in a collective whose peer is gone.
"""
import datetime
import os
import socket
import tempfile
import time

import pytest


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out, announce):
    import torch
    import torch.distributed as dist

    from spar_b200.dp import Heartbeat, RankLost

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    hb = Heartbeat(dist.distributed_c10d._get_default_store(), rank, world, timeout=3.0)
    t = torch.ones(4)
    hb.arrive(1)
    dist.all_reduce(t)  # step 1's collective: every rank is there
    result = f"step1 {t[0].item():.0f}"
    if rank == world - 1:  # this rank leaves between steps
        if announce:
            hb.leave()
        with open(os.path.join(out, f"rank{rank}.txt"), "w") as f:
            f.write(result + " left")
        return  # no destroy_process_group: it just stops
    start = time.monotonic()
    try:
        hb.arrive(2)
        dist.all_reduce(t)  # never reached: the heartbeat fails first
        result += " step2 ran"
    except RankLost as e:
        result += f" lost {e.missing} left {e.left} after {time.monotonic() - start:.1f}s"
    with open(os.path.join(out, f"rank{rank}.txt"), "w") as f:
        f.write(result)


@pytest.mark.parametrize("announce", [True, False])
def test_rank_leaving_between_steps_is_detected_before_the_next_collective(announce):
    import torch.multiprocessing as mp

    world = 3
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_worker, args=(world, _port(), out, announce), nprocs=world, join=True,
                           start_method="spawn")
        lines = [open(os.path.join(out, f"rank{r}.txt")).read() for r in range(world)]
    assert lines[2] == "step1 3 left"
    for line in lines[:2]:
        assert line.startswith("step1 3 lost ["), line
        assert "step2 ran" not in line
        waited = float(line.rsplit("after ", 1)[1].rstrip("s"))
        missing = line.split("lost ", 1)[1].split(" left")[0]
        if announce:  # fails at once; a survivor that has not arrived yet may be listed too
            assert "left [2]" in line and "2]" in missing and waited < 2.0, line
        else:  # at the deadline every survivor has arrived: only the silent rank is missing
            assert missing == "[2]" and "left []" in line and 2.5 <= waited < 10.0, line
