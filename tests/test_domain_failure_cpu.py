"""Failure detection of the decomposed step on CPU ranks (gloo, world size 2), with every failure
made on the host: a rank that stops between steps after posting why, a rank whose step raises
between two of its collectives, a rank that stops without a word.  The surviving rank must end with
an error that names the failed rank (or the missing arrival) instead of waiting for good.  No GPU
is involved."""

import datetime
import json
import os
import socket
import time

import torch

from fsctep_b200 import domain as D

PG_TIMEOUT = 6.0     # process-group timeout: ends a collective whose peer is gone
GUARD_TIMEOUT = 4.0  # how long a step's arrival waits for the other ranks


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _toy_step(rank, world, value, raise_between=False):
    """Two collectives, like a decomposed step: a sum, then an exchange of rows."""
    tot = yield from D.all_reduce_sum(torch.tensor([float(value)], dtype=torch.float64))
    if raise_between:
        raise ValueError("planted failure between the step's collectives")
    recv, _ = yield from D.all_to_all(torch.full((world, 2), float(rank)), [1] * world, [1] * world)
    assert recv[:, 0].tolist() == [float(r) for r in range(world)]
    return float(tot[0])


def _worker(rank, world, port, store_port, scenario, out_dir):
    import torch.distributed as dist

    out = {"rank": rank, "steps": []}
    guard = None
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=PG_TIMEOUT))
        store = dist.TCPStore("127.0.0.1", store_port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
        guard = D.StepGuard(store, rank, world, timeout=GUARD_TIMEOUT)
        for step in range(3):
            if rank == 1 and step == 1 and scenario == "between":
                guard.fail("input check failed before step 2")
                break
            if rank == 1 and step == 1 and scenario == "absent":
                break  # leaves without posting anything
            planted = rank == 1 and step == 1 and scenario == "midstep"
            t0 = time.monotonic()
            out["steps"].append(D.run_dist(_toy_step(rank, world, rank + 1 + 10 * step, planted), guard))
            out["last_step_s"] = time.monotonic() - t0
    except Exception as e:  # recorded for the test; the process ends normally
        out["error"] = type(e).__name__
        out["message"] = str(e)
        out["failed_after_s"] = time.monotonic() - t0
    if guard is not None:
        try:
            out["posted"] = guard.failure()
        except Exception as e:
            out["posted_error"] = repr(e)
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(out, f)
    # no destroy_process_group: the peer may be gone; the process exit closes the connections


def _run(scenario, tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), _free_port(), scenario, str(tmp_path)), nprocs=2, join=True)
    return [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]


def test_guarded_steps_run_normally(tmp_path):
    r0, r1 = _run("ok", tmp_path)
    for r in (r0, r1):
        assert "error" not in r, r
        assert r["steps"] == [3.0, 23.0, 43.0]
        assert r["posted"] is None


def test_failure_posted_between_steps_stops_the_peer_before_its_next_collective(tmp_path):
    r0, r1 = _run("between", tmp_path)
    assert r1["steps"] == [3.0] and "error" not in r1
    assert r0["steps"] == [3.0]
    assert r0["error"] == "RankFailure" and "rank 1: input check failed before step 2" in r0["message"]
    assert r0["failed_after_s"] < GUARD_TIMEOUT  # learnt from the store, not from a timeout


def test_failure_between_collectives_ends_the_peer_collective_and_names_the_rank(tmp_path):
    r0, r1 = _run("midstep", tmp_path)
    assert r1["error"] == "ValueError" and r1["steps"] == [3.0]
    assert r0["steps"] == [3.0] and "error" in r0  # its exchange ended with an error, it did not hang
    assert r0["failed_after_s"] < PG_TIMEOUT + 5.0
    assert r0["posted"].startswith("rank 1: ValueError: planted failure")


def test_rank_that_never_arrives_is_reported_after_the_guard_timeout(tmp_path):
    r0, r1 = _run("absent", tmp_path)
    assert r1["steps"] == [3.0] and "error" not in r1
    assert r0["steps"] == [3.0] and r0["error"] == "RankFailure"
    assert "1 of 2 ranks did not arrive" in r0["message"]
    assert GUARD_TIMEOUT <= r0["failed_after_s"] < GUARD_TIMEOUT + 5.0
