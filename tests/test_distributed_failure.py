"""Failure of a rank in the row-panel multi-GPU path, made on the host (gloo ranks
on CPU, world size 2; no GPU is involved).  Rank 1 either raises before the
all-gather of the C panels or leaves between steps; rank 0 must end with PeerLost
within the short process-group timeout / heartbeat limit, abort its group and exit
cleanly instead of hanging."""
import datetime
import json
import multiprocessing
import os
import socket
import time

import pytest

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, result_dir, mode):
    import numpy as np
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=5))
    from powersparse_b200.distributed import PeerLost, allgather_rows, heartbeat
    cuts = np.array([0, 3, 7])
    local = torch.full((int(cuts[rank + 1] - cuts[rank]), 4), float(rank))
    heartbeat(0, timeout_s=20)
    full = allgather_rows(local, cuts)  # step 0 completes on both ranks
    assert full.shape == (7, 4)
    if rank == 1:
        if mode == "raise":
            raise RuntimeError("failure injected on rank 1 before the all-gather of step 1")
        return  # "leave": rank 1 stops between steps without telling anyone
    t0 = time.monotonic()
    outcome = {"mode": mode}
    try:
        if mode == "leave":
            heartbeat(1, timeout_s=3)  # the host learns of it before step 1 launches anything
        allgather_rows(local, cuts)
        outcome["error"] = None
    except PeerLost as e:
        outcome["error"] = str(e)
    outcome["seconds"] = time.monotonic() - t0
    try:
        dist.destroy_process_group()  # abort the group; with its peer gone this may itself report an error
    except Exception as e:  # noqa: BLE001 - recorded, the rank still exits cleanly
        outcome["destroy_error"] = str(e)[:200]
    with open(os.path.join(result_dir, f"rank0_{mode}.json"), "w") as f:
        json.dump(outcome, f)


@pytest.mark.parametrize("mode", ["raise", "leave"])
def test_surviving_rank_gets_an_error_instead_of_hanging(tmp_path, mode):
    ctx = multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path), mode)) for r in range(WORLD)]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            pytest.fail(f"rank process {p.pid} still running after 60 s")
    assert time.monotonic() - t0 < 60
    assert procs[0].exitcode == 0, "the surviving rank must exit cleanly"
    assert procs[1].exitcode == (1 if mode == "raise" else 0)
    with open(tmp_path / f"rank0_{mode}.json") as f:
        outcome = json.load(f)
    assert outcome["error"], "rank 0 should have raised PeerLost"
    if mode == "leave":
        assert "rank(s) [1]" in outcome["error"] and "step 1" in outcome["error"]
    assert outcome["seconds"] < 20
