"""Multi-rank host logic of the row-panel sharding on CPU (gloo, world size 2):
panel cuts, panel CSR slicing and the padded all-gather of C panels.  Each rank
computes its panel with the CPU oracle; the GPU path is covered by
tests/test_gpu_multi.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import powersparse_b200 as psb
        from oracle import oracle
        from powersparse_b200 import synth
        from powersparse_b200.distributed import allgather_rows, panel_csr
        m = synth.chung_lu(4000, 12, 500, 2.1, seed=21)
        B = synth.dense(m.cols, 32, 5)
        cuts = psb.partition_rows(m.row_ptr, world)
        p = panel_csr(m, int(cuts[rank]), int(cuts[rank + 1]))
        local = torch.from_numpy(oracle.spmm(p.row_ptr, p.col_ind, p.values, B, threads=1))
        full = allgather_rows(local, cuts)
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), full.numpy())
        np.save(os.path.join(result_dir, f"cuts{rank}.npy"), cuts)
        np.save(os.path.join(result_dir, f"nnz{rank}.npy"), np.array([p.nnz]))
    finally:
        dist.destroy_process_group()


def test_row_panels_allgather_on_gloo(tmp_path):
    from oracle import oracle
    from powersparse_b200 import synth
    port = _free_port()
    mp.start_processes(_worker, args=(WORLD, port, str(tmp_path)), nprocs=WORLD, start_method="spawn")
    m = synth.chung_lu(4000, 12, 500, 2.1, seed=21)
    expected = oracle.spmm(m.row_ptr, m.col_ind, m.values, synth.dense(m.cols, 32, 5), threads=1)
    cuts = [np.load(tmp_path / f"cuts{r}.npy") for r in range(WORLD)]
    assert all(np.array_equal(cuts[0], c) for c in cuts)
    nnz = [int(np.load(tmp_path / f"nnz{r}.npy")[0]) for r in range(WORLD)]
    assert sum(nnz) == m.nnz
    assert abs(nnz[0] - nnz[1]) <= m.row_lengths().max() + 1
    for r in range(WORLD):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert got.shape == expected.shape
        assert np.array_equal(got, expected)  # same FP64 loop per row: bit-identical


def test_panel_csr_slices_rows():
    from powersparse_b200 import synth
    from powersparse_b200.distributed import panel_csr
    m = synth.chung_lu(500, 8, 60, 2.1, seed=2)
    p = panel_csr(m, 100, 260)
    assert p.rows == 160 and p.cols == m.cols
    assert p.row_ptr[0] == 0 and p.row_ptr[-1] == p.nnz
    lo, hi = m.row_ptr[100], m.row_ptr[260]
    assert np.array_equal(p.col_ind, m.col_ind[lo:hi])
    assert np.array_equal(np.diff(p.row_ptr), np.diff(m.row_ptr)[100:260])


def _replicas_worker(rank, world, port, result_dir):
    """Replicas on gloo with the CUDA IPC calls replaced by fakes: each rank "exports"
    a handle naming its rank and a made-up base address; opening returns that base."""
    import datetime
    import json
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import powersparse_b200.distributed as D
        base_of = lambda r: (r + 1) << 40  # noqa: E731
        opened, closed = [], []
        D.ipc_export = lambda t: (bytes([rank]) * 64, 256 * (rank + 1))
        D.ipc_open = lambda h: (opened.append(h[0]), base_of(h[0]))[1]
        D.ipc_close = lambda b: closed.append(b)
        reps = D.Replicas(100, 32, "cpu")
        panels = reps.peer_panels(10, 32)
        with pytest.raises(ValueError):
            reps.peer_panels(10, 64)
        reps.close()
        with open(os.path.join(result_dir, f"replicas{rank}.json"), "w") as f:
            json.dump({"opened": opened, "panels": panels, "closed": closed,
                       "shape": list(reps.full.shape)}, f)
    finally:
        dist.destroy_process_group()


def test_replicas_open_peers_in_ring_order_on_gloo(tmp_path):
    """Each rank opens every other rank's replica once, in ring order from itself; the
    panel addresses are the peer's base + its export offset + row0 * N * 4 bytes; close
    releases every mapping."""
    import json
    world = 4
    mp.start_processes(_replicas_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    for rank in range(world):
        with open(tmp_path / f"replicas{rank}.json") as f:
            got = json.load(f)
        ring = [(rank + s) % world for s in range(1, world)]
        assert got["opened"] == ring
        assert got["panels"] == [((r + 1) << 40) + 256 * (r + 1) + 10 * 32 * 4 for r in ring]
        assert got["closed"] == [(r + 1) << 40 for r in ring]
        assert got["shape"] == [100, 32]
