"""GPU multi-rank test of the row-panel sharding (NCCL, one process per GPU):
needs at least two GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import powersparse_b200 as psb
        from powersparse_b200 import synth
        from powersparse_b200.distributed import ShardedPowerSparse, panel_csr
        m = synth.chung_lu(20000, 30, 2000, 2.1, seed=31)
        cuts = psb.partition_rows(m.row_ptr, world)
        panel = panel_csr(m, int(cuts[rank]), int(cuts[rank + 1]))
        shard = ShardedPowerSparse(m.row_ptr, panel, rank, world, sm_count=2)
        B = torch.from_numpy(synth.dense(m.cols, 64, 7)).to(dev)
        C = torch.zeros((panel.rows, 64), device=dev)
        full = shard.spmm(64, B, C, gather=True)
        np.save(os.path.join(result_dir, f"spmm{rank}.npy"), full.cpu().numpy())
        X = torch.from_numpy(synth.dense(m.rows, 32, 8)[cuts[rank]:cuts[rank + 1]].copy()).to(dev)
        Y = torch.from_numpy(synth.dense(m.cols, 32, 9)).to(dev)
        outs = [torch.zeros(max(shard.matrix.workset_size(s), 1), device=dev)
                for s in range(shard.matrix.GroupTypeNum())]
        shard.sddmm(32, X, Y, outs)
        torch.cuda.synchronize()
        for s, o in enumerate(outs):
            np.save(os.path.join(result_dir, f"sddmm{rank}_{s}.npy"), o[: shard.matrix.workset_size(s)].cpu().numpy())
        shard.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_spmm_sddmm_on_two_gpus(tmp_path):
    import powersparse_b200 as psb
    from helpers import ATOL, RTOL
    from oracle import oracle
    from powersparse_b200 import synth
    from powersparse_b200.distributed import panel_csr
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    m = synth.chung_lu(20000, 30, 2000, 2.1, seed=31)
    expected = oracle.spmm(m.row_ptr, m.col_ind, m.values, synth.dense(m.cols, 64, 7))
    for r in range(world):
        assert oracle.close(np.load(tmp_path / f"spmm{r}.npy"), expected, ATOL, RTOL).all()
    cuts = psb.partition_rows(m.row_ptr, world)
    X, Y = synth.dense(m.rows, 32, 8), synth.dense(m.cols, 32, 9)
    for r in range(world):
        p = panel_csr(m, int(cuts[r]), int(cuts[r + 1]))
        L = oracle.build_layout(p.rows, p.cols, p.row_ptr, p.col_ind, p.values, 2)
        exp = oracle.sddmm(L, X[cuts[r]:cuts[r + 1]], Y)
        for s in range(L.S):
            assert oracle.close(np.load(tmp_path / f"sddmm{r}_{s}.npy"), exp[s], ATOL, RTOL).all()


def _push_worker(rank, world, port, result_dir):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import powersparse_b200 as psb
        from powersparse_b200 import synth
        from powersparse_b200.distributed import Replicas, ShardedPowerSparse, panel_csr
        m = synth.chung_lu(20000, 30, 2000, 2.1, seed=37)
        cuts = psb.partition_rows(m.row_ptr, world)
        panel = panel_csr(m, int(cuts[rank]), int(cuts[rank + 1]))
        shard = ShardedPowerSparse(m.row_ptr, panel, rank, world, sm_count=2)
        for n in (32, 128):
            B = torch.from_numpy(synth.dense(m.cols, n, 11 + n)).to(dev)
            reps = Replicas(m.rows, n, dev)
            reps.full.fill_(float("nan"))
            reps.full[shard.row_begin:shard.row_end].zero_()
            dist.barrier()
            full = shard.spmm_replicated(n, B, reps)
            torch.cuda.synchronize()
            np.save(os.path.join(result_dir, f"push{n}_{rank}.npy"), full.cpu().numpy())
            dist.barrier()  # no rank frees its replica while a peer still maps it
            reps.close()
            dist.barrier()
        shard.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_allgather_spmm_on_two_gpus(tmp_path):
    """ps_spmm_push over CUDA IPC: each rank's replica holds every panel, equal across
    ranks bit for bit and to the FP64 product within tolerance."""
    from helpers import ATOL, RTOL
    from oracle import oracle
    from powersparse_b200 import synth
    world = 2
    mp.start_processes(_push_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    m = synth.chung_lu(20000, 30, 2000, 2.1, seed=37)
    for n in (32, 128):
        expected = oracle.spmm(m.row_ptr, m.col_ind, m.values, synth.dense(m.cols, n, 11 + n))
        got = [np.load(tmp_path / f"push{n}_{r}.npy") for r in range(world)]
        for r in range(world):
            assert not np.isnan(got[r]).any(), f"rank {r}: rows missing from the replica (N={n})"
            assert oracle.close(got[r], expected, ATOL, RTOL).all(), f"rank {r} N={n}"
        assert np.array_equal(got[0], got[1]), f"replicas differ between ranks (N={n})"
