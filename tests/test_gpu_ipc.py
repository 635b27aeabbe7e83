"""GPU test of the CUDA IPC path of ps_spmm_push on one GPU: the parent exports a
replica buffer (ps_ipc_export), a child process opens it (ps_ipc_open) and pushes
its SpMM rows into it, then closes the mapping (ps_ipc_close).  The parent's buffer
must hold the child's C exactly, at the row offset the child wrote."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROW0, N = 9, 64


def _matrix():
    from powersparse_b200 import synth
    return synth.config_matrix(2, scale=0.005)


def _child(rank, handle, offset, result_dir):
    import powersparse_b200 as psb
    from helpers import dense_inputs
    torch.cuda.set_device(0)
    A = _matrix()
    base = psb.ipc_open(handle)
    try:
        with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values) as m:
            B = torch.from_numpy(dense_inputs(A.cols, N, 3)).cuda()
            C = torch.zeros((A.rows, N), device="cuda")
            psb.SpMM_push(m, N, B, C, [base + offset + ROW0 * N * 4])
            torch.cuda.synchronize()
            np.save(os.path.join(result_dir, "child_C.npy"), C.cpu().numpy())
    finally:
        psb.ipc_close(base)


def test_push_into_another_process_buffer(tmp_path):
    import powersparse_b200 as psb
    A = _matrix()
    # A slice of a larger tensor, so the export has a non-zero offset to honour.
    backing = torch.full((A.rows + ROW0 + 5 + 16, N), float("nan"), device="cuda")
    replica = backing[16:]
    handle, offset = psb.ipc_export(replica)
    assert len(handle) == psb.PS_IPC_HANDLE_BYTES and offset >= 16 * N * 4
    torch.cuda.synchronize()
    mp.start_processes(_child, args=(handle, offset, str(tmp_path)), nprocs=1, start_method="spawn")
    C = np.load(tmp_path / "child_C.npy")
    got = replica.cpu().numpy()
    assert np.array_equal(got[ROW0:ROW0 + A.rows], C), "pushed rows differ from the child's C"
    assert np.isnan(got[:ROW0]).all() and np.isnan(got[ROW0 + A.rows:]).all(), "wrote outside the panel"
    assert np.isnan(backing[:16].cpu().numpy()).all()
