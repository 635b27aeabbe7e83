"""GPU test of ps_spmm_noalloc, the SpMM entry point that allocates no device memory.

Some callers cannot allocate device memory while they run: engines that reserve
the GPU's memory up front and hand it out from their own pool, and latency-bound
callers that cannot take the synchronization cudaMalloc / cudaFree may imply.
For them ps_spmm_noalloc keeps the FP64 wide-row scratch of SpMM in a fixed
16 MiB device array instead of a buffer grown with cudaMalloc.  This file checks,
through the C ABI, that two calls in a row give the FP64 oracle's results (and
ps_spmm's) within the tolerance of the other GPU tests, that the device's free
memory is the same before and after those calls on a fresh matrix at an N that
ps_spmm never ran, and that a matrix needing more scratch than the array holds is
refused with a clear error.  It is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

import powersparse_b200 as psb
from helpers import ATOL, RTOL
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu

_SCRATCH_DOUBLES = 1 << 21


def _wide_matrix(rows: int, cols: int, row_len: int, seed: int) -> synth.Csr:
    """`rows` rows of `row_len` distinct columns each (every row one wide block group)."""
    rng = np.random.default_rng(seed)
    col = np.argsort(rng.random((rows, cols)), axis=1)[:, :row_len]
    col.sort(axis=1)
    val = rng.uniform(-1, 1, size=(rows, row_len)).astype(np.float32)
    ptr = np.arange(rows + 1, dtype=np.int64) * row_len
    return synth.Csr(rows, cols, ptr.astype(np.int32), col.reshape(-1).astype(np.int32), val.reshape(-1), False)


def _noalloc(m, N, B, C):
    lib = psb.load_library()
    status = lib.ps_spmm_noalloc(m.handle, int(N), ctypes.c_void_p(B.data_ptr()), ctypes.c_void_p(C.data_ptr()),
                                 None)
    return status, lib.ps_last_error().decode()


def _check(actual, expected, tag):
    ok = oracle.close(actual, expected, ATOL, RTOL)
    assert ok.all(), f"{tag}: {int((~ok).sum())} of {ok.size} outside tolerance"


@pytest.mark.parametrize("n", [32, 96, 128, 256])
def test_noalloc_spmm_matches_oracle_and_spmm_on_two_calls(n):
    mtx = synth.chung_lu(3000, 14, 600, 2.1, seed=31)
    wide = _wide_matrix(64, 4096, 2048, 32)
    for A, sm in ((mtx, 1), (wide, 1)):
        with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values, sm_count=sm) as m:
            if A is wide:
                assert m.wide_rows == A.rows
            B_host = synth.dense(A.cols, n, 50 + n)
            B = torch.from_numpy(B_host).cuda()
            outs = [torch.zeros((A.rows, n), device="cuda") for _ in range(2)]
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            for C in outs:  # two calls in a row; this N never ran through ps_spmm on this matrix
                status, err = _noalloc(m, n, B, C)
                assert status == psb.PS_OK, err
            torch.cuda.synchronize()
            assert torch.cuda.mem_get_info()[0] == free_before, "device memory was allocated"
            expected = oracle.spmm(A.row_ptr, A.col_ind, A.values, B_host)
            for call, C in enumerate(outs):
                _check(C.cpu().numpy(), expected, f"N={n} call {call} vs the FP64 oracle")
            C_ref = torch.zeros((A.rows, n), device="cuda")
            psb.SpMM(m, n, B, C_ref)
            torch.cuda.synchronize()
            _check(outs[1].cpu().numpy(), C_ref.cpu().numpy().astype(np.float64), f"N={n} vs ps_spmm")


def test_noalloc_spmm_refuses_more_scratch_than_the_array_holds():
    A = _wide_matrix(4200, 4096, 2048, 33)  # 4200 wide rows: 4200 * 512 > 2^21 doubles
    with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values, sm_count=1) as m:
        assert m.wide_rows == A.rows and A.rows * 512 > _SCRATCH_DOUBLES >= A.rows * 256
        B = torch.zeros((A.cols, 512), device="cuda")
        C = torch.zeros((A.rows, 512), device="cuda")
        status, err = _noalloc(m, 512, B, C)
        assert status == psb.PS_ERR_INVALID_ARGUMENT and "ps_spmm_noalloc" in err and "16 MiB" in err
        # Within the limit the same matrix runs and matches ps_spmm.
        B = torch.from_numpy(synth.dense(A.cols, 256, 7)).cuda()
        C_ref = torch.zeros((A.rows, 256), device="cuda")
        psb.SpMM(m, 256, B, C_ref)
        C = torch.zeros((A.rows, 256), device="cuda")
        status, err = _noalloc(m, 256, B, C)
        torch.cuda.synchronize()
        assert status == psb.PS_OK, err
        _check(C.cpu().numpy(), C_ref.cpu().numpy().astype(np.float64), "N=256, 4200 wide rows")
