"""Dense offsets beyond 2^31 elements.

The reference rejects any shape with rows*N or cols*N above INT_MAX
(utils/matrix_utils.h:72-76, called at PowerSparse_SpMM/spmm_solution.cu:11); this
library computes dense offsets in 64 bits and accepts them, which configuration 5
needs (16.8M x 128 = 2^31).  Here A has n = 2^24 + 2^20 rows and columns, so
n * 128 > 2^31: a few thousand rows, half of them above row 2^24, hold ~200k
nonzeros whose columns are drawn half from [2^24, n).  B (also used as the SDDMM
lhs and rhs) is [n x 128] on the device (9.1 GB); the expected rows are computed on
the host in FP64 from only the B rows the nonzeros touch.  SpMM, SDDMM in workset
order and SDDMM in CSR order are checked at |a - e| <= 1e-5 + 1e-4 |e|.
"""
import numpy as np
import pytest
import torch

import powersparse_b200 as psb
from helpers import ATOL, RTOL
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu

N = 128
SIZE = (1 << 24) + (1 << 20)


def _matrix(seed: int = 64) -> synth.Csr:
    rng = np.random.default_rng(seed)
    low = rng.choice(1 << 24, size=1500, replace=False)
    high = (1 << 24) + rng.choice(SIZE - (1 << 24), size=1500, replace=False)
    rows = np.sort(np.concatenate([low, high]))
    lens = np.minimum(rng.zipf(1.6, size=rows.size) * 8, 3000)
    lens[[7, 1700]] = 3000  # two rows long enough for the block worksets and the FP64 wide-row path
    counts = np.zeros(SIZE, dtype=np.int64)
    cols, vals = [], []
    for r, k in zip(rows, lens):
        c = np.concatenate([rng.integers(0, 1 << 24, size=k // 2), rng.integers(1 << 24, SIZE, size=k - k // 2)])
        c = np.unique(c)
        cols.append(c)
        vals.append(rng.uniform(-1, 1, size=c.size).astype(np.float32))
        counts[r] = c.size
    row_ptr = np.zeros(SIZE + 1, dtype=np.int64)
    np.cumsum(counts, out=row_ptr[1:])
    return synth.Csr(SIZE, SIZE, row_ptr.astype(np.int32), np.concatenate(cols).astype(np.int32),
                     np.concatenate(vals), False)


def _assert_close(actual, expected, tag):
    ok = oracle.close(actual, expected, ATOL, RTOL)
    assert ok.all(), f"{tag}: {int((~ok).sum())} of {ok.size} elements outside tolerance"


def test_dense_offsets_beyond_2_31():
    m = _matrix()
    assert SIZE * N > 2**31 and (m.col_ind >= (1 << 24)).sum() > m.nnz // 3
    free, _ = torch.cuda.mem_get_info()
    if free < 40 << 30:
        pytest.skip("needs ~30 GB of free device memory")
    g = torch.Generator(device="cuda").manual_seed(11)
    B = torch.rand((SIZE, N), generator=g, device="cuda") * 2 - 1
    nz_rows = np.flatnonzero(np.diff(m.row_ptr))
    assert (nz_rows >= (1 << 24)).any()
    rows_of = np.repeat(np.arange(SIZE), np.diff(m.row_ptr))
    Bc = B.index_select(0, torch.from_numpy(m.col_ind.astype(np.int64)).cuda()).double().cpu().numpy()
    Br = B.index_select(0, torch.from_numpy(rows_of.astype(np.int64)).cuda()).double().cpu().numpy()
    vals = m.values.astype(np.float64)
    # sm_count=1 (the workset heuristic's threshold at its smallest) gives this small
    # matrix block worksets, so both kernel paths and the FP64 wide rows run.
    with psb.PowerSparseMatrixGPU(m.rows, m.cols, m.nnz, m.row_ptr, m.col_ind, m.values, sm_count=1) as A:
        assert A.GroupTypeNum() >= 4 and A.wide_rows >= 2
        # SpMM: C[r] = sum over the row's nonzeros of val * B[col].
        C = torch.zeros((SIZE, N), device="cuda")
        psb.SpMM(A, N, B, C)
        torch.cuda.synchronize()
        starts = m.row_ptr[nz_rows].astype(np.int64)
        expected = np.add.reduceat(vals[:, None] * Bc, starts, axis=0)
        got = C.index_select(0, torch.from_numpy(nz_rows.astype(np.int64)).cuda()).cpu().numpy()
        _assert_close(got, expected, "SpMM rows")
        probe = torch.arange(0, SIZE, 4099, device="cuda")
        empty = probe[torch.from_numpy(np.diff(m.row_ptr)[probe.cpu().numpy()] == 0).cuda()]
        assert torch.count_nonzero(C.index_select(0, empty)) == 0, "empty rows must stay zero"
        del C
        # SDDMM (lhs = rhs = B): out_p = val_p * <B[row_p], B[col_p]>.
        e = vals * np.einsum("ij,ij->i", Br, Bc)
        out = torch.empty(m.nnz, device="cuda")
        psb.SDDMM_csr(A, N, B, B, out)
        outs = [torch.zeros(max(A.workset_size(s), 1), device="cuda") for s in range(A.GroupTypeNum())]
        psb.SDDMM(A, N, B, B, outs)
        torch.cuda.synchronize()
        _assert_close(out.cpu().numpy(), e, "SDDMM in CSR order")
        moved = np.empty(m.nnz, dtype=np.float64)
        for s in range(A.GroupTypeNum()):
            size = A.workset_size(s)
            if size:
                pos = psb._device_array(A.CsrPosition()[s], size, torch.int32)
                moved[pos] = outs[s][:size].cpu().numpy()
        _assert_close(moved, e, "SDDMM in workset order")
