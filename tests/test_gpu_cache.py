"""GPU tests of the layout cache (ps_matrix_save / ps_matrix_load): a loaded matrix
has the saved layout bit for bit, gives the oracle's results, and a damaged file is
refused before anything reaches a kernel."""
import struct

import numpy as np
import pytest
import torch

import powersparse_b200 as psb
from helpers import ATOL, RTOL, dense_inputs, golden_names, load_golden
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu


def _same_layout(a: dict, b: dict):
    assert a.keys() == b.keys()
    for k in a:
        if isinstance(a[k], np.ndarray):
            assert a[k].dtype == b[k].dtype and np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)), k
        else:
            assert a[k] == b[k], k


@pytest.mark.parametrize("name", golden_names())
def test_layout_round_trip(name, tmp_path):
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    path = tmp_path / "m.pslayout"
    with psb.PowerSparseMatrixGPU(rows, cols, len(ci), rp, ci, va, sm_count=sm) as m:
        m.save(str(path))
        ref = m.download()
        wide = m.wide_rows
    with psb.PowerSparseMatrixGPU.load(str(path)) as m2:
        assert (m2.MatrixRow(), m2.MatrixCol(), m2.MatrixNNZ()) == (rows, cols, len(ci))
        assert m2.wide_rows == wide
        _same_layout(ref, m2.download())
        B = dense_inputs(cols, 128, 77)
        C = torch.zeros((rows, 128), device="cuda")
        psb.SpMM(m2, 128, torch.from_numpy(B).cuda(), C)
        X, Y = dense_inputs(rows, 32, 78), dense_inputs(cols, 32, 79)
        out = torch.empty(len(ci), device="cuda")
        psb.SDDMM_csr(m2, 32, torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda(), out)
        torch.cuda.synchronize()
    assert oracle.close(C.cpu().numpy(), oracle.spmm(rp, ci, va, B), ATOL, RTOL).all()
    row = np.repeat(np.arange(rows), np.diff(rp))
    exp = va.astype(np.float64) * np.einsum("ij,ij->i", X[row].astype(np.float64), Y[ci].astype(np.float64))
    assert oracle.close(out.cpu().numpy(), exp, ATOL, RTOL).all()


def test_wide_rows_survive_the_round_trip(tmp_path):
    """Four appended rows of 2600 elements: 40 groups of 256 (enough for that workset at
    sm_count=1), 10 slices each, so all four are wide rows."""
    base = synth.chung_lu(3000, 12, 300, 2.1, seed=3)
    rng = np.random.default_rng(3)
    heavy = [np.sort(rng.choice(base.cols, size=2600, replace=False)).astype(np.int32) for _ in range(4)]
    ends = base.nnz + 2600 * np.arange(1, 5)
    rp = np.concatenate([base.row_ptr, ends]).astype(np.int32)
    ci = np.concatenate([base.col_ind] + heavy).astype(np.int32)
    va = np.concatenate([base.values, rng.uniform(-1, 1, 4 * 2600).astype(np.float32)])
    rows = base.rows + 4
    path = tmp_path / "w.pslayout"
    with psb.PowerSparseMatrixGPU(rows, base.cols, len(ci), rp, ci, va, sm_count=1) as m:
        assert m.wide_rows == 4
        m.save(str(path))
    with psb.PowerSparseMatrixGPU.load(str(path)) as m2:
        assert m2.wide_rows == 4
        B = synth.dense(base.cols, 32, 5)
        C = torch.zeros((rows, 32), device="cuda")
        psb.SpMM(m2, 32, torch.from_numpy(B).cuda(), C)
        torch.cuda.synchronize()
    assert oracle.close(C.cpu().numpy(), oracle.spmm(rp, ci, va, B), ATOL, RTOL).all()


def _saved(tmp_path):
    m = synth.chung_lu(2000, 14, 300, 2.1, seed=9)
    path = tmp_path / "c.pslayout"
    with psb.PowerSparseMatrixGPU(m.rows, m.cols, m.nnz, m.row_ptr, m.col_ind, m.values, sm_count=2) as A:
        A.save(str(path))
        S = A.GroupTypeNum()
    return m, path, S


def test_damaged_files_are_refused(tmp_path):
    m, path, S = _saved(tmp_path)
    good = path.read_bytes()
    head = 8 + 7 * 4 + 4 * S + 8 * S          # first int32 of workset 0's column indices
    cases = {
        "column index": good[:head] + struct.pack("<i", m.cols + 5) + good[head + 4:],
        "negative column": good[:head] + struct.pack("<i", -1) + good[head + 4:],
        "truncated": good[: len(good) // 2],
        "trailing": good + b"\0",
    }
    for what, data in cases.items():
        bad = tmp_path / f"{what}.pslayout"
        bad.write_bytes(data)
        with pytest.raises(ValueError, match="layout file"):
            psb.PowerSparseMatrixGPU.load(str(bad))
    with psb.PowerSparseMatrixGPU.load(str(path)) as ok:
        assert ok.MatrixNNZ() == m.nnz
