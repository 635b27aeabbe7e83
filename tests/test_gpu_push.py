"""GPU tests of ps_spmm_push (SpMM whose finished rows are also stored to peer
replicas).  On one GPU the "peers" are other buffers of the same device: every row
of C must arrive in every replica exactly as it ends in C, whichever of the three
finishing paths the row takes (the last add of the SpMM kernel, the wide-row fold,
the copy of rows without elements)."""
import numpy as np
import pytest
import torch

import powersparse_b200 as psb
from helpers import ATOL, RTOL, dense_inputs
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu


def _with_wide_and_empty_rows(seed: int) -> synth.Csr:
    """Chung-Lu rows, three rows of 2500-3500 nnz (wide rows) and every 97th row empty."""
    base = synth.chung_lu(6000, 14, 400, 2.1, seed=seed)
    rng = np.random.default_rng(seed)
    ptr, cols, vals = [0], [], []
    for r in range(base.rows):
        lo, hi = base.row_ptr[r], base.row_ptr[r + 1]
        c, v = list(base.col_ind[lo:hi]), list(base.values[lo:hi])
        if r % 97 == 5:
            c, v = [], []
        elif r % 2000 == 11:
            extra = rng.choice(base.cols, size=2500 + 500 * (r // 2000), replace=False)
            merged = dict(zip(c, v))
            for x in extra:
                merged.setdefault(int(x), float(rng.uniform(-1, 1)))
            c, v = sorted(merged), [merged[k] for k in sorted(merged)]
        cols += c
        vals += v
        ptr.append(len(cols))
    return synth.Csr(base.rows, base.cols, np.array(ptr, np.int32), np.array(cols, np.int32),
                     np.array(vals, np.float32), False)


def _matrices():
    # (matrix, SM count of the workset heuristic): one SM gives the small matrix
    # block worksets with groups of up to 256 elements, so its long rows are wide.
    return {"config2_scaled": (synth.config_matrix(2, scale=0.01), 0),
            "wide_and_empty": (_with_wide_and_empty_rows(3), 1)}


@pytest.mark.parametrize("name", ["config2_scaled", "wide_and_empty"])
@pytest.mark.parametrize("n", [32, 64, 128])
def test_every_row_reaches_every_replica(name, n):
    A, sm = _matrices()[name]
    B_host = dense_inputs(A.cols, n, 31 + n)
    expected = oracle.spmm(A.row_ptr, A.col_ind, A.values, B_host)
    with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values, sm_count=sm) as m:
        if name == "wide_and_empty":
            assert m.wide_rows == 3  # the fold path finishes these rows
        B = torch.from_numpy(B_host).cuda()
        C = torch.zeros((A.rows, n), device="cuda")
        # Replicas hold this panel at an offset, as a full replica of several panels would.
        replicas = [torch.full((A.rows + 7, n), float("nan"), device="cuda") for _ in range(3)]
        peers = [r[5:].data_ptr() for r in replicas]
        psb.SpMM_push(m, n, B, C, peers)
        torch.cuda.synchronize()
        ok = oracle.close(C.cpu().numpy(), expected, ATOL, RTOL)
        assert ok.all(), f"{(~ok).sum()} elements outside tolerance"
        for k, r in enumerate(replicas):
            assert torch.equal(r[5:5 + A.rows], C), f"replica {k} differs from C"
            assert torch.isnan(r[:5]).all() and torch.isnan(r[5 + A.rows:]).all(), "wrote outside the panel"
        # A second call without zeroing C adds into it as SpMM does (rows with a single
        # residue group are stored, the rest added); the replicas get the new rows.
        for r in replicas:
            r.fill_(float("nan"))
        psb.SpMM_push(m, n, B, C, peers)
        C_twice = torch.zeros_like(C)
        psb.SpMM(m, n, B, C_twice)
        psb.SpMM(m, n, B, C_twice)
        torch.cuda.synchronize()
        ok = oracle.close(C.cpu().numpy(), C_twice.cpu().numpy().astype(np.float64), ATOL, RTOL)
        assert ok.all(), f"{(~ok).sum()} elements differ from two plain SpMM calls"
        for k, r in enumerate(replicas):
            assert torch.equal(r[5:5 + A.rows], C), f"replica {k} differs from C after the second call"


def test_push_matches_plain_spmm_and_handles_no_peers():
    A = _with_wide_and_empty_rows(4)
    B_host = dense_inputs(A.cols, 128, 9)
    with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values, sm_count=1) as m:
        assert m.wide_rows > 0
        B = torch.from_numpy(B_host).cuda()
        C_plain = torch.zeros((A.rows, 128), device="cuda")
        psb.SpMM(m, 128, B, C_plain)
        C = torch.zeros((A.rows, 128), device="cuda")
        psb.SpMM_push(m, 128, B, C, [])
        torch.cuda.synchronize()
        ok = oracle.close(C.cpu().numpy(), C_plain.cpu().numpy().astype(np.float64), ATOL, RTOL)
        assert ok.all()


def test_push_from_two_streams_stays_ordered():
    """Eager calls on one matrix share its countdown; the library orders them."""
    A = synth.config_matrix(2, scale=0.01)
    B_host = dense_inputs(A.cols, 32, 5)
    expected = oracle.spmm(A.row_ptr, A.col_ind, A.values, B_host)
    with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values) as m:
        B = torch.from_numpy(B_host).cuda()
        streams = [torch.cuda.Stream(), torch.cuda.Stream()]
        Cs = [torch.zeros((A.rows, 32), device="cuda") for _ in streams]
        reps = [torch.full((A.rows, 32), float("nan"), device="cuda") for _ in streams]
        torch.cuda.synchronize()
        for _ in range(3):
            for s, C, r in zip(streams, Cs, reps):
                with torch.cuda.stream(s):
                    C.zero_()
                    psb.SpMM_push(m, 32, B, C, [r.data_ptr()], stream=s)
        torch.cuda.synchronize()
        for C, r in zip(Cs, reps):
            assert oracle.close(C.cpu().numpy(), expected, ATOL, RTOL).all()
            assert torch.equal(C, r)


def test_push_argument_checks():
    A = synth.config_matrix(2, scale=0.005)
    with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values) as m:
        B = torch.zeros((A.cols, 96), device="cuda")
        C = torch.zeros((A.rows, 96), device="cuda")
        with pytest.raises(ValueError, match="N must be 32, 64 or 128"):
            psb.SpMM_push(m, 96, B, C, [C.data_ptr()])
        B = torch.zeros((A.cols, 32), device="cuda")
        C = torch.zeros((A.rows, 32), device="cuda")
        with pytest.raises(ValueError, match="between 0 and 7 peers"):
            psb.SpMM_push(m, 32, B, C, [C.data_ptr()] * 8)
        with pytest.raises(ValueError, match="null peer"):
            psb.SpMM_push(m, 32, B, C, [0])
