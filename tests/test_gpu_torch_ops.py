"""GPU tests: torch.ops.powersparse.* give the results of the direct entry points."""
import numpy as np
import pytest
import torch

import powersparse_b200 as psb
import powersparse_b200.torch_ops  # noqa: F401
from helpers import ATOL, RTOL
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def graph():
    m = synth.chung_lu(3000, 16, 500, 2.1, seed=17)
    A = psb.PowerSparseMatrixGPU(m.rows, m.cols, m.nnz, m.row_ptr, m.col_ind, m.values, sm_count=2)
    yield m, A
    A.close()


def test_spmm_ops(graph):
    m, A = graph
    for n in (32, 128):
        B = torch.from_numpy(synth.dense(m.cols, n, n)).cuda()
        C = torch.ops.powersparse.spmm(A.handle, B)
        C2 = torch.zeros((m.rows, n), device="cuda")
        torch.ops.powersparse.spmm_(A.handle, B, C2)
        torch.cuda.synchronize()
        exp = oracle.spmm(m.row_ptr, m.col_ind, m.values, B.cpu().numpy())
        assert oracle.close(C.cpu().numpy(), exp, ATOL, RTOL).all()
        assert oracle.close(C2.cpu().numpy(), exp, ATOL, RTOL).all()


def test_sddmm_ops(graph):
    m, A = graph
    for n in (32, 128):
        X = torch.from_numpy(synth.dense(m.rows, n, 3 * n)).cuda()
        Y = torch.from_numpy(synth.dense(m.cols, n, 5 * n)).cuda()
        e = torch.ops.powersparse.sddmm_csr(A.handle, X, Y)
        ref = torch.empty(m.nnz, device="cuda")
        psb.SDDMM_csr(A, n, X, Y, ref)
        outs = [torch.zeros(max(A.workset_size(s), 1), device="cuda") for s in range(A.GroupTypeNum())]
        torch.ops.powersparse.sddmm_(A.handle, X, Y, outs)
        outs2 = [torch.zeros_like(o) for o in outs]
        psb.SDDMM(A, n, X, Y, outs2)
        torch.cuda.synchronize()
        assert torch.equal(e, ref)
        for a, b in zip(outs, outs2):
            assert torch.equal(a, b)


def test_opcheck(graph):
    m, A = graph
    B = torch.from_numpy(synth.dense(m.cols, 32, 9)).cuda()
    X = torch.from_numpy(synth.dense(m.rows, 32, 10)).cuda()
    torch.library.opcheck(torch.ops.powersparse.spmm.default, (A.handle, B),
                          test_utils=("test_schema", "test_faketensor"))
    torch.library.opcheck(torch.ops.powersparse.sddmm_csr.default, (A.handle, X, B),
                          test_utils=("test_schema", "test_faketensor"))
