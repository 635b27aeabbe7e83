"""GPU parity at a benchmark configuration's full size (configuration 2: 2.45M rows,
~61.9M nnz): the GPU layout against the oracle bit for bit, SpMM and SDDMM against
the FP64 oracle at the north-star tolerance, plus size-independent properties
(the layout is a permutation of the CSR; SpMM is linear in B)."""
import numpy as np
import pytest
import torch

import powersparse_b200 as psb
from helpers import ATOL, RTOL, layout_arrays
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cfg2():
    m = synth.config_matrix(2)
    A = psb.PowerSparseMatrixGPU(m.rows, m.cols, m.nnz, m.row_ptr, m.col_ind, m.values)
    yield m, A
    A.close()


def test_full_size_layout_is_bit_exact(cfg2):
    m, A = cfg2
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    L = oracle.build_layout(m.rows, m.cols, m.row_ptr, m.col_ind, m.values, sm)
    assert A.GroupTypeNum() == L.S and A.GroupNum() == list(L.group_num)
    got = A.download()
    for key, arr in layout_arrays(L).items():
        g = got[key]
        assert g.shape == arr.shape, key
        if key.endswith("_val"):
            assert np.array_equal(g.view(np.uint32), arr.view(np.uint32)), key
        else:
            assert np.array_equal(g.astype(arr.dtype), arr), key


def test_full_size_spmm_matches_oracle(cfg2):
    m, A = cfg2
    for n in (32, 128):
        B = synth.dense(m.cols, n, 102)
        C = torch.zeros((m.rows, n), device="cuda")
        psb.SpMM(A, n, torch.from_numpy(B).cuda(), C)
        torch.cuda.synchronize()
        ok = oracle.close(C.cpu().numpy(), oracle.spmm(m.row_ptr, m.col_ind, m.values, B), ATOL, RTOL)
        assert ok.all(), f"N={n}: {int((~ok).sum())} elements outside tolerance"


def test_full_size_sddmm_matches_oracle(cfg2):
    m, A = cfg2
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    L = oracle.build_layout(m.rows, m.cols, m.row_ptr, m.col_ind, m.values, sm)
    for n in (32, 128):
        X, Y = synth.dense(m.rows, n, 202), synth.dense(m.cols, n, 302)
        outs = [torch.zeros(max(A.workset_size(s), 1), device="cuda") for s in range(A.GroupTypeNum())]
        psb.SDDMM(A, n, torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda(), outs)
        torch.cuda.synchronize()
        exp = oracle.sddmm(L, X, Y)
        for s in range(L.S):
            ok = oracle.close(outs[s][: A.workset_size(s)].cpu().numpy(), exp[s], ATOL, RTOL)
            assert ok.all(), f"N={n} workset {s}: {int((~ok).sum())} elements outside tolerance"


def test_full_size_spmm_is_linear(cfg2):
    """A(B1 + 2 B2) = A B1 + 2 A B2 (FP32 on both sides, tolerance scaled to the terms)."""
    m, A = cfg2
    g = torch.Generator(device="cuda").manual_seed(7)
    B1 = torch.rand((m.cols, 128), generator=g, device="cuda") * 2 - 1
    B2 = torch.rand((m.cols, 128), generator=g, device="cuda") * 2 - 1
    out = []
    for B in (B1, B2, B1 + 2 * B2):
        C = torch.zeros((m.rows, 128), device="cuda")
        psb.SpMM(A, 128, B, C)
        out.append(C)
    torch.cuda.synchronize()
    lhs, rhs = out[2], out[0] + 2 * out[1]
    scale = out[0].abs() + 2 * out[1].abs() + 1.0
    assert torch.all((lhs - rhs).abs() <= 1e-4 * scale)


def test_full_size_sddmm_csr_order_is_the_permuted_workset_order(cfg2):
    """CSR-order SDDMM equals the workset-order result moved through the position map,
    bit for bit, and the map is a permutation of [0, nnz)."""
    m, A = cfg2
    pos = [torch.as_tensor(psb._CudaArrayView(A.CsrPosition()[s], A.workset_size(s), "<i4"), device="cuda")
           for s in range(A.GroupTypeNum())]
    allpos = torch.cat(pos)
    assert torch.equal(torch.sort(allpos.long()).values, torch.arange(m.nnz, device="cuda"))
    for n in (32, 128):
        g = torch.Generator(device="cuda").manual_seed(n)
        X = torch.rand((m.rows, n), generator=g, device="cuda")
        Y = torch.rand((m.cols, n), generator=g, device="cuda")
        out = torch.empty(m.nnz, device="cuda")
        psb.SDDMM_csr(A, n, X, Y, out)
        outs = [torch.zeros(max(A.workset_size(s), 1), device="cuda") for s in range(A.GroupTypeNum())]
        psb.SDDMM(A, n, X, Y, outs)
        moved = torch.empty(m.nnz, device="cuda")
        for s in range(A.GroupTypeNum()):
            moved[pos[s].long()] = outs[s][: A.workset_size(s)]
        torch.cuda.synchronize()
        # + 0 folds -0.0 into +0.0: residue outputs are added into zeros there.
        assert torch.equal((out + 0).view(torch.int32), (moved + 0).view(torch.int32)), f"N={n}"
