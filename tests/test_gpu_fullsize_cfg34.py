"""GPU parity at full size for benchmark configurations 3 and 4.

Configuration 3: symmetric Chung-Lu gamma 2.0, 1.57M rows, ~254M nnz (rows up to
~40k nnz, nine worksets at 148 SMs: the FP64 wide-row sums and the deepest radix
keys run here).  Configuration 4: lognormal degrees, 233k rows, ~112M nnz (long
rows).  Both graphs come from the GPU generator (powersparse_b200.synth_gpu) with
the configuration's parameters.  Checked: the GPU layout against the oracle bit for
bit, SpMM and SDDMM (workset order and CSR order) at N = 32 and 128 against the FP64
oracle at |a - e| <= 1e-5 + 1e-4 |e|.
"""
import numpy as np
import pytest
import torch

import powersparse_b200 as psb
from helpers import ATOL, RTOL, layout_arrays
from oracle import oracle
from powersparse_b200 import synth, synth_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=[3, 4], ids=["cfg3", "cfg4"])
def full(request):
    m = synth_gpu.config_matrix(request.param, device="cuda")
    torch.cuda.empty_cache()
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    L = oracle.build_layout(m.rows, m.cols, m.row_ptr, m.col_ind, m.values, sm)
    A = psb.PowerSparseMatrixGPU(m.rows, m.cols, m.nnz, m.row_ptr, m.col_ind, m.values)
    yield request.param, m, L, A
    A.close()


def _assert_close(actual, expected, tag):
    ok = oracle.close(actual, expected, ATOL, RTOL)
    if not ok.all():
        bad = np.argwhere(~ok)[:5]
        where = "; ".join(f"{tuple(int(i) for i in ix)}: got {float(actual[tuple(ix)]):.9g} "
                          f"want {float(expected[tuple(ix)]):.9g}" for ix in bad)
        raise AssertionError(f"{tag}: {int((~ok).sum())} of {ok.size} elements outside tolerance ({where})")


def test_layout_is_bit_exact(full):
    cfg, m, L, A = full
    assert m.nnz > (200_000_000 if cfg == 3 else 100_000_000)
    assert A.GroupTypeNum() == L.S and A.GroupNum() == list(L.group_num)
    got = A.download()
    for key, arr in layout_arrays(L).items():
        g = got[key]
        assert g.shape == arr.shape, f"cfg{cfg} {key}"
        if key.endswith("_val"):
            assert np.array_equal(g.view(np.uint32), arr.view(np.uint32)), f"cfg{cfg} {key}"
        else:
            assert np.array_equal(g.astype(arr.dtype), arr), f"cfg{cfg} {key}"


@pytest.mark.parametrize("n", [32, 128])
def test_spmm_matches_oracle(full, n):
    cfg, m, L, A = full
    B = synth.dense(m.cols, n, 400 + n)
    C = torch.zeros((m.rows, n), device="cuda")
    psb.SpMM(A, n, torch.from_numpy(B).cuda(), C)
    torch.cuda.synchronize()
    _assert_close(C.cpu().numpy(), oracle.spmm(m.row_ptr, m.col_ind, m.values, B), f"cfg{cfg} SpMM N={n}")


@pytest.mark.parametrize("n", [32, 128])
def test_sddmm_matches_oracle(full, n):
    cfg, m, L, A = full
    X, Y = synth.dense(m.rows, n, 500 + n), synth.dense(m.cols, n, 600 + n)
    dX, dY = torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda()
    outs = [torch.zeros(max(A.workset_size(s), 1), device="cuda") for s in range(A.GroupTypeNum())]
    psb.SDDMM(A, n, dX, dY, outs)
    csr = torch.empty(m.nnz, device="cuda")
    psb.SDDMM_csr(A, n, dX, dY, csr)
    torch.cuda.synchronize()
    exp = oracle.sddmm(L, X, Y)
    for s in range(L.S):
        _assert_close(outs[s][: A.workset_size(s)].cpu().numpy(), exp[s], f"cfg{cfg} SDDMM N={n} workset {s}")
    moved = np.empty(m.nnz, dtype=np.float64)
    for s in range(L.S):
        moved[L.csr_pos[s]] = exp[s]
    _assert_close(csr.cpu().numpy(), moved, f"cfg{cfg} SDDMM N={n} CSR order")
