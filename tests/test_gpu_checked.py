"""GPU tests of the bounds-checked debug build (lib/libpowersparse_b200_checked.so):
every operator gives the oracle's results, and an index planted out of range in a
layout is reported as an error by the kernel's own checks (the access is not made)
while the context stays usable.  Each case runs in a fresh process that loads the
debug library through PSB_LIBRARY."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECKED = os.path.join(ROOT, "powersparse_b200", "lib", "libpowersparse_b200_checked.so")

PRELUDE = textwrap.dedent(f"""
    import sys
    sys.path.insert(0, {ROOT!r})
    import numpy as np
    import torch
    import powersparse_b200 as psb
    from oracle import oracle
    from powersparse_b200 import synth
    assert psb.load_library()._name.endswith("_checked.so")
    mtx = synth.chung_lu(4000, 20, 800, 2.1, seed=9)
    A = psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values, sm_count=1)
    assert A.GroupTypeNum() >= 3
    B = synth.dense(mtx.cols, 128, 3)
    dB = torch.from_numpy(B).cuda()
    expected = oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, B)

    def spmm():
        C = torch.zeros((mtx.rows, 128), device="cuda")
        psb.SpMM(A, 128, dB, C)
        torch.cuda.synchronize()
        return C.cpu().numpy()

    def device_ints(ptr, count):
        return torch.as_tensor(psb._CudaArrayView(ptr, count, "<i4"), device="cuda")
""")


def _run(body: str):
    env = dict(os.environ, PSB_LIBRARY=CHECKED)
    r = subprocess.run([sys.executable, "-c", PRELUDE + textwrap.dedent(body)], capture_output=True, text=True,
                       timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_checked_build_matches_the_oracle():
    out = _run("""
        assert oracle.close(spmm(), expected).all()
        X, Y = synth.dense(mtx.rows, 32, 4), synth.dense(mtx.cols, 32, 5)
        e = torch.empty(mtx.nnz, device="cuda")
        psb.SDDMM_csr(A, 32, torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda(), e)
        rows = np.repeat(np.arange(mtx.rows), np.diff(mtx.row_ptr))
        want = mtx.values.astype(np.float64) * np.einsum("ij,ij->i", X[rows].astype(np.float64),
                                                         Y[mtx.col_ind].astype(np.float64))
        torch.cuda.synchronize()
        assert oracle.close(e.cpu().numpy(), want).all()
        psb.edge_softmax_csr(A, e)
        C2 = torch.zeros((mtx.rows, 128), device="cuda")
        psb.SpMM_values(A, 128, e, dB, C2)
        torch.cuda.synchronize()
        assert oracle.close(C2.cpu().numpy(), oracle.spmm(mtx.row_ptr, mtx.col_ind, e.cpu().numpy(), B)).all()
        print("ok")
    """)
    assert "ok" in out


def test_out_of_range_indices_are_reported_not_followed():
    out = _run("""
        cols = device_ints(A.WorksetColInd()[1], A.workset_size(1))
        saved = int(cols[5].item())
        cols[5] = mtx.cols + 7                      # a column past the end of B
        try:
            spmm()
            raise SystemExit("no error for a bad column index")
        except RuntimeError as err:
            assert "column index out of range" in str(err), err
        cols[5] = saved
        des = device_ints(A.GroupDestination()[1], A.GroupNum()[1])
        saved = int(des[0].item())
        des[0] = mtx.rows + 3                       # a destination row past the end of C
        try:
            spmm()
            raise SystemExit("no error for a bad destination row")
        except RuntimeError as err:
            assert "destination row out of range" in str(err), err
        des[0] = saved
        assert oracle.close(spmm(), expected).all()  # the context is still usable
        print("ok")
    """)
    assert "ok" in out
