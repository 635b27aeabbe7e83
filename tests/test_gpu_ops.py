"""GPU tests: fused SpMM / SDDMM against the FP64 oracle and the reference's outputs.

Tolerance (the north star's): |a - e| <= 1e-5 + 1e-4 * |e| for every element,
e the FP64 oracle value (the reference's CheckSpmm / CheckSddmm,
benchmarks/benchmark.cu:64-96, at tighter constants).
"""
import numpy as np
import pytest
import torch

import powersparse_b200 as psb
from helpers import ATOL, RTOL, dense_inputs, golden_names, load_golden
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu


def _assert_close(actual, expected, tag=""):
    ok = oracle.close(actual, expected, ATOL, RTOL)
    if not ok.all():
        bad = np.argwhere(~ok.reshape(-1))[:5].ravel()
        a, e = np.asarray(actual).reshape(-1), np.asarray(expected).reshape(-1)
        raise AssertionError(f"{tag}: {int((~ok).sum())} of {ok.size} outside tolerance; "
                             f"first {[(int(i), float(a[i]), float(e[i])) for i in bad]}")


def _spmm(m, B: np.ndarray, stream=None, C0=None):
    N = B.shape[1]
    dB = torch.from_numpy(B).cuda()
    dC = torch.zeros((m.MatrixRow(), N), dtype=torch.float32, device="cuda") if C0 is None else C0
    psb.SpMM(m, N, dB, dC, stream)
    torch.cuda.synchronize()
    return dC


def _sddmm(m, X: np.ndarray, Y: np.ndarray):
    N = X.shape[1]
    outs = [torch.zeros(max(m.workset_size(s), 1), dtype=torch.float32, device="cuda")
            for s in range(m.GroupTypeNum())]
    psb.SDDMM(m, N, torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda(), outs)
    torch.cuda.synchronize()
    return [o[: m.workset_size(s)].cpu().numpy() for s, o in enumerate(outs)]


@pytest.mark.parametrize("name", golden_names())
def test_spmm_matches_oracle_and_reference(name):
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    with psb.PowerSparseMatrixGPU(rows, cols, len(ci), rp, ci, va, sm_count=sm) as m:
        for n in (32, 64, 96, 128, 256):
            B = dense_inputs(cols, n, 1000 + n)
            C = _spmm(m, B).cpu().numpy()
            _assert_close(C, oracle.spmm(rp, ci, va, B), f"{name} N={n}")
            key = f"spmm{n}"
            if key in z.files:
                assert oracle.close(C, z[key], 1e-4, 1e-4).all()
            if key + "_head" in z.files:
                assert oracle.close(C[: len(z[key + "_head"])], z[key + "_head"], 1e-4, 1e-4).all()


@pytest.mark.parametrize("name", golden_names())
def test_sddmm_matches_oracle_and_reference(name):
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    L = oracle.build_layout(rows, cols, rp, ci, va, sm)
    with psb.PowerSparseMatrixGPU(rows, cols, len(ci), rp, ci, va, sm_count=sm) as m:
        for n in (32, 128):
            X, Y = dense_inputs(rows, n, 2000 + n), dense_inputs(cols, n, 3000 + n)
            got = _sddmm(m, X, Y)
            exp = oracle.sddmm(L, X, Y)
            for s in range(L.S):
                _assert_close(got[s], exp[s], f"{name} N={n} ws{s}")
                key = f"sddmm{n}_ws{s}"
                if key in z.files:
                    assert oracle.close(got[s], z[key], 1e-4, 1e-4).all()


def _sddmm_csr_expected(rp, ci, va, X, Y):
    """FP64 out[p] = val[p] * <X[row(p)], Y[col(p)]> in CSR order."""
    rows = np.repeat(np.arange(len(rp) - 1), np.diff(rp))
    return va.astype(np.float64) * np.einsum("ij,ij->i", X[rows].astype(np.float64), Y[ci].astype(np.float64))


@pytest.mark.parametrize("name", golden_names())
def test_sddmm_csr_order_matches_oracle_and_workset_order(name):
    """SDDMM written in CSR order: within tolerance of the FP64 product and, bit for bit,
    the workset-order result moved through the CSR position map."""
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    with psb.PowerSparseMatrixGPU(rows, cols, len(ci), rp, ci, va, sm_count=sm) as m:
        pos = m.download()
        for n in (32, 128):
            X, Y = dense_inputs(rows, n, 4000 + n), dense_inputs(cols, n, 5000 + n)
            out = torch.full((len(ci),), float("nan"), device="cuda")
            psb.SDDMM_csr(m, n, torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda(), out)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            _assert_close(got, _sddmm_csr_expected(rp, ci, va, X, Y), f"{name} N={n}")
            ws = _sddmm(m, X, Y)
            moved = np.full(len(ci), np.nan, dtype=np.float32)
            for s in range(m.GroupTypeNum()):
                moved[pos[f"ws{s}_pos"]] = ws[s]
            # + 0 folds -0.0 into +0.0: residue outputs are added into zeros there.
            assert np.array_equal((got + np.float32(0)).view(np.uint32),
                                  (moved + np.float32(0)).view(np.uint32)), f"{name} N={n}"


@pytest.mark.parametrize("cfg,scale", [(2, 0.004), (3, 0.004), (4, 0.01)])
@pytest.mark.parametrize("sm", [1, 148])
def test_ops_on_scaled_configs(cfg, scale, sm):
    mtx = synth.config_matrix(cfg, scale=scale)
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values,
                                  sm_count=sm) as m:
        for n in (32, 128):
            B = synth.dense(mtx.cols, n, 100 + cfg)
            _assert_close(_spmm(m, B).cpu().numpy(), oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, B),
                          f"cfg{cfg} spmm N={n}")
        L = oracle.build_layout(mtx.rows, mtx.cols, mtx.row_ptr, mtx.col_ind, mtx.values, sm)
        for n in (32, 128):
            X, Y = synth.dense(mtx.rows, n, 200 + cfg), synth.dense(mtx.cols, n, 300 + cfg)
            got, exp = _sddmm(m, X, Y), oracle.sddmm(L, X, Y)
            for s in range(L.S):
                _assert_close(got[s], exp[s], f"cfg{cfg} sddmm N={n} ws{s}")


def test_spmm_accumulates_like_the_reference_when_not_zeroed():
    """Rows whose groups add atomically accumulate; single-group residue rows are stored
    (spmm_kernel_residue.cu:68-81), so a second call without zeroing doubles only the former."""
    mtx = synth.chung_lu(3000, 14, 600, 2.1, seed=7)
    L = oracle.build_layout(mtx.rows, mtx.cols, mtx.row_ptr, mtx.col_ind, mtx.values, 1)
    stored = np.zeros(mtx.rows, dtype=bool)
    for g in range(L.group_num[0]):
        if not L.residue_atomic[g]:
            stored[L.group_des[0][g]] = True
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values,
                                  sm_count=1) as m:
        B = dense_inputs(mtx.cols, 32, 5)
        C = _spmm(m, B)
        once = C.cpu().numpy().copy()
        psb.SpMM(m, 32, torch.from_numpy(B).cuda(), C)
        torch.cuda.synchronize()
        twice = C.cpu().numpy()
    assert stored.any() and (~stored).any()
    _assert_close(twice[stored], once[stored], "stored rows")
    _assert_close(twice[~stored], 2 * once[~stored].astype(np.float64), "atomic rows")


def _heavy_rows_matrix(seed: int):
    """Light Chung-Lu rows plus four rows of 2100-3600 nnz (wide rows: >= 8 block slices)."""
    base = synth.chung_lu(4000, 12, 300, 2.1, seed=seed)
    rng = np.random.default_rng(seed)
    rows, ptr, cols, vals = [], [0], [], []
    for r in range(base.rows):
        lo, hi = base.row_ptr[r], base.row_ptr[r + 1]
        c, v = list(base.col_ind[lo:hi]), list(base.values[lo:hi])
        if r % 1000 == 3:
            extra = rng.choice(base.cols, size=2100 + 500 * (r // 1000), replace=False)
            merged = dict(zip(c, v))
            for x in extra:
                merged.setdefault(int(x), float(rng.uniform(-1, 1)))
            c, v = sorted(merged), [merged[k] for k in sorted(merged)]
        cols += c
        vals += v
        ptr.append(len(cols))
    return synth.Csr(base.rows, base.cols, np.array(ptr, np.int32), np.array(cols, np.int32),
                     np.array(vals, np.float32), False)


def test_spmm_wide_rows_sum_in_fp64():
    """Wide rows go through the FP64 scratch: results match the oracle at both task orders
    (N = 32 and 128), a second call without zeroing C doubles them (the scratch is zero
    again after each call), and growing N reallocates the scratch."""
    mtx = _heavy_rows_matrix(21)
    L = oracle.build_layout(mtx.rows, mtx.cols, mtx.row_ptr, mtx.col_ind, mtx.values, 1)
    stored = np.zeros(mtx.rows, dtype=bool)  # single-group residue rows are stored, not added
    for g in range(L.group_num[0]):
        if not L.residue_atomic[g]:
            stored[L.group_des[0][g]] = True
    exp = {}
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values,
                                  sm_count=1) as m:
        assert m.wide_rows == 4
        for n in (32, 128, 32, 256):
            B = synth.dense(mtx.cols, n, 40 + n)
            if n not in exp:
                exp[n] = oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, B)
            C = _spmm(m, B)
            _assert_close(C.cpu().numpy(), exp[n], f"N={n}")
            psb.SpMM(m, n, torch.from_numpy(B).cuda(), C)
            torch.cuda.synchronize()
            twice = np.where(stored[:, None], exp[n], 2 * exp[n])
            _assert_close(C.cpu().numpy(), twice, f"N={n} twice")


def test_spmm_wide_rows_from_two_streams():
    """Two SpMM calls on one matrix with wide rows, issued on two streams without a
    host sync in between: the matrix's FP64 scratch is shared, and the calls are
    ordered on the device, so both results are right."""
    mtx = _heavy_rows_matrix(22)
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values,
                                  sm_count=1) as m:
        assert m.wide_rows > 0
        Bs = [synth.dense(mtx.cols, 128, 60 + k) for k in range(2)]
        dB = [torch.from_numpy(b).cuda() for b in Bs]
        dC = [torch.zeros((mtx.rows, 128), device="cuda") for _ in range(2)]
        streams = [torch.cuda.Stream(), torch.cuda.Stream()]
        torch.cuda.synchronize()
        for _ in range(3):
            for k in range(2):
                dC[k].zero_()
                torch.cuda.synchronize()
                psb.SpMM(m, 128, dB[k], dC[k], streams[k])
                psb.SpMM(m, 128, dB[k], dC[k], streams[1 - k])
            torch.cuda.synchronize()
        for k in range(2):
            exp = oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, Bs[k])
            L = oracle.build_layout(mtx.rows, mtx.cols, mtx.row_ptr, mtx.col_ind, mtx.values, 1)
            stored = np.zeros(mtx.rows, dtype=bool)
            for g in range(L.group_num[0]):
                if not L.residue_atomic[g]:
                    stored[L.group_des[0][g]] = True
            _assert_close(dC[k].cpu().numpy(), np.where(stored[:, None], exp, 2 * exp), f"stream {k}")


def test_spmm_on_a_side_stream():
    mtx = synth.chung_lu(2000, 20, 400, 2.1, seed=12)
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values,
                                  sm_count=2) as m:
        B = dense_inputs(mtx.cols, 128, 6)
        s = torch.cuda.Stream()
        dB = torch.from_numpy(B).cuda()
        dC = torch.zeros((mtx.rows, 128), device="cuda")
        torch.cuda.synchronize()
        psb.SpMM(m, 128, dB, dC, s)
        s.synchronize()
        _assert_close(dC.cpu().numpy(), oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, B), "side stream")


def test_operator_errors_match_the_reference():
    mtx = synth.chung_lu(500, 10, 100, 2.1, seed=13)
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values) as m:
        B = torch.zeros((mtx.cols, 64), device="cuda")
        C = torch.zeros((mtx.rows, 64), device="cuda")
        with pytest.raises(ValueError, match="positive multiple of 32"):
            psb.SpMM(m, 48, B, C)
        with pytest.raises(ValueError, match="positive multiple of 32"):
            psb.SpMM(m, 0, B, C)
        with pytest.raises(ValueError, match="Invalid SpMM buffers"):
            psb.SpMM(m, 64, 0, C)
        outs = [torch.zeros(max(m.workset_size(s), 1), device="cuda") for s in range(m.GroupTypeNum())]
        with pytest.raises(ValueError, match="N=32 or N=128"):
            psb.SDDMM(m, 64, B, B, outs)
        bad = list(outs)
        bad[0] = 0
        with pytest.raises(ValueError, match="Missing SDDMM output workset"):
            psb.SDDMM(m, 32, torch.zeros((mtx.rows, 32), device="cuda"), torch.zeros((mtx.cols, 32), device="cuda"),
                      bad)


def test_spmm_large_n_uses_several_slabs():
    mtx = synth.chung_lu(1500, 16, 300, 2.1, seed=14)
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values,
                                  sm_count=1) as m:
        for n in (160, 384, 1024):
            B = dense_inputs(mtx.cols, n, n)
            _assert_close(_spmm(m, B).cpu().numpy(), oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, B), f"N={n}")


def test_spmm_graph_capture_keeps_its_scratch_when_a_larger_n_grows_it():
    """A CUDA graph captured around SpMM on a matrix with wide rows holds the matrix's
    FP64 scratch of that N.  A later eager call at a larger N allocates a larger
    scratch; the captured one stays allocated (retired, freed with the matrix), so
    replays of the graph still give the oracle's result.  Capturing the first call at
    a new N is refused (it would allocate inside the capture)."""
    mtx = _heavy_rows_matrix(23)
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values,
                                  sm_count=1) as m:
        assert m.wide_rows > 0
        B32 = synth.dense(mtx.cols, 32, 71)
        exp32 = oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, B32)
        dB32 = torch.from_numpy(B32).cuda()
        C32 = torch.zeros((mtx.rows, 32), device="cuda")
        psb.SpMM(m, 32, dB32, C32)  # eager call at N=32 sizes the scratch
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            C32.zero_()
            psb.SpMM(m, 32, dB32, C32, torch.cuda.current_stream())
        B128 = synth.dense(mtx.cols, 128, 72)
        C128 = torch.zeros((mtx.rows, 128), device="cuda")
        psb.SpMM(m, 128, torch.from_numpy(B128).cuda(), C128)  # grows the scratch
        torch.cuda.synchronize()
        _assert_close(C128.cpu().numpy(), oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, B128), "eager N=128")
        for replay in range(2):
            C32.fill_(7.0)
            g.replay()
            torch.cuda.synchronize()
            _assert_close(C32.cpu().numpy(), exp32, f"replay {replay}")
        del g
        C256 = torch.zeros((mtx.rows, 256), device="cuda")
        B256 = torch.zeros((mtx.cols, 256), device="cuda")
        g2 = torch.cuda.CUDAGraph()
        with pytest.raises(RuntimeError, match="cannot be captured"):
            with torch.cuda.graph(g2):
                psb.SpMM(m, 256, B256, C256, torch.cuda.current_stream())
        torch.cuda.synchronize()


def test_spmm_rows_longer_than_65536_use_exact_products():
    """Two rows of ~70k and ~120k nonzeros (at least 256 block slices: the exact FP64
    product path) next to light rows and a wide row of ~3k (the compensated FP32 path):
    every output within tolerance of the FP64 oracle, at N = 32 and 128."""
    base = synth.chung_lu(3000, 12, 300, 2.1, seed=24)
    rng = np.random.default_rng(24)
    cols = 200_000
    ptr, col, val = [0], [], []
    for r in range(base.rows):
        lo, hi = base.row_ptr[r], base.row_ptr[r + 1]
        c, v = list(base.col_ind[lo:hi]), list(base.values[lo:hi])
        k = {5: 70_000, 1500: 120_000, 2500: 3_000}.get(r, 0)
        if k:
            c = np.sort(rng.choice(cols, size=k, replace=False)).tolist()
            v = rng.uniform(0, 1, size=k).astype(np.float32).tolist()
        col += c
        val += v
        ptr.append(len(col))
    mtx = synth.Csr(base.rows, cols, np.array(ptr, np.int32), np.array(col, np.int32), np.array(val, np.float32),
                    False)
    with psb.PowerSparseMatrixGPU(mtx.rows, mtx.cols, mtx.nnz, mtx.row_ptr, mtx.col_ind, mtx.values,
                                  sm_count=1) as m:
        assert m.wide_rows >= 3
        for n in (32, 128):
            B = synth.dense(mtx.cols, n, 80 + n)
            _assert_close(_spmm(m, B).cpu().numpy(), oracle.spmm(mtx.row_ptr, mtx.col_ind, mtx.values, B),
                          f"N={n}")
