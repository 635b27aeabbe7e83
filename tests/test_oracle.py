"""CPU tests: the oracle against the reference's own golden outputs, and its host logic.

The fixtures under tests/golden/ were produced by running the reference
(built from its sources) on a B200; see tests/golden/make_golden.py.
"""
import hashlib

import numpy as np
import pytest

from helpers import ATOL, RTOL, dense_inputs, golden_names, layout_arrays, load_golden
from oracle import oracle
from powersparse_b200 import synth


def _digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", golden_names())
def test_oracle_layout_matches_reference_bit_exact(name):
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    L = oracle.build_layout(rows, cols, rp, ci, va, sm)
    assert L.S == int(z["S"])
    assert L.fine == int(z["fine"])
    assert list(L.group_num) == [int(x) for x in z["group_num"]]
    for key, arr in layout_arrays(L).items():
        if key in z.files:
            assert arr.dtype == z[key].dtype or key == "res_atomic"
            assert np.array_equal(arr, z[key]), key
        else:
            assert _digest(arr) == str(z["sha_" + key]), key


@pytest.mark.parametrize("name", golden_names())
def test_oracle_results_match_reference(name):
    """The reference's FP32 outputs agree with the FP64 oracle at the north-star tolerance."""
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    L = oracle.build_layout(rows, cols, rp, ci, va, sm)
    checked = 0
    for k in z.files:
        if k.startswith("spmm"):
            n = int(k[4:].split("_")[0])
            C = oracle.spmm(rp, ci, va, dense_inputs(cols, n, 1000 + n))
            if k.endswith("_head"):
                exp = C[: len(z[k])]
            elif k.endswith("_rowsum") or k.endswith("_sum"):
                exp = C.sum(axis=1)
            else:
                exp = C
            ref = z[k]
            tol = 1e-3 if (k.endswith("sum")) else ATOL
            assert oracle.close(ref, exp, tol, RTOL).all(), k
            checked += 1
        elif k.startswith("sddmm") and "_ws" in k and not k.endswith("_sum"):
            n = int(k[5:].split("_")[0])
            s = int(k.split("_ws")[1])
            outs = oracle.sddmm(L, dense_inputs(rows, n, 2000 + n), dense_inputs(cols, n, 3000 + n))
            assert oracle.close(z[k], outs[s], ATOL, RTOL).all(), k
            checked += 1
    assert checked > 0


def test_oracle_spmm_matches_dense_product():
    m = synth.chung_lu(500, 10, 100, 2.1, seed=3)
    B = dense_inputs(m.cols, 32, 9)
    A = np.zeros((m.rows, m.cols))
    for r in range(m.rows):
        for p in range(m.row_ptr[r], m.row_ptr[r + 1]):
            A[r, m.col_ind[p]] += m.values[p]
    np.testing.assert_allclose(oracle.spmm(m.row_ptr, m.col_ind, m.values, B), A @ B.astype(np.float64),
                               rtol=1e-12, atol=1e-12)


def test_oracle_sddmm_workset_order_covers_every_element():
    m = synth.chung_lu(800, 12, 200, 2.1, seed=4)
    L = oracle.build_layout(m.rows, m.cols, m.row_ptr, m.col_ind, m.values, 1)
    X, Y = dense_inputs(m.rows, 32, 1), dense_inputs(m.cols, 32, 2)
    outs = oracle.sddmm(L, X, Y)
    got = []
    for s in range(L.S):
        off = L.offsets(s)
        for g in range(L.group_num[s]):
            r = L.group_des[s][g]
            for p in range(off[g], off[g + 1]):
                c = L.col_ind[s][p]
                got.append((r, c, L.sp_data[s][p], outs[s][p]))
    assert len(got) == m.nnz
    for r, c, v, o in got[:2000]:
        assert abs(o - float(v) * float(np.dot(X[r].astype(np.float64), Y[c]))) < 1e-9


@pytest.mark.parametrize("sm", [1, 2, 4, 148])
def test_oracle_layout_is_a_permutation_of_the_csr(sm):
    """The reference's own CHECK=1 preprocessing check (benchmarks/benchmark.cu:45-62)."""
    m = synth.chung_lu(2000, 20, 400, 2.1, seed=5)
    L = oracle.build_layout(m.rows, m.cols, m.row_ptr, m.col_ind, m.values, sm)
    got = []
    for s in range(L.S):
        off = L.offsets(s)
        rows = np.repeat(L.group_des[s], np.diff(off))
        got.append(np.stack([rows, L.col_ind[s], L.sp_data[s].view(np.int32)], 1))
    got = np.concatenate(got)
    exp = np.stack([np.repeat(np.arange(m.rows), np.diff(m.row_ptr)), m.col_ind, m.values.view(np.int32)], 1)
    assert np.array_equal(np.unique(got, axis=0, return_counts=True)[1].sum(), m.nnz)
    assert np.array_equal(got[np.lexsort(got.T[::-1])], exp[np.lexsort(exp.T[::-1])])


@pytest.mark.parametrize("name", golden_names())
def test_oracle_csr_positions_map_back_to_the_csr(name):
    """csr_pos is a permutation of [0, nnz) and every element reads its CSR entry:
    same row (the group's destination), same column, same value bits."""
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    L = oracle.build_layout(rows, cols, rp, ci, va, sm)
    pos = np.concatenate([L.csr_pos[s] for s in range(L.S)])
    assert np.array_equal(np.sort(pos), np.arange(len(ci)))
    row_of = np.repeat(np.arange(rows), np.diff(rp))
    for s in range(L.S):
        p = L.csr_pos[s]
        assert np.array_equal(ci[p], L.col_ind[s]), s
        assert np.array_equal(va[p].view(np.uint32), L.sp_data[s].view(np.uint32)), s
        assert np.array_equal(row_of[p], np.repeat(L.group_des[s], np.diff(L.offsets(s)))), s


def test_oracle_rejects_invalid_csr_like_the_reference():
    rp = np.array([0, 1, 2], dtype=np.int32)
    with pytest.raises(ValueError, match="nonempty CSR"):
        oracle.build_layout(0, 2, rp, [0, 1], [1.0, 1.0], 148)
    with pytest.raises(ValueError, match="row-pointer endpoints"):
        oracle.build_layout(2, 2, np.array([0, 1, 3], np.int32), [0, 1], [1.0, 1.0], 148)
    with pytest.raises(ValueError, match="nondecreasing"):
        oracle.build_layout(3, 2, np.array([0, 2, 1, 2], np.int32), [0, 1], [1.0, 1.0], 148)
    with pytest.raises(ValueError, match="column index or sparse value"):
        oracle.build_layout(2, 2, rp, [0, 2], [1.0, 1.0], 148)
    with pytest.raises(ValueError, match="column index or sparse value"):
        oracle.build_layout(2, 2, rp, [0, 1], [1.0, np.nan], 148)


def test_workset_count_follows_sm_threshold():
    """S = 1 + number of consecutive sizes 32, 64, ... with >= 32*SMs floor-groups."""
    rows = 100
    rp = np.arange(rows + 1, dtype=np.int32) * 100  # every row has 100 nnz
    # floor(100/32)=3 -> 300 groups; /64 -> 100; /128 -> 0
    assert oracle.analyze(rp, 1) == 3       # threshold 32: 300 >= 32, 100 >= 32, 0 < 32
    assert oracle.analyze(rp, 4) == 2       # threshold 128: 300 >= 128, 100 < 128
    assert oracle.analyze(rp, 10) == 1      # threshold 320: 300 < 320
    assert oracle.analyze(rp, 148) == 1


def test_config1_generator_shape():
    m = synth.config_matrix(1)
    assert (m.rows, m.cols, m.nnz) == (4096, 4096, 65536)
    lens = m.row_lengths()
    assert (lens == 16).all()
    for r in range(0, 4096, 97):
        cols = m.col_ind[m.row_ptr[r]:m.row_ptr[r + 1]]
        assert len(np.unique(cols)) == 16 and (np.diff(cols) > 0).all()
    assert m.values.min() >= -1 and m.values.max() <= 1


def test_mtx_roundtrip_is_canonical(tmp_path):
    """A symmetric canonical .mtx expands to the same CSR the generator returns."""
    m = synth.chung_lu(300, 6, 60, 2.1, seed=8)
    p = tmp_path / "m.mtx"
    synth.write_mtx(str(p), m)
    lines = p.read_text().splitlines()
    assert lines[0] == "%%MatrixMarket matrix coordinate real symmetric"
    rows, cols, entries = map(int, lines[1].split())
    r_list, c_list, v_list = [], [], []
    for ln in lines[2:]:
        a, b, v = ln.split()
        a, b = int(a) - 1, int(b) - 1
        r_list.append(a); c_list.append(b); v_list.append(np.float32(float(v)))
        if a != b:
            r_list.append(b); c_list.append(a); v_list.append(np.float32(float(v)))
    # two-pass reader semantics: stable bucket by row in file order
    order = np.argsort(np.array(r_list), kind="stable")
    assert np.array_equal(np.array(c_list)[order], m.col_ind)
    assert np.array_equal(np.array(v_list, dtype=np.float32)[order], m.values)


def test_csr_binary_roundtrip(tmp_path):
    m = synth.chung_lu(200, 5, 40, 2.1, seed=9)
    p = str(tmp_path / "m.csr")
    synth.write_csr_bin(p, m)
    r = synth.read_csr_bin(p)
    assert (r.rows, r.cols) == (m.rows, m.cols)
    assert np.array_equal(r.row_ptr, m.row_ptr) and np.array_equal(r.col_ind, m.col_ind)
    assert np.array_equal(r.values, m.values)
