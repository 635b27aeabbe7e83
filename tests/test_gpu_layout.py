"""GPU tests: the CUDA preprocessing builds the reference's layout bit for bit.

Compared against the reference's own golden layouts (tests/golden) and against
the oracle on further seeded cases, edge cases and forced SM counts.
"""
import hashlib

import numpy as np
import pytest

import powersparse_b200 as psb
from helpers import golden_names, layout_arrays, load_golden
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu


def _digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _build(rows, cols, rp, ci, va, sm):
    return psb.PowerSparseMatrixGPU(rows, cols, len(ci), rp, ci, va, sm_count=sm)


def _assert_same_layout(got: dict, exp: dict, tag=""):
    for key, arr in exp.items():
        g = got[key]
        assert g.shape == arr.shape, (tag, key, g.shape, arr.shape)
        if key.endswith("_val"):
            assert np.array_equal(g.view(np.uint32), arr.view(np.uint32)), (tag, key)
        else:
            assert np.array_equal(g.astype(arr.dtype), arr), (tag, key)


@pytest.mark.parametrize("name", golden_names())
def test_layout_matches_reference_golden(name):
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    with _build(rows, cols, rp, ci, va, sm) as m:
        assert m.GroupTypeNum() == int(z["S"])
        assert m.GroupFineSize() == int(z["fine"])
        assert m.GroupNum() == [int(x) for x in z["group_num"]]
        got = m.download()
    # The reference's layout arrays (the CSR position map has no reference counterpart;
    # test_csr_positions_match_the_oracle covers it).
    for key in [k for k in got if k.startswith(("ws", "res_")) and not k.endswith("_pos")]:
        if key in z.files:
            exp = z[key]
            if key.endswith("_val"):
                assert np.array_equal(got[key].view(np.uint32), exp.view(np.uint32)), key
            else:
                assert np.array_equal(got[key].astype(exp.dtype), exp), key
        else:
            assert _digest(got[key].astype(np.uint8 if key == "res_atomic" else got[key].dtype)) == \
                str(z["sha_" + key]), key


def _cases():
    edge_rp = np.array([0, 0, 40, 40, 41, 105], dtype=np.int32)  # empty, 40, empty, 1, 64
    edge_ci = np.concatenate([np.arange(40) % 7, [3], np.arange(64) % 5]).astype(np.int32)
    edge_va = np.linspace(-1, 1, len(edge_ci)).astype(np.float32)
    one_rp = np.array([0, 3000], dtype=np.int32)
    one_ci = (np.arange(3000) * 7919 % 1000).astype(np.int32)
    one_va = np.ones(3000, np.float32)
    mult_rp = (np.arange(301) * 96).astype(np.int32)  # every row 96 = 64 + 32: no residue at S=3
    mult_ci = (np.arange(300 * 96) * 31 % 500).astype(np.int32)
    mult_va = np.full(300 * 96, 0.5, np.float32)
    m4 = synth.config_matrix(4, scale=0.01)
    m3 = synth.config_matrix(3, scale=0.004)
    m2 = synth.config_matrix(2, scale=0.004)
    return {
        "edge": (5, 7, edge_rp, edge_ci, edge_va),
        "one_long_row": (1, 1000, one_rp, one_ci, one_va),
        "single_col": (4, 1, np.array([0, 1, 3, 3, 6], np.int32), np.zeros(6, np.int32),
                       np.arange(6, dtype=np.float32)),
        "no_residue": (300, 500, mult_rp, mult_ci, mult_va),
        "cfg2_small": (m2.rows, m2.cols, m2.row_ptr, m2.col_ind, m2.values),
        "cfg3_small": (m3.rows, m3.cols, m3.row_ptr, m3.col_ind, m3.values),
        "cfg4_small": (m4.rows, m4.cols, m4.row_ptr, m4.col_ind, m4.values),
    }


CASES = _cases()


@pytest.mark.parametrize("sm", [1, 3, 8, 148, 0])
@pytest.mark.parametrize("case", list(CASES))
def test_layout_matches_oracle(case, sm):
    rows, cols, rp, ci, va = CASES[case]
    with _build(rows, cols, rp, ci, va, sm) as m:
        used_sm = sm
        if sm == 0:
            import torch
            used_sm = torch.cuda.get_device_properties(0).multi_processor_count
        L = oracle.build_layout(rows, cols, rp, ci, va, used_sm)
        assert m.GroupTypeNum() == L.S
        assert m.GroupNum() == list(L.group_num)
        got = m.download()
        for s in range(L.S):
            assert m.workset_size(s) == len(L.col_ind[s])
    _assert_same_layout(got, layout_arrays(L), f"{case}/sm{sm}")
    if L.group_num[0] == 0:
        assert got["res_atomic"].size == 0


def test_empty_residue_has_null_atomic_flags():
    rows, cols, rp, ci, va = CASES["no_residue"]
    with _build(rows, cols, rp, ci, va, 1) as m:
        assert m.GroupNum()[0] == 0
        assert m.ResidueAtomic() == 0
        assert m.WorksetColInd()[0] == 0
        assert m.ResidueOffset() != 0


def test_accessor_values():
    rows, cols, rp, ci, va = CASES["cfg4_small"]
    with _build(rows, cols, rp, ci, va, 2) as m:
        assert (m.MatrixRow(), m.MatrixCol(), m.MatrixNNZ()) == (rows, cols, len(ci))
        assert m.preprocess_ms > 0
        assert all(p != 0 for p, g in zip(m.WorksetColInd(), m.GroupNum()) if g)


@pytest.mark.parametrize("name", golden_names())
def test_csr_positions_match_the_oracle(name):
    """The map back to CSR order (ps_matrix_csr_position) equals the oracle's."""
    z, rows, cols, rp, ci, va, sm = load_golden(name)
    L = oracle.build_layout(rows, cols, rp, ci, va, sm)
    with _build(rows, cols, rp, ci, va, sm) as m:
        got = m.download()
    for s in range(L.S):
        assert np.array_equal(got[f"ws{s}_pos"], L.csr_pos[s]), (name, s)


def test_preprocess_trace_reports_every_phase_and_changes_nothing(capfd, monkeypatch):
    """PSB_PREPROCESS_TRACE=1 prints one line of per-phase wall times to stderr; the
    layout built with it is the layout built without it."""
    A = synth.config_matrix(2, scale=0.01)
    monkeypatch.delenv("PSB_PREPROCESS_TRACE", raising=False)
    with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values) as m:
        plain = m.download()
    assert "psb preprocess:" not in capfd.readouterr().err
    monkeypatch.setenv("PSB_PREPROCESS_TRACE", "1")
    with psb.PowerSparseMatrixGPU(A.rows, A.cols, A.nnz, A.row_ptr, A.col_ind, A.values) as m:
        traced = m.download()
    lines = [l for l in capfd.readouterr().err.splitlines() if l.startswith("psb preprocess:")]
    assert len(lines) == 1, lines
    phases = dict(kv.split("=") for kv in lines[0].split(":", 1)[1].split())
    assert list(phases) == ["validate", "upload", "worksets", "col_freq", "freq_sort", "groups", "sig_bits_wait",
                            "signatures", "sig_sort", "residue_meta", "col_sort", "tasks"]
    assert all(float(v) >= 0.0 for v in phases.values())
    assert plain.keys() == traced.keys()
    for k in plain:
        if isinstance(plain[k], np.ndarray):
            assert np.array_equal(plain[k], traced[k]), k
        else:
            assert plain[k] == traced[k], k
