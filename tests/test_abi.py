"""CPU tests of the C ABI surface: the library loads, exports every declared entry
point, and its host-side logic and argument checks work without a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

import powersparse_b200 as psb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "powersparse_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ps_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_operator_surface():
    syms = declared_symbols()
    for s in ("ps_matrix_create", "ps_matrix_destroy", "ps_spmm", "ps_sddmm", "ps_partition_rows",
              "ps_matrix_workset_col_ind", "ps_matrix_residue_atomic", "ps_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = psb.load_library()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_bounds_checked_library_exports_every_declared_symbol():
    """The debug build (bounds-checked kernels) is a drop-in for the release library."""
    path = os.path.join(ROOT, "powersparse_b200", "lib", "libpowersparse_b200_checked.so")
    lib = ctypes.CDLL(path)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    bound = {name for name, _, _ in psb._SIGNATURES}
    assert set(declared_symbols()) <= bound


def test_version_string():
    assert b"sm_100a" in psb.load_library().ps_version()


def test_matrix_create_rejects_invalid_csr_without_touching_the_gpu():
    with pytest.raises(ValueError, match="nonempty CSR"):
        psb.PowerSparseMatrixGPU(0, 3, 0, np.zeros(1, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32))
    with pytest.raises(ValueError, match="row-pointer endpoints"):
        psb.PowerSparseMatrixGPU(2, 3, 2, np.array([0, 1, 1]), np.array([0, 1]), np.array([1.0, 2.0]))
    with pytest.raises(ValueError, match="nondecreasing"):
        psb.PowerSparseMatrixGPU(2, 3, 2, np.array([0, 3, 2]), np.array([0, 1]), np.array([1.0, 2.0]))
    with pytest.raises(ValueError, match="column index or sparse value"):
        psb.PowerSparseMatrixGPU(2, 3, 2, np.array([0, 1, 2]), np.array([0, 3]), np.array([1.0, 2.0]))
    with pytest.raises(ValueError, match="column index or sparse value"):
        psb.PowerSparseMatrixGPU(2, 3, 2, np.array([0, 1, 2]), np.array([0, 1]), np.array([1.0, np.inf]))


def test_operator_argument_checks_without_a_gpu():
    lib = psb.load_library()
    assert lib.ps_spmm(None, 32, None, None, None) == psb.PS_ERR_INVALID_ARGUMENT
    assert lib.ps_sddmm(None, 64, None, None, None, None) == psb.PS_ERR_INVALID_ARGUMENT
    assert b"N=32 or N=128" in lib.ps_last_error()
    assert lib.ps_sddmm(None, 32, None, None, None, None) == psb.PS_ERR_INVALID_ARGUMENT
    out = ctypes.c_void_p()
    assert lib.ps_matrix_create(1, 1, 1, None, None, None, ctypes.byref(out)) == psb.PS_ERR_INVALID_ARGUMENT
    assert out.value is None


@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8])
def test_partition_rows_balances_nnz(parts):
    rng = np.random.default_rng(parts)
    lens = rng.zipf(2.0, size=5000).clip(max=3000)
    rp = np.zeros(5001, dtype=np.int64)
    rp[1:] = np.cumsum(lens)
    cuts = psb.partition_rows(rp.astype(np.int32), parts)
    assert cuts[0] == 0 and cuts[-1] == 5000 and (np.diff(cuts) >= 0).all()
    nnz = rp[-1]
    for p in range(1, parts):
        # cut p is the first row whose start reaches p*nnz/parts
        target = p * nnz // parts
        assert rp[cuts[p]] >= target
        assert cuts[p] == 0 or rp[cuts[p] - 1] < target
    panel = np.diff(rp[cuts])
    assert panel.sum() == nnz
    assert panel.max() <= nnz / parts + lens.max()


def test_partition_rows_more_parts_than_rows():
    rp = np.array([0, 5, 9], dtype=np.int32)
    cuts = psb.partition_rows(rp, 5)
    assert cuts[0] == 0 and cuts[-1] == 2 and (np.diff(cuts) >= 0).all()


def test_group_size_macro():
    assert [psb.GROUP_SIZE(s) for s in range(1, 6)] == [32, 64, 128, 256, 512]


def test_accessors_of_a_null_matrix_do_not_dereference_it():
    """Host-only accessors return 0 / NULL (-1 where -1 already means "invalid")."""
    lib = psb.load_library()
    for name in ("ps_matrix_row", "ps_matrix_col", "ps_matrix_nnz", "ps_matrix_group_type_num",
                 "ps_matrix_group_fine_size", "ps_matrix_wide_rows"):
        assert getattr(lib, name)(None) == 0, name
    for name in ("ps_matrix_group_num", "ps_matrix_workset_col_ind", "ps_matrix_workset_sp_data",
                 "ps_matrix_group_destination", "ps_matrix_csr_position", "ps_matrix_residue_offset",
                 "ps_matrix_residue_atomic"):
        assert not getattr(lib, name)(None), name
    assert lib.ps_matrix_workset_size(None, 0) == -1
    assert lib.ps_matrix_device(None) == -1
    assert lib.ps_matrix_preprocess_ms(None) == 0.0
