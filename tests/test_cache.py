"""CPU tests of the layout-cache loader's header checks (no GPU needed: a file that is
missing, foreign or has a corrupt header is refused before any CUDA call)."""
import ctypes
import struct

import pytest

import powersparse_b200 as psb


def _load_status(path):
    lib = psb.load_library()
    h = ctypes.c_void_p()
    status = lib.ps_matrix_load(str(path).encode(), ctypes.byref(h))
    return status, lib.ps_last_error().decode(), h.value


def test_missing_layout_file_is_an_invalid_argument(tmp_path):
    status, err, h = _load_status(tmp_path / "none.pslayout")
    assert status == psb.PS_ERR_INVALID_ARGUMENT and "Cannot open the layout file" in err and not h


def test_foreign_file_is_refused(tmp_path):
    p = tmp_path / "x.pslayout"
    p.write_bytes(b"PSCSR001" + bytes(64))
    status, err, _ = _load_status(p)
    assert status == psb.PS_ERR_INVALID_ARGUMENT and "Not a PowerSparse layout file" in err


@pytest.mark.parametrize("head", [(0, 10, 10, 1, 16, 148, 32), (10, 10, 10, 0, 16, 148, 32),
                                  (10, 10, 10, 40, 16, 148, 32), (10, 10, 10, 2, 8, 148, 32),
                                  (10, 10, -1, 2, 16, 148, 32)])
def test_corrupt_header_is_refused(tmp_path, head):
    p = tmp_path / "bad.pslayout"
    p.write_bytes(b"PSLAYT01" + struct.pack("<7i", *head))
    status, err, _ = _load_status(p)
    assert status == psb.PS_ERR_INVALID_ARGUMENT and "Corrupt layout file header" in err


def test_truncated_header_is_refused(tmp_path):
    p = tmp_path / "short.pslayout"
    p.write_bytes(b"PSLAYT01" + struct.pack("<3i", 1, 2, 3))
    status, err, _ = _load_status(p)
    assert status == psb.PS_ERR_INVALID_ARGUMENT and "Truncated layout file" in err
