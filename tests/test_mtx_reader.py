"""The CLI's MatrixMarket reader (powersparse_b200/bin/powersparse_mtx2csr, the
same code the powersparse_{spmm,sddmm} CLI reads with) against the reference's own
reader (benchmarks/matrix_market.cpp, compiled from the reference's sources into
oracle/_ref/ref_mtx_dump): the same CSR byte for byte on valid files, and the same
error message on malformed ones, with the text cut into 1 to many chunks."""
import os
import subprocess

import numpy as np
import pytest

from powersparse_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OURS = os.path.join(ROOT, "powersparse_b200", "bin", "powersparse_mtx2csr")
REF = os.path.join(ROOT, "oracle", "_ref", "ref_mtx_dump")

pytestmark = pytest.mark.skipif(not (os.path.exists(OURS) and os.path.exists(REF)),
                                reason="needs the built converter and the reference reader (oracle/_ref)")

# (threads, smallest chunk in bytes): one chunk, and many tiny ones.
SPLITS = [(1, 1 << 22), (3, 1), (8, 16), (5, 200)]


def _run(cmd):
    return subprocess.run(cmd, capture_output=True, timeout=300)


def _read(tool_cmd, path, out):
    r = _run(tool_cmd + [str(path), str(out)] if tool_cmd[0] == REF else
             [OURS, str(path), str(out)] + tool_cmd[1:])
    data = out.read_bytes() if r.returncode == 0 and out.exists() else None
    err = r.stderr.decode(errors="replace").strip()
    if out.exists():
        out.unlink()
    return r.returncode, data, err


def _compare(tmp_path, text: bytes):
    path = tmp_path / "m.mtx"
    path.write_bytes(text)
    want = _read([REF], path, tmp_path / "ref.csr")
    for threads, chunk in SPLITS:
        got = _read([OURS, str(threads), str(chunk)], path, tmp_path / "ours.csr")
        assert got == want, (threads, chunk, got[0], got[2], want[0], want[2])
    return want


VALID = {
    "general_real": b"%%MatrixMarket matrix coordinate real general\n% comment\n\n3 4 5\n"
                    b"1 1 1.5\n3 4 -2.25e-1\n\t2  2\t 7\n% in between\n1 3 .5\n3 1 1E+3\n",
    "crlf_no_final_newline": b"%%MatrixMarket matrix coordinate real general\r\n2 2 2\r\n1 2 3.0\r\n2 1 4.0",
    "symmetric": b"%%MatrixMarket matrix coordinate real symmetric\n4 4 6\n1 1 1\n2 1 2\n3 1 3\n"
                 b"4 2 4\n3 3 5\n4 3 6\n",
    "pattern_general": b"%%MatrixMarket matrix coordinate pattern general\n3 3 4\n1 2\n2 3\n3 1\n1 2\n",
    "pattern_symmetric": b"%%MatrixMarket matrix coordinate pattern symmetric\n3 3 3\n2 1\n3 3\n3 2\n",
    "integer": b"%%MatrixMarket matrix coordinate integer general\n2 3 4\n1 1 -7\n2 3 +12\n1 2 007\n2 1 0\n",
    "notations": b"%%MatrixMarket matrix coordinate real general\n2 2 8\n1 1 +2.5\n1 2 0x1.8p1\n"
                 b"2 1 3.4028234e38\n2 2 1e-320\n1 1 -0\n+1 +2 1.\n2 2 -1.5e-45\n1 1 1e-7\n",
    "nul_ends_line": b"%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 1.0\x00junk\n2 2 2\n",
    "leading_spaces": b"%%MatrixMarket matrix coordinate real general\n   2 2 1  \n   2   1   9.5   \n",
}


@pytest.mark.parametrize("name", sorted(VALID))
def test_valid_files_give_the_reference_csr(tmp_path, name):
    rc, data, err = _compare(tmp_path, VALID[name])
    assert rc == 0 and data, err


BAD = {
    "empty": b"",
    "banner_word": b"%%MatrixMarket matrix array real general\n2 2 1\n1 1 1\n",
    "banner_complex": b"%%MatrixMarket matrix coordinate complex general\n2 2 1\n1 1 1 0\n",
    "banner_extra": b"%%MatrixMarket matrix coordinate real general extra\n2 2 1\n1 1 1\n",
    "banner_missing": b"2 2 1\n1 1 1\n",
    "no_size": b"%%MatrixMarket matrix coordinate real general\n% only a comment\n",
    "size_two_ints": b"%%MatrixMarket matrix coordinate real general\n2 2\n1 1 1\n",
    "size_extra": b"%%MatrixMarket matrix coordinate real general\n2 2 1 1\n1 1 1\n",
    "size_zero": b"%%MatrixMarket matrix coordinate real general\n0 2 1\n1 1 1\n",
    "symmetric_not_square": b"%%MatrixMarket matrix coordinate real symmetric\n2 3 1\n1 1 1\n",
    "row_zero": b"%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 1\n0 1 1\n",
    "col_too_big": b"%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 1\n1 3 1\n",
    "row_float": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n1.5 1 1\n",
    "row_overflow": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n99999999999999999999 1 1\n",
    "value_inf": b"%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 1\n2 2 inf\n",
    "value_nan": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n2 2 nan\n",
    "value_too_big": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n2 2 1e39\n",
    "value_word": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n2 2 abc\n",
    "value_missing": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n2 2\n",
    "extra_field": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n2 2 1.0 5\n",
    "pattern_with_value": b"%%MatrixMarket matrix coordinate pattern general\n2 2 1\n2 2 1.0\n",
    "integer_float": b"%%MatrixMarket matrix coordinate integer general\n2 2 1\n2 2 1.5\n",
    "truncated": b"%%MatrixMarket matrix coordinate real general\n2 2 3\n1 1 1\n2 2 2\n",
    "more_entries": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n1 1 1\n2 2 2\n",
    "more_entries_bad_extra": b"%%MatrixMarket matrix coordinate real general\n2 2 1\n1 1 1\nx y z\n",
    "two_errors": b"%%MatrixMarket matrix coordinate real general\n3 3 6\n1 1 1\n2 2 2\n3 9 1\n"
                  b"1 2 3\n2 3 4\nbad 1 1\n",
}


@pytest.mark.parametrize("name", sorted(BAD))
def test_malformed_files_give_the_reference_error(tmp_path, name):
    rc, data, err = _compare(tmp_path, BAD[name])
    assert rc == 1 and err.startswith("Error: "), err


@pytest.mark.parametrize("seed", [1, 2])
def test_errors_late_in_a_long_file_are_reported_in_file_order(tmp_path, seed):
    """Many small chunks; a malformed record in the middle and another near the end."""
    rng = np.random.default_rng(seed)
    lines = [f"{rng.integers(1, 500)} {rng.integers(1, 500)} {rng.uniform(-1, 1):.6g}" for _ in range(3000)]
    lines[1777] = "17 600 1.0"   # column out of range
    lines[2900] = "17 3 word"    # invalid value, later in the file
    text = ("%%MatrixMarket matrix coordinate real general\n500 500 3000\n" + "\n".join(lines) + "\n").encode()
    rc, data, err = _compare(tmp_path, text)
    assert rc == 1 and "outside the declared dimensions" in err


@pytest.mark.parametrize("seed,symmetric", [(11, True), (12, False)])
def test_generated_power_law_files(tmp_path, seed, symmetric):
    m = synth.chung_lu(20000, 30, 2000, 2.1, seed=seed)
    path = tmp_path / "g.mtx"
    if symmetric:
        synth.write_mtx(str(path), m)
    else:
        rows = np.repeat(np.arange(m.rows), np.diff(m.row_ptr))
        order = np.random.default_rng(seed).permutation(m.nnz)  # unsorted general file
        body = "\n".join(f"{r + 1} {c + 1} {float(v)!r}" for r, c, v in
                         zip(rows[order], m.col_ind[order], m.values[order].astype(float)))
        path.write_text(f"%%MatrixMarket matrix coordinate real general\n{m.rows} {m.cols} {m.nnz}\n{body}\n")
    rc, data, err = _compare(tmp_path, path.read_bytes())
    assert rc == 0 and data, err
