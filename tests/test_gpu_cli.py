"""GPU tests of the drop-in CLI (powersparse_{spmm,sddmm} MATRIX.mtx N DEVICE CHECK REPEATS),
which runs the C++ operator API (include/PowerSparse_*) over the C ABI."""
import csv
import io
import os
import subprocess

import pytest

from powersparse_b200 import synth

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "powersparse_b200", "bin")
REF_BIN = os.path.join(ROOT, "oracle", "_ref")
HEADER = ("algorithm,operator,matrix,rows,cols,nnz,N,device,gpu,compute_capability,cuda_runtime,"
          "cuda_driver,warmup,repeats,seed,check,preprocess_ms,ms,gflops")


def _run(binary, *args):
    return subprocess.run([binary, *map(str, args)], capture_output=True, text=True, timeout=600)


@pytest.fixture(scope="module")
def mtx_files(tmp_path_factory):
    d = tmp_path_factory.mktemp("mtx")
    paths = {}
    paths["cfg1"] = str(d / "cfg1.mtx")
    synth.write_mtx(paths["cfg1"], synth.config_matrix(1))
    paths["cl"] = str(d / "cl.mtx")
    synth.write_mtx(paths["cl"], synth.chung_lu(30000, 40, 3000, 2.1, seed=11))
    paths["cl_bin"] = str(d / "cl.csr")
    synth.write_csr_bin(paths["cl_bin"], synth.chung_lu(30000, 40, 3000, 2.1, seed=11))
    return paths


@pytest.mark.parametrize("op", ["spmm", "sddmm"])
def test_cli_header_and_usage(op):
    binary = os.path.join(BIN, f"powersparse_{op}")
    r = _run(binary, "--header")
    assert r.returncode == 0 and r.stdout.strip() == HEADER
    r = _run(binary, "x.mtx", 64, 0, 0, 1)
    assert r.returncode == 2 and "please use N=32 or N=128" in r.stderr
    assert _run(binary).returncode == 2


@pytest.mark.parametrize("op", ["spmm", "sddmm"])
@pytest.mark.parametrize("n", [32, 128])
@pytest.mark.parametrize("which", ["cfg1", "cl", "cl_bin"])
def test_cli_check_passes(mtx_files, op, n, which):
    r = _run(os.path.join(BIN, f"powersparse_{op}"), mtx_files[which], n, 0, 1, 5)
    assert r.returncode == 0, r.stderr
    assert "checks passed" in r.stderr
    row = next(csv.reader(io.StringIO(r.stdout)))
    fields = dict(zip(HEADER.split(","), row))
    assert fields["operator"] == ("SpMM" if op == "spmm" else "SDDMM")
    assert fields["check"] == "passed" and int(fields["N"]) == n
    assert float(fields["gflops"]) > 0


def test_cli_csv_matches_reference_columns(mtx_files):
    """Same columns and identical matrix fields as the reference's own CLI built here."""
    ref = os.path.join(REF_BIN, "powersparse_spmm")
    if not os.path.exists(ref):
        pytest.skip("reference CLI not built")
    ours = _run(os.path.join(BIN, "powersparse_spmm"), mtx_files["cl"], 32, 0, 0, 3)
    theirs = _run(ref, mtx_files["cl"], 32, 0, 0, 3)
    assert ours.returncode == 0 and theirs.returncode == 0, theirs.stderr
    a = dict(zip(HEADER.split(","), next(csv.reader(io.StringIO(ours.stdout)))))
    b = dict(zip(HEADER.split(","), next(csv.reader(io.StringIO(theirs.stdout)))))
    for k in ("algorithm", "operator", "rows", "cols", "nnz", "N", "warmup", "repeats", "seed", "check"):
        assert a[k] == b[k], k


def test_cli_rejects_bad_input(tmp_path):
    bad = tmp_path / "bad.mtx"
    bad.write_text("%%MatrixMarket matrix coordinate real general\n2 2 1\n3 1 1.0\n")
    r = _run(os.path.join(BIN, "powersparse_spmm"), str(bad), 32, 0, 0, 1)
    assert r.returncode == 1 and "outside the declared dimensions" in r.stderr
