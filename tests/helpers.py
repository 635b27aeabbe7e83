"""Shared test helpers: golden fixtures and their inputs."""
from __future__ import annotations

import glob
import os

import numpy as np

import make_golden as mg

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))

# Tolerance the north star holds results to: |a - e| <= ATOL + RTOL * |e| (FP64 oracle e).
ATOL, RTOL = 1e-5, 1e-4


def golden_names() -> list[str]:
    return [os.path.basename(p)[:-4] for p in GOLDEN]


def load_golden(name: str):
    """(fixture, rows, cols, row_ptr, col_ind, values, sm_count) for one golden case."""
    z = np.load(os.path.join(HERE, "golden", name + ".npz"))
    sm = int(z["sm_count"])
    sm = 148 if sm < 0 else sm
    if "row_ptr" in z.files:
        return z, int(z["rows"]), int(z["cols"]), z["row_ptr"], z["col_ind"], z["values"], sm
    m = mg.cases()[name][0]
    assert mg.csr_digest(m) == str(z["csr_sha256"]), "generator no longer reproduces the golden CSR"
    return z, m.rows, m.cols, m.row_ptr, m.col_ind, m.values, sm


def layout_arrays(L) -> dict:
    """Oracle layout as the fixture keys."""
    out = {"res_off": L.residue_offset, "res_atomic": L.residue_atomic}
    for s in range(L.S):
        out[f"ws{s}_col"] = L.col_ind[s]
        out[f"ws{s}_val"] = L.sp_data[s]
        out[f"ws{s}_des"] = L.group_des[s]
    return out


def close_frac(actual, expected, atol=ATOL, rtol=RTOL):
    from oracle import oracle
    ok = oracle.close(actual, expected, atol, rtol)
    return ok.mean() if ok.size else 1.0, ok


def dense_inputs(rows, n, seed):
    return mg.dense_inputs(rows, n, seed)
