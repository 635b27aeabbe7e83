"""GPU tests of the attention chain after the path: SpMM with per-call edge values
(ps_spmm_values), edge softmax per row (ps_edge_softmax_csr), and the whole
SDDMM -> softmax -> SpMM chain, against FP64 numpy at the tests' tolerance."""
import numpy as np
import pytest
import torch

import powersparse_b200 as psb
from helpers import ATOL, RTOL, golden_names, load_golden
from oracle import oracle
from powersparse_b200 import synth

pytestmark = pytest.mark.gpu


def _rows(rp):
    return np.repeat(np.arange(len(rp) - 1), np.diff(rp))


def _softmax_rows(rp, v):
    v = v.astype(np.float64)
    out = np.empty_like(v)
    for r in range(len(rp) - 1):
        b, e = rp[r], rp[r + 1]
        if b < e:
            x = np.exp(v[b:e] - v[b:e].max())
            out[b:e] = x / x.sum()
    return out


def _close(a, e, tag):
    ok = oracle.close(a, e, ATOL, RTOL)
    assert ok.all(), f"{tag}: {int((~ok).sum())} of {ok.size} outside tolerance"


def _heavy():
    base = synth.chung_lu(3000, 12, 300, 2.1, seed=4)
    rng = np.random.default_rng(4)
    heavy = [np.sort(rng.choice(base.cols, size=2600, replace=False)).astype(np.int32) for _ in range(4)]
    rp = np.concatenate([base.row_ptr, base.nnz + 2600 * np.arange(1, 5)]).astype(np.int32)
    ci = np.concatenate([base.col_ind] + heavy).astype(np.int32)
    va = np.concatenate([base.values, rng.uniform(-1, 1, 4 * 2600).astype(np.float32)])
    return base.rows + 4, base.cols, rp, ci, va


def _cases():
    out = []
    for name in golden_names()[:4]:
        z, rows, cols, rp, ci, va, sm = load_golden(name)
        out.append((name, rows, cols, rp, ci, va, sm))
    rows, cols, rp, ci, va = _heavy()
    out.append(("heavy", rows, cols, rp, ci, va, 1))
    return out


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_spmm_with_per_call_values(case):
    name, rows, cols, rp, ci, va, sm = case
    rng = np.random.default_rng(7)
    w = rng.uniform(-1, 1, len(ci)).astype(np.float32)
    with psb.PowerSparseMatrixGPU(rows, cols, len(ci), rp, ci, va, sm_count=sm) as m:
        if name == "heavy":
            assert m.wide_rows == 4
        for n in (32, 128):
            B = synth.dense(cols, n, 11 + n)
            C = torch.zeros((rows, n), device="cuda")
            psb.SpMM_values(m, n, torch.from_numpy(w).cuda(), torch.from_numpy(B).cuda(), C)
            torch.cuda.synchronize()
            _close(C.cpu().numpy(), oracle.spmm(rp, ci, w, B), f"{name} N={n}")


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_edge_softmax_and_attention_chain(case):
    name, rows, cols, rp, ci, va, sm = case
    n = 32
    X, Y = synth.dense(rows, n, 21), synth.dense(cols, n, 22)
    B = synth.dense(cols, 128, 23)
    logits = va.astype(np.float64) * np.einsum("ij,ij->i", X[_rows(rp)].astype(np.float64), Y[ci].astype(np.float64))
    alpha = _softmax_rows(rp, logits)
    exp_out = oracle.spmm(rp, ci, alpha.astype(np.float32), B)
    with psb.PowerSparseMatrixGPU(rows, cols, len(ci), rp, ci, va, sm_count=sm) as m:
        e = torch.empty(len(ci), device="cuda")
        psb.SDDMM_csr(m, n, torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda(), e)
        psb.edge_softmax_csr(m, e)
        out = torch.zeros((rows, 128), device="cuda")
        psb.SpMM_values(m, 128, e, torch.from_numpy(B).cuda(), out)
        torch.cuda.synchronize()
        _close(e.cpu().numpy(), alpha, f"{name} softmax")
        _close(out.cpu().numpy(), exp_out, f"{name} chain")


def test_edge_softmax_on_a_loaded_layout(tmp_path):
    """A loaded layout rebuilds the row pointer from its groups."""
    rows, cols, rp, ci, va = _heavy()
    v = np.random.default_rng(9).normal(0, 3, len(ci)).astype(np.float32)
    path = tmp_path / "h.pslayout"
    with psb.PowerSparseMatrixGPU(rows, cols, len(ci), rp, ci, va, sm_count=1) as m:
        m.save(str(path))
    with psb.PowerSparseMatrixGPU.load(str(path)) as m2:
        d = torch.from_numpy(v).cuda()
        psb.edge_softmax_csr(m2, d)
        torch.cuda.synchronize()
    _close(d.cpu().numpy(), _softmax_rows(rp, v), "loaded softmax")
