"""Host-side pieces of bench.py: the numpy row partition used by the reference arm
(it must cut exactly like ps_partition_rows) and the sampled FP64 check."""
import numpy as np
import pytest
import torch

import bench
import powersparse_b200 as psb
from powersparse_b200 import synth


@pytest.mark.parametrize("seed", range(6))
def test_numpy_partition_matches_the_c_abi(seed):
    rng = np.random.default_rng(seed)
    rows = int(rng.integers(1, 400))
    lens = rng.integers(0, 50, size=rows) * (rng.random(rows) < 0.7)
    rp = np.zeros(rows + 1, dtype=np.int64)
    np.cumsum(lens, out=rp[1:])
    for parts in (1, 2, 3, 8, rows + 5):
        got = bench.partition_rows_np(rp, parts)
        ref = psb.partition_rows(rp.astype(np.int32), parts)
        assert np.array_equal(got, np.asarray(ref, dtype=np.int64)), (rows, parts)


def test_sampled_check_passes_on_the_exact_product_and_fails_on_an_error():
    m = synth.chung_lu(3000, 12, 300, 2.1, seed=5)
    B = torch.from_numpy(synth.dense(m.cols, 32, 6))
    dense = np.zeros((m.rows, m.cols), dtype=np.float64)
    rows = np.repeat(np.arange(m.rows), np.diff(m.row_ptr))
    np.add.at(dense, (rows, m.col_ind), m.values.astype(np.float64))
    C = torch.from_numpy((dense @ B.double().numpy()).astype(np.float32))
    ok = bench.sampled_check(m, B, C, rows=500)
    assert ok["bad"] == 0 and ok["rows"] > 400 and ok["elements"] == ok["rows"] * 32
    C[:, 3] += 0.01
    bad = bench.sampled_check(m, B, C, rows=500)
    assert bad["bad"] >= bad["rows"] // 2
