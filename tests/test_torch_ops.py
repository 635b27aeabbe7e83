"""CPU test: importing powersparse_b200.torch_ops registers the torch.ops.powersparse ops."""
import torch

import powersparse_b200.torch_ops  # noqa: F401  (registers the ops)


def test_ops_are_registered():
    for name in ("spmm", "spmm_", "sddmm_csr", "sddmm_"):
        assert hasattr(torch.ops.powersparse, name), name
    assert "!) C" in str(torch.ops.powersparse.spmm_.default._schema)  # C is mutated in place
