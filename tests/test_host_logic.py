"""Host-side logic that needs no GPU: lambda broadcasting and gradient reduction, mirrored from
the reference (clean.py:314-325, fused_read.py:504-513), and the oracle's own invariants."""
import numpy as np
import pytest
import torch

import ccq_b200
from oracle import ccq_oracle as O


@pytest.mark.parametrize('shape', [(), (3,), (2, 5, 3, 1), (2, 5, 3)])
def test_lambda_reshape_and_grad_roundtrip(shape):
    q = torch.randn(2, 5, 3, 4)
    lam = torch.rand(shape) if shape else torch.tensor(0.3)
    l3 = ccq_b200.reshape_lambda_3d(lam, q)
    assert l3.shape == (2, 5, 3) and l3.dtype == q.dtype and l3.is_contiguous()
    d3 = torch.randn(2, 5, 3)
    dl = ccq_b200.reduce_lambda_grad(d3, lam)
    assert dl.shape == lam.shape
    # the reduction is the adjoint of the broadcast
    lhs = (l3 * d3).sum()
    rhs = (lam * dl).sum()
    assert torch.allclose(lhs, rhs, rtol=1e-5, atol=1e-6)
    npl = O.reshape_lambda_3d(lam.numpy() if shape else 0.3, 2, 5, 3)
    assert np.allclose(npl, l3.numpy())


def test_lambda_reshape_scalar_and_dtype():
    q = torch.randn(1, 3, 2, 4, dtype=torch.bfloat16)
    l3 = ccq_b200.reshape_lambda_3d(0.25, q)
    assert l3.dtype == torch.bfloat16 and float(l3[0, 0, 0]) == 0.25


def test_oracle_decode_equals_chunked_forward():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 9, 2, 8))
    k = rng.standard_normal((2, 9, 2, 8))
    lam = rng.uniform(size=(2, 9, 2))
    a = O.clean_read_fwd(q, k, lam, 3, None, None, True, True)
    b = O.decode_clean(q, k, lam, 3, None, None, True, True)
    for x, y in zip(a, b):
        assert np.abs(x - y).max() < 1e-12


def test_oracle_lambda_zero_is_identity_with_states():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 70, 2, 8))
    k = rng.standard_normal((1, 70, 2, 8))
    qc, _, _ = O.clean_read_fwd(q, k, 0.0)
    assert np.abs(qc - q).max() == 0.0


def test_chunk_slots_bound():
    # the per-chunk workspace slot of document n starts at floor(bos/BT) + n; slots never overlap
    rng = np.random.default_rng(2)
    for _ in range(200):
        lens = rng.integers(0, 300, size=rng.integers(1, 12))
        bos = np.concatenate([[0], np.cumsum(lens)[:-1]])
        BT = int(rng.choice([32, 64, 128]))
        starts = bos // BT + np.arange(len(lens))
        ends = starts + (lens + BT - 1) // BT
        assert np.all(ends[:-1] <= starts[1:])
        assert ends[-1] <= lens.sum() // BT + len(lens) + 1
