"""Loading and comparing the reference's golden vectors (tests/golden/*.npz)."""
from __future__ import annotations

import os
import sys

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

import gen_golden  # noqa: E402  (input builders only; the reference is not imported)


def rel_err(a, ref):
    """max |a - ref| / max |ref| over the whole tensor (the survey's 'relative error')."""
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    assert a.shape == ref.shape, (a.shape, ref.shape)
    if ref.size == 0:
        return 0.0
    scale = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(a - ref).max() / scale)


def load_case(name):
    """(inputs, options, fixture dict); asserts the regenerated inputs are the ones the reference saw."""
    d, opts = gen_golden.case_inputs(name)
    fx = dict(np.load(os.path.join(GOLDEN, f'{name}.npz')))
    assert str(fx['inputs_sha256']) == gen_golden.inputs_digest(d), f'{name}: input generator drifted'
    return d, opts, fx


def fixture_keys(fx):
    keys = set()
    for k in fx:
        if k == 'inputs_sha256':
            continue
        keys.add(k.split('__')[0])
    return sorted(keys)


def compare(fx, key, value, tol):
    """Compare a full output against a full or sampled fixture entry; returns the relative error."""
    value = np.asarray(value, np.float64)
    if key in fx:
        return rel_err(value, fx[key])
    shape = tuple(int(s) for s in fx[key + '__shape'])
    assert value.shape == shape, (key, value.shape, shape)
    flat = value.reshape(-1)
    ref = fx[key + '__val'].astype(np.float64)
    e = rel_err(flat[fx[key + '__idx']], ref)
    s = float(flat.sum())
    ss = float((flat ** 2).sum())
    # sums of fp32 tensors: compare against the magnitude of the summed terms
    e_sum = abs(s - float(fx[key + '__sum'])) / max(np.sqrt(ss) * np.sqrt(flat.size), 1e-30)
    e_sq = abs(ss - float(fx[key + '__sumsq'])) / max(ss, 1e-30)
    return max(e, e_sum, e_sq)
