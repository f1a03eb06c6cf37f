"""Parity at the exact configuration the benchmark times (bench.py's c2 step).

B=8, T=4096, H=16, d_k=128, bf16 inputs built by bench.c2_inputs with rank 0's seed, the per-head
gate lambda = sigmoid(W[h] . q + b[h]) fused into the kernels, forward and backward through
ops.clean_fwd_raw / ops.clean_bwd_raw as the benchmark calls them.  Checked:
  * the tensor-core path against the exact fp32 SIMT path on every output (q_clean, final states,
    token side outputs, dq, dk, dW, db);
  * three heads across all eight batch rows against the float64 oracle on the same bf16-rounded
    inputs, including the gate gradients dW[h], db[h] summed over the batch.
Bars: 2e-2 max-abs on bf16 outputs against the oracle (each path); between the two paths 4e-2, as
each is within 2e-2 of the exact result (dq reaches ~8 here, where one bf16 ulp is 0.031); 1e-4
relative on the fp32 states (sums of 4096 outer products: the tensor core's fp32 accumulation of
bf16 products differs from a float64 sum by ~1.3e-5 relative at this length); 1e-2 relative on dW / db.
"""
import numpy as np
import pytest
import torch

from golden_util import rel_err
from oracle import ccq_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


@pytest.fixture(scope='module')
def c2():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    import bench
    from ccq_b200 import _lib
    _lib.load()
    dev = torch.device('cuda', 0)
    q, k, W, b, dqc = bench.c2_inputs(dev, 1000)
    return q, k, W, b, dqc


def _run(c2):
    from ccq_b200 import ops
    q, k, W, b, dqc = c2
    B = q.shape[0]
    qc, fc, fm, aux = ops.clean_fwd_raw(q, k, None, W, b, 0, None, None, True, None, B)
    fpath = ops._lib.last_path()
    dq, dk, (dW, db), _, _ = ops.clean_bwd_raw(q, k, None, W, b, 0, None, None, True, None, B, fc, fm, aux, dqc,
                                               None, None)
    bpath = ops._lib.last_path()
    torch.cuda.synchronize()
    return dict(qc=qc, fc=fc, fm=fm, aux=aux, dq=dq, dk=dk, dW=dW, db=db), (fpath, bpath)


def _np(t):
    return t.detach().double().cpu().numpy()


def test_c2_tcgen05_matches_exact_path(c2, monkeypatch):
    tc, paths = _run(c2)
    assert paths == ('tcgen05', 'tcgen05')
    monkeypatch.setenv('CCQ_B200_FORCE_SIMT', '1')
    ex, paths = _run(c2)
    assert paths == ('simt', 'simt')
    monkeypatch.delenv('CCQ_B200_FORCE_SIMT')
    for name in ('qc', 'dq', 'dk'):
        err = (tc[name].float() - ex[name].float()).abs().max().item()
        assert err <= 2 * BF16_TOL, (name, err)
    for name in ('fc', 'fm'):
        assert rel_err(_np(tc[name]), _np(ex[name])) <= 1e-4, name
    assert rel_err(_np(tc['aux']), _np(ex['aux'])) <= 1e-3
    for name in ('dW', 'db'):
        assert rel_err(_np(tc[name]), _np(ex[name])) <= 1e-2, (name, rel_err(_np(tc[name]), _np(ex[name])))


@pytest.mark.parametrize('path', ['tcgen05', 'simt'])
@pytest.mark.parametrize('h', [0, 7, 15])
def test_c2_heads_against_oracle(c2, h, path, monkeypatch):
    if path == 'simt':
        monkeypatch.setenv('CCQ_B200_FORCE_SIMT', '1')
    tc, paths = _run(c2)
    assert paths == (path, path)
    q, k, W, b, dqc = c2
    qn, kn, gn = (_np(t[:, :, h:h + 1]) for t in (q, k, dqc))
    Wn, bn = _np(W[h:h + 1]), _np(b[h:h + 1])
    lam = O.lambda_headwise_fwd(qn, Wn, bn)
    oq, ofc, ofm = O.clean_read_fwd(qn, kn, lam, output_final_state=True)
    odq, odk, odl, _, _ = O.clean_read_bwd(qn, kn, lam, gn)
    dqx, odW, odb = O.lambda_headwise_bwd(qn, Wn, lam, odl)
    assert np.abs(_np(tc['qc'][:, :, h:h + 1]) - oq).max() <= BF16_TOL
    assert np.abs(_np(tc['dq'][:, :, h:h + 1]) - (odq + dqx)).max() <= BF16_TOL
    assert np.abs(_np(tc['dk'][:, :, h:h + 1]) - odk).max() <= BF16_TOL
    assert rel_err(_np(tc['fc'][:, h:h + 1]), ofc) <= 1e-4
    assert rel_err(_np(tc['fm'][:, h:h + 1]), ofm) <= 1e-4
    assert rel_err(_np(tc['dW'][h:h + 1]), odW) <= 1e-2
    assert rel_err(_np(tc['db'][h:h + 1]), odb) <= 1e-2
