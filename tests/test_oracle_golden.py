"""The CPU oracle against the reference's own outputs (golden vectors), fp32 bar 1e-5 relative."""
import numpy as np
import pytest

from golden_util import compare, fixture_keys, load_case
from oracle import ccq_oracle as O

TOL = 1e-5
CLEAN_CASES = ['dense', 'varlen', 'nomean', 'lamh', 'scalar', 'k128']


def oracle_outputs(name, d, opts):
    out = {}
    lam = d.get('lam')
    h0 = d.get('initial_cov_state')
    m0 = d.get('initial_mean_state')
    kw = dict(position_offset=opts['position_offset'], initial_cov_state=h0, initial_mean_state=m0,
              subtract_mean=opts['subtract_mean'], cu_seqlens=opts['cu_seqlens'])
    if name == 'cfg1':
        lam = O.lambda_headwise_fwd(d['q'], d['W'], d['b'])
    qc, fc, fm = O.clean_read_fwd(d['q'], d['k'], lam, output_final_state=opts['output_final_state'], **kw)
    dfc = d.get('dfinal_cov') if fc is not None else None
    dfm = d.get('dfinal_mean') if fm is not None else None
    dq, dk, dl3, dh0, dm0 = O.clean_read_bwd(d['q'], d['k'], lam, d['dqc'], dfinal_cov=dfc, dfinal_mean=dfm, **kw)
    out.update(q_clean=qc, dq=dq, dk=dk)
    if fc is not None:
        out['final_cov'] = fc
    if fm is not None:
        out['final_mean'] = fm
    if name == 'cfg1':
        dqx, dW, db = O.lambda_headwise_bwd(d['q'], d['W'], lam, dl3)
        out['dq'] = dq + dqx
        out['dW'] = dW
        out['db'] = db
    elif isinstance(lam, np.ndarray):
        out['dlam'] = O.reduce_dlambda(dl3, lam.shape)
    if dh0 is not None:
        out['dh0'] = dh0
    if dm0 is not None:
        out['dm0'] = dm0
    return out


@pytest.mark.parametrize('name', CLEAN_CASES + ['cfg1'])
def test_oracle_matches_reference(name):
    d, opts, fx = load_case(name)
    out = oracle_outputs(name, d, opts)
    assert set(out) == set(fixture_keys(fx)), (sorted(out), fixture_keys(fx))
    for key, val in out.items():
        e = compare(fx, key, val, TOL)
        assert e <= TOL, f'{name}.{key}: rel err {e:.3e}'


def test_oracle_decode_matches_reference():
    d, opts, fx = load_case('decode')
    P, S = opts['prefix'], opts['steps']
    _, C, m = O.clean_read_fwd(d['prefix_q'], d['prefix_k'], d['prefix_lam'], output_final_state=True)
    assert compare(fx, 'prefix_cov', C, TOL) <= TOL
    assert compare(fx, 'prefix_mean', m, TOL) <= TOL
    qcs = []
    off = P
    for i in range(S):
        qc, C, m = O.decode_clean(d['step_q'][i], d['step_k'][i], d['step_lam'][i], off, C, m)
        qcs.append(qc)
        off += 1
    assert compare(fx, 'step_q_clean', np.stack(qcs), TOL) <= TOL
    assert compare(fx, 'steps_cov', C, TOL) <= TOL
    assert compare(fx, 'steps_mean', m, TOL) <= TOL
    qc, C, m = O.decode_clean(d['multi_q'], d['multi_k'], d['multi_lam'], off, C, m)
    assert compare(fx, 'multi_q_clean', qc, TOL) <= TOL
    assert compare(fx, 'multi_cov', C, TOL) <= TOL
    assert compare(fx, 'multi_mean', m, TOL) <= TOL
    qc, C2, m2 = O.decode_clean(d['var_q'], d['var_k'], d['var_lam'], 3, C[:2], m[:2],
                                cu_seqlens=opts['var_cu'])
    assert compare(fx, 'var_q_clean', qc, TOL) <= TOL
    assert compare(fx, 'var_cov', C2, TOL) <= TOL
    assert compare(fx, 'var_mean', m2, TOL) <= TOL


def test_oracle_chunk_size_independent():
    d, opts, _ = load_case('varlen')
    kw = dict(position_offset=7, initial_cov_state=d['initial_cov_state'],
              initial_mean_state=d['initial_mean_state'], cu_seqlens=opts['cu_seqlens'])
    a = O.clean_read_fwd(d['q'], d['k'], d['lam'], output_final_state=True, chunk=64, **kw)
    b = O.clean_read_fwd(d['q'], d['k'], d['lam'], output_final_state=True, chunk=17, **kw)
    for x, y in zip(a, b):
        assert np.abs(x - y).max() < 1e-12
