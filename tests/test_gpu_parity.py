"""Parity of the CUDA operator (through the C ABI) with the reference's golden vectors and the oracle.

Bars (the operator's stated tolerances): fp32 within 1e-5 relative error (max |a - b| / max |b|);
bf16 within 2e-2 max-abs error against the float64 oracle evaluated on the bf16-rounded inputs.
"""
import numpy as np
import pytest
import torch

from golden_util import compare, fixture_keys, load_case, rel_err
from oracle import ccq_oracle as O

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
BF16_TOL = 2e-2


@pytest.fixture(scope='module', autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    import ccq_b200  # noqa: F401
    from ccq_b200 import _lib as L
    L.load()
    yield


def dev(x, dtype=torch.float32, grad=False):
    if x is None:
        return None
    t = torch.tensor(np.asarray(x), dtype=dtype, device='cuda')
    if grad:
        t.requires_grad_(True)
    return t


def np64(t):
    return t.detach().double().cpu().numpy()


# ------------------------------------------------------------------------------------------
# golden vectors of the reference (fp32)
# ------------------------------------------------------------------------------------------

def run_ours_fp32(name, d, opts, gated=False):
    import ccq_b200
    q, k = dev(d['q'], grad=True), dev(d['k'], grad=True)
    h0 = dev(d.get('initial_cov_state'), grad=True)
    m0 = dev(d.get('initial_mean_state'), grad=True)
    cu = dev(opts['cu_seqlens'], torch.int64) if opts['cu_seqlens'] is not None else None
    W = b = lam = None
    if name == 'cfg1':
        W, b = dev(d['W'], grad=True), dev(d['b'], grad=True)
        if gated:
            qc, fc, fm = ccq_b200.fused_ccq_clean_gated(
                q, k, W, b, position_offset=opts['position_offset'], output_final_state=opts['output_final_state'],
                subtract_mean=opts['subtract_mean'], cu_seqlens=cu)
        else:
            lam = torch.sigmoid(torch.einsum('bthk,hk->bth', q, W) + b)
    if not gated:
        if lam is None:
            lam = d['lam']
            lam = dev(lam, grad=True) if isinstance(lam, np.ndarray) else lam
        qc, fc, fm = ccq_b200.fused_ccq_clean_read(
            q, k, lam, position_offset=opts['position_offset'], initial_cov_state=h0, initial_mean_state=m0,
            output_final_state=opts['output_final_state'], subtract_mean=opts['subtract_mean'], cu_seqlens=cu)
    loss = (qc * dev(d['dqc'])).sum()
    if fc is not None and 'dfinal_cov' in d:
        loss = loss + (fc * dev(d['dfinal_cov'])).sum()
    if fm is not None and 'dfinal_mean' in d:
        loss = loss + (fm * dev(d['dfinal_mean'])).sum()
    loss.backward()
    out = {'q_clean': qc, 'dq': q.grad, 'dk': k.grad}
    if fc is not None:
        out['final_cov'] = fc
    if fm is not None:
        out['final_mean'] = fm
    if name == 'cfg1':
        out['dW'] = W.grad
        out['db'] = b.grad
    elif isinstance(lam, torch.Tensor):
        out['dlam'] = lam.grad
    if h0 is not None:
        out['dh0'] = h0.grad
    if m0 is not None and m0.grad is not None:
        out['dm0'] = m0.grad
    return {key: np64(v) for key, v in out.items()}


@pytest.mark.parametrize('name', ['dense', 'varlen', 'nomean', 'lamh', 'scalar', 'cfg1', 'k128'])
def test_golden_fp32(name):
    d, opts, fx = load_case(name)
    out = run_ours_fp32(name, d, opts)
    assert set(out) == set(fixture_keys(fx)), (sorted(out), fixture_keys(fx))
    for key, val in out.items():
        e = compare(fx, key, val, FP32_TOL)
        assert e <= FP32_TOL, f'{name}.{key}: rel err {e:.3e}'


def test_golden_cfg1_gated_fp32():
    d, opts, fx = load_case('cfg1')
    out = run_ours_fp32('cfg1', d, opts, gated=True)
    for key, val in out.items():
        e = compare(fx, key, val, FP32_TOL)
        assert e <= FP32_TOL, f'cfg1(gated).{key}: rel err {e:.3e}'


def test_golden_decode_fp32():
    import ccq_b200
    d, opts, fx = load_case('decode')
    P, S = opts['prefix'], opts['steps']
    _, C, m = ccq_b200.fused_ccq_clean_read(dev(d['prefix_q']), dev(d['prefix_k']), dev(d['prefix_lam']),
                                            output_final_state=True)
    assert compare(fx, 'prefix_cov', np64(C), FP32_TOL) <= FP32_TOL
    assert compare(fx, 'prefix_mean', np64(m), FP32_TOL) <= FP32_TOL
    qcs = []
    off = P
    for i in range(S):
        qc, _, C, m, _ = ccq_b200.fused_ccq_clean(dev(d['step_q'][i]), dev(d['step_k'][i]), dev(d['step_lam'][i]),
                                                  initial_cov_state=C, initial_mean_state=m, output_final_state=True,
                                                  position_offset=off, use_chunk=False)
        assert ccq_b200.last_path() == 'decode'
        qcs.append(np64(qc))
        off += 1
    assert compare(fx, 'step_q_clean', np.stack(qcs), FP32_TOL) <= FP32_TOL
    assert compare(fx, 'steps_cov', np64(C), FP32_TOL) <= FP32_TOL
    assert compare(fx, 'steps_mean', np64(m), FP32_TOL) <= FP32_TOL
    qc, _, C, m, _ = ccq_b200.fused_ccq_clean(dev(d['multi_q']), dev(d['multi_k']), dev(d['multi_lam']),
                                              initial_cov_state=C, initial_mean_state=m, output_final_state=True,
                                              position_offset=off, use_chunk=False)
    assert compare(fx, 'multi_q_clean', np64(qc), FP32_TOL) <= FP32_TOL
    assert compare(fx, 'multi_cov', np64(C), FP32_TOL) <= FP32_TOL
    assert compare(fx, 'multi_mean', np64(m), FP32_TOL) <= FP32_TOL
    qc, _, C2, m2, _ = ccq_b200.fused_ccq_clean(dev(d['var_q']), dev(d['var_k']), dev(d['var_lam']),
                                                initial_cov_state=C[:2].contiguous(),
                                                initial_mean_state=m[:2].contiguous(), output_final_state=True,
                                                position_offset=3, use_chunk=False,
                                                cu_seqlens=dev(opts['var_cu'], torch.int64))
    assert compare(fx, 'var_q_clean', np64(qc), FP32_TOL) <= FP32_TOL
    assert compare(fx, 'var_cov', np64(C2), FP32_TOL) <= FP32_TOL
    assert compare(fx, 'var_mean', np64(m2), FP32_TOL) <= FP32_TOL


# ------------------------------------------------------------------------------------------
# seeded inputs against the oracle: fp32 at 1e-5, bf16 / fp16 at 2e-2 max-abs
# ------------------------------------------------------------------------------------------

def unit(rng, shape):
    x = rng.standard_normal(shape)
    return x / np.linalg.norm(x, axis=-1, keepdims=True)


def make_case(seed, B, T, H, K, lens=None, states=False, offset=0, final_grads=False, subtract_mean=True):
    rng = np.random.default_rng(seed)
    if lens is not None:
        T = int(sum(lens))
        B = 1
    d = dict(q=unit(rng, (B, T, H, K)), k=unit(rng, (B, T, H, K)), lam=rng.uniform(0, 1, (B, T, H)),
             dqc=rng.standard_normal((B, T, H, K)))
    N = B if lens is None else len(lens)
    cu = None if lens is None else np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    if states:
        kk = unit(rng, (N, 16, H, K))
        d['h0'] = np.einsum('nthk,nthv->nhkv', kk, kk)
        d['m0'] = kk.sum(1)
    if final_grads:
        # state gradients of realistic size: (dC + dC^T) k stays O(1) like the other gradient terms
        d['dfc'] = rng.standard_normal((N, H, K, K)) / np.sqrt(K)
        d['dfm'] = rng.standard_normal((N, H, K)) / np.sqrt(K) if subtract_mean else None
    return d, cu, offset, subtract_mean


def round_to(x, dtype):
    return torch.tensor(x, dtype=torch.float32).to(dtype).double().numpy()


def check_against_oracle(d, cu, offset, subtract_mean, dtype, tol, rel):
    import ccq_b200
    q, k = dev(d['q'], dtype, True), dev(d['k'], dtype, True)
    lam = dev(d['lam'], dtype, True)
    h0 = dev(d.get('h0'), torch.float32, True)
    m0 = dev(d.get('m0'), torch.float32, True) if subtract_mean else None
    cut = dev(cu, torch.int64) if cu is not None else None
    want_final = 'dfc' in d
    qc, fc, fm = ccq_b200.fused_ccq_clean_read(q, k, lam, position_offset=offset, initial_cov_state=h0,
                                               initial_mean_state=m0, output_final_state=want_final,
                                               subtract_mean=subtract_mean, cu_seqlens=cut)
    g = dev(d['dqc'], dtype)
    loss = (qc.float() * g.float()).sum()
    if want_final:
        loss = loss + (fc * dev(d['dfc'])).sum()
        if fm is not None and d.get('dfm') is not None:
            loss = loss + (fm * dev(d['dfm'])).sum()
    loss.backward()
    # oracle on the rounded inputs
    qr, kr, lr, gr = (round_to(d[x], dtype) for x in ('q', 'k', 'lam', 'dqc'))
    oq, ofc, ofm = O.clean_read_fwd(qr, kr, lr, offset, d.get('h0'), d.get('m0') if subtract_mean else None,
                                    want_final, subtract_mean, cu)
    odq, odk, odl, odh0, odm0 = O.clean_read_bwd(qr, kr, lr, gr, offset, d.get('h0'),
                                                 d.get('m0') if subtract_mean else None, subtract_mean, cu,
                                                 d.get('dfc') if want_final else None,
                                                 d.get('dfm') if (want_final and subtract_mean) else None)
    pairs = [('q_clean', qc, oq), ('dq', q.grad, odq), ('dk', k.grad, odk), ('dlam', lam.grad, odl)]
    if want_final:
        pairs.append(('final_cov', fc, ofc))
        if subtract_mean:
            pairs.append(('final_mean', fm, ofm))
    if h0 is not None:
        pairs.append(('dh0', h0.grad, odh0))
    if m0 is not None and odm0 is not None:
        pairs.append(('dm0', m0.grad, odm0))
    for name, ours, ref in pairs:
        ours = np64(ours)
        err = rel_err(ours, ref) if rel else float(np.abs(ours - ref).max())
        assert err <= tol, f'{name}: {"rel" if rel else "max-abs"} err {err:.3e} > {tol}'


SHAPES = [
    # (B, T, H, K, lens, states, offset, final_grads, subtract_mean)
    (2, 130, 2, 64, None, False, 0, True, True),
    (1, 1, 3, 128, None, True, 9, True, True),
    (2, 63, 2, 128, None, False, 0, False, True),
    (2, 64, 2, 128, None, False, 0, False, True),
    (2, 65, 2, 128, None, True, 2, True, True),
    (1, 0, 2, 128, [200, 1, 64, 129, 3], True, 7, True, True),
    (2, 300, 2, 128, None, False, -5, False, False),
    (1, 150, 2, 100, None, True, 0, True, True),
    (1, 97, 2, 256, None, True, 3, True, True),
    (2, 77, 3, 16, None, False, 0, True, True),
]


@pytest.mark.parametrize('shape', SHAPES, ids=[f's{i}' for i in range(len(SHAPES))])
def test_oracle_fp32(shape):
    B, T, H, K, lens, states, off, fg, sm = shape
    d, cu, off, sm = make_case(1, B, T, H, K, lens, states, off, fg, sm)
    check_against_oracle(d, cu, off, sm, torch.float32, FP32_TOL, rel=True)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16], ids=['bf16', 'fp16'])
@pytest.mark.parametrize('shape', SHAPES, ids=[f's{i}' for i in range(len(SHAPES))])
def test_oracle_half(shape, dtype):
    B, T, H, K, lens, states, off, fg, sm = shape
    d, cu, off, sm = make_case(2, B, T, H, K, lens, states, off, fg, sm)
    check_against_oracle(d, cu, off, sm, dtype, BF16_TOL, rel=False)


def test_bf16_long_sequence():
    # gradient magnitudes grow with T (C entries ~ T / K): check the bf16 bar at T = 4096
    d, cu, off, sm = make_case(3, 1, 4096, 2, 128)
    check_against_oracle(d, cu, off, sm, torch.bfloat16, BF16_TOL, rel=False)


def test_gated_against_oracle_bf16():
    import ccq_b200
    rng = np.random.default_rng(4)
    B, T, H, K = 2, 333, 4, 128
    qn, kn = unit(rng, (B, T, H, K)), unit(rng, (B, T, H, K))
    W = rng.normal(0, 0.02, (H, K))
    b = rng.uniform(-1, 1, H)
    g = rng.standard_normal((B, T, H, K))
    q, k = dev(qn, torch.bfloat16, True), dev(kn, torch.bfloat16, True)
    Wt, bt = dev(W, grad=True), dev(b, grad=True)
    qc, _, _ = ccq_b200.fused_ccq_clean_gated(q, k, Wt, bt)
    (qc.float() * dev(g)).sum().backward()
    qr, kr, gr = round_to(qn, torch.bfloat16), round_to(kn, torch.bfloat16), round_to(g, torch.bfloat16)
    lam = O.lambda_headwise_fwd(qr, W, b)
    oq, _, _ = O.clean_read_fwd(qr, kr, lam)
    odq, odk, odl, _, _ = O.clean_read_bwd(qr, kr, lam, gr)
    dqx, dW, db = O.lambda_headwise_bwd(qr, W, lam, odl)
    assert np.abs(np64(qc) - oq).max() <= BF16_TOL
    assert np.abs(np64(q.grad) - (odq + dqx)).max() <= BF16_TOL
    assert np.abs(np64(k.grad) - odk).max() <= BF16_TOL
    assert rel_err(np64(Wt.grad), dW) <= 1e-2
    assert rel_err(np64(bt.grad), db) <= 1e-2


def test_decode_against_oracle_bf16():
    import ccq_b200
    rng = np.random.default_rng(5)
    N, H, K = 4, 3, 128
    kk = unit(rng, (N, 50, H, K))
    C0 = np.einsum('nthk,nthv->nhkv', kk, kk)
    m0 = kk.sum(1)
    C, m = dev(C0), dev(m0)
    Cn, mn = C0.copy(), m0.copy()
    for step in range(5):
        q, k = unit(rng, (N, 1, H, K)), unit(rng, (N, 1, H, K))
        lam = rng.uniform(0, 1, (N, 1, H))
        qc, C, m = ccq_b200.decode_step(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(lam, torch.bfloat16),
                                        C, m, position_offset=50 + step)
        oq, Cn, mn = O.decode_clean(round_to(q, torch.bfloat16), round_to(k, torch.bfloat16),
                                    round_to(lam, torch.bfloat16), 50 + step, Cn, mn)
        assert np.abs(np64(qc) - oq).max() <= BF16_TOL
    assert rel_err(np64(C), Cn) <= 1e-5
    assert rel_err(np64(m), mn) <= 1e-5


@pytest.mark.parametrize('N,H,K', [(3, 2, 64), (8, 4, 256)])
def test_decode_inplace_and_gate(N, H, K):
    # K = 256 runs as 4 column tiles per (sequence, head) that share the mean state updated in place
    import ccq_b200
    rng = np.random.default_rng(6)
    kk = unit(rng, (N, 10, H, K))
    C0 = np.einsum('nthk,nthv->nhkv', kk, kk)
    m0 = kk.sum(1)
    C, m = dev(C0), dev(m0)
    W, b = rng.normal(0, 0.1, (H, K)), rng.uniform(-1, 1, H)
    q, k = unit(rng, (N, 3, H, K)), unit(rng, (N, 3, H, K))
    cptr = C.data_ptr()
    qc, C2, m2 = ccq_b200.decode_step(dev(q), dev(k), None, C, m, position_offset=10, gate_w=dev(W), gate_b=dev(b),
                                      inplace=True)
    assert C2.data_ptr() == cptr
    lam = O.lambda_headwise_fwd(q, W, b)
    oq, oC, om = O.decode_clean(q, k, lam, 10, C0, m0)
    assert rel_err(np64(qc), oq) <= FP32_TOL
    assert rel_err(np64(C2), oC) <= FP32_TOL
    assert rel_err(np64(m2), om) <= FP32_TOL


def test_errors_raise():
    import ccq_b200
    q = torch.randn(2, 8, 2, 300, device='cuda')
    with pytest.raises(ccq_b200.CCQError):
        ccq_b200.fused_ccq_clean_read(q, q, 0.5)
    q = torch.randn(2, 8, 2, 64, device='cuda')
    with pytest.raises(ValueError):
        ccq_b200.fused_ccq_clean_read(q, q, 0.5, cu_seqlens=torch.tensor([0, 8], device='cuda'))
    with pytest.raises(RuntimeError):
        ccq_b200.fused_ccq_clean_read(q.cpu(), q.cpu(), 0.5)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16], ids=['bf16', 'fp16'])
@pytest.mark.parametrize('case', [
    dict(B=2, T=1000, H=3, lens=None, states=True, off=0, gate=False, sm=True),
    dict(B=1, T=0, H=2, lens=[300, 1, 128, 129, 7, 256], states=True, off=4, gate=False, sm=True),
    dict(B=3, T=257, H=2, lens=None, states=False, off=-3, gate=True, sm=True),
    dict(B=2, T=200, H=2, lens=None, states=True, off=0, gate=False, sm=False),
], ids=['dense', 'varlen', 'gate', 'nomean'])
def test_tcgen05_forward_path(case, dtype, monkeypatch):
    """bf16/fp16 with K = 128 runs the tcgen05 forward; it agrees with the exact SIMT forward and the oracle."""
    import ccq_b200
    from ccq_b200 import ops
    rng = np.random.default_rng(7)
    lens = case['lens']
    B, T, H, K = case['B'], case['T'], case['H'], 128
    if lens is not None:
        B, T = 1, int(sum(lens))
    N = B if lens is None else len(lens)
    cu = None if lens is None else dev(np.concatenate([[0], np.cumsum(lens)]), torch.int64)
    q = dev(unit(rng, (B, T, H, K)), dtype)
    k = dev(unit(rng, (B, T, H, K)), dtype)
    lam = dev(rng.uniform(0, 1, (B, T, H)), dtype)
    W = dev(rng.normal(0, 0.05, (H, K)))
    b = dev(rng.uniform(-1, 1, H))
    h0 = m0 = None
    if case['states']:
        kk = unit(rng, (N, 20, H, K))
        h0 = dev(np.einsum('nthk,nthv->nhkv', kk, kk))
        m0 = dev(kk.sum(1)) if case['sm'] else None
    cu_, _ = ops._seqs(B, cu)

    def run():
        if case['gate']:
            return ops.clean_fwd_raw(q, k, None, W, b, case['off'], h0, m0, case['sm'], cu_, N)
        return ops.clean_fwd_raw(q, k, lam, None, None, case['off'], h0, m0, case['sm'], cu_, N)

    qc, fc, fm, aux = run()
    assert ccq_b200.last_path() == 'tcgen05'
    monkeypatch.setenv('CCQ_B200_FORCE_SIMT', '1')
    qs, fcs, fms, auxs = run()
    assert ccq_b200.last_path() == 'simt'
    monkeypatch.delenv('CCQ_B200_FORCE_SIMT')
    assert (qc.float() - qs.float()).abs().max().item() <= BF16_TOL
    assert rel_err(np64(fc), np64(fcs)) <= 1e-5
    if case['sm']:
        assert rel_err(np64(fm), np64(fms)) <= 1e-5
    assert rel_err(np64(aux), np64(auxs)) <= 1e-3
    # and the oracle on the rounded inputs
    lam_np = (O.lambda_headwise_fwd(np64(q), np64(W), np64(b)) if case['gate'] else np64(lam))
    oq, ofc, ofm = O.clean_read_fwd(np64(q), np64(k), lam_np, case['off'], None if h0 is None else np64(h0),
                                    None if m0 is None else np64(m0), True, case['sm'],
                                    None if cu is None else cu.cpu().numpy())
    assert np.abs(np64(qc) - oq).max() <= BF16_TOL
    assert rel_err(np64(fc), ofc) <= 1e-5


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16], ids=['bf16', 'fp16'])
@pytest.mark.parametrize('case', [
    dict(B=2, T=1000, H=3, lens=None, states=True, off=0, gate=False, sm=True, fg=True),
    dict(B=1, T=0, H=2, lens=[300, 1, 64, 65, 7, 256], states=True, off=4, gate=False, sm=True, fg=True),
    dict(B=3, T=257, H=2, lens=None, states=False, off=-3, gate=True, sm=True, fg=False),
    dict(B=2, T=200, H=2, lens=None, states=True, off=0, gate=False, sm=False, fg=True),
    dict(B=1, T=63, H=4, lens=None, states=False, off=0, gate=True, sm=True, fg=False),
], ids=['dense', 'varlen', 'gate', 'nomean', 'short'])
def test_tcgen05_backward_path(case, dtype, monkeypatch):
    """bf16/fp16 with K = 128 runs the tcgen05 backward; it agrees with the exact SIMT backward and the oracle."""
    import ccq_b200
    from ccq_b200 import ops
    rng = np.random.default_rng(11)
    lens = case['lens']
    B, T, H, K = case['B'], case['T'], case['H'], 128
    if lens is not None:
        B, T = 1, int(sum(lens))
    N = B if lens is None else len(lens)
    cu = None if lens is None else dev(np.concatenate([[0], np.cumsum(lens)]), torch.int64)
    q = dev(unit(rng, (B, T, H, K)), dtype)
    k = dev(unit(rng, (B, T, H, K)), dtype)
    lam = dev(rng.uniform(0, 1, (B, T, H)), dtype)
    g = dev(rng.standard_normal((B, T, H, K)), dtype)
    W = dev(rng.normal(0, 0.05, (H, K)))
    b = dev(rng.uniform(-1, 1, H))
    h0 = m0 = dfc = dfm = None
    if case['states']:
        kk = unit(rng, (N, 20, H, K))
        h0 = dev(np.einsum('nthk,nthv->nhkv', kk, kk))
        m0 = dev(kk.sum(1)) if case['sm'] else None
    if case['fg']:
        dfc = dev(rng.standard_normal((N, H, K, K)) / np.sqrt(K))
        dfm = dev(rng.standard_normal((N, H, K)) / np.sqrt(K)) if case['sm'] else None
    cu_, _ = ops._seqs(B, cu)
    gw, gb = (W, b) if case['gate'] else (None, None)
    lam3 = None if case['gate'] else lam

    qc, fc, fm, aux = ops.clean_fwd_raw(q, k, lam3, gw, gb, case['off'], h0, m0, case['sm'], cu_, N)
    res = ops.clean_bwd_raw(q, k, lam3, gw, gb, case['off'], h0, m0, case['sm'], cu_, N, fc, fm, aux, g, dfc, dfm)
    assert ccq_b200.last_path() == 'tcgen05'
    monkeypatch.setenv('CCQ_B200_FORCE_SIMT', '1')
    ref = ops.clean_bwd_raw(q, k, lam3, gw, gb, case['off'], h0, m0, case['sm'], cu_, N, fc, fm, aux, g, dfc, dfm)
    assert ccq_b200.last_path() == 'simt'
    monkeypatch.delenv('CCQ_B200_FORCE_SIMT')
    dq, dk, dl, dh0, dm0 = res
    rdq, rdk, rdl, rdh0, rdm0 = ref
    assert (dq.float() - rdq.float()).abs().max().item() <= BF16_TOL
    assert (dk.float() - rdk.float()).abs().max().item() <= BF16_TOL
    if case['gate']:
        assert rel_err(np64(dl[0]), np64(rdl[0])) <= 1e-2
        assert rel_err(np64(dl[1]), np64(rdl[1])) <= 1e-2
    else:
        assert (dl - rdl).abs().max().item() <= BF16_TOL
    if h0 is not None:
        assert rel_err(np64(dh0), np64(rdh0)) <= 1e-2
    if dm0 is not None:
        assert rel_err(np64(dm0), np64(rdm0)) <= 1e-2
    # oracle on the rounded inputs
    qn, kn, gn = np64(q), np64(k), np64(g)
    lam_np = O.lambda_headwise_fwd(qn, np64(W), np64(b)) if case['gate'] else np64(lam)
    cun = None if cu is None else cu.cpu().numpy()
    odq, odk, odl, _, _ = O.clean_read_bwd(qn, kn, lam_np, gn, case['off'], None if h0 is None else np64(h0),
                                           None if m0 is None else np64(m0), case['sm'], cun,
                                           None if dfc is None else np64(dfc), None if dfm is None else np64(dfm))
    if case['gate']:
        dqx, oW, ob = O.lambda_headwise_bwd(qn, np64(W), lam_np, odl)
        odq = odq + dqx
        assert rel_err(np64(dl[0]), oW) <= 1e-2
    assert np.abs(np64(dq) - odq).max() <= BF16_TOL
    assert np.abs(np64(dk) - odk).max() <= BF16_TOL


@pytest.mark.parametrize('gate', [False, True], ids=['lambda', 'gate'])
def test_tcgen05_deterministic(gate):
    """Repeated runs of the tensor-core forward and backward give bitwise-equal outputs: every
    hand-off between warps is ordered (a race shows up here long before it breaks a tolerance)."""
    import ccq_b200
    from ccq_b200 import ops
    rng = np.random.default_rng(21)
    B, T, H, K = 2, 1500, 4, 128
    q = dev(unit(rng, (B, T, H, K)), torch.bfloat16)
    k = dev(unit(rng, (B, T, H, K)), torch.bfloat16)
    lam = None if gate else dev(rng.uniform(0, 1, (B, T, H)), torch.bfloat16)
    W = dev(rng.normal(0, 0.05, (H, K))) if gate else None
    b = dev(rng.uniform(-1, 1, H)) if gate else None
    g = dev(rng.standard_normal((B, T, H, K)), torch.bfloat16)
    dfc = dev(rng.standard_normal((B, H, K, K)) / np.sqrt(K))
    dfm = dev(rng.standard_normal((B, H, K)) / np.sqrt(K))
    runs = []
    for _ in range(4):
        qc, fc, fm, aux = ops.clean_fwd_raw(q, k, lam, W, b, 0, None, None, True, None, B)
        assert ccq_b200.last_path() == 'tcgen05'
        dq, dk, dl, _, _ = ops.clean_bwd_raw(q, k, lam, W, b, 0, None, None, True, None, B, fc, fm, aux, g, dfc, dfm)
        assert ccq_b200.last_path() == 'tcgen05'
        runs.append((qc, fc, fm, aux, dq, dk, dl))
    for other in runs[1:]:
        for x, y in zip(runs[0][:6], other[:6]):
            assert torch.equal(x, y)
        if gate:  # dW sums per-document partials in a fixed order; db also adds per-warp atomics
            assert torch.equal(runs[0][6][0], other[6][0])
            assert rel_err(np64(other[6][1]), np64(runs[0][6][1])) <= 1e-5
        else:
            assert torch.equal(runs[0][6], other[6])
