"""The L2 normalisation of q and k fused into the operator (ccq_clean_l2norm_fwd / _bwd through
ops.fused_ccq_clean_read_l2norm), against the float64 oracle of fla's l2norm followed by the operator.

The oracle normalises the raw inputs in float64 and rounds the result to the activation dtype (what
the reference's l2norm stores and its operator reads), runs the operator's forward and backward on
those, adds the gradient arriving on the normalised keys from the backbone, and maps both gradients
back through the normalisation (fla/modules/l2norm.py:49-72).  Bars as elsewhere: fp32 1e-5 relative,
bf16 / fp16 2e-2 max-abs.  16-bit inputs with K = 128 run the tensor-core kernels, which normalise the
tiles they load; they are also checked against the exact path.
"""
import numpy as np
import pytest
import torch

from golden_util import rel_err
from oracle import ccq_oracle as O

pytestmark = pytest.mark.gpu

CASES = {
    'dense': dict(B=2, T=300, H=3, K=128, lens=None, states=False, off=0, sm=True, fg=False),
    'varlen_states': dict(B=1, T=0, H=2, K=128, lens=[200, 1, 77, 129, 3], states=True, off=5, sm=True, fg=True),
    'nomean': dict(B=2, T=130, H=2, K=128, lens=None, states=False, off=0, sm=False, fg=False),
    'k64': dict(B=2, T=150, H=2, K=64, lens=None, states=True, off=2, sm=True, fg=True),
}


@pytest.fixture(scope='module', autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from ccq_b200 import _lib as L
    L.load()


def _np(t):
    return None if t is None else t.detach().double().cpu().numpy()


def _run(case, dtype, seed=3, key_grad=True):
    import ccq_b200
    c = CASES[case]
    g = torch.Generator(device='cuda').manual_seed(seed)
    lens = c['lens']
    B, T, H, K = c['B'], (sum(lens) if lens else c['T']), c['H'], c['K']
    N = len(lens) if lens else B
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int64, device='cuda') if lens else None
    # raw inputs of varied norms (the layer's projections are not unit vectors)
    q0 = torch.randn(B, T, H, K, generator=g, device='cuda') * (0.5 + torch.rand(B, T, H, 1, generator=g, device='cuda'))
    k0 = torch.randn(B, T, H, K, generator=g, device='cuda') * (0.5 + torch.rand(B, T, H, 1, generator=g, device='cuda'))
    lam0 = torch.rand(B, T, H, generator=g, device='cuda')
    dqc = torch.randn(B, T, H, K, generator=g, device='cuda').to(dtype)
    dkn = torch.randn(B, T, H, K, generator=g, device='cuda').to(dtype)
    if not key_grad:  # nothing downstream reads the normalised keys: no gradient arrives on them
        dkn = torch.zeros_like(dkn)
    h00 = m00 = dfc = dfm = None
    if c['states']:
        kk = torch.nn.functional.normalize(torch.randn(N, 16, H, K, generator=g, device='cuda'), dim=-1)
        h00 = torch.einsum('nthk,nthv->nhkv', kk, kk)
        m00 = kk.sum(1)
    if c['fg']:
        dfc = torch.randn(N, H, K, K, generator=g, device='cuda') / K ** 0.5
        dfm = torch.randn(N, H, K, generator=g, device='cuda') / K ** 0.5 if c['sm'] else None
    q = q0.to(dtype).requires_grad_(True)
    k = k0.to(dtype).requires_grad_(True)
    lam = lam0.to(dtype).requires_grad_(True)
    h0 = h00.clone().requires_grad_(True) if h00 is not None else None
    m0 = m00.clone().requires_grad_(True) if (m00 is not None and c['sm']) else None
    qc, kn, fc, fm = ccq_b200.fused_ccq_clean_read_l2norm(q, k, lam, position_offset=c['off'], initial_cov_state=h0,
                                                          initial_mean_state=m0, output_final_state=True,
                                                          subtract_mean=c['sm'], cu_seqlens=cu)
    path = ccq_b200.last_path()
    loss = (qc.float() * dqc.float()).sum()
    if key_grad:
        loss = loss + (kn.float() * dkn.float()).sum()
    if dfc is not None:
        loss = loss + (fc * dfc).sum()
    if dfm is not None:
        loss = loss + (fm * dfm).sum()
    loss.backward()
    out = dict(q_clean=qc, k_norm=kn, final_cov=fc, final_mean=fm, dq=q.grad, dk=k.grad, dlam=lam.grad,
               dh0=None if h0 is None else h0.grad, dm0=None if m0 is None else m0.grad)
    inp = dict(q=q, k=k, lam=lam, dqc=dqc, dkn=dkn, h0=h00, m0=m00 if c['sm'] else None, dfc=dfc, dfm=dfm, cu=cu)
    return out, inp, path


def _oracle(case, inp, dtype):
    c = CASES[case]
    rnd = (lambda x: torch.tensor(x, dtype=torch.float64).to(dtype).double().numpy())
    qh, rq = O.l2norm_fwd(_np(inp['q']), round_to=rnd)
    kh, rk = O.l2norm_fwd(_np(inp['k']), round_to=rnd)
    cun = None if inp['cu'] is None else inp['cu'].cpu().numpy()
    lam = _np(inp['lam'])
    oq, ofc, ofm = O.clean_read_fwd(qh, kh, lam, c['off'], _np(inp['h0']), _np(inp['m0']), True, c['sm'], cun)
    dqh, dkh, dl, dh0, dm0 = O.clean_read_bwd(qh, kh, lam, _np(inp['dqc']), c['off'], _np(inp['h0']), _np(inp['m0']),
                                              c['sm'], cun, _np(inp['dfc']), _np(inp['dfm']))
    dk_tot = rnd(rnd(dkh) + _np(inp['dkn'])) if dtype != torch.float32 else dkh + _np(inp['dkn'])
    return dict(q_clean=oq, k_norm=kh, final_cov=ofc, final_mean=ofm, dq=O.l2norm_bwd(qh, rq, dqh),
                dk=O.l2norm_bwd(kh, rk, dk_tot), dlam=dl, dh0=dh0, dm0=dm0)


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16, torch.float16], ids=['fp32', 'bf16', 'fp16'])
@pytest.mark.parametrize('case', list(CASES), ids=list(CASES))
def test_l2norm_fused_against_oracle(case, dtype):
    out, inp, path = _run(case, dtype)
    expect_tc = dtype != torch.float32 and CASES[case]['K'] == 128
    assert path == ('tcgen05' if expect_tc else 'simt')
    ref = _oracle(case, inp, dtype)
    for name, val in out.items():
        if val is None:
            assert ref[name] is None, name
            continue
        a = _np(val)
        if dtype == torch.float32 or name in ('final_cov', 'final_mean', 'dh0', 'dm0'):
            tol = 1e-5 if dtype == torch.float32 else 1e-2
            e = rel_err(a, ref[name])
            assert e <= tol, f'{case}.{name}: rel err {e:.3e}'
        else:
            e = float(np.abs(a - ref[name]).max())
            assert e <= 2e-2, f'{case}.{name}: max-abs err {e:.3e}'


@pytest.mark.parametrize('case', ['dense', 'varlen_states'])
def test_l2norm_without_key_gradient(case):
    """The normalised keys feed nothing downstream, so the backward gets no gradient on them (a null
    pointer through the C ABI): the key gradient is the operator's own, mapped through the norm."""
    out, inp, path = _run(case, torch.bfloat16, seed=11, key_grad=False)
    assert path == 'tcgen05'
    ref = _oracle(case, inp, torch.bfloat16)
    for name in ('q_clean', 'dq', 'dk', 'dlam'):
        e = float(np.abs(_np(out[name]) - ref[name]).max())
        assert e <= 2e-2, f'{case}.{name}: max-abs err {e:.3e}'


@pytest.mark.parametrize('case', ['dense', 'varlen_states'])
def test_l2norm_tcgen05_matches_exact_path(case, monkeypatch):
    out, _, path = _run(case, torch.bfloat16, seed=8)
    assert path == 'tcgen05'
    monkeypatch.setenv('CCQ_B200_FORCE_SIMT', '1')
    ref, _, path = _run(case, torch.bfloat16, seed=8)
    assert path == 'simt'
    monkeypatch.delenv('CCQ_B200_FORCE_SIMT')
    for name in ('q_clean', 'k_norm', 'dq', 'dk', 'dlam'):
        e = (out[name].float() - ref[name].float()).abs().max().item()
        assert e <= 2e-2, (name, e)
    assert torch.equal(out['k_norm'], ref['k_norm']) or (out['k_norm'].float() - ref['k_norm'].float()).abs().max() <= 8e-3


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16], ids=['fp32', 'bf16'])
@pytest.mark.parametrize('K', [64, 128, 256])
def test_decode_l2norm_against_oracle(dtype, K):
    """decode_step_l2norm (ccq_decode_step_l2norm): raw q, k of a few tokens normalised in the decode
    kernel, on a cache built from a prefix; the cache update uses the normalised keys."""
    import ccq_b200
    g = torch.Generator(device='cuda').manual_seed(21)
    N, H, T, P = 3, 2, 2, 30
    kk = torch.nn.functional.normalize(torch.randn(N, P, H, K, generator=g, device='cuda'), dim=-1)
    C0 = torch.einsum('nthk,nthv->nhkv', kk, kk)
    m0 = kk.sum(1)
    q = (torch.randn(N, T, H, K, generator=g, device='cuda') * 3).to(dtype)
    k = (torch.randn(N, T, H, K, generator=g, device='cuda') * 3).to(dtype)
    lam = torch.rand(N, T, H, generator=g, device='cuda').to(dtype)
    qc, kn, C1, m1 = ccq_b200.decode_step_l2norm(q, k, lam, C0, m0, position_offset=P)
    assert ccq_b200.last_path() == 'decode'
    rnd = (lambda a: torch.tensor(a).to(dtype).double().numpy())
    qh, _ = O.l2norm_fwd(_np(q), round_to=rnd)
    kh, _ = O.l2norm_fwd(_np(k), round_to=rnd)
    oq, oC, om = O.decode_clean(qh, kh, _np(lam), P, _np(C0), _np(m0))
    if dtype == torch.float32:
        assert rel_err(_np(qc), oq) <= 1e-5
        assert rel_err(_np(kn), kh) <= 1e-6
    else:
        assert np.abs(_np(qc) - oq).max() <= 2e-2
        assert np.abs(_np(kn) - kh).max() <= 8e-3
    assert rel_err(_np(C1), oC) <= 1e-5
    assert rel_err(_np(m1), om) <= 1e-5
