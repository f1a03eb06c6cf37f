"""The drop-in, run on the GPU through the reference's own entry points.

The reference package (its pip install under baseline/_ref, or CCQ_REFERENCE_PATH) runs here
natively: its Triton kernels JIT-compile on the B200.  Each test calls a reference entry point twice
on the same seeded inputs, once as shipped and once after ``ccq_b200.integration.install()`` has
routed its cleaning operator to this library, and compares every output and gradient.  The strict
bars are against the float64 oracle (fp32: 1e-5 relative; bf16 / fp16: 2e-2 max-abs on the
inputs the operator actually received); the reference's own outputs are compared at looser bounds
and the differences printed.

The reference compiles its Triton kernels (and fla's, which it calls) on first use, and autotunes
each over many configurations; on the B200 that costs seconds per kernel for the operator itself but
tens of minutes for fla's backbones, and far more for fp32 under TRITON_F32_DEFAULT=ieee.  So:
  * the operator-level tests run by default, at K = 128, in bf16 and in fp32; the fp32 reference
    runs with Triton's default TF32 dots, so it is compared at a TF32-sized bound (the strict fp32 bar
    is against the oracle);
  * the entry points that run fla's backbones (the attn_mode orchestrators and the decode routes)
    run only with CCQ_TEST_REFERENCE_BACKBONES=1, in bf16.
"""
import os
import sys

import numpy as np
import pytest
import torch

from golden_util import rel_err
from oracle import ccq_oracle as O

pytestmark = pytest.mark.gpu

backbones = pytest.mark.skipif(os.environ.get('CCQ_TEST_REFERENCE_BACKBONES') != '1',
                               reason='compiles fla backbones for many minutes; set CCQ_TEST_REFERENCE_BACKBONES=1')

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope='module')
def ref():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    sys.path.insert(0, ROOT)
    from bench import reference_path
    path = reference_path()
    if path is None:
        pytest.skip('reference package not installed (baseline/_ref or CCQ_REFERENCE_PATH)')
    if path not in sys.path:
        sys.path.insert(0, path)
    import ccq.ops.ccq_gdn.fused_chunk as gdn_chunk
    import ccq.ops.ccq_gdn.fused_recurrent as gdn_rec
    import ccq.ops.ccq_gla.fused_chunk as gla_chunk
    import ccq.ops.ccq_gla.fused_recurrent as gla_rec
    import ccq.ops.common.fused_read as fused_read

    from ccq_b200 import _lib, integration
    _lib.load()
    integration.uninstall()
    yield dict(fused_read=fused_read, gdn_chunk=gdn_chunk, gla_chunk=gla_chunk, gdn_rec=gdn_rec, gla_rec=gla_rec)
    integration.uninstall()


def _np(t):
    return None if t is None else t.detach().double().cpu().numpy()


def _unit(g, shape):
    x = torch.randn(shape, generator=g, device='cuda')
    return x / x.norm(dim=-1, keepdim=True)


def _leaf(x, dtype):
    return None if x is None else x.to(dtype).detach().requires_grad_(True)


def _check(name, ours, ref_out, oracle, dtype, ref_tol):
    """ours vs the oracle at the operator's bar, ours vs the reference at `ref_tol`; prints both."""
    ours = _np(ours)
    if oracle is not None:
        if dtype == torch.float32:
            e = rel_err(ours, oracle)
            assert e <= 1e-5, f'{name}: rel err vs oracle {e:.3e}'
        else:
            e = float(np.abs(ours - oracle).max())
            assert e <= 2e-2, f'{name}: max-abs err vs oracle {e:.3e}'
    if ref_out is not None:
        r = _np(ref_out)
        e_abs = float(np.abs(ours - r).max())
        e_rel = rel_err(ours, r)
        print(f'{name} [{dtype}]: vs reference max-abs {e_abs:.3e}, rel {e_rel:.3e}')
        assert e_rel <= ref_tol, f'{name}: rel diff vs reference {e_rel:.3e} > {ref_tol}'


# ------------------------------------------------------------------------------------------------
# the operator itself: ccq.ops.common.fused_read.fused_ccq_clean_read (fused_read.py:517-531)
# ------------------------------------------------------------------------------------------------

OP_CASES = {
    'dense_states': dict(B=2, T=300, H=4, K=128, lens=None, states=True, off=3, sm=True),
    'varlen': dict(B=1, T=0, H=2, K=128, lens=[200, 1, 77, 129], states=True, off=0, sm=True),
}


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16], ids=['fp32', 'bf16'])
@pytest.mark.parametrize('case', list(OP_CASES), ids=list(OP_CASES))
def test_fused_ccq_clean_read_against_reference(ref, case, dtype):
    import ccq_b200
    c = OP_CASES[case]
    g = torch.Generator(device='cuda').manual_seed(11)
    lens = c['lens']
    B, T, H, K = c['B'], (sum(lens) if lens else c['T']), c['H'], c['K']
    N = len(lens) if lens else B
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int64, device='cuda') if lens else None
    q0, k0 = _unit(g, (B, T, H, K)), _unit(g, (B, T, H, K))
    lam0 = torch.rand(B, T, H, generator=g, device='cuda')
    dqc = torch.randn(B, T, H, K, generator=g, device='cuda').to(dtype)
    h00 = m00 = dfc = dfm = None
    if c['states']:
        kk = _unit(g, (N, 16, H, K))
        h00 = torch.einsum('nthk,nthv->nhkv', kk, kk)
        m00 = kk.sum(1)
        dfc = torch.randn(N, H, K, K, generator=g, device='cuda') / K ** 0.5
        dfm = torch.randn(N, H, K, generator=g, device='cuda') / K ** 0.5 if c['sm'] else None

    def run(fn):
        q, k, lam = _leaf(q0, dtype), _leaf(k0, dtype), _leaf(lam0, dtype)
        h0, m0 = _leaf(h00, torch.float32), _leaf(m00 if c['sm'] else None, torch.float32)
        qc, fc, fm = fn(q, k, lam, position_offset=c['off'], initial_cov_state=h0, initial_mean_state=m0,
                        output_final_state=True, subtract_mean=c['sm'], cu_seqlens=cu)
        loss = (qc.float() * dqc.float()).sum()
        if dfc is not None:
            loss = loss + (fc * dfc).sum()
        if dfm is not None and fm is not None:
            loss = loss + (fm * dfm).sum()
        loss.backward()
        return dict(q_clean=qc, final_cov=fc, final_mean=fm, dq=q.grad, dk=k.grad, dlam=lam.grad,
                    dh0=None if h0 is None else h0.grad, dm0=None if m0 is None else m0.grad)

    theirs = run(ref['fused_read'].fused_ccq_clean_read)
    ours = run(ccq_b200.fused_ccq_clean_read)
    rd = lambda t: _np(t.to(dtype))  # noqa: E731  inputs as the operator saw them
    cun = None if cu is None else cu.cpu().numpy()
    oq, ofc, ofm = O.clean_read_fwd(rd(q0), rd(k0), rd(lam0), c['off'], _np(h00), _np(m00) if c['sm'] else None,
                                    True, c['sm'], cun)
    odq, odk, odl, odh0, odm0 = O.clean_read_bwd(rd(q0), rd(k0), rd(lam0), _np(dqc), c['off'], _np(h00),
                                                 _np(m00) if c['sm'] else None, c['sm'], cun, _np(dfc), _np(dfm))
    oracle = dict(q_clean=oq, final_cov=ofc, final_mean=ofm, dq=odq, dk=odk, dlam=odl, dh0=odh0, dm0=odm0)
    ref_tol = 1e-2 if dtype == torch.float32 else 3e-2  # fp32 reference: TF32 dots
    for name, val in ours.items():
        if val is None:
            assert theirs[name] is None, name
            continue
        orc = oracle[name]
        if dtype != torch.float32 and name in ('final_cov', 'final_mean', 'dh0', 'dm0'):
            # fp32 outputs of a 16-bit call: relative bar, the states sum thousands of products
            assert rel_err(_np(val), orc) <= 1e-2, name
            orc = None
        _check(f'{case}.{name}', val, theirs[name], orc, dtype, ref_tol)


# ------------------------------------------------------------------------------------------------
# the layers' attn_mode "fused_chunk" orchestrators and the decode routes, patched vs as shipped
# ------------------------------------------------------------------------------------------------

class _Recorder:
    """Wraps ops.fused_ccq_clean_read_l2norm (what the B200 orchestrators call) to keep the raw inputs
    and outputs of its last call."""

    def __init__(self):
        from ccq_b200 import ops
        self.ops = ops
        self.fn = ops.fused_ccq_clean_read_l2norm
        self.last = None

    def __call__(self, q, k, lambda_h, **kw):
        out = self.fn(q, k, lambda_h, **kw)
        self.last = (q.detach().clone(), k.detach().clone(), lambda_h.detach().clone(), kw, out[0].detach().clone(),
                     out[1].detach().clone())
        return out

    def __enter__(self):
        self.ops.fused_ccq_clean_read_l2norm = self
        return self

    def __exit__(self, *exc):
        self.ops.fused_ccq_clean_read_l2norm = self.fn


def _orchestrator_inputs(dtype, B=2, T=200, H=4, K=128, V=64, seed=5):
    import torch.nn.functional as F
    g = torch.Generator(device='cuda').manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, device='cuda')  # noqa: E731
    return dict(q=r(B, T, H, K), k=r(B, T, H, K), v=r(B, T, H, V), lam=torch.rand(B, T, H, generator=g, device='cuda'),
                g=F.logsigmoid(r(B, T, H)) * 0.1, gk=F.logsigmoid(r(B, T, H, K)) * 0.1, beta=torch.sigmoid(r(B, T, H)),
                do=r(B, T, H, V), dfs=r(B, H, K, V) * 0.1, dfc=r(B, H, K, K) / K ** 0.5, dfm=r(B, H, K) / K ** 0.5)


def _run_orchestrator(fn, x, dtype, gla):
    q, k, v, lam = (_leaf(x[n], dtype) for n in ('q', 'k', 'v', 'lam'))
    if gla:
        gk = _leaf(x['gk'], torch.float32)
        o, fs, fc, fm = fn(q, k, v, lam, g=gk, output_final_state=True)
        extra = dict(dgk=gk)
    else:
        g_, beta = _leaf(x['g'], torch.float32), _leaf(x['beta'], dtype)
        o, fs, fc, fm = fn(q, k, v, lam, g_, beta, output_final_state=True, use_qk_l2norm_in_kernel=True)
        extra = dict(dg=g_, dbeta=beta)
    loss = (o.float() * x['do']).sum() + (fs.float() * x['dfs']).sum() + (fc * x['dfc']).sum() + (fm * x['dfm']).sum()
    loss.backward()
    out = dict(o=o, final_state=fs, final_cov=fc, final_mean=fm, dq=q.grad, dk=k.grad, dv=v.grad, dlam=lam.grad)
    out.update({n: t.grad for n, t in extra.items()})
    return out


@backbones
@pytest.mark.parametrize('dtype', [torch.bfloat16], ids=['bf16'])
@pytest.mark.parametrize('attn_mode', ['fused_chunk', 'chunk'])
@pytest.mark.parametrize('mode', ['gdn', 'gla'])
def test_orchestrator_patched_vs_shipped(ref, mode, attn_mode, dtype):
    """The layers' attn_mode entry points: fused_chunk_ccq_gdn (ccq/ops/ccq_gdn/fused_chunk.py:16-59),
    fused_chunk_ccq_gla (ccq/ops/ccq_gla/fused_chunk.py:16-46), chunk_ccq_gdn (ccq/ops/ccq_gdn/chunk.py:11-87)
    and chunk_ccq_gla (ccq/ops/ccq_gla/chunk.py:17-64), looked up by name in the reference's package as its
    layers do (ccq/gdn/layer.py:14-18), as shipped and after install()."""
    import importlib

    from ccq_b200 import integration
    pkg = importlib.import_module(f'ccq.ops.ccq_{mode}')
    fname = f'{attn_mode}_ccq_{mode}'
    x = _orchestrator_inputs(dtype)
    shipped = _run_orchestrator(getattr(pkg, fname), x, dtype, mode == 'gla')
    integration.install()
    try:
        assert getattr(pkg, fname) is getattr(integration, fname)
        with _Recorder() as rec:
            patched = _run_orchestrator(getattr(pkg, fname), x, dtype, mode == 'gla')
    finally:
        integration.uninstall()
    assert rec.last is not None, 'the patched orchestrator did not reach the fused l2norm + cleaning operator'
    # the operator's outputs against the oracle: fla's l2norm then the cleaning, on the raw inputs it got
    q, k, lam, kw, qc, kn = rec.last
    rnd = (lambda a: torch.tensor(a).to(dtype).double().numpy())
    qh, _ = O.l2norm_fwd(_np(q), round_to=rnd)
    kh, _ = O.l2norm_fwd(_np(k), round_to=rnd)
    oq, _, _ = O.clean_read_fwd(qh, kh, _np(lam), kw.get('position_offset', 0), None, None, False,
                                kw.get('subtract_mean', True), None)
    _check(f'{mode}.{attn_mode}.k_norm', kn, None, kh, dtype, None)
    _check(f'{mode}.{attn_mode}.q_clean', qc, None, oq, dtype, None)
    # chunk mode's reference reads z through fla's chunk_simple_gla (a different summation than its
    # fused_chunk kernels): a slightly looser bound against it in fp32
    tol = 3e-2
    for name, val in patched.items():
        _check(f'{mode}.{attn_mode}.{name}', val, shipped[name], None, dtype, tol)


@backbones
@pytest.mark.parametrize('dtype', [torch.bfloat16], ids=['bf16'])
@pytest.mark.parametrize('mode', ['gdn', 'gla'])
def test_decode_route_patched_vs_shipped(ref, mode, dtype):
    """fused_recurrent_ccq_gdn (ccq/ops/ccq_gdn/fused_recurrent.py:18-75) and fused_recurrent_ccq_gla
    (ccq/ops/ccq_gla/fused_recurrent.py:9-51): one decode token on a cache built from a prefix."""
    from ccq_b200 import integration
    B, H, K, V, P = 3, 4, 128, 64, 40
    g = torch.Generator(device='cuda').manual_seed(9)
    kk = _unit(g, (B, P, H, K))
    cov = torch.einsum('nthk,nthv->nhkv', kk, kk)
    mean = kk.sum(1)
    S0 = torch.randn(B, H, K, V, generator=g, device='cuda') * 0.1
    q = torch.randn(B, 1, H, K, generator=g, device='cuda').to(dtype)
    k = torch.randn(B, 1, H, K, generator=g, device='cuda').to(dtype)
    v = torch.randn(B, 1, H, V, generator=g, device='cuda').to(dtype)
    lam = torch.rand(B, 1, H, generator=g, device='cuda').to(dtype)
    gg = torch.nn.functional.logsigmoid(torch.randn(B, 1, H, generator=g, device='cuda'))
    gk = torch.nn.functional.logsigmoid(torch.randn(B, 1, H, K, generator=g, device='cuda'))
    beta = torch.sigmoid(torch.randn(B, 1, H, generator=g, device='cuda')).to(dtype)

    def call():
        kw = dict(initial_state=S0.clone(), initial_cov_state=cov.clone(), initial_mean_state=mean.clone(),
                  output_final_state=True, position_offset=P)
        with torch.no_grad():
            if mode == 'gdn':
                return ref['gdn_rec'].fused_recurrent_ccq_gdn(q, k, v, lam, g=gg, beta=beta,
                                                             use_qk_l2norm_in_kernel=True, **kw)
            return ref['gla_rec'].fused_recurrent_ccq_gla(q, k, v, lam, gk=gk, **kw)

    shipped = call()
    integration.install()
    try:
        if mode == 'gla':  # the layer module imported the name before install(): call the rebound one
            import ccq.ops.ccq_gla.fused_recurrent as m
            assert m.fused_recurrent_ccq_gla is integration.fused_recurrent_ccq_gla
        patched = call()
    finally:
        integration.uninstall()
    tol = 3e-2
    for name, a, b in zip(('o', 'final_state', 'final_cov', 'final_mean'), patched, shipped):
        _check(f'{mode}-decode.{name}', a, b, None, dtype, tol)
