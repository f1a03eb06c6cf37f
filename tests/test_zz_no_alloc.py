"""ccq_clean_bwd_noalloc (fixed scratch in the library's device data) against ccq_clean_bwd with a
caller-provided workspace, both called through the C ABI on the same inputs.

Collected last on purpose: it must pass in a fresh process and after every other test, whatever
those left in the shared scratch."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _case(dtype, gate, B, T, H, K, seed):
    from ccq_b200 import ops
    dev = torch.device('cuda', 0)
    g = torch.Generator(device=dev).manual_seed(seed)

    def unit(shape):
        x = torch.randn(shape, generator=g, device=dev)
        return (x / x.norm(dim=-1, keepdim=True)).to(dtype)

    q, k = unit((B, T, H, K)), unit((B, T, H, K))
    dqc = (torch.randn(B, T, H, K, generator=g, device=dev) * 0.5).to(dtype)
    if gate:
        W = torch.randn(H, K, generator=g, device=dev) * 0.02
        b = torch.rand(H, generator=g, device=dev) * 2 - 1
        lam = None
    else:
        W = b = None
        lam = torch.rand(B, T, H, generator=g, device=dev).to(dtype)
    qc, fcov, fmean, aux = ops.clean_fwd_raw(q, k, lam, W, b, 0, None, None, True, None, B)
    return dict(q=q, k=k, dqc=dqc, W=W, b=b, lam=lam, fcov=fcov, fmean=fmean, aux=aux, B=B, T=T, H=H, K=K)


def _outputs(c):
    dev = c['q'].device
    gate = c['W'] is not None
    return dict(dq=torch.empty_like(c['q']), dk=torch.empty_like(c['k']),
                dlam=None if gate else torch.empty(c['B'], c['T'], c['H'], device=dev),
                dW=torch.empty_like(c['W']) if gate else None,
                db=torch.empty_like(c['b']) if gate else None)


def _bwd(c, noalloc):
    from ccq_b200 import _lib
    lib = _lib.load()
    o = _outputs(c)
    dt = _lib.CCQ_BF16 if c['q'].dtype == torch.bfloat16 else (_lib.CCQ_F16 if c['q'].dtype == torch.float16
                                                                else _lib.CCQ_F32)
    mode = _lib.CCQ_LAMBDA_GATE if c['W'] is not None else _lib.CCQ_LAMBDA_TOKEN
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    head = (dt, c['B'], c['T'], c['H'], c['K'], _p(c['q']), _p(c['k']), mode, _p(c['lam']), _p(c['W']),
            _p(c['b']), None, c['B'], 0, 1, None, None, _p(c['fcov']), _p(c['fmean']), _p(c['aux']),
            _p(c['dqc']), None, None, _p(o['dq']), _p(o['dk']), _p(o['dlam']), _p(o['dW']), _p(o['db']), None, None)
    if noalloc:
        st = lib.ccq_clean_bwd_noalloc(*head, stream)
    else:
        nbytes = lib.ccq_workspace_size(_lib.CCQ_OP_BWD, dt, c['B'], c['T'], c['H'], c['K'], c['B'])
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=c['q'].device)
        st = lib.ccq_clean_bwd(*head, _p(ws), nbytes, stream)
    assert st == 0, lib.ccq_last_error().decode()
    torch.cuda.synchronize()
    return o


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize('dtype,gate,shape,tol', [
    (torch.bfloat16, True, (2, 600, 4, 128), 1e-3),    # tensor-core backward, gate gradients
    (torch.float32, False, (2, 200, 3, 64), 1e-5),     # exact fp32 backward, per-token lambda
])
def test_noalloc_matches_workspace_entry_point(dtype, gate, shape, tol):
    c = _case(dtype, gate, *shape, seed=7)
    ref = _bwd(c, noalloc=False)
    from ccq_b200 import _lib
    lib = _lib.load()
    for _ in range(2):  # two calls in a row reuse the one static scratch
        got = _bwd(c, noalloc=True)
        # the scratch's error word: every bounded pipeline wait of the call completed
        code = ctypes.c_int(-1)
        st = lib.ccq_noalloc_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(code))
        assert st == 0 and code.value == 0, (st, code.value)
        for name in ('dq', 'dk', 'dlam', 'dW', 'db'):
            if ref[name] is None:
                continue
            assert torch.isfinite(got[name]).all(), name
            assert _rel(got[name], ref[name]) <= tol, (name, _rel(got[name], ref[name]))


def test_noalloc_rejects_calls_beyond_the_fixed_scratch():
    from ccq_b200 import _lib
    lib = _lib.load()
    # 4096 one-token documents of one head: the gate partials alone need 4096 * 516 bytes > 1 MiB
    n, H, K = 4096, 1, 128
    dev = torch.device('cuda', 0)
    q = torch.nn.functional.normalize(torch.randn(1, n, H, K, device=dev), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(1, n, H, K, device=dev), dim=-1).bfloat16()
    W = torch.randn(H, K, device=dev) * 0.02
    b = torch.zeros(H, device=dev)
    cu = torch.arange(n + 1, device=dev, dtype=torch.int64)
    from ccq_b200 import ops
    qc, fcov, fmean, aux = ops.clean_fwd_raw(q, k, None, W, b, 0, None, None, True, cu, n)
    assert 256 + 516 * n * H > 1 << 20  # scratch of the tensor-core backward for this call
    dq, dk, dW, db = torch.empty_like(q), torch.empty_like(k), torch.empty_like(W), torch.empty_like(b)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = lib.ccq_clean_bwd_noalloc(_lib.CCQ_BF16, 1, n, H, K, _p(q), _p(k), _lib.CCQ_LAMBDA_GATE, None, _p(W), _p(b),
                                   _p(cu), n, 0, 1, None, None, _p(fcov), _p(fmean), _p(aux), _p(qc), None, None,
                                   _p(dq), _p(dk), None, _p(dW), _p(db), None, None, stream)
    assert st == _lib.CCQ_ERR_WORKSPACE
    msg = lib.ccq_last_error().decode()
    assert 'fixed 1048576 bytes' in msg and 'ccq_clean_bwd with a workspace' in msg
