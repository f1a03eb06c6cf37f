"""Parity at the sizes of the benchmark configurations that are not the timed one.

* c3: a variable-length packed batch of 32 documents with lengths ~ U[128, 8192], H=16, d_k=128,
  bf16, per-head gate: the tensor-core path against the exact fp32 SIMT path over the whole batch,
  and against the float64 oracle on three sampled documents (states reset at boundaries, so a
  document is checked on its own rows).
* c4: 1024 decode steps at batch 256, H=16, d_k=128 from a 2048-token prefix: the final cache
  against a float64 sum of the same rank-1 updates, q_clean of two sequences against the oracle at
  every step.
* c5 (single GPU, reduced heads): T = 16384 fwd+bwd against the SIMT path and, on one head, the
  oracle.

Bars as in test_gpu_parity: 2e-2 max-abs for bf16 outputs and gradients against the float64
oracle, relative errors for fp32 states and the gate-parameter gradients.  Two bf16 results of
the same value may round to neighbouring bf16 numbers, so the tensor-core path is held to the SIMT
path within 2e-2 or one bf16 ulp at the largest magnitude, whichever is larger (|dq| reaches ~6
at c3, where an ulp is 2^-5; both paths stay within 2e-2 of the oracle there).  The fp32 states
of the tensor-core path are accumulated by the MMA (fp32, not in IEEE sequential order): after
8192 tokens they differ from the SIMT path's sequential sums by ~2e-5 relative (~1e-3 absolute
on entries near 50), so states are held to 1e-4 relative, against the SIMT path and the oracle.
dW and db are sums over every token of the batch with heavy cancellation (db ~ 0.1 from 16k terms);
they are held to the bf16 bar, 2e-2 max-abs.
"""
import math

import numpy as np
import pytest
import torch

from golden_util import rel_err
from oracle import ccq_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
STATE_TOL = 1e-4


@pytest.fixture(scope='module', autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from ccq_b200 import _lib as L
    L.load()
    yield


def np64(t):
    return t.detach().double().cpu().numpy()


def unit_t(gen, shape, dtype):
    x = torch.randn(shape, generator=gen, device='cuda')
    return (x / x.norm(dim=-1, keepdim=True)).to(dtype)


def run_both(q, k, W, b, g, cu, N, monkeypatch):
    """fwd+bwd of the gated operator on the tensor-core path and on the exact SIMT path."""
    import ccq_b200
    from ccq_b200 import ops
    out = {}
    for path in ('tcgen05', 'simt'):
        if path == 'simt':
            monkeypatch.setenv('CCQ_B200_FORCE_SIMT', '1')
        qc, fc, fm, aux = ops.clean_fwd_raw(q, k, None, W, b, 0, None, None, True, cu, N)
        assert ccq_b200.last_path() == path
        dq, dk, (dW, db), _, _ = ops.clean_bwd_raw(q, k, None, W, b, 0, None, None, True, cu, N, fc, fm, aux, g,
                                                   None, None)
        assert ccq_b200.last_path() == path
        out[path] = dict(qc=qc, fc=fc, fm=fm, dq=dq, dk=dk, dW=dW, db=db)
        if path == 'simt':
            monkeypatch.delenv('CCQ_B200_FORCE_SIMT')
    return out['tcgen05'], out['simt']


def bf16_pair_tol(ref):
    top = ref.float().abs().max().item()
    ulp = 2.0 ** (math.floor(math.log2(top)) - 7) if top > 0 else 0.0
    return max(BF16_TOL, ulp)


def assert_paths_agree(tc, ref):
    for name in ('qc', 'dq', 'dk'):
        err = (tc[name].float() - ref[name].float()).abs().max().item()
        assert err <= bf16_pair_tol(ref[name]), (name, err)
    assert rel_err(np64(tc['fc']), np64(ref['fc'])) <= STATE_TOL
    assert rel_err(np64(tc['fm']), np64(ref['fm'])) <= STATE_TOL
    assert (tc['dW'] - ref['dW']).abs().max().item() <= BF16_TOL
    assert (tc['db'] - ref['db']).abs().max().item() <= BF16_TOL


def check_document(q, k, W, b, g, tc, r0, r1, n=None):
    """Rows r0:r1 of a packed batch (document n) against the float64 oracle."""
    qn, kn, gn = (np64(x[:, r0:r1]) for x in (q, k, g))
    Wn, bn = np64(W), np64(b)
    lam = O.lambda_headwise_fwd(qn, Wn, bn)
    oq, ofc, ofm = O.clean_read_fwd(qn, kn, lam, output_final_state=True)
    odq, odk, odl, _, _ = O.clean_read_bwd(qn, kn, lam, gn)
    dqx, odW, odb = O.lambda_headwise_bwd(qn, Wn, lam, odl)
    if n is None:  # a whole sequence: the gate-parameter gradients too
        assert np.abs(np64(tc['dW']) - odW).max() <= BF16_TOL
        assert np.abs(np64(tc['db']) - odb).max() <= BF16_TOL
    else:
        assert rel_err(np64(tc['fc'][n:n + 1]), ofc) <= STATE_TOL
        assert rel_err(np64(tc['fm'][n:n + 1]), ofm) <= STATE_TOL
    assert np.abs(np64(tc['qc'][:, r0:r1]) - oq).max() <= BF16_TOL
    assert np.abs(np64(tc['dq'][:, r0:r1]) - (odq + dqx)).max() <= BF16_TOL
    assert np.abs(np64(tc['dk'][:, r0:r1]) - odk).max() <= BF16_TOL


def test_c3_varlen_packed_full_size(monkeypatch):
    rng = np.random.default_rng(30)
    lens = rng.integers(128, 8193, size=32)
    cu_np = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    T, H, K, N = int(cu_np[-1]), 16, 128, len(lens)
    gen = torch.Generator(device='cuda').manual_seed(30)
    q, k = unit_t(gen, (1, T, H, K), torch.bfloat16), unit_t(gen, (1, T, H, K), torch.bfloat16)
    W = torch.randn(H, K, generator=gen, device='cuda') * 0.02
    b = torch.rand(H, generator=gen, device='cuda') * 2 - 1
    g = torch.randn(1, T, H, K, generator=gen, device='cuda').to(torch.bfloat16)
    cu = torch.tensor(cu_np, device='cuda')
    tc, ref = run_both(q, k, W, b, g, cu, N, monkeypatch)
    assert_paths_agree(tc, ref)
    order = np.argsort(lens)
    for n in (order[0], order[N // 2], order[-1]):  # the shortest, a median and the longest document
        check_document(q, k, W, b, g, tc, int(cu_np[n]), int(cu_np[n + 1]), n)


def test_c5_long_context_single_gpu(monkeypatch):
    T, H, K = 16384, 4, 128
    gen = torch.Generator(device='cuda').manual_seed(50)
    q, k = unit_t(gen, (1, T, H, K), torch.bfloat16), unit_t(gen, (1, T, H, K), torch.bfloat16)
    W = torch.randn(H, K, generator=gen, device='cuda') * 0.02
    b = torch.rand(H, generator=gen, device='cuda') * 2 - 1
    g = torch.randn(1, T, H, K, generator=gen, device='cuda').to(torch.bfloat16)
    tc, ref = run_both(q, k, W, b, g, None, 1, monkeypatch)
    assert_paths_agree(tc, ref)
    # head 0 against the oracle over the whole sequence
    h = slice(0, 1)
    one = {name: tc[name][:, :, h] for name in ('qc', 'dq', 'dk')}
    one['dW'], one['db'] = tc['dW'][h], tc['db'][h]
    check_document(q[:, :, h], k[:, :, h], W[h], b[h], g[:, :, h], one, 0, T)


def test_c4_decode_1024_steps():
    import ccq_b200
    N, H, K, P, S = 256, 16, 128, 2048, 1024
    gen = torch.Generator(device='cuda').manual_seed(40)
    pre = unit_t(gen, (N, P, H, K), torch.float32)
    C = torch.einsum('nthk,nthv->nhkv', pre, pre).contiguous()
    m = pre.sum(1).contiguous()
    Cd, md = C.double(), m.double()
    picks = [0, N - 1]
    oC = [np64(C[n:n + 1]) for n in picks]
    om = [np64(m[n:n + 1]) for n in picks]
    del pre
    worst = 0.0
    for step in range(S):
        q = unit_t(gen, (N, 1, H, K), torch.bfloat16)
        k = unit_t(gen, (N, 1, H, K), torch.bfloat16)
        lam = torch.rand(N, 1, H, generator=gen, device='cuda').to(torch.bfloat16)
        qc, C, m = ccq_b200.decode_step(q, k, lam, C, m, position_offset=P + step, inplace=True)
        kd = k[:, 0].double()
        Cd += torch.einsum('nhk,nhv->nhkv', kd, kd)
        md += kd
        for i, n in enumerate(picks):
            oq, oC[i], om[i] = O.decode_clean(np64(q[n:n + 1]), np64(k[n:n + 1]), np64(lam[n:n + 1]), P + step,
                                              oC[i], om[i])
            worst = max(worst, float(np.abs(np64(qc[n:n + 1]) - oq).max()))
    assert worst <= BF16_TOL, worst
    assert rel_err(np64(C), Cd.cpu().numpy()) <= 1e-5
    assert rel_err(np64(m), md.cpu().numpy()) <= 1e-5
