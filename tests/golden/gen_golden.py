"""Generate the golden vectors in this folder by running the REFERENCE implementation.

Run once in a container that has the reference checkout and its dependencies
(flash-linear-attention 0.5.1, triton 3.6) but no GPU:

    python tests/golden/gen_golden.py --reference <path to the CCQ checkout>

The reference's Triton kernels run on the CPU under ``TRITON_INTERPRET=1`` in
fp32, with two harness shims and no change to the reference:
  * ``torch.cpu.device`` becomes a no-op context (fla's ``input_guard`` calls it);
  * Triton's autotuner keeps its first config (it cannot benchmark without a GPU).

Every input is drawn from ``numpy.random.default_rng(seed)`` (PCG64, stable
streams), so the tests regenerate inputs bit-exactly and the fixtures only need
the outputs; each fixture also stores the SHA-256 of its inputs so that a change
in the generator is detected rather than silently compared.  Small cases store
full outputs; the two larger cases store a fixed random sample of each output
plus its sum and sum of squares.

Cases (the list follows the reference's behaviour surface for this path):
  dense         B=2 T=130 H=2 K=32, lambda [B,T,H,1], final states + their grads
  varlen        cu_seqlens (70, 5, 130), initial cov/mean states, offset 7, final-state grads
  nomean        subtract_mean=False, 0-d lambda, initial cov state and its grad
  lamh          lambda [H], negative offset -3 (position clamp), T=65 (ragged chunk)
  scalar        lambda as a Python float (no lambda grad), T=1 after a 4-token state, offset 4
  cfg1          config 1 (B=2 T=512 H=4 K=64) with the per-head gate sigmoid(W q + b)
  k128          B=1 T=200 H=2 K=128 with states, offset 5 (the fast path's head size)
  decode        40 single-token decode steps from a 20-token prefix, then a 5-token
                step and a varlen step (the generation-cache path)
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def unit(rng, shape):
    x = rng.standard_normal(shape)
    return x / np.linalg.norm(x, axis=-1, keepdims=True)


def sym_state(rng, N, H, K, n_tok):
    """A covariance state sum_j k_j k_j^T over n_tok unit keys (symmetric PSD), and the matching key sum."""
    kk = unit(rng, (N, n_tok, H, K))
    C = np.einsum('nthk,nthv->nhkv', kk, kk)
    m = kk.sum(1)
    return C, m


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(np.asarray(a, np.float32)).tobytes())
    return h.hexdigest()


# --------------------------------------------------------------------------------------
# input builders (shared with the tests, which import this module without the reference)
# --------------------------------------------------------------------------------------

def case_inputs(name):
    """Deterministic inputs of a golden case as float32 numpy arrays plus call options."""
    if name == 'dense':
        rng = np.random.default_rng(100)
        B, T, H, K = 2, 130, 2, 32
        d = dict(q=unit(rng, (B, T, H, K)), k=unit(rng, (B, T, H, K)),
                 lam=rng.uniform(0, 1, (B, T, H, 1)))
        d['dqc'] = rng.standard_normal((B, T, H, K))
        d['dfinal_cov'] = rng.standard_normal((B, H, K, K))
        d['dfinal_mean'] = rng.standard_normal((B, H, K))
        opts = dict(position_offset=0, output_final_state=True, subtract_mean=True, cu_seqlens=None)
    elif name == 'varlen':
        rng = np.random.default_rng(101)
        lens = [70, 5, 130]
        T, H, K = sum(lens), 2, 32
        d = dict(q=unit(rng, (1, T, H, K)), k=unit(rng, (1, T, H, K)), lam=rng.uniform(0, 1, (1, T, H)))
        C0, m0 = sym_state(rng, 3, H, K, 20)
        d['initial_cov_state'] = C0
        d['initial_mean_state'] = m0
        d['dqc'] = rng.standard_normal((1, T, H, K))
        d['dfinal_cov'] = rng.standard_normal((3, H, K, K))
        d['dfinal_mean'] = rng.standard_normal((3, H, K))
        opts = dict(position_offset=7, output_final_state=True, subtract_mean=True,
                    cu_seqlens=np.array([0, 70, 75, 205], dtype=np.int64))
    elif name == 'nomean':
        rng = np.random.default_rng(102)
        B, T, H, K = 1, 97, 2, 32
        d = dict(q=unit(rng, (B, T, H, K)), k=unit(rng, (B, T, H, K)), lam=np.array(0.37))
        C0, _ = sym_state(rng, B, H, K, 10)
        d['initial_cov_state'] = C0
        d['dqc'] = rng.standard_normal((B, T, H, K))
        d['dfinal_cov'] = rng.standard_normal((B, H, K, K))
        opts = dict(position_offset=0, output_final_state=True, subtract_mean=False, cu_seqlens=None)
    elif name == 'lamh':
        rng = np.random.default_rng(103)
        B, T, H, K = 2, 65, 3, 16
        d = dict(q=unit(rng, (B, T, H, K)), k=unit(rng, (B, T, H, K)), lam=rng.uniform(0, 1, (H,)))
        d['dqc'] = rng.standard_normal((B, T, H, K))
        opts = dict(position_offset=-3, output_final_state=False, subtract_mean=True, cu_seqlens=None)
    elif name == 'scalar':
        rng = np.random.default_rng(104)
        B, T, H, K = 3, 1, 2, 16
        d = dict(q=unit(rng, (B, T, H, K)), k=unit(rng, (B, T, H, K)), lam=0.3)
        C0, m0 = sym_state(rng, B, H, K, 4)
        d['initial_cov_state'] = C0
        d['initial_mean_state'] = m0
        d['dqc'] = rng.standard_normal((B, T, H, K))
        d['dfinal_cov'] = rng.standard_normal((B, H, K, K))
        d['dfinal_mean'] = rng.standard_normal((B, H, K))
        opts = dict(position_offset=4, output_final_state=True, subtract_mean=True, cu_seqlens=None)
    elif name == 'cfg1':
        rng = np.random.default_rng(0)
        B, T, H, K = 2, 512, 4, 64
        d = dict(q=unit(rng, (B, T, H, K)), k=unit(rng, (B, T, H, K)))
        d['W'] = rng.normal(0.0, 0.02, (H, K))
        d['b'] = np.zeros(H)
        d['dqc'] = rng.standard_normal((B, T, H, K))
        opts = dict(position_offset=0, output_final_state=False, subtract_mean=True, cu_seqlens=None)
    elif name == 'k128':
        rng = np.random.default_rng(105)
        B, T, H, K = 1, 200, 2, 128
        d = dict(q=unit(rng, (B, T, H, K)), k=unit(rng, (B, T, H, K)), lam=rng.uniform(0, 1, (B, T, H)))
        C0, m0 = sym_state(rng, B, H, K, 30)
        d['initial_cov_state'] = C0
        d['initial_mean_state'] = m0
        d['dqc'] = rng.standard_normal((B, T, H, K))
        d['dfinal_cov'] = rng.standard_normal((B, H, K, K))
        d['dfinal_mean'] = rng.standard_normal((B, H, K))
        opts = dict(position_offset=5, output_final_state=True, subtract_mean=True, cu_seqlens=None)
    elif name == 'decode':
        rng = np.random.default_rng(106)
        N, H, K, P, S = 3, 2, 32, 20, 40
        d = dict(prefix_q=unit(rng, (N, P, H, K)), prefix_k=unit(rng, (N, P, H, K)),
                 prefix_lam=rng.uniform(0, 1, (N, P, H, 1)))
        d['step_q'] = unit(rng, (S, N, 1, H, K))
        d['step_k'] = unit(rng, (S, N, 1, H, K))
        d['step_lam'] = rng.uniform(0, 1, (S, N, 1, H, 1))
        d['multi_q'] = unit(rng, (N, 5, H, K))
        d['multi_k'] = unit(rng, (N, 5, H, K))
        d['multi_lam'] = rng.uniform(0, 1, (N, 5, H, 1))
        d['var_q'] = unit(rng, (1, 7, H, K))
        d['var_k'] = unit(rng, (1, 7, H, K))
        d['var_lam'] = rng.uniform(0, 1, (1, 7, H, 1))
        opts = dict(prefix=P, steps=S, var_cu=np.array([0, 2, 7], dtype=np.int64))
    else:
        raise KeyError(name)
    out = {}
    for key, v in d.items():
        out[key] = np.asarray(v, np.float32) if isinstance(v, np.ndarray) else v
    return out, opts


CASES = ['dense', 'varlen', 'nomean', 'lamh', 'scalar', 'cfg1', 'k128', 'decode']
SAMPLED = {'cfg1', 'k128'}


def inputs_digest(d):
    return digest(*[d[k] for k in sorted(d) if isinstance(d[k], np.ndarray)])


def sample_index(size, n=2048, seed=7):
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(size, size=min(n, size), replace=False))


# --------------------------------------------------------------------------------------
# running the reference (only here, never in the tests)
# --------------------------------------------------------------------------------------

def _setup_reference(path):
    os.environ['TRITON_INTERPRET'] = '1'
    import torch
    torch.cpu.device = lambda i=None: contextlib.nullcontext()
    from triton.runtime.autotuner import Autotuner
    orig = Autotuner.run

    def run_first_config(self, *a, **k):
        self.configs = self.configs[:1]
        return orig(self, *a, **k)
    Autotuner.run = run_first_config
    sys.path.insert(0, path)


def _t(x, grad=False):
    import torch
    if x is None:
        return None
    if not isinstance(x, np.ndarray):
        return x
    t = torch.tensor(x)
    if grad:
        t.requires_grad_(True)
    return t


def run_clean_read(name, d, opts):
    import torch
    from ccq.ops.common.fused_read import fused_ccq_clean_read
    q, k = _t(d['q'], True), _t(d['k'], True)
    if name == 'cfg1':
        W, b = _t(d['W'], True), _t(d['b'], True)
        # contiguous like the layer's Linear output: the reference copies a non-contiguous
        # lambda inside its autograd forward and then returns no lambda gradient
        lam = torch.sigmoid(torch.einsum('bthk,hk->bth', q, W) + b).contiguous()
    else:
        lam = d['lam']
        lam = torch.tensor(lam, requires_grad=True) if isinstance(lam, np.ndarray) else lam
    h0 = _t(d.get('initial_cov_state'), True)
    m0 = _t(d.get('initial_mean_state'), True)
    cu = opts['cu_seqlens']
    cu = torch.tensor(cu) if cu is not None else None
    qc, fc, fm = fused_ccq_clean_read(
        q, k, lam, position_offset=opts['position_offset'], initial_cov_state=h0,
        initial_mean_state=m0, output_final_state=opts['output_final_state'],
        subtract_mean=opts['subtract_mean'], cu_seqlens=cu)
    loss = (qc * _t(d['dqc'])).sum()
    if fc is not None and 'dfinal_cov' in d:
        loss = loss + (fc * _t(d['dfinal_cov'])).sum()
    if fm is not None and 'dfinal_mean' in d:
        loss = loss + (fm * _t(d['dfinal_mean'])).sum()
    loss.backward()
    out = {'q_clean': qc, 'dq': q.grad, 'dk': k.grad}
    if fc is not None:
        out['final_cov'] = fc
    if fm is not None:
        out['final_mean'] = fm
    if name == 'cfg1':
        out['dW'] = W.grad
        out['db'] = b.grad
    elif isinstance(lam, torch.Tensor) and lam.grad is not None:
        out['dlam'] = lam.grad
    if h0 is not None and h0.grad is not None:
        out['dh0'] = h0.grad
    if m0 is not None and m0.grad is not None:
        out['dm0'] = m0.grad
    return {k_: v.detach().numpy().astype(np.float32) for k_, v in out.items()}


def run_decode(d, opts):
    import torch
    from ccq.ops.common.fused_read import fused_ccq_clean_read
    from ccq.ops.ccq_gdn.fused_clean import fused_ccq_clean
    P, S = opts['prefix'], opts['steps']
    with torch.no_grad():
        _, C, m = fused_ccq_clean_read(_t(d['prefix_q']), _t(d['prefix_k']), _t(d['prefix_lam']),
                                       output_final_state=True)
        out = {'prefix_cov': C.numpy().copy(), 'prefix_mean': m.numpy().copy()}
        qcs = []
        off = P
        for i in range(S):
            qc, _, C, m, _ = fused_ccq_clean(_t(d['step_q'][i]), _t(d['step_k'][i]), _t(d['step_lam'][i]),
                                             initial_cov_state=C, initial_mean_state=m,
                                             output_final_state=True, position_offset=off,
                                             subtract_mean=True, use_chunk=False)
            qcs.append(qc.numpy())
            off += 1
        out['step_q_clean'] = np.stack(qcs)
        out['steps_cov'] = C.numpy().copy()
        out['steps_mean'] = m.numpy().copy()
        qc, _, C, m, _ = fused_ccq_clean(_t(d['multi_q']), _t(d['multi_k']), _t(d['multi_lam']),
                                         initial_cov_state=C, initial_mean_state=m,
                                         output_final_state=True, position_offset=off,
                                         subtract_mean=True, use_chunk=False)
        out['multi_q_clean'] = qc.numpy()
        out['multi_cov'] = C.numpy().copy()
        out['multi_mean'] = m.numpy().copy()
        C2 = C[:2].contiguous()
        m2 = m[:2].contiguous()
        qc, _, C2, m2, _ = fused_ccq_clean(_t(d['var_q']), _t(d['var_k']), _t(d['var_lam']),
                                           initial_cov_state=C2, initial_mean_state=m2,
                                           output_final_state=True, position_offset=3,
                                           subtract_mean=True, use_chunk=False,
                                           cu_seqlens=torch.tensor(opts['var_cu']))
        out['var_q_clean'] = qc.numpy()
        out['var_cov'] = C2.numpy().copy()
        out['var_mean'] = m2.numpy().copy()
    return {k_: np.asarray(v, np.float32) for k_, v in out.items()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True)
    ap.add_argument('--cases', nargs='*', default=CASES)
    args = ap.parse_args()
    _setup_reference(args.reference)
    for name in args.cases:
        d, opts = case_inputs(name)
        out = run_decode(d, opts) if name == 'decode' else run_clean_read(name, d, opts)
        save = {'inputs_sha256': np.array(inputs_digest(d))}
        for key, v in out.items():
            if name in SAMPLED:
                idx = sample_index(v.size)
                save[key + '__idx'] = idx.astype(np.int64)
                save[key + '__val'] = v.reshape(-1)[idx]
                save[key + '__sum'] = np.array(v.astype(np.float64).sum())
                save[key + '__sumsq'] = np.array((v.astype(np.float64) ** 2).sum())
                save[key + '__shape'] = np.array(v.shape, dtype=np.int64)
            else:
                save[key] = v
        path = os.path.join(HERE, f'{name}.npz')
        np.savez_compressed(path, **save)
        print(name, {k_: v.shape for k_, v in out.items()}, os.path.getsize(path))


if __name__ == '__main__':
    main()
