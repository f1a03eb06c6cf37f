"""Context-parallel cleaning (ccq_b200.distributed.cp_clean_read) on gloo ranks against one process.

A packed varlen batch is split over 3 ranks exactly as fla's build_cp_context splits it (documents
cut at rank boundaries).  Each rank runs cp_clean_read with a float64 torch restatement of the
operator standing in for the CUDA kernels (this host has no GPU), so the test checks the exchange:
the prefix of (C, m) over ranks, the positions a cut document continues at, and the gradients that
flow back through the all-gather.  Outputs and gradients must equal the single-process result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

LENS = [37, 50, 21, 9, 36]  # 153 tokens = 3 ranks x 51
H, K = 2, 8
WORLD = 3


def torch_clean(q, k, lam, *, position_offset=0, initial_cov_state=None, initial_mean_state=None,
                output_final_state=False, subtract_mean=True, cu_seqlens=None):
    """The operator (ccq/ops/common/fused_read.py:11-16) restated with autograd, per document."""
    cu = [int(x) for x in cu_seqlens.tolist()]
    outs, fcs, fms = [], [], []
    for n in range(len(cu) - 1):
        a, b = cu[n], cu[n + 1]
        qs, ks, ls = q[0, a:b], k[0, a:b], lam[0, a:b]
        C = torch.cumsum(torch.einsum('thk,thv->thkv', ks, ks), 0)
        m = torch.cumsum(ks, 0)
        if initial_cov_state is not None:
            C = C + initial_cov_state[n]
        if initial_mean_state is not None:
            m = m + initial_mean_state[n]
        pos = (torch.arange(1, b - a + 1, dtype=q.dtype) + position_offset).clamp_min(1.0)[:, None, None]
        corr = torch.einsum('thk,thkv->thv', qs, C) / pos
        if subtract_mean:
            s = (m * qs).sum(-1, keepdim=True)
            corr = corr - s * m / pos ** 2
        outs.append(qs - ls[..., None] * corr)
        fcs.append(C[-1] if b > a else torch.zeros(H, K, K, dtype=q.dtype))
        fms.append(m[-1] if b > a else torch.zeros(H, K, dtype=q.dtype))
    qc = torch.cat(outs, 0)[None]
    if not output_final_state:
        return qc, None, None
    return qc, torch.stack(fcs), torch.stack(fms) if subtract_mean else None


def _inputs():
    g = torch.Generator().manual_seed(0)
    T = sum(LENS)
    q = torch.randn(1, T, H, K, generator=g, dtype=torch.float64)
    k = torch.randn(1, T, H, K, generator=g, dtype=torch.float64)
    lam = torch.rand(1, T, H, generator=g, dtype=torch.float64)
    dqc = torch.randn(1, T, H, K, generator=g, dtype=torch.float64)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(LENS)]), dtype=torch.int64)
    return q, k, lam, dqc, cu


def _worker(rank, port, out):
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=WORLD)
    try:
        from fla.ops.cp import build_cp_context

        from ccq_b200.distributed import cp_clean_read
        q, k, lam, dqc, cu = _inputs()
        ctx = build_cp_context(cu, group=dist.group.WORLD)
        per = sum(LENS) // WORLD
        lo, hi = rank * per, (rank + 1) * per
        ql = q[:, lo:hi].clone().requires_grad_(True)
        kl = k[:, lo:hi].clone().requires_grad_(True)
        ll = lam[:, lo:hi].clone().requires_grad_(True)
        qc, kn, fc, fm = cp_clean_read(ql, kl, ll, ctx, l2norm_qk=True, position_offset=2, output_final_state=True,
                                       clean_fn=torch_clean)
        (qc * dqc[:, lo:hi]).sum().backward()
        out[rank] = (qc.detach().numpy(), ql.grad.numpy(), kl.grad.numpy(), ll.grad.numpy(), fc.detach().numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_cp_clean_read_matches_single_process():
    pytest.importorskip('fla')
    ctx = mp.get_context('spawn')
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    from ccq_b200 import ops
    q, k, lam, dqc, cu = _inputs()
    q.requires_grad_(True)
    k.requires_grad_(True)
    lam.requires_grad_(True)
    qc, fc, _ = torch_clean(ops.l2norm(q), ops.l2norm(k), lam, position_offset=2, output_final_state=True,
                            cu_seqlens=cu)
    (qc * dqc).sum().backward()
    got = [np.concatenate([out[r][i] for r in range(WORLD)], axis=1) for i in range(4)]
    for name, a, b in zip(('q_clean', 'dq', 'dk', 'dlam'), got, (qc.detach(), q.grad, k.grad, lam.grad)):
        assert np.abs(a - b.numpy()).max() <= 1e-10 * max(1.0, np.abs(b.numpy()).max()), name
    # the last rank's final state of the document that ends there equals the single-process final state
    assert np.allclose(out[WORLD - 1][4][-1], fc.detach().numpy()[-1], atol=1e-10)
