"""Torch transcription of CCQ's cleaning operator, used as the timed CPU baseline.

Test infrastructure only (see ``oracle/ccq_oracle.py``): ``bench.py``'s CPU
baseline leg times this module on the host cores, and the tests use its
autograd gradients as an independent cross-check of the explicit backward in
``ccq_oracle``.  The reference ships no pure-PyTorch path, so this is a direct
transcription of the formula at ccq/ops/common/fused_read.py:11-16 plus the
lambda gate ``sigmoid(erase_lambda_proj(q))`` (ccq/gdn/layer.py:292), in the
chunked (BT=64) einsum form; gradients come from autograd.
"""
from __future__ import annotations

import torch

BT = 64


def clean_read_dense_batch(q, k, lam, subtract_mean=True, position_offset=0, chunk=BT):
    """q_clean for dense [B,T,H,K] inputs with lambda [B,T,H]; all (b, h) in one batched chunk loop."""
    B, T, H, K = q.shape
    qh = q.permute(0, 2, 1, 3).reshape(B * H, T, K)
    kh = k.permute(0, 2, 1, 3).reshape(B * H, T, K)
    lh = lam.permute(0, 2, 1).reshape(B * H, T)
    C = q.new_zeros(B * H, K, K)
    m = q.new_zeros(B * H, K)
    outs = []
    for c0 in range(0, T, chunk):
        c1 = min(c0 + chunk, T)
        Q = qh[:, c0:c1]
        Kc = kh[:, c0:c1]
        pos = torch.arange(c0 + 1, c1 + 1, dtype=q.dtype) + position_offset
        pos = pos.clamp_min(1.0)
        A = torch.tril(Q @ Kc.transpose(1, 2))
        z = Q @ C + A @ Kc
        corr = z / pos[None, :, None]
        if subtract_mean:
            mc = m[:, None, :] + torch.cumsum(Kc, dim=1)
            s = (mc * Q).sum(-1)
            corr = corr - (s / pos ** 2)[..., None] * mc
        outs.append(Q - lh[:, c0:c1, None] * corr)
        C = C + Kc.transpose(1, 2) @ Kc
        m = m + Kc.sum(1)
    out = torch.cat(outs, dim=1)
    return out.reshape(B, H, T, K).permute(0, 2, 1, 3)


def clean_read_dense_cumsum(q, k, lam, subtract_mean=True, position_offset=0):
    """The T*K^2 'dense' variant: materialise every C_t by a cumulative sum (small shapes only)."""
    B, T, H, K = q.shape
    C = torch.cumsum(torch.einsum('bthk,bthv->bthkv', k, k), dim=1)
    z = torch.einsum('bthk,bthkv->bthv', q, C)
    pos = (torch.arange(1, T + 1, dtype=q.dtype) + position_offset).clamp_min(1.0)[None, :, None]
    corr = z / pos[..., None]
    if subtract_mean:
        m = torch.cumsum(k, dim=1)
        s = (m * q).sum(-1)
        corr = corr - (s / pos ** 2)[..., None] * m
    return q - lam[..., None] * corr


def headwise_lambda(q, W, b):
    """lambda[b,t,h] = sigmoid(W[h] . q[b,t,h] + b[h])."""
    return torch.sigmoid(torch.einsum('bthk,hk->bth', q, W) + b)


def clean_step_fwd_bwd(q, k, W, b, dqc, chunk=BT):
    """One fwd+bwd of the op with the per-head gate; returns (q_clean, dq, dk, dW, db)."""
    q = q.detach().requires_grad_(True)
    k = k.detach().requires_grad_(True)
    W = W.detach().requires_grad_(True)
    b = b.detach().requires_grad_(True)
    lam = headwise_lambda(q, W, b)
    qc = clean_read_dense_batch(q, k, lam, chunk=chunk)
    qc.backward(dqc)
    return qc.detach(), q.grad, k.grad, W.grad, b.grad
