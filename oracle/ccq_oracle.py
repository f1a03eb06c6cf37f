"""CPU oracle for CCQ's read-side cleaning operator (test infrastructure only).

This module is a float64 numpy restatement of the reference's cleaning path.
It exists to check the CUDA kernels; nothing in the product imports it.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
use it, and only as the checker.

Math (per document, 1-based positions, pos_t = t + position_offset clamped >= 1),
restated from ccq/ops/common/fused_read.py:11-25 of the reference:

    C_t = C_0 + sum_{j<=t} k_j k_j^T     (fla state layout [K, V] with V = K)
    m_t = m_0 + sum_{j<=t} k_j
    z_t[v] = sum_k q_t[k] C_t[k, v]       (fla read: o = q @ h)
    s_t = m_t . q_t
    corr_t = z_t / pos_t - s_t m_t / pos_t^2       (mean term only if subtract_mean)
    q_clean_t = q_t - lambda_t corr_t

Backward (fused_read.py:18-25 and the kernel at :177-307):

    dlambda_t = -dqc_t . corr_t
    dz_t = -lambda_t dqc_t / pos_t
    ds_t = lambda_t (dqc_t . m_t) / pos_t^2
    dm_t = lambda_t s_t dqc_t / pos_t^2 + ds_t q_t
    dq_t = dqc_t + ds_t m_t + dz_t @ C_t            (row-vector form, as the kernel at :262)
    dk_j = sum_{t>=j} [q_t (k_j . dz_t) + dz_t (k_j . q_t) + dm_t] + (dC_T + dC_T^T) k_j + dm_T
    dC_0 = dC_T + sum_t q_t dz_t^T                  (fla chunk_bwd_dh orientation)
    dm_0 = dm_T + sum_t dm_t                        (fused_read.py:444-450)

Two pins hold this restatement to the reference: ``tests/golden/*.npz`` was
produced by running the reference's own Triton kernels (interpreter mode, fp32)
with ``tests/golden/gen_golden.py``; ``tests/test_oracle_golden.py`` checks this
module against every one of those fixtures.

Note on the state orientation: the reference's dq term is ``dz_t @ C_t``
(fused_read.py:262), which is the exact gradient only when C_t is symmetric.
Every state the operator or the decode step produces is symmetric (a sum of
outer products), so the two agree for all states reachable through the API; the
oracle follows the reference's form.
"""
from __future__ import annotations

import numpy as np

BT_REF = 64  # reference chunk size, fused_read.py:41 (math is chunk-size independent)


def segments(B, T, cu_seqlens):
    """(batch row, start, end, state row) per document.

    Dense batches have one document per row; varlen batches (B == 1) have one
    per cu_seqlens interval (fused_read.py:111-120).
    """
    if cu_seqlens is None:
        return [(b, 0, T, b) for b in range(B)]
    cu = [int(x) for x in np.asarray(cu_seqlens).reshape(-1)]
    return [(0, cu[i], cu[i + 1], i) for i in range(len(cu) - 1)]


def positions(n, position_offset):
    """Segment-relative positions 1..n plus the offset, clamped at 1 (fused_read.py:130-131, :463-471)."""
    pos = np.arange(1, n + 1, dtype=np.float64) + float(position_offset)
    return np.maximum(pos, 1.0)


def reshape_lambda_3d(lam, B, T, H):
    """Broadcast lambda (float, 0-d, [H], [B,T,H,1] or [B,T,H]) to [B,T,H] (clean.py:314-325)."""
    if np.isscalar(lam) or (isinstance(lam, np.ndarray) and lam.ndim == 0):
        return np.full((B, T, H), float(lam), dtype=np.float64)
    lam = np.asarray(lam, dtype=np.float64)
    if lam.ndim == 1 and lam.shape[0] == H:
        return np.broadcast_to(lam.reshape(1, 1, H), (B, T, H)).copy()
    if lam.ndim == 4 and lam.shape[-1] == 1:
        return lam[..., 0].copy()
    return lam.reshape(B, T, H).copy()


def reduce_dlambda(dlam3, lam_shape):
    """Reduce the [B,T,H] lambda gradient back to the lambda shape (fused_read.py:504-513)."""
    if lam_shape is None:
        return None
    nd = len(lam_shape)
    if nd == 0:
        return np.asarray(dlam3.sum())
    if nd == 1:
        return dlam3.sum(axis=(0, 1))
    if nd == 4 and lam_shape[-1] == 1:
        return dlam3[..., None]
    return dlam3


def clean_read_fwd(q, k, lam, position_offset=0, initial_cov_state=None, initial_mean_state=None,
                   output_final_state=False, subtract_mean=True, cu_seqlens=None, chunk=BT_REF):
    """Forward of ``fused_ccq_clean_read`` (fused_read.py:517-531, :379-403).

    Returns (q_clean, final_cov, final_mean); final_cov is None unless
    output_final_state, final_mean is None unless output_final_state and
    subtract_mean (fused_read.py:389-393).
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    B, T, H, K = q.shape
    lam3 = reshape_lambda_3d(lam, B, T, H)
    segs = segments(B, T, cu_seqlens)
    N = len(segs)
    qc = np.zeros_like(q)
    fcov = np.zeros((N, H, K, K))
    fmean = np.zeros((N, H, K))
    for (b, bos, eos, n) in segs:
        pos_all = positions(eos - bos, position_offset)
        for h in range(H):
            C = np.zeros((K, K)) if initial_cov_state is None else np.asarray(initial_cov_state, np.float64)[n, h].copy()
            m = np.zeros(K)
            if subtract_mean and initial_mean_state is not None:
                m = np.asarray(initial_mean_state, np.float64)[n, h].copy()
            for c0 in range(bos, eos, chunk):
                c1 = min(c0 + chunk, eos)
                Q = q[b, c0:c1, h]
                Kc = k[b, c0:c1, h]
                pos = pos_all[c0 - bos:c1 - bos]
                A = np.tril(Q @ Kc.T)
                z = Q @ C + A @ Kc
                corr = z / pos[:, None]
                if subtract_mean:
                    mc = m[None, :] + np.cumsum(Kc, axis=0)
                    s = (mc * Q).sum(1)
                    corr = corr - (s / pos ** 2)[:, None] * mc
                qc[b, c0:c1, h] = Q - lam3[b, c0:c1, h][:, None] * corr
                C = C + Kc.T @ Kc
                m = m + Kc.sum(0)
            fcov[n, h] = C
            fmean[n, h] = m
    final_cov = fcov if output_final_state else None
    final_mean = fmean if (output_final_state and subtract_mean) else None
    return qc, final_cov, final_mean


def clean_read_bwd(q, k, lam, dqc, position_offset=0, initial_cov_state=None, initial_mean_state=None,
                   subtract_mean=True, cu_seqlens=None, dfinal_cov=None, dfinal_mean=None, chunk=BT_REF):
    """Backward of ``fused_ccq_clean_read`` (fused_read.py:406-460, :496-514).

    Returns (dq, dk, dlam3 [B,T,H], dh0 or None, dm0 or None).  dh0 exists only
    when an initial cov state was given; dm0 only when an initial mean state was
    given and subtract_mean (or a final-mean gradient) is active.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    dqc = np.asarray(dqc, np.float64)
    B, T, H, K = q.shape
    lam3 = reshape_lambda_3d(lam, B, T, H)
    segs = segments(B, T, cu_seqlens)
    N = len(segs)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dlam = np.zeros((B, T, H))
    dh0 = np.zeros((N, H, K, K)) if initial_cov_state is not None else None
    use_carry = subtract_mean or dfinal_mean is not None
    dm0 = np.zeros((N, H, K)) if (initial_mean_state is not None and use_carry) else None
    for (b, bos, eos, n) in segs:
        pos_all = positions(eos - bos, position_offset)
        bounds = [(c0, min(c0 + chunk, eos)) for c0 in range(bos, eos, chunk)]
        for h in range(H):
            # forward sweep: states at chunk starts
            C = np.zeros((K, K)) if initial_cov_state is None else np.asarray(initial_cov_state, np.float64)[n, h].copy()
            m = np.zeros(K)
            if subtract_mean and initial_mean_state is not None:
                m = np.asarray(initial_mean_state, np.float64)[n, h].copy()
            Cs, ms = [], []
            for (c0, c1) in bounds:
                Cs.append(C.copy())
                ms.append(m.copy())
                Kc = k[b, c0:c1, h]
                C = C + Kc.T @ Kc
                m = m + Kc.sum(0)
            G = np.zeros((K, K)) if dfinal_cov is None else np.asarray(dfinal_cov, np.float64)[n, h].copy()
            carry = np.zeros(K) if dfinal_mean is None else np.asarray(dfinal_mean, np.float64)[n, h].copy()
            for ci in range(len(bounds) - 1, -1, -1):
                c0, c1 = bounds[ci]
                Cp, mp = Cs[ci], ms[ci]
                Q = q[b, c0:c1, h]
                Kc = k[b, c0:c1, h]
                Gc = dqc[b, c0:c1, h]
                pos = pos_all[c0 - bos:c1 - bos]
                lm = lam3[b, c0:c1, h]
                dz = -(lm / pos)[:, None] * Gc
                A = np.tril(Q @ Kc.T)
                Bm = np.tril(dz @ Kc.T)
                z = Q @ Cp + A @ Kc
                u = (Gc * z).sum(1)
                dqt = Gc + dz @ Cp + Bm @ Kc
                dkt = A.T @ dz + Bm.T @ Q + Kc @ (G + G.T)
                dl = -u / pos
                if subtract_mean:
                    mc = mp[None, :] + np.cumsum(Kc, axis=0)
                    s = (mc * Q).sum(1)
                    w = (mc * Gc).sum(1)
                    ds = lm * w / pos ** 2
                    dmg = lm * s / pos ** 2
                    dqt = dqt + ds[:, None] * mc
                    dm = dmg[:, None] * Gc + ds[:, None] * Q
                    suffix = np.cumsum(dm[::-1], axis=0)[::-1]
                    dkt = dkt + suffix
                    dl = dl + s * w / pos ** 2
                    dkt = dkt + carry[None, :]
                    carry = carry + dm.sum(0)
                elif dfinal_mean is not None:
                    dkt = dkt + carry[None, :]
                dq[b, c0:c1, h] = dqt
                dk[b, c0:c1, h] = dkt
                dlam[b, c0:c1, h] = dl
                G = G + Q.T @ dz
            if dh0 is not None:
                dh0[n, h] = G
            if dm0 is not None:
                dm0[n, h] = carry
    return dq, dk, dlam, dh0, dm0


def decode_clean(q, k, lam, position_offset=0, initial_cov_state=None, initial_mean_state=None,
                 output_final_state=True, subtract_mean=True, cu_seqlens=None):
    """Recurrent (decode) cleaning: fla ``fused_recurrent_gla(q, k, v=k, scale=1)`` followed by
    ``_CCQCleanQ`` (ccq/ops/ccq_gdn/fused_clean.py:34-83 with use_chunk=False,
    ccq/ops/ccq_gla/fused_recurrent.py:26-38; clean.py:220-311, :341-384).

    The state includes the current token (inclusive read).  Returns
    (q_clean, final_cov or None, final_mean or None).
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    B, T, H, K = q.shape
    lam3 = reshape_lambda_3d(lam, B, T, H)
    segs = segments(B, T, cu_seqlens)
    N = len(segs)
    qc = np.zeros_like(q)
    fcov = np.zeros((N, H, K, K))
    fmean = np.zeros((N, H, K))
    for (b, bos, eos, n) in segs:
        pos_all = positions(eos - bos, position_offset)
        for h in range(H):
            C = np.zeros((K, K)) if initial_cov_state is None else np.asarray(initial_cov_state, np.float64)[n, h].copy()
            m = np.zeros(K)
            if initial_mean_state is not None:
                m = np.asarray(initial_mean_state, np.float64)[n, h].copy()
            for t in range(bos, eos):
                kt = k[b, t, h]
                qt = q[b, t, h]
                C = C + np.outer(kt, kt)
                m = m + kt
                pos = pos_all[t - bos]
                z = qt @ C
                corr = z / pos
                if subtract_mean:
                    corr = corr - (m @ qt) / pos ** 2 * m
                qc[b, t, h] = qt - lam3[b, t, h] * corr
            fcov[n, h] = C
            fmean[n, h] = m
    return (qc, fcov if output_final_state else None,
            fmean if (output_final_state and subtract_mean) else None)


def lambda_headwise_fwd(q, W, bias):
    """Per-head gate lambda[b,t,h] = sigmoid(W[h] . q[b,t,h] + bias[h]).

    This is the block-diagonal form of the layer's ``sigmoid(erase_lambda_proj(q))``
    (ccq/gdn/layer.py:174, :292) that the benchmark configurations use (W_lambda is H x d_k).
    """
    pre = np.einsum('bthk,hk->bth', np.asarray(q, np.float64), np.asarray(W, np.float64)) + np.asarray(bias, np.float64)
    return 1.0 / (1.0 + np.exp(-pre))


def lambda_headwise_bwd(q, W, lam, dlam):
    """Gradients of the per-head gate: returns (dq_extra, dW, db)."""
    dpre = np.asarray(dlam, np.float64) * lam * (1.0 - lam)
    dq = dpre[..., None] * np.asarray(W, np.float64)[None, None]
    dW = np.einsum('bth,bthk->hk', dpre, np.asarray(q, np.float64))
    db = dpre.sum(axis=(0, 1))
    return dq, dW, db


def lambda_dense_fwd(q_pre, W, bias):
    """Dense gate of the layer: sigmoid(q_pre.reshape(B,T,H*K) @ W^T + bias), W [H, H*K] (gdn/layer.py:292)."""
    B, T, H, K = q_pre.shape
    x = np.asarray(q_pre, np.float64).reshape(B, T, H * K)
    pre = x @ np.asarray(W, np.float64).T + np.asarray(bias, np.float64)
    return 1.0 / (1.0 + np.exp(-pre))


def lambda_dense_bwd(q_pre, W, lam, dlam):
    """Gradients of the dense gate: returns (dq_pre, dW, db)."""
    B, T, H, K = q_pre.shape
    dpre = np.asarray(dlam, np.float64) * lam * (1.0 - lam)
    x = np.asarray(q_pre, np.float64).reshape(B * T, H * K)
    dx = dpre.reshape(B * T, H) @ np.asarray(W, np.float64)
    dW = dpre.reshape(B * T, H).T @ x
    db = dpre.sum(axis=(0, 1))
    return dx.reshape(B, T, H, K), dW, db


def l2norm_fwd(x, eps=1e-6, round_to=None):
    """fla's l2norm (fla/modules/l2norm.py:26-46, :266): y = x / sqrt(sum(x^2) + eps) per row.

    Returns (y, r) with r = 1 / sqrt(sum(x^2) + eps).  ``round_to`` (a callable) rounds y to the
    activation dtype the way the kernels store it; the backward then uses the rounded y, as fla's
    saves its stored output."""
    x = np.asarray(x, np.float64)
    r = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True) + eps)
    y = x * r
    if round_to is not None:
        y = round_to(y)
    return y, r[..., 0]


def l2norm_bwd(y, r, dy):
    """fla's l2norm backward (fla/modules/l2norm.py:49-72): dx = r (dy - y sum(dy * y))."""
    y = np.asarray(y, np.float64)
    dy = np.asarray(dy, np.float64)
    return r[..., None] * (dy - y * (dy * y).sum(-1, keepdims=True))
