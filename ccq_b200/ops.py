"""PyTorch-facing operators over the C ABI (same names, arguments and outputs as the reference).

``fused_ccq_clean_read`` / ``FusedCCQCleanRead`` replace ccq/ops/common/fused_read.py:474-531;
``fused_ccq_clean`` replaces the decode cleaning of ccq/ops/ccq_gdn/fused_clean.py:34-83.
``fused_ccq_clean_gated`` is the same operator with the per-head gate
lambda = sigmoid(W[h] . q + b[h]) fused into the kernels (returns dW, db directly).

Every call goes to the sm_100a kernels in ``libccq_b200.so``; tensors must be on a CUDA device.
There is no CPU or eager fallback: a missing library or a CPU tensor raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

_DT = {torch.float32: _lib.CCQ_F32, torch.bfloat16: _lib.CCQ_BF16, torch.float16: _lib.CCQ_F16}


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dtype_code(t):
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f'unsupported activation dtype {t.dtype}; use float32, bfloat16 or float16') from None


def _check_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError('ccq_b200 operators run on CUDA tensors only (got a CPU tensor)')
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f'tensors on different devices: {dev} and {t.device}')
    return dev


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _state(t, shape):
    """An optional fp32 state tensor, contiguous, checked against its expected shape."""
    if t is None:
        return None
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f'state has shape {tuple(t.shape)}, expected {tuple(shape)}')
    return t.detach().float().contiguous()


def _seqs(B, cu_seqlens, T=None):
    """(int64 cu_seqlens, number of documents).  With CCQ_B200_CHECK=1 the offsets are also checked
    (start at 0, never decrease, end at T), which reads them back to the host."""
    if cu_seqlens is None:
        return None, B
    cu = cu_seqlens.to(torch.int64).contiguous()
    if B != 1:
        raise ValueError(f'varlen inputs (cu_seqlens given) must have batch size 1, got {B}')
    if cu.ndim != 1 or cu.numel() < 2:
        raise ValueError('cu_seqlens must be a 1-D tensor with at least two offsets')
    if T is not None and os.environ.get('CCQ_B200_CHECK') == '1':
        c = cu.cpu()
        if int(c[0]) != 0 or int(c[-1]) != T or bool((c[1:] < c[:-1]).any()):
            raise ValueError(f'cu_seqlens must start at 0, never decrease and end at T={T}')
    return cu, cu.numel() - 1


def reshape_lambda_3d(lam, q):
    """lambda broadcast to [B, T, H] in q's dtype (ccq/ops/common/clean.py:314-325)."""
    B, T, H = q.shape[:3]
    if not isinstance(lam, torch.Tensor):
        return torch.full((B, T, H), float(lam), device=q.device, dtype=q.dtype)
    if lam.ndim == 0:
        return lam.detach().expand(B, T, H).contiguous().to(q.dtype)
    if lam.ndim == 1 and lam.shape[0] == H:
        return lam.detach().view(1, 1, H).expand(B, T, H).contiguous().to(q.dtype)
    if lam.ndim == 4 and lam.shape[-1] == 1:
        return lam.detach().squeeze(-1).contiguous().to(q.dtype)
    return lam.detach().to(q.dtype).reshape(B, T, H).contiguous()


def reduce_lambda_grad(dlam3, lam):
    """The [B,T,H] lambda gradient reduced to lambda's own shape and dtype (fused_read.py:504-513)."""
    if lam.ndim == 0:
        dl = dlam3.sum()
    elif lam.ndim == 1:
        dl = dlam3.sum(dim=(0, 1))
    elif lam.ndim == 4 and lam.shape[-1] == 1:
        dl = dlam3.unsqueeze(-1)
    else:
        dl = dlam3.reshape(lam.shape)
    return dl.to(lam.dtype)


def device_status(ws):
    """Error word of the tensor-core kernels that last used workspace ``ws`` (0 = every bounded
    pipeline wait completed).  Waits for the current stream.  With CCQ_B200_CHECK=1 the C entry
    points check it themselves and the operators raise CCQError on a non-zero code."""
    if ws is None:
        return 0
    code = ctypes.c_int(0)
    _lib.check(_lib.load().ccq_device_status(_p(ws), _stream(ws.device), ctypes.byref(code)))
    return code.value


def _workspace(op, dtype, B, T, H, K, N, device, flags=0):
    """A workspace sized for the path the call takes (the tensor-core backward needs a few hundred
    bytes per (document, head); only the exact backward needs per-chunk state checkpoints)."""
    nbytes = _lib.load().ccq_workspace_size_for(op, dtype, B, T, H, K, N, flags)
    if nbytes == 0:
        return None, 0
    return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes


def clean_fwd_raw(q, k, lam3, gate_w, gate_b, position_offset, h0, m0, subtract_mean, cu, N):
    """One ccq_clean_fwd call; returns (q_clean, final_cov, final_mean, token_aux [B,T,H,2] fp32)."""
    B, T, H, K = q.shape
    dev = q.device
    dt = _dtype_code(q)
    qc = torch.empty_like(q)
    fcov = torch.empty(N, H, K, K, device=dev, dtype=torch.float32)
    fmean = torch.empty(N, H, K, device=dev, dtype=torch.float32) if subtract_mean else None
    aux = torch.empty(B, T, H, 2, device=dev, dtype=torch.float32)
    ws, nbytes = _workspace(_lib.CCQ_OP_FWD, dt, B, T, H, K, N, dev)
    mode = _lib.CCQ_LAMBDA_GATE if gate_w is not None else _lib.CCQ_LAMBDA_TOKEN
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.ccq_clean_fwd(dt, B, T, H, K, _p(q), _p(k), mode, _p(lam3), _p(gate_w), _p(gate_b), _p(aux),
                               _p(cu), N, int(position_offset), int(bool(subtract_mean)), _p(h0), _p(m0),
                               _p(qc), _p(fcov), _p(fmean), _p(ws), nbytes, _stream(dev))
    _lib.check(st)
    return qc, fcov, fmean, aux


def clean_bwd_raw(q, k, lam3, gate_w, gate_b, position_offset, h0, m0, subtract_mean, cu, N, fcov, fmean, aux,
                  dqc, dfinal_cov, dfinal_mean, want_dlam=True, gate_out=None):
    """One ccq_clean_bwd call; returns (dq, dk, dlam3 | (dW, db), dh0, dm0).

    ``gate_out``: optional contiguous fp32 (dW [H, K], db [H]) tensors the gate gradients are
    written into (for instance views of a buffer that is all-reduced next)."""
    B, T, H, K = q.shape
    dev = q.device
    dt = _dtype_code(q)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    gate = gate_w is not None
    dlam = torch.empty(B, T, H, device=dev, dtype=torch.float32) if (want_dlam and not gate) else None
    if gate and gate_out is not None:
        dW, db = gate_out
        if not (dW.is_contiguous() and db.is_contiguous() and dW.dtype == torch.float32 and db.dtype == torch.float32
                and tuple(dW.shape) == (H, K) and tuple(db.shape) == (H,)):
            raise ValueError('gate_out must be contiguous fp32 tensors of shapes [H, K] and [H]')
    else:
        dW = torch.empty_like(gate_w) if gate else None
        db = torch.empty_like(gate_b) if gate else None
    dh0 = torch.empty(N, H, K, K, device=dev, dtype=torch.float32) if h0 is not None else None
    use_carry = bool(subtract_mean) or dfinal_mean is not None
    dm0 = torch.empty(N, H, K, device=dev, dtype=torch.float32) if (m0 is not None and use_carry) else None
    have_fwd = fcov is not None and aux is not None and (fmean is not None or not subtract_mean)
    ws, nbytes = _workspace(_lib.CCQ_OP_BWD, dt, B, T, H, K, N, dev,
                            _lib.CCQ_WS_HAVE_FWD_OUTPUTS if have_fwd else 0)
    mode = _lib.CCQ_LAMBDA_GATE if gate else _lib.CCQ_LAMBDA_TOKEN
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.ccq_clean_bwd(dt, B, T, H, K, _p(q), _p(k), mode, _p(lam3), _p(gate_w), _p(gate_b), _p(cu), N,
                               int(position_offset), int(bool(subtract_mean)), _p(h0), _p(m0), _p(fcov),
                               _p(fmean), _p(aux), _p(dqc), _p(dfinal_cov), _p(dfinal_mean), _p(dq), _p(dk), _p(dlam),
                               _p(dW), _p(db), _p(dh0), _p(dm0), _p(ws), nbytes, _stream(dev))
    _lib.check(st)
    return dq, dk, ((dW, db) if gate else dlam), dh0, dm0


def clean_l2norm_fwd_raw(q, k, lam3, gate_w, gate_b, position_offset, h0, m0, subtract_mean, cu, N):
    """One ccq_clean_l2norm_fwd call on raw q, k; returns
    (q_clean, k_norm, final_cov, final_mean, token_aux [B,T,H,2], norm_aux [B,T,H,2])."""
    B, T, H, K = q.shape
    dev = q.device
    dt = _dtype_code(q)
    qc = torch.empty_like(q)
    kn = torch.empty_like(k)
    fcov = torch.empty(N, H, K, K, device=dev, dtype=torch.float32)
    fmean = torch.empty(N, H, K, device=dev, dtype=torch.float32) if subtract_mean else None
    aux = torch.empty(B, T, H, 2, device=dev, dtype=torch.float32)
    naux = torch.empty(B, T, H, 2, device=dev, dtype=torch.float32)
    ws, nbytes = _workspace(_lib.CCQ_OP_FWD, dt, B, T, H, K, N, dev, _lib.CCQ_WS_L2NORM)
    mode = _lib.CCQ_LAMBDA_GATE if gate_w is not None else _lib.CCQ_LAMBDA_TOKEN
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.ccq_clean_l2norm_fwd(dt, B, T, H, K, _p(q), _p(k), mode, _p(lam3), _p(gate_w), _p(gate_b), _p(aux),
                                      _p(naux), _p(cu), N, int(position_offset), int(bool(subtract_mean)), _p(h0),
                                      _p(m0), _p(qc), _p(kn), _p(fcov), _p(fmean), _p(ws), nbytes, _stream(dev))
    _lib.check(st)
    return qc, kn, fcov, fmean, aux, naux


def clean_l2norm_bwd_raw(q, kn, lam3, gate_w, gate_b, position_offset, h0, m0, subtract_mean, cu, N, fcov, fmean,
                         aux, naux, dqc, dkn, dfinal_cov, dfinal_mean, want_dlam=True):
    """One ccq_clean_l2norm_bwd call; returns (dq, dk, dlam3 | (dW, db), dh0, dm0), dq and dk on the raw
    q and k (``dkn``: gradient arriving on the normalised keys, or None)."""
    B, T, H, K = q.shape
    dev = q.device
    dt = _dtype_code(q)
    dq = torch.empty_like(q)
    dk = torch.empty_like(kn)
    gate = gate_w is not None
    dlam = torch.empty(B, T, H, device=dev, dtype=torch.float32) if (want_dlam and not gate) else None
    dW = torch.empty_like(gate_w) if gate else None
    db = torch.empty_like(gate_b) if gate else None
    dh0 = torch.empty(N, H, K, K, device=dev, dtype=torch.float32) if h0 is not None else None
    use_carry = bool(subtract_mean) or dfinal_mean is not None
    dm0 = torch.empty(N, H, K, device=dev, dtype=torch.float32) if (m0 is not None and use_carry) else None
    ws, nbytes = _workspace(_lib.CCQ_OP_BWD, dt, B, T, H, K, N, dev,
                            _lib.CCQ_WS_HAVE_FWD_OUTPUTS | _lib.CCQ_WS_L2NORM)
    mode = _lib.CCQ_LAMBDA_GATE if gate else _lib.CCQ_LAMBDA_TOKEN
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.ccq_clean_l2norm_bwd(dt, B, T, H, K, _p(q), _p(kn), mode, _p(lam3), _p(gate_w), _p(gate_b), _p(cu), N,
                                      int(position_offset), int(bool(subtract_mean)), _p(h0), _p(m0), _p(fcov),
                                      _p(fmean), _p(aux), _p(naux), _p(dqc), _p(dkn), _p(dfinal_cov), _p(dfinal_mean),
                                      _p(dq), _p(dk), _p(dlam), _p(dW), _p(db), _p(dh0), _p(dm0), _p(ws), nbytes,
                                      _stream(dev))
    _lib.check(st)
    return dq, dk, ((dW, db) if gate else dlam), dh0, dm0


class FusedCCQCleanRead(torch.autograd.Function):
    """q_clean, final covariance and final key-sum states from (q, k, lambda) (fused_read.py:474-514)."""

    @staticmethod
    def forward(ctx, q, k, lambda_h, position_offset, initial_cov_state, initial_mean_state,
                output_final_state, subtract_mean, cu_seqlens):
        _check_cuda(q, k, lambda_h if isinstance(lambda_h, torch.Tensor) else None,
                    initial_cov_state, initial_mean_state, cu_seqlens)
        q = q.contiguous()
        k = k.contiguous() if k.dtype == q.dtype else k.to(q.dtype).contiguous()
        B, T, H, K = q.shape
        cu, N = _seqs(B, cu_seqlens, T)
        h0 = _state(initial_cov_state, (N, H, K, K))
        m0 = _state(initial_mean_state, (N, H, K)) if subtract_mean else None
        lam3 = reshape_lambda_3d(lambda_h, q)
        qc, fcov, fmean, aux = clean_fwd_raw(q, k, lam3, None, None, position_offset, h0, m0, subtract_mean, cu, N)
        ctx.save_for_backward(q, k, lam3, h0, m0, cu, fcov, fmean, aux)
        ctx.lambda_h = lambda_h if isinstance(lambda_h, torch.Tensor) else None
        ctx.position_offset = int(position_offset)
        ctx.subtract_mean = bool(subtract_mean)
        ctx.N = N
        ctx.has_m0 = initial_mean_state is not None and bool(subtract_mean)
        if not output_final_state:
            return qc, None, None
        return qc, fcov.clone(), (fmean.clone() if fmean is not None else None)

    @staticmethod
    def backward(ctx, dqc, dfinal_cov, dfinal_mean):
        q, k, lam3, h0, m0, cu, fcov, fmean, aux = ctx.saved_tensors
        lam_t = ctx.lambda_h
        need_dl = lam_t is not None and ctx.needs_input_grad[2]
        dqc = dqc.contiguous() if dqc.dtype == q.dtype else dqc.to(q.dtype).contiguous()
        dfc = dfinal_cov.float().contiguous() if dfinal_cov is not None else None
        dfm = dfinal_mean.float().contiguous() if dfinal_mean is not None else None
        dq, dk, dlam3, dh0, dm0 = clean_bwd_raw(q, k, lam3, None, None, ctx.position_offset, h0, m0,
                                                ctx.subtract_mean, cu, ctx.N, fcov, fmean, aux, dqc, dfc, dfm,
                                                want_dlam=need_dl)
        dl = reduce_lambda_grad(dlam3, lam_t) if need_dl else None
        if dm0 is not None and not ctx.has_m0:
            dm0 = None
        return dq, dk, dl, None, dh0, dm0, None, None, None


def fused_ccq_clean_read(q, k, lambda_h, *, position_offset=0, initial_cov_state=None, initial_mean_state=None,
                         output_final_state=False, subtract_mean=True, cu_seqlens=None):
    """Drop-in for ccq.ops.common.fused_read.fused_ccq_clean_read (fused_read.py:517-531).

    Returns (q_clean, final_cov_state, final_mean_state); the states are None unless requested.
    """
    qc, final_cov, final_mean = FusedCCQCleanRead.apply(
        q, k, lambda_h, int(position_offset), initial_cov_state, initial_mean_state,
        bool(output_final_state), bool(subtract_mean), cu_seqlens,
    )
    if not output_final_state:
        final_cov, final_mean = None, None
    return qc, final_cov, final_mean


class FusedCCQCleanReadL2Norm(torch.autograd.Function):
    """l2norm(q), l2norm(k) and the cleaning operator in one: (q_clean, k_norm, final_cov, final_mean)
    from the raw q and k.  Replaces fla's l2norm of both plus FusedCCQCleanRead as the fused_chunk
    orchestrators chain them (ccq/ops/ccq_gdn/fused_chunk.py:42-53, ccq/ops/ccq_gla/fused_chunk.py:31-41)."""

    @staticmethod
    def forward(ctx, q, k, lambda_h, position_offset, initial_cov_state, initial_mean_state,
                output_final_state, subtract_mean, cu_seqlens):
        _check_cuda(q, k, lambda_h if isinstance(lambda_h, torch.Tensor) else None,
                    initial_cov_state, initial_mean_state, cu_seqlens)
        ctx.set_materialize_grads(False)
        q = q.contiguous()
        k = k.contiguous() if k.dtype == q.dtype else k.to(q.dtype).contiguous()
        B, T, H, K = q.shape
        cu, N = _seqs(B, cu_seqlens, T)
        h0 = _state(initial_cov_state, (N, H, K, K))
        m0 = _state(initial_mean_state, (N, H, K)) if subtract_mean else None
        lam3 = reshape_lambda_3d(lambda_h, q)
        qc, kn, fcov, fmean, aux, naux = clean_l2norm_fwd_raw(q, k, lam3, None, None, position_offset, h0, m0,
                                                              subtract_mean, cu, N)
        ctx.save_for_backward(q, kn, lam3, h0, m0, cu, fcov, fmean, aux, naux)
        ctx.lambda_h = lambda_h if isinstance(lambda_h, torch.Tensor) else None
        ctx.position_offset = int(position_offset)
        ctx.subtract_mean = bool(subtract_mean)
        ctx.N = N
        ctx.has_m0 = initial_mean_state is not None and bool(subtract_mean)
        if not output_final_state:
            return qc, kn, None, None
        return qc, kn, fcov.clone(), (fmean.clone() if fmean is not None else None)

    @staticmethod
    def backward(ctx, dqc, dkn, dfinal_cov, dfinal_mean):
        q, kn, lam3, h0, m0, cu, fcov, fmean, aux, naux = ctx.saved_tensors
        lam_t = ctx.lambda_h
        need_dl = lam_t is not None and ctx.needs_input_grad[2]
        if dqc is None:
            dqc = torch.zeros_like(q)
        dqc = dqc.contiguous() if dqc.dtype == q.dtype else dqc.to(q.dtype).contiguous()
        if dkn is not None:
            dkn = dkn.contiguous() if dkn.dtype == q.dtype else dkn.to(q.dtype).contiguous()
        dfc = dfinal_cov.float().contiguous() if dfinal_cov is not None else None
        dfm = dfinal_mean.float().contiguous() if dfinal_mean is not None else None
        dq, dk, dlam3, dh0, dm0 = clean_l2norm_bwd_raw(q, kn, lam3, None, None, ctx.position_offset, h0, m0,
                                                       ctx.subtract_mean, cu, ctx.N, fcov, fmean, aux, naux, dqc, dkn,
                                                       dfc, dfm, want_dlam=need_dl)
        dl = reduce_lambda_grad(dlam3, lam_t) if need_dl else None
        if dm0 is not None and not ctx.has_m0:
            dm0 = None
        return dq, dk, dl, None, dh0, dm0, None, None, None


def fused_ccq_clean_read_l2norm(q, k, lambda_h, *, position_offset=0, initial_cov_state=None,
                                initial_mean_state=None, output_final_state=False, subtract_mean=True,
                                cu_seqlens=None):
    """``q, k = l2norm(q), l2norm(k)`` (fla, eps 1e-6) followed by ``fused_ccq_clean_read`` in one call.

    Takes the raw q and k; returns (q_clean, k_norm, final_cov_state, final_mean_state), where k_norm
    is the normalised keys the backbone reads next.  Gradients reach the raw q and k (including the
    gradient the backbone sends back through k_norm).  On the tensor-core path the normalised q
    never goes to memory: the kernels normalise the tiles they load.
    """
    qc, kn, final_cov, final_mean = FusedCCQCleanReadL2Norm.apply(
        q, k, lambda_h, int(position_offset), initial_cov_state, initial_mean_state,
        bool(output_final_state), bool(subtract_mean), cu_seqlens,
    )
    if not output_final_state:
        final_cov, final_mean = None, None
    return qc, kn, final_cov, final_mean


class FusedCCQCleanGated(torch.autograd.Function):
    """The cleaning operator with the per-head gate lambda = sigmoid(W[h] . q + b[h]) in the kernels."""

    @staticmethod
    def forward(ctx, q, k, gate_w, gate_b, position_offset, initial_cov_state, initial_mean_state,
                output_final_state, subtract_mean, cu_seqlens):
        _check_cuda(q, k, gate_w, gate_b, initial_cov_state, initial_mean_state, cu_seqlens)
        q = q.contiguous()
        k = k.contiguous() if k.dtype == q.dtype else k.to(q.dtype).contiguous()
        B, T, H, K = q.shape
        if tuple(gate_w.shape) != (H, K) or tuple(gate_b.shape) != (H,):
            raise ValueError(f'gate_w must be [H, K] = [{H}, {K}] and gate_b [H]')
        W = gate_w.detach().float().contiguous()
        bb = gate_b.detach().float().contiguous()
        cu, N = _seqs(B, cu_seqlens, T)
        h0 = _state(initial_cov_state, (N, H, K, K))
        m0 = _state(initial_mean_state, (N, H, K)) if subtract_mean else None
        qc, fcov, fmean, aux = clean_fwd_raw(q, k, None, W, bb, position_offset, h0, m0, subtract_mean, cu, N)
        ctx.save_for_backward(q, k, W, bb, h0, m0, cu, fcov, fmean, aux)
        ctx.position_offset = int(position_offset)
        ctx.subtract_mean = bool(subtract_mean)
        ctx.N = N
        ctx.w_dtype = gate_w.dtype
        ctx.has_m0 = initial_mean_state is not None and bool(subtract_mean)
        if not output_final_state:
            return qc, None, None
        return qc, fcov.clone(), (fmean.clone() if fmean is not None else None)

    @staticmethod
    def backward(ctx, dqc, dfinal_cov, dfinal_mean):
        q, k, W, bb, h0, m0, cu, fcov, fmean, aux = ctx.saved_tensors
        dqc = dqc.contiguous() if dqc.dtype == q.dtype else dqc.to(q.dtype).contiguous()
        dfc = dfinal_cov.float().contiguous() if dfinal_cov is not None else None
        dfm = dfinal_mean.float().contiguous() if dfinal_mean is not None else None
        dq, dk, (dW, db), dh0, dm0 = clean_bwd_raw(q, k, None, W, bb, ctx.position_offset, h0, m0,
                                                   ctx.subtract_mean, cu, ctx.N, fcov, fmean, aux, dqc, dfc, dfm)
        if dm0 is not None and not ctx.has_m0:
            dm0 = None
        return dq, dk, dW.to(ctx.w_dtype), db.to(ctx.w_dtype), None, dh0, dm0, None, None, None


def fused_ccq_clean_gated(q, k, gate_w, gate_b, *, position_offset=0, initial_cov_state=None,
                          initial_mean_state=None, output_final_state=False, subtract_mean=True, cu_seqlens=None):
    """The cleaning operator with lambda = sigmoid(gate_w[h] . q + gate_b[h]) computed in the kernels.

    gate_w is [H, K] and gate_b [H] (the per-head, block-diagonal form of the layer's
    erase_lambda_proj, ccq/gdn/layer.py:174, :292).  Gradients reach gate_w and gate_b directly.
    """
    qc, final_cov, final_mean = FusedCCQCleanGated.apply(
        q, k, gate_w, gate_b, int(position_offset), initial_cov_state, initial_mean_state,
        bool(output_final_state), bool(subtract_mean), cu_seqlens,
    )
    if not output_final_state:
        final_cov, final_mean = None, None
    return qc, final_cov, final_mean


def ccq_gate_lambda(q, gate_w, gate_b):
    """lambda = sigmoid(gate_w[h] . q + gate_b[h]) as the gated kernels compute it (fp32), for inspection."""
    return torch.sigmoid(torch.einsum('bthk,hk->bth', q.float(), gate_w.float()) + gate_b.float())


def decode_step(q, k, lambda_h, cov_state=None, mean_state=None, *, position_offset=0, subtract_mean=True,
                cu_seqlens=None, gate_w=None, gate_b=None, inplace=False):
    """Recurrent cleaning over the generation cache (inference; no autograd).

    Returns (q_clean, cov_state_after [N,H,K,K] fp32, mean_state_after [N,H,K] fp32 or None).
    ``inplace=True`` updates the given cache tensors instead of allocating new ones.
    """
    qc, _, cov, mean = _decode(q, k, lambda_h, cov_state, mean_state, position_offset, subtract_mean, cu_seqlens,
                               gate_w, gate_b, inplace, False)
    return qc, cov, mean


def decode_step_l2norm(q, k, lambda_h, cov_state=None, mean_state=None, *, position_offset=0, subtract_mean=True,
                       cu_seqlens=None, gate_w=None, gate_b=None, inplace=False):
    """decode_step on RAW q and k, with fla's l2norm of both (eps 1e-6) done inside the kernel.

    Returns (q_clean, k_norm, cov_state_after, mean_state_after); k_norm is what the backbone reads."""
    return _decode(q, k, lambda_h, cov_state, mean_state, position_offset, subtract_mean, cu_seqlens, gate_w, gate_b,
                   inplace, True)


def _decode(q, k, lambda_h, cov_state, mean_state, position_offset, subtract_mean, cu_seqlens, gate_w, gate_b,
            inplace, l2norm_qk):
    _check_cuda(q, k, lambda_h if isinstance(lambda_h, torch.Tensor) else None, cov_state, mean_state,
                cu_seqlens, gate_w, gate_b)
    q = q.detach().contiguous()
    k = k.detach().to(q.dtype).contiguous()
    B, T, H, K = q.shape
    cu, N = _seqs(B, cu_seqlens, T)
    dev = q.device
    if cov_state is not None and tuple(cov_state.shape) != (N, H, K, K):
        raise ValueError(f'cov_state has shape {tuple(cov_state.shape)}, expected {(N, H, K, K)}')
    if mean_state is not None and tuple(mean_state.shape) != (N, H, K):
        raise ValueError(f'mean_state has shape {tuple(mean_state.shape)}, expected {(N, H, K)}')
    cov_in = cov_state.detach() if cov_state is not None else None
    if cov_in is not None and (cov_in.dtype != torch.float32 or not cov_in.is_contiguous()):
        cov_in = cov_in.float().contiguous()
        inplace = False
    mean_in = None
    if subtract_mean and mean_state is not None:
        mean_in = mean_state.detach()
        if mean_in.dtype != torch.float32 or not mean_in.is_contiguous():
            mean_in = mean_in.float().contiguous()
    if inplace and cov_in is not None:
        cov_out = cov_in
    else:
        cov_out = torch.empty(N, H, K, K, device=dev, dtype=torch.float32)
    mean_out = None
    if subtract_mean:
        mean_out = mean_in if (inplace and mean_in is not None) else torch.empty(N, H, K, device=dev,
                                                                                  dtype=torch.float32)
    qc = torch.empty_like(q)
    gate = gate_w is not None
    lam3 = None if gate else reshape_lambda_3d(lambda_h, q)
    W = gate_w.detach().float().contiguous() if gate else None
    bb = gate_b.detach().float().contiguous() if gate else None
    mode = _lib.CCQ_LAMBDA_GATE if gate else _lib.CCQ_LAMBDA_TOKEN
    kn = torch.empty_like(k) if l2norm_qk else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.ccq_decode_step_l2norm(_dtype_code(q), B, T, H, K, _p(q), _p(k), mode, _p(lam3), _p(W), _p(bb), _p(cu),
                                        N, int(position_offset), int(bool(subtract_mean)), _p(cov_in), _p(mean_in),
                                        _p(cov_out), _p(mean_out), _p(qc), _p(kn), _stream(dev))
    _lib.check(st)
    return qc, kn, cov_out, mean_out


def l2norm(x, eps=1e-6):
    """x / sqrt(sum(x^2) + eps) over the last dim, computed in fp32 (fla/modules/l2norm.py:266)."""
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)


def fused_ccq_clean(q, k, lambda_h, *, initial_cov_state=None, initial_mean_state=None, output_final_state=False,
                    cu_seqlens=None, use_qk_l2norm_in_kernel=False, position_offset=0, subtract_mean=True,
                    use_chunk=True, chunk_size=64):
    """Drop-in for ccq.ops.ccq_gdn.fused_clean.fused_ccq_clean (fused_clean.py:34-83).

    Returns (q_clean, k, final_cov_state, final_mean_state, use_qk_l2norm_in_kernel).  Inference
    calls run the decode kernel; calls that need gradients run the chunked operator, whose math
    is identical (the inclusive read z_t = C_t q_t at pos_t = t + 1 + position_offset).  With
    ``use_qk_l2norm_in_kernel`` the normalisation of q and k happens inside those kernels and the
    returned k is the normalised one (as the reference returns it), with the flag cleared.
    """
    norm = bool(use_qk_l2norm_in_kernel)
    needs_grad = torch.is_grad_enabled() and any(
        isinstance(t, torch.Tensor) and t.requires_grad
        for t in (q, k, lambda_h, initial_cov_state, initial_mean_state))
    m0 = initial_mean_state if subtract_mean else None
    if needs_grad or (use_chunk and q.shape[1] > chunk_size):
        kw = dict(position_offset=position_offset, initial_cov_state=initial_cov_state, initial_mean_state=m0,
                  output_final_state=output_final_state, subtract_mean=subtract_mean, cu_seqlens=cu_seqlens)
        if norm:
            qc, k, fc, fm = fused_ccq_clean_read_l2norm(q, k, lambda_h, **kw)
        else:
            qc, fc, fm = fused_ccq_clean_read(q, k, lambda_h, **kw)
        return qc, k, fc, fm, False
    if norm:
        qc, k, fc, fm = decode_step_l2norm(q, k, lambda_h, initial_cov_state, initial_mean_state,
                                           position_offset=position_offset, subtract_mean=subtract_mean,
                                           cu_seqlens=cu_seqlens)
    else:
        qc, fc, fm = decode_step(q, k, lambda_h, initial_cov_state, initial_mean_state,
                                 position_offset=position_offset, subtract_mean=subtract_mean, cu_seqlens=cu_seqlens)
    if not output_final_state:
        fc, fm = None, None
    return qc, k, fc, fm, False
