"""Drop-in wiring into the reference package (``ccq``): ``attn_mode`` "fused_chunk" and "chunk", and
the decode step.

``install()`` rebinds, inside an imported reference package, exactly the names its layers reach
for this path, so the unchanged layers run the B200 kernels:

* the orchestrators ``fused_chunk_ccq_gdn`` / ``fused_chunk_ccq_gla`` (ccq/ops/ccq_gdn/fused_chunk.py:16-59,
  ccq/ops/ccq_gla/fused_chunk.py:16-46) and ``chunk_ccq_gdn`` / ``chunk_ccq_gla``
  (ccq/ops/ccq_gdn/chunk.py:11-87, ccq/ops/ccq_gla/chunk.py:17-64), in their modules, their packages
  and the layer modules that imported them (ccq/gdn/layer.py:14-18, ccq/gla/layer.py:14-18), which
  the layers' ``attn_mode`` dispatch calls (gdn/layer.py:337-390, gla/layer.py:274-320).  The B200
  versions keep the reference's signatures and return tuples, call the fused l2norm + cleaning
  operator (``ops.fused_ccq_clean_read_l2norm``: no separate normalisation pass over q and k) and
  hand q_clean and the normalised keys, in the layout the backbone reads, to the same fla
  backbone the reference calls (chunk_gated_delta_rule / chunk_gla, with ``cp_context`` passed
  through);
* ``ccq.ops.common.fused_read.fused_ccq_clean_read`` / ``FusedCCQCleanRead``
  (fused_read.py:474-531) and the imported copies in the reference's own orchestrators
  (fused_chunk.py:13 of both), for callers that use the operator directly;
* the GDN decode cleaning ``fused_ccq_clean`` (ccq/ops/ccq_gdn/fused_clean.py:34-83) as imported by
  ``ccq.ops.ccq_gdn.fused_recurrent`` (fused_recurrent.py:15, called at :53);
* the GLA decode orchestrator ``fused_recurrent_ccq_gla`` (ccq/ops/ccq_gla/fused_recurrent.py:9-51),
  rebuilt here around the B200 decode step and fla's ``fused_recurrent_gla`` backbone, and its
  imported copy in ``ccq.gla.layer``.

The backbones (fla's chunk_gated_delta_rule, chunk_gla, fused_recurrent_*) are untouched.
``uninstall()`` restores the reference's own functions.
"""
from __future__ import annotations

import importlib

from . import ops

_saved = {}


def _set(module_name, attr, value):
    mod = importlib.import_module(module_name)
    key = (module_name, attr)
    if key not in _saved:
        _saved[key] = getattr(mod, attr)
    setattr(mod, attr, value)


def fused_recurrent_ccq_gla(q, k, v, lambda_h, gk=None, gv=None, scale=None, initial_state=None,
                            initial_cov_state=None, initial_mean_state=None, output_final_state=False,
                            reverse=False, cu_seqlens=None, position_offset=0, subtract_mean=True):
    """GLA decode step (ccq/ops/ccq_gla/fused_recurrent.py:9-51) with the B200 cleaning.

    Same arguments and returns: (o, final_state, final_cov_state, final_mean_state).
    """
    from fla.ops.gla.fused_recurrent import fused_recurrent_gla
    q_clean, k, final_cov_state, final_mean_state, _ = ops.fused_ccq_clean(
        q, k, lambda_h, initial_cov_state=initial_cov_state,
        initial_mean_state=initial_mean_state if subtract_mean else None,
        output_final_state=output_final_state, cu_seqlens=cu_seqlens, use_qk_l2norm_in_kernel=True,
        position_offset=position_offset, subtract_mean=subtract_mean, use_chunk=False)
    o, final_state = fused_recurrent_gla(q=q_clean, k=k, v=v, gk=gk, gv=gv, scale=scale,
                                         initial_state=initial_state, output_final_state=output_final_state,
                                         reverse=reverse, cu_seqlens=cu_seqlens)
    return o, final_state, final_cov_state, final_mean_state


def fused_chunk_ccq_gdn(q, k, v, lambda_h, g, beta, scale=None, initial_state=None, initial_cov_state=None,
                        initial_mean_state=None, output_final_state=False, use_qk_l2norm_in_kernel=False,
                        cu_seqlens=None, position_offset=0, subtract_mean=True, enable_ccq=True, **kwargs):
    """CCQ-GDN, attn_mode "fused_chunk" (ccq/ops/ccq_gdn/fused_chunk.py:16-59): the B200 cleaning, with
    the l2norm of q and k fused into it, then fla's chunk_gated_delta_rule on (q_clean, k_norm).

    Same arguments and returns: (o, final_state, final_cov_state, final_mean_state)."""
    from fla.ops.gated_delta_rule import chunk_gated_delta_rule
    if not enable_ccq:
        o, final_state = chunk_gated_delta_rule(q=q, k=k, v=v, g=g, beta=beta, scale=scale, initial_state=initial_state,
                                                output_final_state=output_final_state,
                                                use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
                                                cu_seqlens=cu_seqlens, **kwargs)
        return o, final_state, None, None
    q_clean, k, final_cov_state, final_mean_state = _clean(q, k, lambda_h, use_qk_l2norm_in_kernel, position_offset,
                                                           initial_cov_state, initial_mean_state, output_final_state,
                                                           subtract_mean, cu_seqlens)
    o, final_state = chunk_gated_delta_rule(q=q_clean, k=k, v=v, g=g, beta=beta, scale=scale,
                                            initial_state=initial_state, output_final_state=output_final_state,
                                            use_qk_l2norm_in_kernel=False, cu_seqlens=cu_seqlens, **kwargs)
    return o, final_state, final_cov_state, final_mean_state


def fused_chunk_ccq_gla(q, k, v, lambda_h, g=None, scale=None, initial_state=None, initial_cov_state=None,
                        initial_mean_state=None, output_final_state=False, cu_seqlens=None, position_offset=0,
                        subtract_mean=True):
    """CCQ-GLA, attn_mode "fused_chunk" (ccq/ops/ccq_gla/fused_chunk.py:16-46): l2norm + cleaning in one
    B200 operator, then fla's chunk_gla on (q_clean, k_norm).  Same arguments and returns."""
    from fla.ops.gla.chunk import chunk_gla
    q_clean, k, final_cov_state, final_mean_state = _clean(q, k, lambda_h, True, position_offset, initial_cov_state,
                                                           initial_mean_state, output_final_state, subtract_mean,
                                                           cu_seqlens)
    o, final_state = chunk_gla(q=q_clean, k=k, v=v, g=g, scale=scale, initial_state=initial_state,
                               output_final_state=output_final_state, cu_seqlens=cu_seqlens)
    return o, final_state, final_cov_state, final_mean_state


def chunk_ccq_gdn(q, k, v, lambda_h, g, beta, scale=None, initial_state=None, initial_cov_state=None,
                  initial_mean_state=None, output_final_state=False, use_qk_l2norm_in_kernel=False, cu_seqlens=None,
                  cp_context=None, transpose_state_layout=False, position_offset=0, subtract_mean=True,
                  enable_ccq=True, **kwargs):
    """CCQ-GDN, attn_mode "chunk" (ccq/ops/ccq_gdn/chunk.py:11-87).  The reference computes the same
    q_clean there from fla's chunk_simple_gla read plus _CCQCleanQ; here it is the B200 operator, and the
    backbone call (with ``cp_context`` and ``transpose_state_layout``) is the reference's.  With a
    context-parallel ``cp_context`` the cleaning carries its (C, m) state across the ranks
    (``distributed.cp_clean_read``), which the reference's chunk path does not do.
    Same arguments and returns: (o, final_state, final_cov_state, final_mean_state)."""
    from fla.ops.gated_delta_rule import chunk_gated_delta_rule
    if not enable_ccq:
        o, final_state = chunk_gated_delta_rule(q=q, k=k, v=v, g=g, beta=beta, scale=scale, initial_state=initial_state,
                                                output_final_state=output_final_state,
                                                use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
                                                cu_seqlens=cu_seqlens, cp_context=cp_context,
                                                transpose_state_layout=transpose_state_layout, **kwargs)
        return o, final_state, None, None
    q_clean, k, final_cov_state, final_mean_state = _clean(q, k, lambda_h, use_qk_l2norm_in_kernel, position_offset,
                                                           initial_cov_state, initial_mean_state, output_final_state,
                                                           subtract_mean, cu_seqlens, cp_context)
    o, final_state = chunk_gated_delta_rule(q=q_clean, k=k, v=v, g=g, beta=beta, scale=scale,
                                            initial_state=initial_state, output_final_state=output_final_state,
                                            use_qk_l2norm_in_kernel=False, cu_seqlens=cu_seqlens,
                                            cp_context=cp_context, transpose_state_layout=transpose_state_layout,
                                            **kwargs)
    return o, final_state, final_cov_state, final_mean_state


def chunk_ccq_gla(q, k, v, lambda_h, g=None, scale=None, initial_state=None, initial_cov_state=None,
                  initial_mean_state=None, output_final_state=False, cu_seqlens=None, position_offset=0,
                  subtract_mean=True):
    """CCQ-GLA, attn_mode "chunk" (ccq/ops/ccq_gla/chunk.py:17-64): same mathematics as fused_chunk, so the
    same B200 operator; then fla's chunk_gla.  Same arguments and returns."""
    return fused_chunk_ccq_gla(q, k, v, lambda_h, g=g, scale=scale, initial_state=initial_state,
                               initial_cov_state=initial_cov_state, initial_mean_state=initial_mean_state,
                               output_final_state=output_final_state, cu_seqlens=cu_seqlens,
                               position_offset=position_offset, subtract_mean=subtract_mean)


def _clean(q, k, lambda_h, l2norm_qk, position_offset, initial_cov_state, initial_mean_state, output_final_state,
           subtract_mean, cu_seqlens, cp_context=None):
    """(q_clean, k as the backbone reads it, final_cov, final_mean) through the B200 operator."""
    m0 = initial_mean_state if subtract_mean else None
    if cp_context is not None and getattr(cp_context, 'group', None) is not None:
        from .distributed import cp_clean_read
        return cp_clean_read(q, k, lambda_h, cp_context, l2norm_qk=l2norm_qk, position_offset=position_offset,
                             initial_cov_state=initial_cov_state, initial_mean_state=m0,
                             output_final_state=output_final_state, subtract_mean=subtract_mean)
    if l2norm_qk:
        return ops.fused_ccq_clean_read_l2norm(q, k, lambda_h, position_offset=position_offset,
                                               initial_cov_state=initial_cov_state, initial_mean_state=m0,
                                               output_final_state=output_final_state, subtract_mean=subtract_mean,
                                               cu_seqlens=cu_seqlens)
    qc, fc, fm = ops.fused_ccq_clean_read(q, k, lambda_h, position_offset=position_offset,
                                          initial_cov_state=initial_cov_state, initial_mean_state=m0,
                                          output_final_state=output_final_state, subtract_mean=subtract_mean,
                                          cu_seqlens=cu_seqlens)
    return qc, k, fc, fm


def install():
    """Route the reference package's cleaning operator, its attn_mode orchestrators and decode step to
    the B200 kernels."""
    _set('ccq.ops.common.fused_read', 'fused_ccq_clean_read', ops.fused_ccq_clean_read)
    _set('ccq.ops.common.fused_read', 'FusedCCQCleanRead', ops.FusedCCQCleanRead)
    _set('ccq.ops.ccq_gdn.fused_chunk', 'fused_ccq_clean_read', ops.fused_ccq_clean_read)
    _set('ccq.ops.ccq_gla.fused_chunk', 'fused_ccq_clean_read', ops.fused_ccq_clean_read)
    _set('ccq.ops.ccq_gdn.fused_clean', 'fused_ccq_clean', ops.fused_ccq_clean)
    _set('ccq.ops.ccq_gdn.fused_recurrent', 'fused_ccq_clean', ops.fused_ccq_clean)
    _set('ccq.ops.ccq_gla.fused_recurrent', 'fused_recurrent_ccq_gla', fused_recurrent_ccq_gla)
    _set('ccq.ops.ccq_gla', 'fused_recurrent_ccq_gla', fused_recurrent_ccq_gla)
    orchestrators = {
        'ccq.ops.ccq_gdn': {'fused_chunk_ccq_gdn': fused_chunk_ccq_gdn, 'chunk_ccq_gdn': chunk_ccq_gdn},
        'ccq.ops.ccq_gla': {'fused_chunk_ccq_gla': fused_chunk_ccq_gla, 'chunk_ccq_gla': chunk_ccq_gla},
    }
    for pkg, names in orchestrators.items():
        for name, fn in names.items():
            _set(pkg, name, fn)
            _set(f'{pkg}.{name.split("_ccq_")[0]}', name, fn)  # the defining module
    for layer, names in (('ccq.gdn.layer', orchestrators['ccq.ops.ccq_gdn']),
                         ('ccq.gla.layer', dict(orchestrators['ccq.ops.ccq_gla'],
                                                fused_recurrent_ccq_gla=fused_recurrent_ccq_gla))):
        try:
            for name, fn in names.items():
                _set(layer, name, fn)
        except ImportError:  # layers need transformers; the ops above are enough without them
            pass


def uninstall():
    """Restore every name install() replaced."""
    for (module_name, attr), value in list(_saved.items()):
        setattr(importlib.import_module(module_name), attr, value)
    _saved.clear()
