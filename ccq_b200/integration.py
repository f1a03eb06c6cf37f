"""Drop-in wiring into the reference package (``ccq``): ``attn_mode: "fused_chunk"`` and the decode step.

``install()`` rebinds, inside an imported reference package, exactly the names its layers reach
for this path, so the unchanged layers run the B200 kernels:

* ``ccq.ops.common.fused_read.fused_ccq_clean_read`` / ``FusedCCQCleanRead``
  (fused_read.py:474-531) and the imported copies in the orchestrators
  ``ccq.ops.ccq_gdn.fused_chunk`` (fused_chunk.py:13, called at :45) and
  ``ccq.ops.ccq_gla.fused_chunk`` (fused_chunk.py:13, called at :33), which the layers'
  ``attn_mode`` dispatch calls (ccq/gdn/layer.py:355-372, ccq/gla/layer.py:289-303);
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
    q = ops.l2norm(q, eps=1e-6)
    k = ops.l2norm(k, eps=1e-6)
    q_clean, _, final_cov_state, final_mean_state, _ = ops.fused_ccq_clean(
        q, k, lambda_h, initial_cov_state=initial_cov_state,
        initial_mean_state=initial_mean_state if subtract_mean else None,
        output_final_state=output_final_state, cu_seqlens=cu_seqlens, position_offset=position_offset,
        subtract_mean=subtract_mean, use_chunk=False)
    o, final_state = fused_recurrent_gla(q=q_clean, k=k, v=v, gk=gk, gv=gv, scale=scale,
                                         initial_state=initial_state, output_final_state=output_final_state,
                                         reverse=reverse, cu_seqlens=cu_seqlens)
    return o, final_state, final_cov_state, final_mean_state


def install():
    """Route the reference package's cleaning operator and decode step to the B200 kernels."""
    _set('ccq.ops.common.fused_read', 'fused_ccq_clean_read', ops.fused_ccq_clean_read)
    _set('ccq.ops.common.fused_read', 'FusedCCQCleanRead', ops.FusedCCQCleanRead)
    _set('ccq.ops.ccq_gdn.fused_chunk', 'fused_ccq_clean_read', ops.fused_ccq_clean_read)
    _set('ccq.ops.ccq_gla.fused_chunk', 'fused_ccq_clean_read', ops.fused_ccq_clean_read)
    _set('ccq.ops.ccq_gdn.fused_clean', 'fused_ccq_clean', ops.fused_ccq_clean)
    _set('ccq.ops.ccq_gdn.fused_recurrent', 'fused_ccq_clean', ops.fused_ccq_clean)
    _set('ccq.ops.ccq_gla.fused_recurrent', 'fused_recurrent_ccq_gla', fused_recurrent_ccq_gla)
    _set('ccq.ops.ccq_gla', 'fused_recurrent_ccq_gla', fused_recurrent_ccq_gla)
    try:
        _set('ccq.gla.layer', 'fused_recurrent_ccq_gla', fused_recurrent_ccq_gla)
    except ImportError:  # layers need transformers; the ops above are enough without them
        pass


def uninstall():
    """Restore every name install() replaced."""
    for (module_name, attr), value in list(_saved.items()):
        setattr(importlib.import_module(module_name), attr, value)
    _saved.clear()
