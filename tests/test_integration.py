"""The attn_mode drop-in rebinds exactly the reference's names for this path (CPU: wiring only).

The reference package is found under baseline/_ref (its pip install) or CCQ_REFERENCE_PATH; where
neither exists the test is skipped.  Nothing here runs a kernel.
"""
import contextlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
from bench import reference_path  # noqa: E402

REF = reference_path()


@pytest.fixture
def ccq_ref():
    if REF is None:
        pytest.skip('reference package not installed (baseline/_ref or CCQ_REFERENCE_PATH)')
    import torch
    torch.cpu.device = getattr(torch.cpu, 'device', None) or (lambda i=None: contextlib.nullcontext())
    sys.path.insert(0, REF)
    try:
        import ccq.ops.ccq_gdn.fused_chunk  # noqa: F401
        import ccq.ops.ccq_gla.fused_chunk  # noqa: F401
        import ccq.ops.ccq_gdn.fused_recurrent  # noqa: F401
        import ccq.ops.ccq_gla.fused_recurrent  # noqa: F401
    except Exception as exc:  # pragma: no cover - dependency missing
        pytest.skip(f'reference not importable: {exc}')
    yield
    sys.path.remove(REF)


def test_install_rebinds_and_uninstall_restores(ccq_ref):
    import importlib

    from ccq_b200 import integration, ops
    fr = importlib.import_module('ccq.ops.common.fused_read')
    gdn = importlib.import_module('ccq.ops.ccq_gdn.fused_chunk')
    gla = importlib.import_module('ccq.ops.ccq_gla.fused_chunk')
    gdn_rec = importlib.import_module('ccq.ops.ccq_gdn.fused_recurrent')
    gla_rec = importlib.import_module('ccq.ops.ccq_gla.fused_recurrent')
    orig = (fr.fused_ccq_clean_read, gdn.fused_ccq_clean_read, gla.fused_ccq_clean_read, gdn_rec.fused_ccq_clean,
            gla_rec.fused_recurrent_ccq_gla)
    integration.install()
    try:
        assert fr.fused_ccq_clean_read is ops.fused_ccq_clean_read
        assert fr.FusedCCQCleanRead is ops.FusedCCQCleanRead
        assert gdn.fused_ccq_clean_read is ops.fused_ccq_clean_read
        assert gla.fused_ccq_clean_read is ops.fused_ccq_clean_read
        assert gdn_rec.fused_ccq_clean is ops.fused_ccq_clean
        assert gla_rec.fused_recurrent_ccq_gla is integration.fused_recurrent_ccq_gla
        # the attn_mode orchestrators, in their modules and packages
        for mod, name in (('ccq.ops.ccq_gdn.fused_chunk', 'fused_chunk_ccq_gdn'), ('ccq.ops.ccq_gdn', 'fused_chunk_ccq_gdn'),
                          ('ccq.ops.ccq_gdn.chunk', 'chunk_ccq_gdn'), ('ccq.ops.ccq_gdn', 'chunk_ccq_gdn'),
                          ('ccq.ops.ccq_gla.fused_chunk', 'fused_chunk_ccq_gla'), ('ccq.ops.ccq_gla', 'fused_chunk_ccq_gla'),
                          ('ccq.ops.ccq_gla.chunk', 'chunk_ccq_gla'), ('ccq.ops.ccq_gla', 'chunk_ccq_gla')):
            assert getattr(importlib.import_module(mod), name) is getattr(integration, name), (mod, name)
    finally:
        integration.uninstall()
    now = (fr.fused_ccq_clean_read, gdn.fused_ccq_clean_read, gla.fused_ccq_clean_read, gdn_rec.fused_ccq_clean,
           gla_rec.fused_recurrent_ccq_gla)
    assert all(a is b for a, b in zip(orig, now))
    assert importlib.import_module('ccq.ops.ccq_gdn.fused_chunk').fused_chunk_ccq_gdn is not integration.fused_chunk_ccq_gdn


def test_signatures_match_reference(ccq_ref):
    import inspect

    from ccq_b200 import integration, ops
    from ccq.ops.ccq_gdn.fused_clean import fused_ccq_clean as ref_clean
    from ccq.ops.ccq_gla.fused_recurrent import fused_recurrent_ccq_gla as ref_gla
    from ccq.ops.common.fused_read import fused_ccq_clean_read as ref_read
    from ccq.ops.ccq_gdn.chunk import chunk_ccq_gdn as ref_chunk_gdn
    from ccq.ops.ccq_gdn.fused_chunk import fused_chunk_ccq_gdn as ref_fc_gdn
    from ccq.ops.ccq_gla.chunk import chunk_ccq_gla as ref_chunk_gla
    from ccq.ops.ccq_gla.fused_chunk import fused_chunk_ccq_gla as ref_fc_gla
    for ours, ref in ((ops.fused_ccq_clean_read, ref_read), (ops.fused_ccq_clean, ref_clean),
                      (integration.fused_recurrent_ccq_gla, ref_gla), (integration.fused_chunk_ccq_gdn, ref_fc_gdn),
                      (integration.fused_chunk_ccq_gla, ref_fc_gla), (integration.chunk_ccq_gdn, ref_chunk_gdn),
                      (integration.chunk_ccq_gla, ref_chunk_gla)):
        a = inspect.signature(ours).parameters
        b = inspect.signature(ref).parameters
        assert list(a) == list(b), (ours.__name__, list(a), list(b))
        for name in b:
            assert a[name].kind == b[name].kind, name
            assert a[name].default == b[name].default, name
