"""The C-ABI library loads on a CPU-only host, exports every symbol include/ccq_b200.h declares,
and rejects bad arguments with a status and a message before touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, 'include', 'ccq_b200.h')


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r'/\*.*?\*/', '', src, flags=re.S)
    return sorted(set(re.findall(r'\b(ccq_[a-z_0-9]+)\s*\(', src)))


@pytest.fixture(scope='module')
def lib():
    from ccq_b200 import _lib
    from ccq_b200.build import build
    build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ('ccq_clean_fwd', 'ccq_clean_bwd', 'ccq_decode_step', 'ccq_workspace_size', 'ccq_last_error'):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    from ccq_b200 import _lib
    out = subprocess.run(['nm', '-D', '--defined-only', _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r'\bT (ccq_[a-z_0-9]+)$', out, flags=re.M))
    for name in declared_functions():
        assert name in exported, f'{name} declared but not exported'
        assert hasattr(lib, name)
    assert set(_lib.EXPORTS) == set(declared_functions())


def test_version_and_workspace(lib):
    assert lib.ccq_version() >= 100
    assert lib.ccq_workspace_size(1, 1, 8, 4096, 16, 128, 8) > 0
    assert lib.ccq_workspace_size(1, 1, 0, 4096, 16, 128, 8) == 0
    assert lib.ccq_workspace_size(0, 0, 2, 64, 2, 300, 2) == 0


def _fwd(lib, dtype=1, B=2, T=8, H=2, K=64, q=1, k=1, mode=0, lam=1, w=None, b=None, cu=None, n=2):
    P = lambda x: None if x is None else ctypes.c_void_p(x)  # noqa: E731
    return lib.ccq_clean_fwd(dtype, B, T, H, K, P(q), P(k), mode, P(lam), P(w), P(b), None, P(cu), n, 0, 1,
                             None, None, P(16), None, None, None, 0, None)


@pytest.mark.parametrize('kw,status,msg', [
    (dict(dtype=9), 1, 'dtype'),
    (dict(K=300), 2, 'K=300'),
    (dict(B=0), 1, 'bad sizes'),
    (dict(q=None), 1, 'q and k'),
    (dict(lam=None), 1, 'lambda'),
    (dict(mode=1), 1, 'gate_w'),
    (dict(mode=5), 1, 'lambda_mode'),
    (dict(n=3), 1, 'n_seqs'),
    (dict(cu=64, B=2), 1, 'B == 1'),
])
def test_validation_errors_without_gpu(lib, kw, status, msg):
    st = _fwd(lib, **kw)
    assert st == status
    assert msg in lib.ccq_last_error().decode()


def test_decode_validation(lib):
    P = ctypes.c_void_p
    st = lib.ccq_decode_step(1, 2, 1, 2, 66, P(16), P(16), 0, P(16), None, None, None, 2, 0, 1, None, None,
                             P(16), None, P(16), None)
    assert st == 2 and 'K % 4' in lib.ccq_last_error().decode()
    st = lib.ccq_decode_step(1, 2, 1, 2, 64, P(16), P(16), 0, P(16), None, None, None, 2, 0, 1, None, None,
                             None, None, P(16), None)
    assert st == 1 and 'cov_out' in lib.ccq_last_error().decode()


def test_python_ops_reject_cpu_tensors():
    import torch

    import ccq_b200
    q = torch.randn(1, 4, 1, 16)
    with pytest.raises(RuntimeError, match='CUDA'):
        ccq_b200.fused_ccq_clean_read(q, q, 0.5)
    with pytest.raises(RuntimeError, match='CUDA'):
        ccq_b200.decode_step(q, q, 0.5)
