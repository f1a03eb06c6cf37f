"""The tensor-core kernels' bounded pipeline waits: a wait that runs out is reported, and the library
and the CUDA context stay usable.

CCQ_B200_DEBUG_STALL_CYCLES makes the forward kernel's first wait, on an mbarrier that nothing ever
arrives on, give up after that many clock cycles before any copy or MMA is issued.  No fault and no
hang is involved: the kernel sets its abort flag, records code 0x100 in the workspace's error word,
every warp role unwinds through its named barriers, and the CTA frees its TMEM and exits.  The test
checks that the C ABI reports it (CCQ_ERR_CUDA under CCQ_B200_CHECK=1, the code through
ccq_device_status otherwise) and that the next normal call succeeds with the usual result.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope='module')
def setup():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from ccq_b200 import _lib
    lib = _lib.load()
    dev = torch.device('cuda', 0)
    g = torch.Generator(device=dev).manual_seed(17)
    B, T, H, K = 2, 300, 2, 128
    q = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g, device=dev), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g, device=dev), dim=-1).bfloat16()
    W = torch.randn(H, K, generator=g, device=dev) * 0.02
    b = torch.zeros(H, device=dev)
    nbytes = lib.ccq_workspace_size_for(_lib.CCQ_OP_FWD, _lib.CCQ_BF16, B, T, H, K, B, 0)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    return dict(lib=lib, L=_lib, q=q, k=k, W=W, b=b, ws=ws, nbytes=nbytes, shape=(B, T, H, K))


def _fwd(s):
    B, T, H, K = s['shape']
    L, q = s['L'], s['q']
    qc = torch.empty_like(q)
    fc = torch.empty(B, H, K, K, device=q.device)
    fm = torch.empty(B, H, K, device=q.device)
    aux = torch.empty(B, T, H, 2, device=q.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = s['lib'].ccq_clean_fwd(L.CCQ_BF16, B, T, H, K, _p(q), _p(s['k']), L.CCQ_LAMBDA_GATE, None, _p(s['W']),
                                _p(s['b']), _p(aux), None, B, 0, 1, None, None, _p(qc), _p(fc), _p(fm), _p(s['ws']),
                                s['nbytes'], stream)
    return st, qc, fc


def _status(s):
    code = ctypes.c_int(-1)
    st = s['lib'].ccq_device_status(_p(s['ws']), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                    ctypes.byref(code))
    assert st == 0
    return code.value


def test_forced_wait_timeout_is_reported_and_the_next_call_succeeds(setup, monkeypatch):
    s = setup
    monkeypatch.delenv('CCQ_B200_DEBUG_STALL_CYCLES', raising=False)
    monkeypatch.setenv('CCQ_B200_CHECK', '1')
    st, ref_qc, ref_fc = _fwd(s)
    assert st == 0, s['lib'].ccq_last_error().decode()
    assert s['L'].last_path() == 'tcgen05'
    assert _status(s) == 0

    # checked mode: the call waits for its kernel and returns the timeout
    monkeypatch.setenv('CCQ_B200_DEBUG_STALL_CYCLES', str(1 << 22))
    st, _, _ = _fwd(s)
    msg = s['lib'].ccq_last_error().decode()
    assert st == s['L'].CCQ_ERR_CUDA, (st, msg)
    assert 'timeout' in msg and '0x100' in msg, msg

    # unchecked: the call returns at once; the error word tells the caller afterwards
    monkeypatch.setenv('CCQ_B200_CHECK', '0')
    st, _, _ = _fwd(s)
    assert st == 0
    assert _status(s) == 0x100
    torch.cuda.synchronize()  # the context is intact

    # knob off: the next call is normal and gives the same result as before
    monkeypatch.delenv('CCQ_B200_DEBUG_STALL_CYCLES')
    monkeypatch.setenv('CCQ_B200_CHECK', '1')
    st, qc, fc = _fwd(s)
    assert st == 0, s['lib'].ccq_last_error().decode()
    assert _status(s) == 0
    assert torch.equal(qc, ref_qc)
    assert torch.equal(fc, ref_fc)
