"""Build the in-tree C-ABI library ``ccq_b200/lib/libccq_b200.so`` for sm_100a with nvcc.

    python -m ccq_b200.build        # or: from ccq_b200.build import build; build()

The library has no torch dependency: plain nvcc, static CUDA runtime, -fPIC -shared.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, 'csrc')
LIBDIR = os.path.join(PKG, 'lib')
LIB = os.path.join(LIBDIR, 'libccq_b200.so')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def nvcc_path():
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError('nvcc not found')


def sources():
    return sorted(glob.glob(os.path.join(CSRC, '*.cu')))


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, '*.h')) + glob.glob(os.path.join(CSRC, '*.cuh'))
    deps.append(os.path.join(os.path.dirname(PKG), 'include', 'ccq_b200.h'))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, extra=()):
    if not force and not needs_build():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = os.path.join(LIBDIR, '_obj')
    os.makedirs(objdir, exist_ok=True)
    nvcc = nvcc_path()
    common = ARCH + ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC,-O2', '--expt-relaxed-constexpr',
                     '-I', os.path.join(os.path.dirname(PKG), 'include')] + list(extra)
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + '.o')
        cmd = [nvcc] + common + ['-c', src, '-o', obj]
        if verbose:
            print(' '.join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode != 0:
            sys.stdout.write(out.decode(errors='replace'))
        if p.returncode != 0:
            failed.append(src)
    if failed:
        raise RuntimeError('nvcc failed for: ' + ', '.join(os.path.basename(f) for f in failed))
    tmp = LIB + '.tmp'
    cmd = [nvcc] + ARCH + ['-shared', '-o', tmp] + objs + ['-cudart', 'static']
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    build(force='--force' in sys.argv, verbose='-v' in sys.argv)
    print(LIB)
