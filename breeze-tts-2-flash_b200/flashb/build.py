"""Ahead-of-time build of ``libflashb.so`` (the sm_100a kernels + C ABI) with nvcc, in-tree.

The reference JIT-compiles pybind11 torch extensions per process (``flash/kernels.py:64-79``); here the kernels are
one plain shared library with an ``extern "C"`` interface (``include/flashb.h``), built once for sm_100a and loaded
with ctypes.  Objects go to ``flashb/_build/``, the library to ``flashb/_lib/libflashb.so``; both are rebuilt only
when a source, header or flag changes.

    python -m flashb.build [--force] [--verbose]
"""
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)                      # breeze-tts-2-flash_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, 'csrc')
INCLUDE = os.path.join(REPO, 'include')
BUILD = os.path.join(PKG, '_build')
LIBDIR = os.path.join(PKG, '_lib')
LIB = os.path.join(LIBDIR, 'libflashb.so')

SOURCES = ['fb_api.cu', 'fb_gemv.cu', 'fb_attn.cu', 'fb_aux.cu', 'fb_sample.cu', 'fb_depth.cu', 'fb_prefill.cu',
           'fb_gemv_narrow.cu', 'fb_gemv_tc.cu', 'fb_gemv_rows.cu', 'fb_attn_mma.cu']
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr', '-I', CSRC, '-I', INCLUDE]


def nvcc():
    for c in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if c and os.path.exists(c):
            return c
    raise RuntimeError('nvcc not found: set NVCC or put the CUDA toolkit on PATH')


def _headers():
    hs = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith(('.cuh', '.h'))]
    return hs + [os.path.join(INCLUDE, f) for f in sorted(os.listdir(INCLUDE)) if f.endswith('.h')]


def _stamp(src, extra=()):
    h = hashlib.sha256()
    for f in [src, *_headers(), *extra]:
        with open(f, 'rb') as fh:
            h.update(fh.read())
    h.update(' '.join(ARCH + FLAGS).encode())
    return h.hexdigest()


def _compile(src, verbose):
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, src.replace('.cu', '.o'))
    stamp_file = obj + '.stamp'
    stamp = _stamp(path)
    if os.path.exists(obj) and os.path.exists(stamp_file) and open(stamp_file).read() == stamp:
        return obj, False
    cmd = [nvcc(), *ARCH, *FLAGS, '-c', path, '-o', obj]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
        print(' '.join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f'nvcc failed on {src}:\n{r.stdout}\n{r.stderr}')
    if verbose and r.stderr:
        print(r.stderr, flush=True)
    with open(stamp_file, 'w') as f:
        f.write(stamp)
    return obj, True


def build(force=False, verbose=False):
    """Compile every source for sm_100a and link libflashb.so; returns the library path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    if force:
        for f in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, f))
    with ThreadPoolExecutor(max_workers=max(1, min(len(SOURCES), os.cpu_count() or 1))) as ex:
        res = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    objs = [o for o, _ in res]
    if any(ch for _, ch in res) or not os.path.exists(LIB) or force:
        tmp = LIB + '.tmp'
        cmd = [nvcc(), *ARCH, '-shared', '-o', tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f'link failed:\n{r.stdout}\n{r.stderr}')
        os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='--verbose' in sys.argv))
