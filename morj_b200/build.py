"""Build the native library `morj_b200/_morj_b200.so` from `morj_b200/csrc/*.cu` (device code for sm_100a, nvcc)
and `morj_b200/csrc/*.cpp` (host code, g++), in-tree.

    python -m morj_b200.build [--force] [--verbose]

The library is a plain C-ABI shared object (no torch types); it links the CUDA runtime statically and resolves
driver entry points (cuTensorMapEncodeTiled) at run time, so it loads on any machine with the NVIDIA driver and
cross-compiles on a machine without a GPU. Device code is relocatable (-rdc) so that all kernels share the one
device error word.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, 'csrc')
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, '_morj_b200.so')
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
CXX = os.environ.get('CXX', 'g++')
CXXFLAGS = ['-O3', '-std=c++17', '-fPIC', '-Wall', '-I', os.path.join(ROOT, 'include')]
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-rdc=true', '-Xcompiler', '-fPIC,-O3', '--expt-relaxed-constexpr',
         '-I', os.path.join(ROOT, 'include')]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, '*.cu')) + glob.glob(os.path.join(CSRC, '*.cpp')))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, '*.cuh')) + glob.glob(os.path.join(ROOT, 'include', '*.h')))


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(f) > t for f in sources() + headers() + [__file__])


def build(force=False, verbose=False):
    """Compile every source to an object (in parallel) and link the shared library; returns its path."""
    if not force and not stale():
        return LIB
    objdir = os.path.join(HERE, '_build')
    os.makedirs(objdir, exist_ok=True)
    procs, objs = [], []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + '.o')
        objs.append(obj)
        if src.endswith('.cpp'):
            cmd = [CXX, *CXXFLAGS, '-c', src, '-o', obj]
        else:
            cmd = [NVCC, *ARCH, *FLAGS, '-c', src, '-o', obj]
            if verbose:
                cmd += ['-Xptxas', '-v']
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stderr.write(out)
        if p.returncode:
            failed.append(src)
    if failed:
        raise RuntimeError('nvcc failed for ' + ', '.join(os.path.basename(f) for f in failed))
    tmp = LIB + '.tmp'
    cmd = [NVCC, *ARCH, '-shared', '-o', tmp, *objs, '-Xcompiler', '-fPIC']
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout)
        raise RuntimeError('nvcc link failed')
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='--verbose' in sys.argv))
