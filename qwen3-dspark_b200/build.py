"""Build the in-tree CUDA library ``lib/libdspark_b200.so`` for sm_100a with nvcc.

Run ``python qwen3-dspark_b200/build.py`` (or ``__graft_entry__.build()``). The
library is plain C ABI (no torch types), so a cgo/JNI/ctypes caller can link it.
"""
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_DIR = os.path.join(PKG, 'lib')
LIB_PATH = os.path.join(LIB_DIR, 'libdspark_b200.so')
SOURCES = [os.path.join(PKG, 'csrc', 'dspark_b200.cu')]
# every header under csrc/ (a new .cuh is picked up without editing this list) and the C-ABI header
DEPENDS = sorted(os.path.join(PKG, 'csrc', f) for f in os.listdir(os.path.join(PKG, 'csrc')) if f.endswith('.cuh')) + \
    [os.path.join(ROOT, 'include', 'dspark_b200.h')]
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def nvcc():
    path = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    if not os.path.exists(path):
        raise RuntimeError('nvcc not found; the CUDA library cannot be built')
    return path


def up_to_date():
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in SOURCES + DEPENDS)


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + '.tmp'
    cmd = [nvcc(), *ARCH, '-lineinfo', '-O3', '-std=c++17', '-Xcompiler', '-fPIC', '-shared',
           '-I', os.path.join(ROOT, 'include'), *SOURCES, '-o', tmp]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'nvcc failed ({res.returncode}):\n{res.stderr}')
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='-v' in sys.argv))
