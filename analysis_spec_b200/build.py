"""Builds libspeckv.so (all CUDA sources under csrc/) for sm_100a with nvcc.

The library is built in-tree next to this file so that it ships with the
package. A rebuild happens only when a source, header or flag changed (a hash
of them is kept beside the library).
"""
import hashlib
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
INCLUDE = HERE.parent / 'include'
LIB = HERE / 'libspeckv.so'
OBJDIR = HERE / '_build'

NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '-Xcompiler', '-O2',
         '--expt-relaxed-constexpr', '-I', str(INCLUDE)]


def _sources():
    return sorted(CSRC.glob('*.cu'))


def _digest():
    h = hashlib.sha256()
    h.update(' '.join(ARCH + FLAGS).encode())
    for path in sorted(list(CSRC.glob('*')) + list(INCLUDE.glob('*.h'))):
        if path.is_file():
            h.update(path.name.encode())
            h.update(path.read_bytes())
    return h.hexdigest()


def build(force=False, verbose=False):
    """Compile and link libspeckv.so; returns its path."""
    stamp = LIB.with_suffix('.so.hash')
    digest = _digest()
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == digest:
        return LIB
    OBJDIR.mkdir(exist_ok=True)

    def compile_one(src):
        obj = OBJDIR / (src.stem + '.o')
        cmd = [NVCC, *ARCH, *FLAGS, '-c', str(src), '-o', str(obj)]
        if verbose:
            print(' '.join(cmd), file=sys.stderr)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f'nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}')
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(compile_one, _sources()))
    tmp = LIB.with_suffix('.so.tmp')
    cmd = [NVCC, *ARCH, '-shared', '-o', str(tmp), *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f'nvcc link failed:\n{proc.stdout}\n{proc.stderr}')
    os.replace(tmp, LIB)
    stamp.write_text(digest)
    return LIB


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='-v' in sys.argv))
