"""Build the sm_100a library: every .cu/.cpp under csrc/ into one shared object.

  python colabfold-legacy-kernels_b200/build.py [--jobs N] [--verbose]

Output: src/colabfold_legacy_kernels/kernels/sm100/libcflk_sm100.so (in-tree, git-ignored).
nvcc links cudart statically; libstdc++ and libgcc are linked statically too, so the library
needs only libc and the CUDA driver at run time, as the reference's own libraries do.
"""
import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, 'csrc')
OUT_DIR = os.path.join(HERE, 'src', 'colabfold_legacy_kernels', 'kernels', 'sm100')
LIB = os.path.join(OUT_DIR, 'libcflk_sm100.so')
BUILD = os.path.join(HERE, '_build')

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ARCH + ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC',
                     '-Xcompiler', '-fvisibility=hidden', '-Xptxas', '-warn-spills',
                     '--expt-relaxed-constexpr', '-I', CSRC, '-I', os.path.join(HERE, '..', 'include')]


def nvcc():
    path = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    if not os.path.exists(path):
        raise RuntimeError('nvcc not found')
    return path


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(('.cu', '.cpp')))


def compile_one(src, verbose):
    obj = os.path.join(BUILD, src + '.o')
    cmd = [nvcc()] + NVCC_FLAGS + ['-c', os.path.join(CSRC, src), '-o', obj]
    if verbose:
        cmd += ['-Xptxas', '-v']
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError('nvcc failed on %s:\n%s%s' % (src, r.stdout, r.stderr))
    return obj, r.stderr


def build(jobs=None, verbose=False):
    """Compile and link; returns the library path. Raises on any compiler error."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
        results = list(ex.map(lambda s: compile_one(s, verbose), srcs))
    for _, log in results:
        if verbose or 'spill' in log:
            sys.stderr.write(log)
    objs = [o for o, _ in results]
    tmp = LIB + '.tmp'
    cmd = [nvcc()] + ARCH + ['-shared', '-o', tmp] + objs + [
        '-Xcompiler', '-static-libstdc++', '-Xcompiler', '-static-libgcc']
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError('link failed:\n%s%s' % (r.stdout, r.stderr))
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--jobs', type=int, default=None)
    ap.add_argument('--verbose', action='store_true')
    a = ap.parse_args()
    print(build(a.jobs, a.verbose))
