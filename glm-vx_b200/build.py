"""Build libglmvx_cuda.so in-tree for sm_100a (B200).

    python glm-vx_b200/build.py [--force] [--verbose]

Steps: regenerate the GGML codebooks from gguf-py (codebooks.py), compile
each csrc/*.cu with nvcc for `-gencode arch=compute_100a,code=sm_100a`, and
link one shared library next to this file.  Objects go to _build/.  The
library is what the Python boundary (kernels/, gpu/) loads; nothing is
installed into site-packages and no JIT cache is used.
"""
import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / 'csrc'
OBJ = HERE / '_build'
LIB = HERE / 'libglmvx_cuda.so'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++20', '-lineinfo', '-Xcompiler', '-fPIC,-fvisibility=hidden',
         '--expt-relaxed-constexpr', '-I', str(ROOT / 'include'), '-I', str(CSRC)]


def nvcc():
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError('nvcc not found; the CUDA library cannot be built')


def _stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force=False, verbose=False, extra_flags=()):
    sys.path.insert(0, str(HERE))
    import codebooks
    inc = CSRC / 'ggml_tables.inc'
    binf = HERE / 'kernels' / 'ggml_tables.bin'
    if force or not inc.exists() or not binf.exists():
        codebooks.write_outputs(binf, inc)
    OBJ.mkdir(exist_ok=True)
    headers = list(CSRC.glob('*.cuh')) + [inc, ROOT / 'include' / 'glmvx.h', Path(__file__)]
    sources = sorted(CSRC.glob('*.cu'))
    cc = nvcc()
    flags = FLAGS + list(extra_flags)

    def compile_one(src):
        obj = OBJ / (src.stem + '.o')
        if force or _stale(obj, [src] + headers):
            cmd = [cc, *ARCH, *flags, '-c', str(src), '-o', str(obj)]
            if verbose:
                print(' '.join(cmd), flush=True)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode:
                raise RuntimeError(f'nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}')
            if verbose and (res.stdout or res.stderr):
                print(res.stdout + res.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(compile_one, sources))
    if force or _stale(LIB, objs):
        cmd = [cc, *ARCH, '-shared', '-o', str(LIB), *map(str, objs), '-lcudart_static', '-ldl', '-lpthread', '-lrt']
        if verbose:
            print(' '.join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode:
            raise RuntimeError(f'link failed:\n{res.stdout}\n{res.stderr}')
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--ptxas-info', action='store_true', help='print registers/spills per kernel (-Xptxas -v)')
    a = ap.parse_args()
    print(build(a.force or a.ptxas_info, a.verbose or a.ptxas_info, ['-Xptxas', '-v'] if a.ptxas_info else []))
