"""Locate (and, if needed, build) the oracle libraries -- TEST INFRASTRUCTURE ONLY.

serial():   oracle/_build/libglm_vx_ref.so      -- the reference's single-thread numerics
parallel(): oracle/_build/libglm_vx_ref_omp.so  -- same loops, rows over OpenMP threads
Both export the reference's C ABI (kernels/kernels.h of gakonst/glm-vx) plus
glm_vx_fp8_decode / glm_vx_fp8_matvec_reference (gpu/fp8.vx:3-38).
"""
import ctypes as C
import subprocess
from functools import lru_cache
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / '_build'


def build():
    res = subprocess.run(['make', '-s', '-C', str(HERE)], capture_output=True, text=True)
    if res.returncode:
        raise RuntimeError('oracle build failed:\n' + res.stdout + res.stderr)


def _path(name):
    path = BUILD / name
    sources = list(HERE.glob('*.c')) + [HERE / 'Makefile']
    if not path.exists() or any(s.stat().st_mtime > path.stat().st_mtime for s in sources):
        build()
    return path


def serial():
    return _path('libglm_vx_ref.so')


def parallel():
    return _path('libglm_vx_ref_omp.so')


@lru_cache(maxsize=None)
def cdll(which='serial'):
    lib = C.CDLL(str(serial() if which == 'serial' else parallel()))
    lib.glm_vx_fp8_decode.argtypes, lib.glm_vx_fp8_decode.restype = [C.c_uint8], C.c_float
    return lib
