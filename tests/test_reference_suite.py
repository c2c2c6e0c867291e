"""The reference's own tests, unmodified, against the libraries here.

CPU: the reference's packed-path tests (tests/test_packed_matvec.py,
test_packed_batch.py, test_packed_model.py, test_backend_oracle.py) and its
kernel tests (kernels/test_backend.py, kernels/test_kernels.py) run with
GLM_VX_LIBRARY pointing at the CPU oracle -- the check that the oracle IS
the reference's numerics.  The reference's tests/ directory is only present
where the reference checkout is (this test skips elsewhere); the tests that
need a native GGML build or the trained GGUF skip inside the reference's own
suite.

GPU: the reference's kernel tests that ship with its installed package
(baseline/_ref/kernels/test_backend.py and test_kernels.py) run with
GLM_VX_LIBRARY pointing at libglmvx_cuda.so, i.e. the reference's own
VxBackend and C-ABI checks drive the B200 library.  One test of that file
imports the reference's tests/ package, absent on a GPU box; it runs only
where the checkout is."""
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF_PKG = ROOT / 'baseline' / '_ref'
REF_CHECKOUT = Path(os.environ.get('GLM_VX_REFERENCE_CHECKOUT', '/nonexistent'))
PACKED_TESTS = ('tests/test_packed_matvec.py', 'tests/test_packed_batch.py', 'tests/test_packed_model.py',
                'tests/test_backend_oracle.py')


def _run(cmd, library, extra_path=()):
    env = dict(os.environ, GLM_VX_LIBRARY=str(library),
               PYTHONPATH=os.pathsep.join([str(REF_PKG), *map(str, extra_path)]))
    return subprocess.run(cmd, cwd='/tmp', env=env, capture_output=True, text=True, timeout=900)


def _passed(out):
    m = re.search(r'(\d+) passed', out)
    return int(m.group(1)) if m else 0


@pytest.mark.skipif(not (REF_CHECKOUT / 'tests').is_dir() or not (REF_PKG / 'glm_vx').is_dir(),
                    reason='set GLM_VX_REFERENCE_CHECKOUT to a reference checkout (and install baseline/_ref)')
def test_reference_packed_suite_on_oracle():
    from oracle import loader
    lib = loader.serial()
    tests = [str(REF_CHECKOUT / t) for t in PACKED_TESTS] + [str(REF_PKG / 'kernels' / 'test_backend.py')]
    res = _run([sys.executable, '-m', 'pytest', '-q', '-p', 'no:cacheprovider', *tests], lib,
               extra_path=(REF_CHECKOUT, REF_CHECKOUT / 'tests'))
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-2000:]
    assert _passed(res.stdout) >= 61, res.stdout[-500:]
    res = _run([sys.executable, str(REF_PKG / 'kernels' / 'test_kernels.py'), str(lib)], lib)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]


@pytest.mark.gpu
@pytest.mark.skipif(not (REF_PKG / 'kernels' / 'test_backend.py').exists(), reason='reference not installed')
def test_reference_kernel_tests_on_b200_library(cuda_lib):
    from gpu.runtime import library_path
    lib = library_path()
    res = _run([sys.executable, '-m', 'pytest', '-q', '-p', 'no:cacheprovider',
                str(REF_PKG / 'kernels' / 'test_backend.py'), '-k', 'not independent_oracle'], lib)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-2000:]
    assert _passed(res.stdout) >= 5, res.stdout[-500:]
    res = _run([sys.executable, str(REF_PKG / 'kernels' / 'test_kernels.py'), str(lib)], lib)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert '"max_absolute_error"' in res.stdout
