"""Host boundary checks that need no GPU: argument validation wording (the
reference's tests/test_packed_matvec.py:132-143 and tests/test_packed_batch.py
:294-323 cases), codebook pinning, and the C-ABI library's exported symbols."""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import PACKAGE, ROOT
from kernels import packed
from kernels.packed import LAYOUTS, _buffers, batch_input


@pytest.mark.parametrize('change,error', [
    ({'raw': np.zeros(49, np.uint8)}, 'byte count'),
    ({'raw': np.zeros(50, np.float32)}, 'uint8'),
    ({'raw': np.zeros(100, np.uint8)[::2]}, 'contiguous'),
    ({'shape': (1, 255)}, 'block-aligned'), ({'shape': (-1, 256)}, 'nonnegative'),
    ({'shape': (2**31, 256)}, 'int32'), ({'shape': (1, 0)}, 'positive'),
    ({'shape': (True, 256)}, 'integer'), ({'kind': 999}, 'unsupported'),
    ({'x': np.ones(255, np.float32)}, 'columns'),
    ({'x': np.full(256, np.nan, np.float32)}, 'finite')])
def test_matvec_bounds_before_kernel(oracle, change, error):
    args = dict(raw=np.zeros(50, np.uint8), kind=19, shape=(1, 256), x=np.ones(256, np.float32))
    args.update(change)
    with pytest.raises(ValueError, match=error):
        oracle.packed_matvec(**args)


@pytest.mark.parametrize('change,message', [
    ({'x': np.zeros((65, 256), np.float32)}, '64'),
    ({'x': np.zeros(256, np.float32)}, 'columns'),
    ({'x': np.zeros((2, 255), np.float32)}, 'columns'),
    ({'x': np.full((2, 256), np.nan, np.float32)}, 'finite'),
    ({'raw': np.zeros(49, np.uint8)}, 'byte count'),
    ({'raw': np.zeros(100, np.uint8)[::2]}, 'contiguous'),
    ({'kind': 999}, 'unsupported'),
    ({'shape': (2**31, 256)}, 'int32')])
def test_batch_bounds(oracle, change, message):
    args = dict(raw=np.zeros(50, np.uint8), kind=19, shape=(1, 256), x=np.ones((2, 256), np.float32))
    args.update(change)
    with pytest.raises(ValueError, match=message):
        oracle.packed_linear_batch(**args)


def test_capacity_counts_f32_elements():
    with pytest.raises(ValueError, match='byte count'):
        _buffers(np.empty(0, np.uint8), 0, (154880, 6144))
    with pytest.raises(ValueError, match='int32'):
        _buffers(np.empty(0, np.uint8), 0, (2**30, 2))
    with pytest.raises(ValueError, match='int32'):
        _buffers(np.empty(0, np.uint8), 1, (2**30, 1))


def test_empty_rows_and_batch(oracle):
    assert oracle.packed_linear_batch(np.zeros(0, np.uint8), 19, (0, 256), np.zeros((7, 256), np.float32)).shape == (7, 0)
    assert oracle.packed_linear_batch(np.zeros(50, np.uint8), 19, (1, 256), np.zeros((0, 256), np.float32)).shape == (0, 1)


def test_corrupt_scale_fails_closed(oracle):
    raw = np.zeros(50, np.uint8)
    raw[:2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    with pytest.raises(ValueError, match='nonfinite'):
        oracle.packed_matvec(raw, 19, (1, 256), np.ones(256, np.float32))


def test_supports_checks_symbols():
    class OldLibrary:
        pass
    assert packed.supports(OldLibrary(), 0)
    assert not packed.supports(OldLibrary(), 19)
    assert not packed.supports(OldLibrary(), 999)


def test_codebooks_rebuild_from_gguf_py_matches_pin():
    import codebooks
    assert packed.lookup_tables()[1].tobytes() == codebooks.build_blob()


def test_missing_library_is_an_error():
    from kernels.backend import VxBackend
    with pytest.raises(RuntimeError):
        VxBackend('/nonexistent/libglmvx_cuda.so')


def _header_functions():
    text = (ROOT / 'include' / 'glmvx.h').read_text()
    names = set(re.findall(r'^\s*(?:const\s+)?(?:int32_t|int64_t|char)\s*\*?\s*(glmvx_\w+|glm_vx_\w+)\(', text, re.M))
    body = re.search(r'#define GLMVX_REFERENCE_PACKED_DECL\(kind\)(.*?)\n\n', text, re.S).group(1)
    stems = re.findall(r'(glm_vx_\w+?)##kind', body)
    kinds = re.findall(r'^GLMVX_REFERENCE_PACKED_DECL\((\w+)\)', text, re.M)
    names |= {s + k for s in stems for k in kinds}
    return names


def test_library_exports_every_header_symbol():
    """The C-ABI library loads (no GPU needed) and exports all of include/glmvx.h."""
    lib = PACKAGE / 'libglmvx_cuda.so'
    assert lib.exists(), 'run python glm-vx_b200/build.py'
    import ctypes
    ctypes.CDLL(str(lib))
    out = subprocess.run(['nm', '-D', '--defined-only', str(lib)], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if ' T ' in line}
    declared = _header_functions()
    assert len(declared) > 90
    assert declared <= exported, sorted(declared - exported)


def test_reference_abi_symbol_set_matches_reference_header():
    """Every glm_vx_* the reference's kernels.h declares is declared here too
    (the list is restated from kernels/kernels.h:168-207)."""
    reference = {'glm_vx_' + n for n in (
        'rmsnorm layernorm softmax swiglu add axpy matvec matmul_nt rope router topk attention '
        'sparse_attention rope_offset index_scores rope_glm').split()}
    for suffix in ('f16', 'q8_0', 'q2_k', 'q3_k', 'q4_k', 'q5_k', 'q6_k', 'iq1_s', 'iq2_xxs', 'iq3_xxs', 'iq4_xs'):
        reference |= {f'glm_vx_packed_{suffix}', f'glm_vx_packed_batch_v2_{suffix}', f'glm_vx_unpack_{suffix}'}
    assert reference <= _header_functions()
