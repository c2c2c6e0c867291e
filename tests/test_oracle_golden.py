"""Pin the CPU oracle against golden vectors made from the reference's own
fixtures and gguf-py 0.19 (tests/golden/make_golden.py).  CPU only."""
import ctypes as C
import struct

import numpy as np
import pytest

from helpers import sha
from kernels.packed import LAYOUTS, unpack_for_validation, matmul

NAMES = {kind: name for kind, (_, _, name) in LAYOUTS.items()}


@pytest.mark.parametrize('kind', list(LAYOUTS))
def test_decode_bit_exact(oracle, golden, kind):
    name = NAMES[kind]
    raw, dec = golden[f'raw_{name}'], golden[f'dec_{name}']
    got = unpack_for_validation(oracle.lib, raw, kind, dec.shape)
    assert got.tobytes() == dec.tobytes()


@pytest.mark.parametrize('kind', list(LAYOUTS))
def test_ordered_dot_bit_exact(oracle, golden, kind):
    name = NAMES[kind]
    raw, dec = golden[f'raw_{name}'], golden[f'dec_{name}']
    for i in range(2):
        got = oracle.packed_matvec(raw, kind, dec.shape, golden[f'x{i}_{name}'])
        assert got.tobytes() == golden[f'dot{i}_{name}'].tobytes()


@pytest.mark.parametrize('kind', list(LAYOUTS))
@pytest.mark.parametrize('batch', [2, 3, 5, 8, 17, 64])
def test_batch_tiles_bit_exact(oracle, golden, kind, batch):
    """batch_v2 token tiles (64/32/.../1) keep each lane's ordered sum."""
    name = NAMES[kind]
    block = LAYOUTS[kind][0]
    x = np.random.default_rng(4400 + kind + batch).normal(size=(batch, 4 * block)).astype(np.float32)
    x[:, ::2] *= np.float32(2**12)
    assert sha(x) == golden[f'bsha_{name}_{batch}'].tobytes(), 'activation RNG drifted from the fixture'
    got = matmul(oracle.lib, golden[f'raw_{name}'], kind, (3, 4 * block), x)
    assert got.tobytes() == golden[f'bout_{name}_{batch}'].tobytes()


def test_iq1_every_grid_index(oracle, golden):
    got = unpack_for_validation(oracle.lib, golden['iq1_grid_raw'], 19, (64, 256))
    assert got.tobytes() == golden['iq1_grid_dec'].tobytes()


def test_half_table_every_finite_pattern(oracle):
    bits = np.arange(65536, dtype=np.uint16)
    bits = bits[(bits & 0x7c00) != 0x7c00]
    got = unpack_for_validation(oracle.lib, bits.view(np.uint8), 1, (1, len(bits))).ravel()
    assert got.tobytes() == bits.view(np.float16).astype(np.float32).tobytes()


def test_router_known_answers(oracle, ops_golden):
    ids, w = oracle.route(ops_golden['kat_logits'], ops_golden['kat_bias'], 2, 2.5)
    assert ids.tolist() == [0, 1] == ops_golden['kat_ids'].tolist()
    assert w[0] < w[1]  # the bias picks expert 0 but never raises its weight
    np.testing.assert_allclose(w, ops_golden['kat_w'], rtol=1e-6)
    ids, w = oracle.route(ops_golden['r256_logits'], ops_golden['r256_bias'], 8, 2.5)
    assert ids.tolist() == ops_golden['r256_ids'].tolist()
    np.testing.assert_allclose(w, ops_golden['r256_w'], rtol=1e-6)


def test_topk_stable_ties(oracle):
    assert oracle.topk(np.array([3, 1, 3, -2], np.float32), 3).tolist() == [0, 2, 1]
    assert oracle.topk(np.array([0.0, -0.0, 1.0], np.float32), 3).tolist() == [2, 0, 1]


def test_fp8_decode_all_encodings(ops_golden):
    from oracle import loader
    lib = loader.cdll()
    got = np.array([lib.glm_vx_fp8_decode(b) for b in range(256)], np.float32)
    want = ops_golden['fp8_decode']
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert got[ok].tobytes() == want[ok].tobytes()


def test_parallel_oracle_is_bit_identical():
    """The OpenMP build used for the all-core CPU baseline changes no bits."""
    from oracle import loader
    from kernels.backend import VxBackend
    from helpers import payload
    serial, par = VxBackend(str(loader.serial())), VxBackend(str(loader.parallel()))
    for kind in (8, 12, 19):
        block = LAYOUTS[kind][0]
        raw = payload(kind, blocks=64 * 2048 // block, seed=7)
        x = np.random.default_rng(1).normal(size=2048).astype(np.float32)
        a = serial.packed_matvec(raw, kind, (64, 2048), x)
        b = par.packed_matvec(raw, kind, (64, 2048), x)
        assert a.tobytes() == b.tobytes()
