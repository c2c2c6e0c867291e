"""Absorbed-MLA decode attention (csrc/mla.cu, glmvx_mla_decode) and the
drop-in GPUBackend.compressed_attention against a float64 NumPy restatement
of the reference's contract (gpu/backend.py:233-254, kernels
gpu/kernels.vx:204-310, model glm_vx/model.py:209-221): the reference's own
split-boundary case, the config-3 shape, selected-id lists shared and per
head with masked ids, an empty selection, and argument validation."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def mla_ref(q, qr, latent, rope, scale, ids=None):
    """float64 softmax attention of every head over the rows `ids` (valid only)."""
    q, qr, latent, rope = (np.asarray(a, np.float64) for a in (q, qr, latent, rope))
    out = np.zeros(q.shape)
    for h in range(q.shape[0]):
        sel = np.arange(latent.shape[0]) if ids is None else np.asarray(ids[h])
        sel = sel[(sel >= 0) & (sel < latent.shape[0])]
        if sel.size == 0:
            continue
        s = (latent[sel] @ q[h] + rope[sel] @ qr[h]) * scale
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ latent[sel]
    return out


def test_reference_split_boundary_case(gpu_backend):
    """gpu/test_backend.py:193-207 of the reference, same seed and tolerance."""
    rng = np.random.default_rng(381)
    heads, rank, rdim, count = 2, 33, 8, 257
    q = rng.normal(0, .1, (heads, rank)).astype('f4')
    qr = rng.normal(0, .1, (heads, rdim)).astype('f4')
    latent = rng.normal(0, .1, (count, rank)).astype('f4')
    rotary = rng.normal(0, .1, (count, rdim)).astype('f4')
    actual = gpu_backend.compressed_attention(q, qr, latent, rotary, .125)
    assert actual.shape == (heads, rank)
    np.testing.assert_allclose(actual, mla_ref(q, qr, latent, rotary, .125), rtol=5e-5, atol=3e-6)


@pytest.mark.parametrize('heads,rank,rdim,count', [(64, 512, 64, 2048), (7, 1000, 100, 33), (3, 64, 0, 5),
                                                    (20, 256, 100, 777), (17, 510, 62, 95), (1, 1, 1, 1)])
def test_compressed_attention_shapes(gpu_backend, heads, rank, rdim, count):
    rng = np.random.default_rng(heads + rank + count)
    q = rng.normal(0, 1, (heads, rank)).astype('f4') * np.float32(0.05)
    qr = rng.normal(0, 1, (heads, rdim)).astype('f4') * np.float32(0.05)
    latent = rng.normal(0, 1, (count, rank)).astype('f4')
    rotary = rng.normal(0, 1, (count, rdim)).astype('f4')
    scale = (192 + 64) ** -0.5
    np.testing.assert_allclose(gpu_backend.compressed_attention(q, qr, latent, rotary, scale),
                               mla_ref(q, qr, latent, rotary, scale), rtol=5e-5, atol=3e-6)


def _device(cuda_lib, q, qr, latent, rope, ids, stride, count, scale):
    from gpu.runtime import DeviceBuffer, check
    heads, rank = q.shape
    rdim = qr.shape[1]
    need = int(cuda_lib.glmvx_mla_scratch_bytes(heads, rank, count))
    arrays = [q, qr, latent, rope] + ([ids] if ids is not None else [])
    bufs = [DeviceBuffer(max(a.nbytes, 16)) for a in arrays]
    out_d, scratch = DeviceBuffer(4 * heads * rank), DeviceBuffer(max(need, 16))
    try:
        for b, a in zip(bufs, arrays):
            b.upload(np.ascontiguousarray(a))
        check(cuda_lib, cuda_lib.glmvx_mla_decode(out_d.ptr, bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                                  bufs[4].ptr if ids is not None else None, heads, rank, rdim,
                                                  latent.shape[0], count, stride, scale, scratch.ptr, need, None),
              'glmvx_mla_decode')
        out = np.empty((heads, rank), np.float32)
        out_d.download(out)
        return out
    finally:
        for b in bufs + [out_d, scratch]:
            b.close()


def test_selected_ids_shared_and_per_head(cuda_lib):
    rng = np.random.default_rng(5)
    heads, rank, rdim, tokens, count = 16, 512, 64, 3000, 700
    q = (rng.normal(size=(heads, rank)) * 0.05).astype('f4')
    qr = (rng.normal(size=(heads, rdim)) * 0.05).astype('f4')
    latent = rng.normal(size=(tokens, rank)).astype('f4')
    rope = rng.normal(size=(tokens, rdim)).astype('f4')
    shared = rng.choice(tokens, count, replace=False).astype(np.int32)
    got = _device(cuda_lib, q, qr, latent, rope, shared, 0, count, 0.0625)
    np.testing.assert_allclose(got, mla_ref(q, qr, latent, rope, 0.0625, [shared] * heads), rtol=5e-5, atol=3e-6)
    masked = shared.copy()
    masked[::9] = -1            # skipped in the shared list too
    masked[1::11] = tokens
    got = _device(cuda_lib, q, qr, latent, rope, masked, 0, count, 0.0625)
    np.testing.assert_allclose(got, mla_ref(q, qr, latent, rope, 0.0625, [masked] * heads), rtol=5e-5, atol=3e-6)
    per = np.stack([rng.choice(tokens, count, replace=False) for _ in range(heads)]).astype(np.int32)
    per[3, ::5] = -1          # padding ids are skipped
    per[4, ::7] = tokens + 9  # as are ids past the cache
    per[5, :] = -1            # a head with nothing selected outputs zeros
    got = _device(cuda_lib, q, qr, latent, rope, per, count, count, 0.0625)
    want = mla_ref(q, qr, latent, rope, 0.0625, per)
    np.testing.assert_allclose(got, want, rtol=5e-5, atol=3e-6)
    assert np.all(got[5] == 0.0)


def test_empty_selection_and_validation(cuda_lib, gpu_backend):
    rng = np.random.default_rng(6)
    q, qr = rng.normal(size=(4, 64)).astype('f4'), rng.normal(size=(4, 8)).astype('f4')
    latent, rope = rng.normal(size=(10, 64)).astype('f4'), rng.normal(size=(10, 8)).astype('f4')
    assert np.all(_device(cuda_lib, q, qr, latent, rope, None, 0, 0, 0.5) == 0.0)
    for args, msg in [((q[0], qr, latent, rope, 0.5), 'matrices'), ((q, qr[:3], latent, rope, 0.5), 'shape'),
                      ((q, qr, latent[:, :5], rope, 0.5), 'shape'), ((q, qr, latent, rope, 0.0), 'positive'),
                      ((q, qr, latent, rope, np.inf), 'positive')]:
        with pytest.raises(ValueError, match=msg):
            gpu_backend.compressed_attention(*args)


@pytest.mark.parametrize('heads,rank,rdim,tokens,count', [(64, 512, 64, 9000, 6144), (17, 510, 62, 7000, 6200),
                                                          (5, 96, 0, 6500, 6500), (64, 512, 64, 8192, 8192)])
def test_tensor_core_partials(cuda_lib, heads, rank, rdim, tokens, count):
    """From 6144 selected rows a shared selection takes the tcgen05 partials
    (3xTF32 split): same contract, same tolerance; masked ids included."""
    rng = np.random.default_rng(heads + rank + count)
    q = (rng.normal(size=(heads, rank)) * 0.05).astype('f4')
    qr = (rng.normal(size=(heads, rdim)) * 0.05).astype('f4')
    latent = rng.normal(size=(tokens, rank)).astype('f4')
    rope = rng.normal(size=(tokens, rdim)).astype('f4')
    ids = rng.choice(tokens, count, replace=False).astype(np.int32)
    ids[::13] = -1
    ids[5::17] = tokens + 3
    got = _device(cuda_lib, q, qr, latent, rope, ids, 0, count, (192 + 64) ** -0.5)
    want = mla_ref(q, qr, latent, rope, (192 + 64) ** -0.5, [ids] * heads)
    np.testing.assert_allclose(got, want, rtol=5e-5, atol=3e-6)
