"""GPU parity of the f32 model primitives (reference ABI glm_vx_* on the
B200) against the CPU oracle.  Tolerances follow the reference's backend
tests (kernels/test_backend.py: rtol=3e-5, atol=3e-5); router ids and top-k
ids must match exactly."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = dict(rtol=3e-5, atol=3e-5)


def test_router_known_answers(gpu_vx, ops_golden):
    ids, w = gpu_vx.route(ops_golden['kat_logits'], ops_golden['kat_bias'], 2, 2.5)
    assert ids.tolist() == [0, 1] and w[0] < w[1]
    np.testing.assert_allclose(w, ops_golden['kat_w'], rtol=3e-6)
    ids, w = gpu_vx.route(ops_golden['r256_logits'], ops_golden['r256_bias'], 8, 2.5)
    assert ids.tolist() == ops_golden['r256_ids'].tolist()
    np.testing.assert_allclose(w, ops_golden['r256_w'], rtol=3e-6)


def test_router_ties_pick_lower_id(gpu_vx, oracle):
    logits = np.zeros(64, np.float32)
    bias = np.zeros(64, np.float32)
    bias[[5, 9, 40]] = 1.0
    for b in (gpu_vx, oracle):
        assert b.route(logits, bias, 4, 1.0)[0].tolist() == [5, 9, 40, 0]


def test_router_many_tokens_vs_oracle(gpu_backend, oracle):
    rng = np.random.default_rng(11)
    for _ in range(32):
        logits = rng.normal(size=256).astype(np.float32)
        bias = (rng.normal(size=256) * 0.01).astype(np.float32)
        a, wa = gpu_backend.route(logits, bias, 8, 2.5)
        b, wb = oracle.route(logits, bias, 8, 2.5)
        assert a.tolist() == b.tolist()
        np.testing.assert_allclose(wa, wb, rtol=3e-6)


@pytest.mark.parametrize('backend_name', ['gpu_vx', 'gpu_backend'])
def test_elementwise_and_norms(request, oracle, backend_name):
    b = request.getfixturevalue(backend_name)
    rng = np.random.default_rng(531)
    x = rng.normal(size=(3, 1000)).astype(np.float32)
    w = rng.normal(size=1000).astype(np.float32)
    bias = rng.normal(size=1000).astype(np.float32)
    np.testing.assert_allclose(b.rmsnorm(x, w, 1e-5), oracle.rmsnorm(x, w, 1e-5), **TOL)
    np.testing.assert_allclose(b.layernorm(x, w, bias), oracle.layernorm(x, w, bias), **TOL)
    np.testing.assert_allclose(b.softmax(x), oracle.softmax(x), **TOL)
    np.testing.assert_allclose(b.swiglu(x[0], x[1]), oracle.swiglu(x[0], x[1]), **TOL)
    for pos in (0, 7, 131071):
        np.testing.assert_allclose(b.rope(x[:, :64], pos, 8e6), oracle.rope(x[:, :64], pos, 8e6), **TOL)


@pytest.mark.parametrize('backend_name', ['gpu_vx', 'gpu_backend'])
def test_f32_matvec_and_linear_batch(request, oracle, backend_name):
    b = request.getfixturevalue(backend_name)
    rng = np.random.default_rng(81)
    w = rng.normal(size=(257, 129)).astype(np.float32)
    x = rng.normal(size=(9, 129)).astype(np.float32)
    np.testing.assert_allclose(b.matvec(w, x[0]), oracle.matvec(w, x[0]), **TOL)
    np.testing.assert_allclose(b.linear_batch(w, x), oracle.linear_batch(w, x), **TOL)


@pytest.mark.parametrize('n,k', [(4, 3), (100, 10), (4096, 2048), (40000, 2048), (32768, 2048), (65536, 4096),
                                 (5000, 1), (9000, 4097), (36864, 4096), (36865, 7), (20000, 2000), (4100, 33)])
def test_topk_exact(gpu_vx, oracle, n, k):
    """Small inputs sort in shared memory; above 4096 scores (k <= 4096) the
    radix selection runs, with the keys staged in shared memory up to 36864
    scores and re-read from the scores above; all give the stable order of
    the oracle."""
    rng = np.random.default_rng(n)
    scores = rng.integers(-50, 50, size=n).astype(np.float32)  # many ties
    assert gpu_vx.topk(scores, k).tolist() == oracle.topk(scores, k).tolist()
    scores = rng.normal(size=n).astype(np.float32)
    scores[::11] = 0.0
    scores[::13] = -0.0  # -0 and +0 tie, lower index first
    assert gpu_vx.topk(scores, k).tolist() == oracle.topk(scores, k).tolist()


@pytest.mark.parametrize('heads,dim', [(32, 128), (40, 100), (5, 300), (64, 64), (1, 1)])
def test_index_scores(gpu_vx, oracle, heads, dim):
    """Blocks of 32 heads x 256 columns, vector and scalar key loads."""
    rng = np.random.default_rng(532 + heads + dim)
    q = rng.normal(size=(heads, dim)).astype(np.float32)
    keys = rng.normal(size=(777, dim)).astype(np.float32)
    w = rng.normal(size=heads).astype(np.float32) / 2
    np.testing.assert_allclose(gpu_vx.index_scores(q, keys, w), oracle.index_scores(q, keys, w), **TOL)


def test_attention_and_sparse_attention(gpu_vx, oracle):
    import ctypes as C
    rng = np.random.default_rng(7)
    tokens, dim, vdim = 300, 96, 80
    q = rng.normal(size=dim).astype(np.float32)
    keys = rng.normal(size=(tokens, dim)).astype(np.float32)
    values = rng.normal(size=(tokens, vdim)).astype(np.float32)
    sel = np.array([5, 299, 0, 17, 17], np.int32)
    F = C.POINTER(C.c_float)
    I = C.POINTER(C.c_int32)
    outs = []
    for lib in (gpu_vx.lib, oracle.lib):
        o1, s1 = np.empty(vdim, np.float32), np.empty(tokens, np.float32)
        assert lib.glm_vx_attention(o1.ctypes.data_as(F), s1.ctypes.data_as(F), q.ctypes.data_as(F),
                                    keys.ctypes.data_as(F), values.ctypes.data_as(F), tokens, dim, vdim,
                                    C.c_float(dim ** -0.5)) == 0
        o2, s2 = np.empty(vdim, np.float32), np.empty(len(sel), np.float32)
        assert lib.glm_vx_sparse_attention(o2.ctypes.data_as(F), s2.ctypes.data_as(F), q.ctypes.data_as(F),
                                           keys.ctypes.data_as(F), values.ctypes.data_as(F), sel.ctypes.data_as(I),
                                           len(sel), tokens, dim, vdim, C.c_float(dim ** -0.5)) == 0
        bad = np.array([1, tokens], np.int32)
        assert lib.glm_vx_sparse_attention(o2.ctypes.data_as(F), s2.ctypes.data_as(F), q.ctypes.data_as(F),
                                           keys.ctypes.data_as(F), values.ctypes.data_as(F), bad.ctypes.data_as(I),
                                           2, tokens, dim, vdim, C.c_float(1.0)) == -1
        outs.append((o1, o2))
    np.testing.assert_allclose(outs[0][0], outs[1][0], **TOL)
    np.testing.assert_allclose(outs[0][1], outs[1][1], **TOL)


def test_mlp_resident(gpu_backend, oracle):
    rng = np.random.default_rng(9)
    gate = rng.normal(size=(64, 48)).astype(np.float32)
    up = rng.normal(size=(64, 48)).astype(np.float32)
    down = rng.normal(size=(40, 64)).astype(np.float32)
    x = rng.normal(size=48).astype(np.float32)
    want = oracle.matvec(down, oracle.swiglu(oracle.matvec(gate, x), oracle.matvec(up, x)))
    np.testing.assert_allclose(gpu_backend.mlp(gate, up, down, x), want, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize('n', [1, 7, 4096, 4099, 1_000_003])
@pytest.mark.parametrize('shift', [0, 1])
def test_nonfinite_flag(gpu_backend, n, shift):
    """glmvx_nonfinite_flag sets the flag for a NaN or infinity at the first,
    a middle or the last element (16-byte aligned and unaligned starts, ragged
    tails, one and many blocks) and leaves a zeroed flag at 0 otherwise."""
    from gpu import runtime as rt
    lib, s = gpu_backend.lib, gpu_backend.stream.handle
    x = np.random.default_rng(n).normal(size=n + shift).astype(np.float32)
    buf, flag = rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(16)
    got = np.zeros(1, np.uint32)

    def run(values):
        buf.upload(values, s)
        rt.call('glmvx_memset', flag.ptr, 0, 4, s)
        rt.call('glmvx_nonfinite_flag', buf.ptr + 4 * shift, n, flag.ptr, s)
        gpu_backend.stream.synchronize()
        flag.download(got)
        return int(got[0])

    try:
        assert run(x) == 0
        for pos in {0, n // 2, n - 1}:
            for bad in (np.nan, np.inf, -np.inf):
                xb = x.copy()
                xb[shift + pos] = bad
                assert run(xb) == 1, (pos, bad)
        if shift:  # a non-finite value just outside the range is not seen
            xb = x.copy()
            xb[0] = np.nan
            assert run(xb) == 0
    finally:
        buf.close()
        flag.close()
