"""MoE feed-forward layer on the GPU vs the reference model's semantics
composed from oracle calls (glm_vx/model.py:289-324): routing must pick the
same experts; outputs agree within the f32 tolerance."""
import numpy as np
import pytest

from helpers import RTOL
from kernels.packed import LAYOUTS

pytestmark = pytest.mark.gpu


def synthetic_layer(experts, hidden, inter, kind=19, seed=0):
    """BASELINE config-2 style weights: IQ1_S d=|N|*0.02, random qs/qh;
    router N(0, 0.02), bias N(0, 0.01)."""
    rng = np.random.default_rng(seed)
    block, size, _ = LAYOUTS[kind]

    def packed(n_rows, cols, count):
        blocks = count * n_rows * cols // block
        raw = rng.integers(0, 256, size=(blocks, size), dtype=np.uint8)
        raw[:, :2] = (np.abs(rng.normal(size=(blocks, 1))) * 0.02).astype(np.float16).view(np.uint8)
        if kind == 12:  # Q4_K dmin
            raw[:, 2:4] = (np.abs(rng.normal(size=(blocks, 1))) * 0.02).astype(np.float16).view(np.uint8)
        return raw.reshape(-1)

    layer = dict(router=(rng.normal(size=(experts, hidden)) * 0.02).astype(np.float32),
                 bias=(rng.normal(size=experts) * 0.01).astype(np.float32),
                 gate=packed(inter, hidden, experts), up=packed(inter, hidden, experts),
                 down=packed(hidden, inter, experts),
                 shared=(packed(inter, hidden, 1), packed(inter, hidden, 1), packed(hidden, inter, 1)))
    return layer


def reference_ffn(cpu, layer, x, experts, hidden, inter, k, scale, kind=19):
    """glm_vx/model.py:289-324 with every primitive on the CPU oracle."""
    block, size, _ = LAYOUTS[kind]
    gu = inter * (hidden // block) * size
    dn = hidden * (inter // block) * size

    def mlp(g, u, d, v):
        gate = cpu.packed_matvec(g, kind, (inter, hidden), v)
        up = cpu.packed_matvec(u, kind, (inter, hidden), v)
        return cpu.packed_matvec(d, kind, (hidden, inter), cpu.swiglu(gate, up))

    ys, all_ids = [], []
    for v in x:
        logits = cpu.matvec(layer['router'], v)
        ids, w = cpu.route(logits, layer['bias'], k, scale)
        result = np.zeros(hidden, np.float32)
        for slot in np.argsort(ids, kind='stable'):
            e = int(ids[slot])
            out = mlp(layer['gate'][e * gu:(e + 1) * gu], layer['up'][e * gu:(e + 1) * gu],
                      layer['down'][e * dn:(e + 1) * dn], v)
            result += out * float(w[slot])
        result += mlp(*layer['shared'], v)
        ys.append(result)
        all_ids.append(ids)
    return np.stack(ys), np.stack(all_ids)


@pytest.mark.parametrize('tokens', [1, 3, 8])
@pytest.mark.parametrize('H,I', [(512, 256), (2048, 2048)])  # generic job path / streaming path
def test_moe_small(gpu_backend, oracle, tokens, H, I):
    from gpu.moe import MoELayer
    E, K = 16, 4
    layer = synthetic_layer(E, H, I, seed=tokens)
    moe = MoELayer(gpu_backend, layer['router'], layer['bias'], 19, layer['gate'], layer['up'], layer['down'],
                   H, I, K, 2.5, shared=layer['shared'])
    try:
        x = np.random.default_rng(100 + tokens).normal(size=(tokens, H)).astype(np.float32)
        y, ids, w = moe.forward(x)
        want, want_ids = reference_ffn(oracle, layer, x, E, H, I, K, 2.5)
        assert ids.tolist() == want_ids.tolist()
        err = np.linalg.norm(y - want) / np.linalg.norm(want)
        assert err <= RTOL, err
    finally:
        moe.close()


@pytest.fixture(scope='module')
def config2_layer(gpu_backend):
    """BASELINE config 2 at full width: 256 experts + shared, hidden 6144,
    inter 2048, IQ1_S, top-8, scale 2.5 (the benchmarked layer's shapes)."""
    from gpu.moe import MoELayer
    E, H, I, K = 256, 6144, 2048, 8
    layer = synthetic_layer(E, H, I, seed=2)
    moe = MoELayer(gpu_backend, layer['router'], layer['bias'], 19, layer['gate'], layer['up'], layer['down'],
                   H, I, K, 2.5, shared=layer['shared'])
    yield layer, moe
    moe.close()


def _job_counts(moe, tokens):
    import ctypes as C
    counts = (C.c_int32 * 4)()
    moe.backend.lib.glmvx_moe_job_counts(tokens, moe.hidden, moe.inter, moe.experts, moe.top_k, 1, moe._ws.ptr,
                                         counts, moe.backend.stream.handle)
    return list(counts)


@pytest.mark.parametrize('T', [1, 2, 8, 32])
def test_moe_config2_full_width(config2_layer, T):
    """The benchmarked layer (config 2, full width) at 1, 2, 8 and 32 tokens
    against the reference's sparse feed-forward (glm_vx/model.py:289-324) on
    the CPU oracle: identical routing, outputs within 1e-5.  At 32 tokens the
    IQ1_S experts routed three or more tokens and the shared expert run in
    the four-token job list (mma_rows_kernel<IQ1_S, S=12> with two token pairs
    per fragment), the path the headline number times; the job counts show
    both lists were used.  Repeated calls are bit-identical."""
    from oracle import loader
    from kernels.backend import VxBackend
    layer, moe = config2_layer
    cpu = VxBackend(str(loader.parallel()))
    E, H, I, K = 256, 6144, 2048, 8
    x = np.random.default_rng(7 + T).normal(size=(T, H)).astype(np.float32)
    y, ids, _ = moe.forward(x)
    counts = _job_counts(moe, T)
    want, want_ids = reference_ffn(cpu, layer, x, E, H, I, K, 2.5)
    assert ids.tolist() == want_ids.tolist()
    err = np.linalg.norm(y - want) / np.linalg.norm(want)
    assert err <= RTOL, err
    row_err = np.linalg.norm(y - want, axis=1) / np.linalg.norm(want, axis=1)
    assert row_err.max() <= RTOL, row_err.max()
    assert counts[0] == 2 * counts[1] and counts[2] == 2 * counts[3]
    if T >= 16:
        # the shared expert alone fills ceil(T/4) four-token jobs
        assert counts[3] >= (T + 3) // 4, counts
    else:
        assert counts[3] == 0, counts
    y2, _, _ = moe.forward(x)
    assert y2.tobytes() == y.tobytes()


def _check_layer(gpu_backend, oracle, E, H, I, K, T, kind, seed):
    from gpu.moe import MoELayer
    layer = synthetic_layer(E, H, I, kind=kind, seed=seed)
    moe = MoELayer(gpu_backend, layer['router'], layer['bias'], kind, layer['gate'], layer['up'], layer['down'],
                   H, I, K, 2.5, shared=layer['shared'])
    try:
        x = np.random.default_rng(seed).normal(size=(T, H)).astype(np.float32)
        y, ids, _ = moe.forward(x)
        want, want_ids = reference_ffn(oracle, layer, x, E, H, I, K, 2.5, kind=kind)
        assert ids.tolist() == want_ids.tolist()
        err = np.linalg.norm(y - want) / np.linalg.norm(want)
        assert err <= RTOL, err
    finally:
        moe.close()


@pytest.mark.parametrize('T', [1, 2, 5, 9, 17, 23])
def test_moe_tokens_share_experts(gpu_backend, oracle, T):
    """4 experts, top-2: most experts serve several tokens, with odd and even
    counts, so expert jobs take two tokens and some a single one; experts with
    three or more tokens and the shared expert run as four-token jobs, full
    and partial, from 16 tokens per call."""
    _check_layer(gpu_backend, oracle, 4, 2048, 2048, 2, T, 19, seed=30 + T)


@pytest.mark.parametrize('T', [17, 23])
def test_moe_result_independent_of_batch(gpu_backend, T):
    """A token's output does not depend on the job it lands in (two- or
    four-token jobs compute each token with the same arithmetic): the batch
    equals token-by-token calls bit for bit."""
    from gpu.moe import MoELayer
    E, H, I, K = 4, 2048, 2048, 2
    layer = synthetic_layer(E, H, I, seed=50 + T)
    moe = MoELayer(gpu_backend, layer['router'], layer['bias'], 19, layer['gate'], layer['up'], layer['down'],
                   H, I, K, 2.5, shared=layer['shared'])
    try:
        x = np.random.default_rng(60 + T).normal(size=(T, H)).astype(np.float32)
        y, _, _ = moe.forward(x)
        singles = np.stack([moe.forward(x[i:i + 1])[0][0] for i in range(T)])
        assert y.tobytes() == singles.tobytes()
    finally:
        moe.close()


@pytest.mark.parametrize('kind', [8, 12])
def test_moe_other_formats(gpu_backend, oracle, kind):
    """Q8_0 and Q4_K expert stacks through the same layer (tensor-core path)."""
    _check_layer(gpu_backend, oracle, 8, 2048, 2048, 3, 4, kind, seed=kind)


def test_moe_pinned_io_and_nonfinite_input(gpu_backend, oracle):
    """forward_pinned on rows written into the layer's pinned buffers equals
    forward; a non-finite activation runs safely (the router ranks NaN scores
    last, every slot still a distinct expert in range) and is reported as
    ValueError, after which the layer keeps working."""
    from gpu.moe import MoELayer
    E, H, I, K, T = 8, 2048, 2048, 4, 5
    layer = synthetic_layer(E, H, I, seed=71)
    moe = MoELayer(gpu_backend, layer['router'], layer['bias'], 19, layer['gate'], layer['up'], layer['down'],
                   H, I, K, 2.5, shared=layer['shared'])
    try:
        x = np.random.default_rng(72).normal(size=(T, H)).astype(np.float32)
        y, ids, w = moe.forward(x)
        io = moe.pinned_io(T)
        np.copyto(io['x'], x)
        yp, idp, wp = moe.forward_pinned(T)
        assert yp.tobytes() == y.tobytes() and idp.tolist() == ids.tolist() and wp.tobytes() == w.tobytes()
        for bad in (np.nan, np.inf):
            xb = x.copy()
            xb[2, 10] = bad
            with pytest.raises(ValueError, match='must be finite'):
                moe.forward(xb)
        xb = np.full_like(x, np.nan)
        with pytest.raises(ValueError, match='must be finite'):
            moe.forward(xb)
        gpu_backend.device.check_device_error()
        y2, _, _ = moe.forward(x)
        assert y2.tobytes() == y.tobytes()
        want, _ = reference_ffn(oracle, layer, x, E, H, I, K, 2.5)
        assert np.linalg.norm(y - want) / np.linalg.norm(want) <= RTOL
    finally:
        moe.close()


@pytest.mark.parametrize('T', [1, 2, 3, 32, 65])
def test_layer_routing_equals_router_kernel(gpu_backend, T):
    """Up to 2 tokens over up to 256 experts the grouping kernel routes the
    tokens itself (every (token, expert) score ranked by one thread); beyond,
    the separate router kernel runs.  Either way the layer's ids and weights are byte-identical to
    glmvx_router on the same logits (glmvx_matmul_nt of the same rows)."""
    import ctypes as C
    from gpu import runtime as rt
    from gpu.moe import MoELayer
    E, H, I, K = 256, 2048, 2048, 8
    layer = synthetic_layer(E, H, I, seed=90)
    # ties and extremes in the router: duplicate expert rows tie their scores
    layer['router'][7] = layer['router'][3]
    layer['bias'][7] = layer['bias'][3]
    moe = MoELayer(gpu_backend, layer['router'], layer['bias'], 19, layer['gate'], layer['up'], layer['down'],
                   H, I, K, 2.5, shared=layer['shared'])
    lib, s = gpu_backend.lib, gpu_backend.stream.handle
    x = np.random.default_rng(T).normal(size=(T, H)).astype(np.float32)
    x[0] = layer['router'][3] * 40.0  # a token that favours the tied pair
    bufs = [rt.DeviceBuffer(n) for n in (x.nbytes, 4 * T * E, 4 * T * K, 4 * T * K)]
    try:
        y, ids, w = moe.forward(x)
        xd, ld, idd, wd = bufs
        xd.upload(x, s)
        rt.check(lib, lib.glmvx_matmul_nt(ld.ptr, xd.ptr, moe.router_w, T, E, H, s), 'matmul_nt')
        rt.check(lib, lib.glmvx_router(idd.ptr, wd.ptr, ld.ptr, moe.router_bias, T, E, K, C.c_float(2.5), s),
                 'router')
        want_ids, want_w = np.empty((T, K), np.int32), np.empty((T, K), np.float32)
        gpu_backend.stream.synchronize()
        idd.download(want_ids)
        wd.download(want_w)
        assert ids.tolist() == want_ids.tolist()
        assert w.tobytes() == want_w.tobytes()
        assert 3 in ids[0] and 7 in ids[0] and list(ids[0]).index(3) < list(ids[0]).index(7)
    finally:
        gpu_backend.stream.synchronize()
        for b in bufs:
            b.close()
        moe.close()
