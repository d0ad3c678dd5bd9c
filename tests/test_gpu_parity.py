"""Parity of the CUDA path (called through the C-ABI) with the CPU oracle:
bit-identical outputs on the same seeded inputs, for every weight format of
the benchmark models, token counts 1..512, both src1 shapes (ne11 = 1 and
ne11 = k), strided id views, slot churn, and the error paths."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q6_K, Q8_K, IQ1_S, MXFP4 = 8, 12, 14, 15, 19, 39
# (type, ne00, ne01) of the expert matrices of the benchmark models
SHAPES = {
    "q8_0-gate": (Q8_0, 2048, 768), "q8_0-down": (Q8_0, 768, 2048),
    "q4_K-gate": (Q4_K, 2048, 1024), "q6_K-down": (Q6_K, 1024, 2048),
    "q4_K-gate-4096": (Q4_K, 4096, 1536), "q6_K-down-1536": (Q6_K, 1536, 4096),
    "mxfp4": (MXFP4, 2880, 2880), "iq1_s-gate": (IQ1_S, 7168, 2048), "iq1_s-down": (IQ1_S, 2048, 7168),
}


def D(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def H(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def no_device_error(gxlib):
    from galactus_b200.moe import device_error
    assert device_error() == 0


@pytest.fixture(autouse=True)
def clear_device_error(gxlib):
    """Each test starts with the device error word cleared."""
    try:
        import torch as _t
        if _t.cuda.is_available():
            from galactus_b200.moe import device_error
            gxlib.lib().gx_device_init(0)
            device_error()
    except Exception:
        pass
    yield


@pytest.mark.parametrize("t", [Q8_0, Q4_K, Q6_K, MXFP4, IQ1_S])
def test_synth_weights_bytes(gxlib, orc, dev, t):
    ne00 = 2880 if t == MXFP4 else 2048
    rows = 12
    want = orc.synth_weights(t, ne00, rows, seed=3, stream_id=99)
    buf = torch.zeros(want.size, dtype=torch.uint8, device=dev)
    gxlib.check(gxlib.lib().gx_synth_weights(t, buf.data_ptr(), ne00, rows, 3, 99, 0.02, None))
    np.testing.assert_array_equal(H(buf), want)
    x = torch.zeros(10000, dtype=torch.float32, device=dev)
    gxlib.check(gxlib.lib().gx_synth_normal(x.data_ptr(), 10000, 7, 5, 1.0, None))
    np.testing.assert_array_equal(bits(H(x)), bits(orc.synth_normal(10000, 7, 5, 1.0)))


def test_expf_bitwise(gxlib, orc, dev):
    rng = np.random.default_rng(1)
    xs = np.concatenate([
        rng.uniform(-110, 95, 1 << 21), rng.uniform(-2, 2, 1 << 20),
        np.arange(-(1 << 16), 1 << 16, dtype=np.int64).astype(np.float32) * np.float32(1 / 512),
        np.array([0, -0.0, np.inf, -np.inf, np.nan, 88.72283935546875, 88.7228317, -103.972084, -87.33655], np.float32),
    ]).astype(np.float32)
    xd = D(xs)
    yd = torch.empty_like(xd)
    gxlib.check(gxlib.lib().gx_expf(xd.data_ptr(), yd.data_ptr(), xs.size, None))
    got, want = H(yd), orc.expf(xs)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(bits(got)[~nan], bits(want)[~nan])


@pytest.mark.parametrize("vdt,n", [(Q8_0, 2048), (Q8_0, 2880), (Q8_K, 2048), (Q8_K, 7168)])
def test_quantize_rows_bitwise(gxlib, orc, dev, vdt, n):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((9, n)).astype(np.float32)
    x[1] = 0.0
    x[2, :64] = np.float32(0.5)          # ties in |x|
    x[3] *= np.float32(1e-30)            # tiny magnitudes
    want = orc.quantize(vdt, x)
    pitch = (want.shape[1] + 15) // 16 * 16
    out = torch.zeros(9 * pitch, dtype=torch.uint8, device=dev)
    xd = D(x)
    gxlib.check(gxlib.lib().gx_quantize_rows(vdt, xd.data_ptr(), n, 9, n * 4, out.data_ptr(), pitch, None))
    got = H(out).reshape(9, pitch)[:, :want.shape[1]]
    np.testing.assert_array_equal(got, want)


def test_activations_and_combine_bitwise(gxlib, orc, dev):
    rng = np.random.default_rng(3)
    g = (rng.standard_normal(1 << 18) * 6).astype(np.float32)
    u = (rng.standard_normal(1 << 18) * 6).astype(np.float32)
    g[:4] = [np.nan, 100.0, -100.0, 7.0]
    gd, ud = D(g), D(u)
    out = torch.empty_like(gd)
    gxlib.check(gxlib.lib().gx_swiglu(gd.data_ptr(), ud.data_ptr(), out.data_ptr(), g.size, None))
    w = orc.swiglu(g, u)
    np.testing.assert_array_equal(bits(H(out))[4:], bits(w)[4:])
    gxlib.check(gxlib.lib().gx_swiglu_oai(gd.data_ptr(), ud.data_ptr(), out.data_ptr(), g.size, 1.702, 7.0, None))
    w = orc.swiglu_oai(g, u, 1.702, 7.0)
    got = H(out)
    assert np.array_equal(np.isnan(got), np.isnan(w))
    np.testing.assert_array_equal(bits(got)[~np.isnan(w)], bits(w)[~np.isnan(w)])
    y = rng.standard_normal((5, 8, 2048)).astype(np.float32)
    wt = rng.random((5, 8)).astype(np.float32)
    o = torch.empty((5, 2048), dtype=torch.float32, device=dev)
    yd, wd = D(y), D(wt)          # keep the device copies alive until the kernel has run
    gxlib.check(gxlib.lib().gx_combine(yd.data_ptr(), wd.data_ptr(), o.data_ptr(), 2048, 8, 5, None))
    np.testing.assert_array_equal(bits(H(o)), bits(orc.combine(y, wt)))


def _experts(orc, t, ne00, ne01, n_as, seed):
    rb = orc.row_bytes(t, ne00)
    nb02 = (rb * ne01 + 16383) // 16384 * 16384 + 16384   # a record stride wider than the matrix
    ex = np.zeros((n_as, nb02), np.uint8)
    for e in range(n_as):
        ex[e, :rb * ne01] = orc.synth_weights(t, ne00, ne01, seed, 1000 + e)
    return ex, rb, nb02


def _run_mmid(gxlib, t, ex, ne00, ne01, rb, nb02, b, ids_full, k):
    T, ne11, _ = b.shape
    dst = torch.zeros((T, k, ne01), dtype=torch.float32, device="cuda")
    exd, bd, idd = D(ex), D(b), D(ids_full)
    gxlib.mul_mat_id(t, exd, ne00, ne01, rb, nb02, ex.shape[0], bd, ne11, T, ne00 * 4, ne11 * ne00 * 4,
                     idd, k, T, ids_full.shape[1] * 4, dst)
    return H(dst)


@pytest.mark.parametrize("shape", list(SHAPES))
@pytest.mark.parametrize("T", [1, 2, 3, 8, 32])
def test_mul_mat_id_bitwise(gxlib, orc, dev, shape, T):
    t, ne00, ne01 = SHAPES[shape]
    k, n_as, n_exp_row = 4, 6, 16
    rng = np.random.default_rng(T * 31 + ne00)
    ex, rb, nb02 = _experts(orc, t, ne00, ne01, n_as, seed=T)
    # ids as a view into a wider argsort row (nb1 = 16 ints), the case the
    # reference's stride fix is about
    ids_full = np.full((T, n_exp_row), -7, np.int32)
    for i in range(T):
        ids_full[i, :k] = rng.choice(n_as, k, replace=False)
    ids = ids_full[:, :k]
    for ne11 in (1, k):
        b = rng.standard_normal((T, ne11, ne00)).astype(np.float32)
        got = _run_mmid(gxlib, t, ex, ne00, ne01, rb, nb02, b, ids_full, k)
        want = orc.mul_mat_id(t, ex, ne00, ne01, b, ids, nb01=rb)
        np.testing.assert_array_equal(bits(got), bits(want), err_msg=f"{shape} T={T} ne11={ne11}")
    no_device_error(gxlib)


@pytest.mark.parametrize("shape", list(SHAPES))
def test_mul_mat_id_512_tokens(gxlib, orc, dev, shape):
    """A 512-token micro-batch (the reference's full-residency micro-batch,
    app/src-tauri/src/lib.rs:3342-3346) for every expert format, both src1
    shapes (ne11 = 1 and ne11 = k)."""
    t, ne00, ne01 = SHAPES[shape]
    k, n_as, T = 8, 16, 512
    rng = np.random.default_rng(512 + ne00)
    ex, rb, nb02 = _experts(orc, t, ne00, ne01, n_as, seed=9)
    ids = np.stack([rng.choice(n_as, k, replace=False) for _ in range(T)]).astype(np.int32)
    for ne11 in (1, k):
        b = rng.standard_normal((T, ne11, ne00)).astype(np.float32)
        got = _run_mmid(gxlib, t, ex, ne00, ne01, rb, nb02, b, ids, k)
        want = orc.mul_mat_id(t, ex, ne00, ne01, b, ids, nb01=rb)
        np.testing.assert_array_equal(bits(got), bits(want), err_msg=f"{shape} ne11={ne11}")
    no_device_error(gxlib)


def test_layer_2048_token_prefill_qwen3_235b(gxlib, orc, dev):
    """BASELINE cfg 4's 2048-token prefill on one Qwen3-235B-A22B-shaped layer
    (Q4_K gate/up, Q6_K down, 16 resident experts, Zipf routes): the layer
    output equals the oracle's bit for bit."""
    m = _small_model(gxlib, "qwen3-235b", experts=16, layers=1)
    k, T = m.used, 2048
    arena = gxlib.Arena(m, capacity_bytes=m.experts * m.record, policy=gxlib.POLICY_AUTO, max_tokens=T)
    try:
        recs = np.stack([orc.synth_record(m, m.seed, 0, e) for e in range(m.experts)])
        for e in range(m.experts):
            arena.load_record(0, e, recs[e])
        rng = np.random.default_rng(2048)
        ids, w = _zipf_routes(rng, T, m.experts, k)
        x = rng.standard_normal((T, m.hidden)).astype(np.float32)
        out = torch.full((T, m.hidden), float("nan"), dtype=torch.float32, device=dev)
        arena.layer_forward(0, D(x), ids, D(w), out, stream=torch.cuda.current_stream())
        got = H(out)
        want = orc.moe_layer(m, recs, x, ids, w)
        np.testing.assert_array_equal(bits(got), bits(want))
        no_device_error(gxlib)
    finally:
        arena.close()


def test_out_of_domain_id_is_reported_not_read(gxlib, orc, dev):
    from galactus_b200.moe import device_error
    device_error()
    t, ne00, ne01 = SHAPES["q8_0-down"]
    k, n_as, T = 2, 3, 2
    ex, rb, nb02 = _experts(orc, t, ne00, ne01, n_as, seed=1)
    ids = np.array([[0, 1], [2, 3]], np.int32)      # 3 is outside [0, 3)
    b = np.random.default_rng(0).standard_normal((T, 1, ne00)).astype(np.float32)
    got = _run_mmid(gxlib, t, ex, ne00, ne01, rb, nb02, b, ids, k)
    assert np.isnan(got[1, 1]).all()
    want = orc.mul_mat_id(t, ex, ne00, ne01, b, np.array([[0, 1], [2, 0]], np.int32), nb01=rb)
    np.testing.assert_array_equal(bits(got[:, 0]), bits(want[:, 0]))
    assert device_error() == 1
    assert device_error() == 0


def _small_model(gxlib, name, experts=12, layers=2):
    m = gxlib.MODELS[name]
    from galactus_b200.models import ModelShape
    return ModelShape(**{**m.__dict__, "experts": experts, "layers": layers})


def _zipf_routes(rng, T, experts, k):
    p = 1.0 / np.arange(1, experts + 1) ** 1.1
    p /= p.sum()
    ids = np.stack([rng.choice(experts, k, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    w /= w.sum(axis=1, keepdims=True)
    return ids, w.astype(np.float32)


@pytest.mark.parametrize("name", ["qwen3-30b", "olmoe", "gpt-oss-120b", "qwen3-235b", "deepseek-v3"])
def test_layer_forward_bitwise_with_churn(gxlib, orc, dev, name):
    """remap (policy + host->HBM miss copies) + fused gate/up/act + fused
    down/combine, against the oracle layer on expert-indexed records, with a
    cache small enough that slots are evicted and reused; micro-batches whose
    distinct routes exceed the policy's batch bound run in waves."""
    m = _small_model(gxlib, name)
    k = m.used
    rng = np.random.default_rng(sum(map(ord, name)))
    cap_slots = k + 2 if k + 2 < m.experts else m.experts
    arena = gxlib.Arena(m, capacity_bytes=cap_slots * m.record * m.layers, policy=gxlib.POLICY_AUTO,
                        max_tokens=16)
    records = np.stack([orc.synth_record(m, m.seed, 0, e) for e in range(m.experts)])
    records2 = np.stack([orc.synth_record(m, m.seed, 1, e) for e in range(m.experts)])
    for e in range(m.experts):
        arena.load_record(0, e, records[e])
        arena.load_record(1, e, records2[e])
    q, prot, prob = arena.quota(0)
    bound = min(q, prob)
    stream = torch.cuda.current_stream()
    waved = 0
    for step, T in enumerate([1, 1, 2, 1, 4, 1, 16, 1, 3]):
        layer = step % 2
        recs = records if layer == 0 else records2
        ids, w = _zipf_routes(rng, T, m.experts, k)
        waved += len(set(ids.ravel().tolist())) > bound   # served in expert-major waves
        x = rng.standard_normal((T, m.hidden)).astype(np.float32)
        out = torch.zeros((T, m.hidden), dtype=torch.float32, device=dev)
        arena.layer_forward(layer, D(x), ids, D(w), out, stream=stream)
        got = H(out)
        want = orc.moe_layer(m, recs, x, ids, w)
        np.testing.assert_array_equal(bits(got), bits(want), err_msg=f"{name} step {step} T={T}")
    st = arena.stats()
    assert st["misses"] > 0 and st["hits"] > 0
    assert waved > 0
    no_device_error(gxlib)
    arena.close()


@pytest.mark.parametrize("T", [16, 64, 257, 512])
def test_grouped_prefill_matches_oracle(gxlib, orc, dev, T):
    """Micro-batches of >= 128 (token, slot) pairs take the expert-grouped
    path: by default the tensor-core kernels (tcgen05 int8 MMA, 16 pairs of
    one expert x 128 weight rows per unit), with GX_PREFILL_MMA=0 the
    CUDA-core grouped kernels, with GX_GROUPED=0 the per-pair decode kernels;
    all three give the oracle's bits, including experts with one token, with
    a partial last chunk and with many chunks."""
    import os
    m = _small_model(gxlib, "qwen3-30b", experts=12, layers=1)
    k = m.used
    arena = gxlib.Arena(m, capacity_bytes=m.experts * m.record, policy=gxlib.POLICY_AUTO, max_tokens=T)
    recs = np.stack([orc.synth_record(m, m.seed, 0, e) for e in range(m.experts)])
    for e in range(m.experts):
        arena.load_record(0, e, recs[e])
    rng = np.random.default_rng(900 + T)
    ids, w = _zipf_routes(rng, T, m.experts, k)
    x = rng.standard_normal((T, m.hidden)).astype(np.float32)
    stream = torch.cuda.current_stream()
    out = torch.full((T, m.hidden), float("nan"), dtype=torch.float32, device=dev)
    arena.layer_forward(0, D(x), ids, D(w), out, stream=stream)
    got = H(out)
    variants = {}
    for env in ("GX_PREFILL_MMA", "GX_GROUPED"):
        os.environ[env] = "0"
        try:
            out2 = torch.full((T, m.hidden), float("nan"), dtype=torch.float32, device=dev)
            arena.layer_forward(0, D(x), ids, D(w), out2, stream=stream)
            variants[env] = H(out2)
        finally:
            del os.environ[env]
    want = orc.moe_layer(m, recs, x, ids, w)
    np.testing.assert_array_equal(bits(got), bits(want), err_msg=f"tensor-core T={T}")
    np.testing.assert_array_equal(bits(variants["GX_PREFILL_MMA"]), bits(want), err_msg=f"CUDA-core grouped T={T}")
    np.testing.assert_array_equal(bits(variants["GX_GROUPED"]), bits(want), err_msg=f"per-pair T={T}")
    no_device_error(gxlib)
    arena.close()


def test_route_trace_of_layer_calls(gxlib, orc, dev, tmp_path):
    """The arena path records each layer call with its (tokens, k) shape, the
    residency sampled before the serve and whole records per miss."""
    from galactus_b200.route_trace import close_trace, open_trace, read_trace
    m = _small_model(gxlib, "qwen3-30b", experts=12, layers=2)
    k = m.used
    arena = gxlib.Arena(m, capacity_bytes=(k + 2) * m.record * m.layers, policy=gxlib.POLICY_AUTO, max_tokens=2)
    for L in range(m.layers):
        for e in range(m.experts):
            arena.load_record(L, e, orc.synth_record(m, m.seed, L, e))
    path = tmp_path / "routes.txt"
    open_trace(str(path), arch="qwen3moe")
    rng = np.random.default_rng(4)
    stream = torch.cuda.current_stream()
    calls = []
    for step in range(8):
        L = step % 2
        ids, w = _zipf_routes(rng, 1, m.experts, k)
        before = [arena.slot_of(L, int(e)) >= 0 for e in ids.ravel()]
        x = rng.standard_normal((1, m.hidden)).astype(np.float32)
        out = torch.zeros((1, m.hidden), dtype=torch.float32, device=dev)
        s0 = arena.stats()["misses"]
        arena.layer_forward(L, D(x), ids, D(w), out, stream=stream)
        calls.append((L, ids.ravel().tolist(), before, arena.stats()["misses"] - s0))
    torch.cuda.synchronize()
    close_trace()
    tr = read_trace(str(path))
    assert len(tr["entries"]) == len(calls)
    for e, (L, ids, before, misses) in zip(tr["entries"], calls):
        assert (e["layer"], e["tokens"], e["k"]) == (L, 1, k)
        assert e["ids"] == ids and e["resident"] == [int(b) for b in before]
        assert e["bytes_read"] == misses * m.record
    arena.close()


def test_remap_serve_strided_and_slot_bytes(gxlib, orc, dev):
    """The remap node reads and writes through strides, and every served slot
    holds exactly its record's bytes after churn (the serve-check pattern)."""
    m = _small_model(gxlib, "qwen3-30b", experts=16, layers=1)
    arena = gxlib.Arena(m, capacity_bytes=10 * m.record, policy=gxlib.POLICY_AUTO, max_tokens=4)
    recs = [orc.synth_record(m, 11, 0, e) for e in range(m.experts)]
    for e in range(m.experts):
        arena.load_record(0, e, recs[e])
    rng = np.random.default_rng(4)
    stream = torch.cuda.current_stream()
    q, _, prob = arena.quota(0)
    for _ in range(30):
        full = np.full((2, 16), -1, np.int32)            # argsort rows of 16, top-k view of 4
        full[0, :4] = rng.choice(16, 4, replace=False)
        full[1, :4] = full[0, :4][::-1]
        view = full[:, :4]
        slots_full = np.full((2, 8), -5, np.int32)
        slots = slots_full[:, ::2]                        # strided destination
        arena.remap(0, view, stream=stream, slots=slots)
        assert (slots_full[:, 1::2] == -5).all()
        for i in range(2):
            for j in range(4):
                assert slots[i, j] == arena.slot_of(0, int(view[i, j]))
    torch.cuda.synchronize()
    seen = 0
    for e in range(m.experts):
        s = arena.slot_of(0, e)
        if s >= 0:
            np.testing.assert_array_equal(arena.read_slot(0, s), recs[e][:m.record_raw])
            seen += 1
    assert seen > 0
    arena.close()


@pytest.mark.parametrize("name,T,layers,layerwise", [
    ("qwen3-30b", 1, 3, False), ("olmoe", 1, 3, False), ("gpt-oss-120b", 1, 3, False),
    ("qwen3-235b", 1, 3, False), ("deepseek-v3", 1, 2, False), ("qwen3-30b", 1, 10, False),
    ("qwen3-30b", 3, 3, False), ("gpt-oss-120b", 5, 3, False), ("olmoe", 4, 3, False), ("olmoe", 1, 10, False),
    ("qwen3-235b", 3, 2, False), ("deepseek-v3", 2, 2, False),
    ("qwen3-30b", 1, 3, True), ("olmoe", 2, 3, True),
])
def test_stack_plan_graph_matches_oracle(gxlib, orc, dev, name, T, layers, layerwise):
    """The captured decode plan (CUDA graph, slot ids from a device array) gives
    the oracle's bits, with misses and evictions between runs (T = 1), and the
    per-layer C-ABI path gives the same bits. Without GX_PLAN_LAYERWISE the
    graph is the single persistent stack kernel, which streams every layer's
    expert rows through one bulk-copy ring."""
    from galactus_b200.moe import StackCall, StackPlan
    m = _small_model(gxlib, name, experts=12, layers=layers)
    k = m.used
    slots = k + 2 if T == 1 else m.experts
    arena = gxlib.Arena(m, capacity_bytes=slots * m.record * m.layers, policy=gxlib.POLICY_AUTO, max_tokens=T)
    recs = [np.stack([orc.synth_record(m, m.seed, L, e) for e in range(m.experts)]) for L in range(m.layers)]
    for L in range(m.layers):
        for e in range(m.experts):
            arena.load_record(L, e, recs[L][e])
    x = torch.zeros((m.layers, T, m.hidden), dtype=torch.float32, device=dev)
    w = torch.zeros((m.layers, T, k), dtype=torch.float32, device=dev)
    out = torch.zeros((m.layers, T, m.hidden), dtype=torch.float32, device=dev)
    ptr = lambda t: [t[L].data_ptr() for L in range(m.layers)]
    plan = StackPlan(arena, 0, m.layers, ptr(x), ptr(w), ptr(out), k, T, layerwise=layerwise)
    info = plan.info()
    stack_types = {(gxlib.TYPE_Q8_0, gxlib.TYPE_Q8_0), (gxlib.TYPE_Q4_K, gxlib.TYPE_Q6_K),
                   (gxlib.TYPE_MXFP4, gxlib.TYPE_MXFP4), (gxlib.TYPE_IQ1_S, gxlib.TYPE_IQ1_S)}
    expect = not layerwise and (m.type_gate, m.type_down) in stack_types
    assert info["stack_kernel"] == (1 if expect else 0), info
    if expect:
        # each ring stage belongs to one of the two weight-producer warps; the
        # tensor-core MXFP4 jobs (k = 4) run on the TMA-fed row mode by default
        # (its ring a multiple of 4 stages), or with one producer (GX_STACK_MMA=1)
        env = os.environ.get("GX_STACK_MMA")
        mx = m.type_gate == gxlib.TYPE_MXFP4 and k == 4
        want_tc = (1 if env == "1" else 0 if env == "0" else 2) if mx else 0
        assert info["tensor_cores"] == want_tc, info
        assert info["stages"] % {0: 2, 1: 1, 2: 4}[want_tc] == 0, info
    call = StackCall(arena, 0, m.layers, ptr(x), ptr(w), ptr(out), k, T)
    rng = np.random.default_rng(5 + T)
    stream = torch.cuda.current_stream()
    for step in range(6):
        xs = rng.standard_normal((m.layers, T, m.hidden)).astype(np.float32)
        ids = np.stack([_zipf_routes(rng, T, m.experts, k)[0] for _ in range(m.layers)]).astype(np.int32)  # [L,T,k]
        ws = rng.random((m.layers, T, k)).astype(np.float32)
        x.copy_(torch.from_numpy(xs))
        w.copy_(torch.from_numpy(ws))
        out.fill_(float("nan"))
        runner = plan if step % 2 == 0 else call
        runner(np.ascontiguousarray(ids), stream)
        got = H(out)
        no_device_error(gxlib)
        for L in range(m.layers):
            want = orc.moe_layer(m, recs[L], xs[L], ids[L], ws[L])
            np.testing.assert_array_equal(bits(got[L]), bits(want), err_msg=f"{name} T={T} step {step} layer {L}")
    if T == 1:
        assert arena.stats()["misses"] > 0
    no_device_error(gxlib)
    plan.close()
    arena.close()


@pytest.mark.parametrize("tc", ["2", "1", "0"])
@pytest.mark.parametrize("T,layers,experts", [(1, 4, 16), (2, 3, 12), (8, 2, 16)])
def test_stack_plan_mxfp4_tensor_and_cuda_cores(gxlib, orc, dev, monkeypatch, tc, T, layers, experts):
    """gpt-oss-shaped MXFP4 stacks (hidden 2880, top-4) with the block dots on
    the tensor cores (tcgen05 kind::f8f6f4, e4m3 activation digits) fed by TMA
    from the slots' tensor-core copies (GX_STACK_MMA=2) or repacked by the CUDA
    cores (1), and on the CUDA cores (the default, 0): all give the oracle's
    bits, through the captured plan and after slot churn (the copies follow
    the arena's fills)."""
    from galactus_b200.moe import StackPlan
    monkeypatch.setenv("GX_STACK_MMA", tc)
    m = _small_model(gxlib, "gpt-oss-120b", experts=experts, layers=layers)
    k = m.used
    slots = k + 3 if T == 1 else m.experts   # churn at one token; every expert resident at more
    arena = gxlib.Arena(m, capacity_bytes=slots * m.record * m.layers, policy=gxlib.POLICY_AUTO, max_tokens=T)
    recs = [np.stack([orc.synth_record(m, m.seed, L, e) for e in range(m.experts)]) for L in range(m.layers)]
    for L in range(m.layers):
        for e in range(m.experts):
            arena.load_record(L, e, recs[L][e])
    x = torch.zeros((m.layers, T, m.hidden), dtype=torch.float32, device=dev)
    w = torch.zeros((m.layers, T, k), dtype=torch.float32, device=dev)
    out = torch.zeros((m.layers, T, m.hidden), dtype=torch.float32, device=dev)
    ptr = lambda t: [t[L].data_ptr() for L in range(m.layers)]
    plan = StackPlan(arena, 0, m.layers, ptr(x), ptr(w), ptr(out), k, T)
    info = plan.info()
    assert info["stack_kernel"] == 1 and info["tensor_cores"] == int(tc), info
    rng = np.random.default_rng(90 + T)
    stream = torch.cuda.current_stream()
    for step in range(3):
        xs = (rng.standard_normal((m.layers, T, m.hidden)) * (1.0 + 3.0 * step)).astype(np.float32)
        ids = np.stack([_zipf_routes(rng, T, m.experts, k)[0] for _ in range(m.layers)]).astype(np.int32)
        ws = rng.random((m.layers, T, k)).astype(np.float32)
        x.copy_(torch.from_numpy(xs))
        w.copy_(torch.from_numpy(ws))
        out.fill_(float("nan"))
        plan(np.ascontiguousarray(ids), stream)
        got = H(out)
        no_device_error(gxlib)
        for L in range(m.layers):
            want = orc.moe_layer(m, recs[L], xs[L], ids[L], ws[L])
            np.testing.assert_array_equal(bits(got[L]), bits(want), err_msg=f"tc={tc} T={T} step {step} layer {L}")
    plan.close()
    arena.close()


def test_stack_kernel_timing(gxlib, orc, dev):
    """A timing plan of the stack kernel reports one positive duration (events
    recorded inside the graph around the kernel) and the oracle's bits."""
    from galactus_b200.moe import StackPlan
    m = _small_model(gxlib, "qwen3-30b", experts=12, layers=2)
    k = m.used
    arena = gxlib.Arena(m, capacity_bytes=m.experts * m.record * m.layers, policy=gxlib.POLICY_AUTO, max_tokens=1)
    recs = [np.stack([orc.synth_record(m, m.seed, L, e) for e in range(m.experts)]) for L in range(m.layers)]
    for L in range(m.layers):
        for e in range(m.experts):
            arena.load_record(L, e, recs[L][e])
    rng = np.random.default_rng(17)
    xs = rng.standard_normal((m.layers, 1, m.hidden)).astype(np.float32)
    ws = rng.random((m.layers, 1, k)).astype(np.float32)
    x = torch.from_numpy(xs).to(dev)
    w = torch.from_numpy(ws).to(dev)
    out = torch.zeros((m.layers, 1, m.hidden), dtype=torch.float32, device=dev)
    ptr = lambda t: [t[L].data_ptr() for L in range(m.layers)]
    plan = StackPlan(arena, 0, m.layers, ptr(x), ptr(w), ptr(out), k, 1, timing=True)
    assert plan.info()["stack_kernel"] == 1
    ids = np.stack([_zipf_routes(rng, 1, m.experts, k)[0] for _ in range(m.layers)]).astype(np.int32)
    stream = torch.cuda.current_stream()
    plan(np.ascontiguousarray(ids), stream)
    torch.cuda.synchronize()
    ms, zero = plan.timing()
    assert ms > 0.0 and zero == 0.0
    for L in range(m.layers):
        want = orc.moe_layer(m, recs[L], xs[L], ids[L], ws[L])
        np.testing.assert_array_equal(bits(H(out)[L]), bits(want))
    plan.close()
    arena.close()
    no_device_error(gxlib)
