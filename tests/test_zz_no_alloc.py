"""The allocation-free layer entry point (gx_moe_ffn_noalloc).

It serves callers that may not call cudaMalloc -- a host framework that owns
every device allocation, a plugin inside such a process, or a latency-bound
path -- by keeping its scratch in a fixed device array inside the library.
This file is collected last on purpose, so that a run stopping at the first
failure has run every other test first; it also passes alone in a fresh
process. The reference has no counterpart: the comparison is with the
library's own gx_moe_layer_forward on the same slots, which the other GPU tests
hold bit-identical to the CPU oracle."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["qwen3-30b", "olmoe", "gpt-oss-120b", "deepseek-v3"])
def test_noalloc_matches_layer_forward_on_two_calls(gxlib, orc, name):
    from galactus_b200 import _lib as L
    from galactus_b200.models import ModelShape
    gxlib.check(gxlib.lib().gx_device_init(0), "gx_device_init")
    base = gxlib.MODELS[name]
    m = ModelShape(**{**base.__dict__, "experts": 12, "layers": 1})
    k = m.used
    arena = gxlib.Arena(m, capacity_bytes=m.experts * m.record, policy=gxlib.POLICY_AUTO, max_tokens=4)
    for e in range(m.experts):
        arena.load_record(0, e, orc.synth_record(m, m.seed, 0, e))
    stream = torch.cuda.current_stream()
    arena.warm_all(stream)
    slab, record, n_slots = arena.layer_view(0)
    rng = np.random.default_rng(17)
    fn = gxlib.lib().gx_moe_ffn_noalloc
    for call, T in enumerate([2, 1]):                  # two calls in a row, different shapes
        ids = np.stack([rng.choice(m.experts, k, replace=False) for _ in range(T)]).astype(np.int32)
        x = torch.from_numpy(rng.standard_normal((T, m.hidden)).astype(np.float32)).cuda()
        w = torch.from_numpy(rng.random((T, k)).astype(np.float32)).cuda()
        want = torch.zeros((T, m.hidden), dtype=torch.float32, device="cuda")
        arena.layer_forward(0, x, ids, w, want, stream=stream)
        slots = np.array([[arena.slot_of(0, int(e)) for e in row] for row in ids], dtype=np.int32)
        got = torch.full((T, m.hidden), float("nan"), dtype=torch.float32, device="cuda")
        rc = fn(C.byref(arena.desc), slab, record, n_slots, x.data_ptr(), slots.ctypes.data, w.data_ptr(), k, T,
                got.data_ptr(), stream.cuda_stream)
        assert rc == L.GX_OK, (call, rc)
        torch.cuda.synchronize()
        g, wnt = got.cpu().numpy(), want.cpu().numpy()
        # the same kernels on the same bytes: bit for bit
        np.testing.assert_array_equal(g.view(np.uint32), wnt.view(np.uint32), err_msg=f"{name} call {call} T={T}")
    from galactus_b200.moe import device_error
    assert device_error() == 0
    arena.close()


def test_noalloc_rejects_sizes_beyond_its_array(gxlib):
    from galactus_b200 import _lib as L
    gxlib.check(gxlib.lib().gx_device_init(0), "gx_device_init")
    m = gxlib.MODELS["qwen3-30b"]
    desc = L.gx_layer_desc(m.type_gate, m.type_up, m.type_down, m.act, m.alpha, m.limit, m.hidden, m.intermediate,
                           m.off_gate, m.off_up)
    slots = np.zeros((9, 8), np.int32)                  # 72 (token, slot) pairs > 64
    buf = torch.zeros(16, dtype=torch.float32, device="cuda")
    rc = gxlib.lib().gx_moe_ffn_noalloc(C.byref(desc), buf.data_ptr(), m.record, 1, buf.data_ptr(), slots.ctypes.data,
                                        buf.data_ptr(), 8, 9, buf.data_ptr(), None)
    assert rc == L.GX_ERR_INVALID


def test_noalloc_at_its_limits_matches_the_oracle(gxlib, orc):
    """The largest call the array admits -- 64 (token, slot) pairs, hidden
    8192, expert intermediate 4096 -- where the carve-up of the array is
    tightest, on Q4_K gate/up and Q6_K down records: bit-identical to the CPU
    oracle and to gx_moe_layer_forward, on two calls in a row."""
    from galactus_b200 import _lib as L
    from galactus_b200.models import ModelShape
    gxlib.check(gxlib.lib().gx_device_init(0), "gx_device_init")
    m = ModelShape("limits", 1, 8192, 8, 8, 4096, gxlib.TYPE_Q4_K, gxlib.TYPE_Q4_K, gxlib.TYPE_Q6_K, seed=21)
    k, T = m.used, 8
    recs = np.stack([orc.synth_record(m, m.seed, 0, e) for e in range(m.experts)])
    arena = gxlib.Arena(m, capacity_bytes=m.experts * m.record, policy=gxlib.POLICY_AUTO, max_tokens=T)
    try:
        for e in range(m.experts):
            arena.load_record(0, e, recs[e])
        stream = torch.cuda.current_stream()
        arena.warm_all(stream)
        slab, record, n_slots = arena.layer_view(0)
        rng = np.random.default_rng(64)
        fn = gxlib.lib().gx_moe_ffn_noalloc
        for call in range(2):
            ids = np.stack([rng.permutation(m.experts)[:k] for _ in range(T)]).astype(np.int32)
            xh = rng.standard_normal((T, m.hidden)).astype(np.float32)
            wh = rng.random((T, k)).astype(np.float32)
            x, w = torch.from_numpy(xh).cuda(), torch.from_numpy(wh).cuda()
            want = torch.zeros((T, m.hidden), dtype=torch.float32, device="cuda")
            arena.layer_forward(0, x, ids, w, want, stream=stream)
            slots = np.array([[arena.slot_of(0, int(e)) for e in row] for row in ids], dtype=np.int32)
            got = torch.full((T, m.hidden), float("nan"), dtype=torch.float32, device="cuda")
            rc = fn(C.byref(arena.desc), slab, record, n_slots, x.data_ptr(), slots.ctypes.data, w.data_ptr(), k, T,
                    got.data_ptr(), stream.cuda_stream)
            assert rc == L.GX_OK, (call, rc)
            torch.cuda.synchronize()
            g = got.cpu().numpy()
            np.testing.assert_array_equal(g.view(np.uint32), want.cpu().numpy().view(np.uint32), err_msg=f"call {call}")
            oracle = orc.moe_layer(m, recs, xh, ids, wh)
            np.testing.assert_array_equal(g.view(np.uint32), oracle.view(np.uint32), err_msg=f"oracle call {call}")
        from galactus_b200.moe import device_error
        assert device_error() == 0
    finally:
        arena.close()
