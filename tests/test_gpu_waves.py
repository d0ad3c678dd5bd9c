"""Micro-batches with more distinct experts than the slot policy serves at once
(min(quota, probation) per layer, the reference's micro-batch bound,
src/h4/h4-expert-cache.cpp:105-124) run in expert-major waves; the layer
output is bit-identical to the oracle's one-shot layer. The shapes are the
benchmark configurations' own: real expert counts (128 and 256, so slot ids
and slab offsets are wide) and their small slot caches (10 slots per layer
for gpt-oss-120b at 5 GB and Qwen3-235B-A22B at 12 GB per GPU)."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def fill_tier_on_device(gxlib, arena, m, layer=0):
    """Every record of `layer` written into the arena's pinned host tier by the
    library's generator (the same bytes as the oracle's synth_record, pinned
    by test_synth_weights_bytes), returned as an [E, record] view."""
    lib = gxlib.lib()
    stage = torch.empty(m.record, dtype=torch.uint8, device="cuda")
    for e in range(m.experts):
        stage.zero_()
        sid = (layer * m.experts + e) * 3
        base = stage.data_ptr()
        gxlib.check(lib.gx_synth_weights(m.type_down, base, m.intermediate, m.hidden, m.seed, sid + 0, 0.02, None))
        gxlib.check(lib.gx_synth_weights(m.type_gate, base + m.off_gate, m.hidden, m.intermediate, m.seed, sid + 1,
                                         0.02, None))
        gxlib.check(lib.gx_synth_weights(m.type_up, base + m.off_up, m.hidden, m.intermediate, m.seed, sid + 2, 0.02,
                                         None))
        torch.cuda.synchronize()
        arena.host_record(layer, e)[:] = stage.cpu().numpy()
    p = arena.host_record_ptr(layer, 0)
    return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(m.experts, m.record))


def zipf_routes(rng, T, experts, k):
    p = 1.0 / np.arange(1, experts + 1) ** 1.1
    p /= p.sum()
    perm = rng.permutation(experts)          # popular experts spread over the id range
    ids = np.stack([perm[rng.choice(experts, k, replace=False, p=p)] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    return ids, (w / w.sum(axis=1, keepdims=True)).astype(np.float32)


@pytest.mark.parametrize("name,slots,batches", [
    ("gpt-oss-120b", 10, [8, 64, 1, 8]),     # BASELINE cfg 3 at 5 GB: 10 slots of 128, batches of 1, 8, 64
    ("qwen3-235b", 10, [32, 1, 32]),         # cfg 4: 10 slots per layer per GPU, batch-32 decode
    ("deepseek-v3", 29, [16, 1, 16]),        # cfg 5: 256 experts, batch-16 decode, 29 slots
])
def test_waves_real_expert_counts(gxlib, orc, dev, name, slots, batches):
    m = gxlib.MODELS[name].with_layers(1)
    k = m.used
    Tmax = max(batches)
    arena = gxlib.Arena(m, capacity_bytes=slots * m.record, policy=gxlib.POLICY_AUTO, max_tokens=Tmax)
    try:
        recs = fill_tier_on_device(gxlib, arena, m)
        q, _, prob = arena.quota(0)
        bound = min(q, prob)
        rng = np.random.default_rng(sum(map(ord, name)) + slots)
        stream = torch.cuda.current_stream()
        waved = 0
        for T in batches:
            ids, w = zipf_routes(rng, T, m.experts, k)
            waved += len(set(ids.ravel().tolist())) > bound
            x = rng.standard_normal((T, m.hidden)).astype(np.float32)
            out = torch.full((T, m.hidden), float("nan"), dtype=torch.float32, device=dev)
            st = arena.layer_forward(0, torch.from_numpy(x).to(dev), ids, torch.from_numpy(w).to(dev), out,
                                     stream=stream)
            torch.cuda.synchronize()
            want = orc.moe_layer(m, recs, x, ids, w)
            np.testing.assert_array_equal(bits(out.cpu().numpy()), bits(want), err_msg=f"{name} T={T}")
            assert st.distinct == len(set(ids.ravel().tolist()))
        assert waved > 0, "no batch exceeded the policy's batch bound"
        s = arena.stats()
        assert s["misses"] > 0 and s["evictions"] > 0
        from galactus_b200.moe import device_error
        assert device_error() == 0
    finally:
        arena.close()


def test_waves_match_one_shot_and_slots_stay_consistent(gxlib, orc, dev):
    """The same micro-batch through a cache that holds it whole (one shot) and
    through a 10-slot cache (waves) gives the same bits; afterwards every
    resident expert's slot holds its own record."""
    m = gxlib.MODELS["qwen3-30b"].with_layers(1).with_experts(64)
    k = m.used
    T = 12
    rng = np.random.default_rng(3)
    ids, w = zipf_routes(rng, T, m.experts, k)
    x = rng.standard_normal((T, m.hidden)).astype(np.float32)
    outs = []
    want = None
    for slots in (m.experts, 10):
        arena = gxlib.Arena(m, capacity_bytes=slots * m.record, policy=gxlib.POLICY_AUTO, max_tokens=T)
        try:
            recs = fill_tier_on_device(gxlib, arena, m)
            if want is None:
                want = orc.moe_layer(m, recs, x, ids, w)
            out = torch.zeros((T, m.hidden), dtype=torch.float32, device=dev)
            arena.layer_forward(0, torch.from_numpy(x).to(dev), ids, torch.from_numpy(w).to(dev), out,
                                stream=torch.cuda.current_stream())
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
            if slots == 10:
                for e in range(m.experts):
                    s = arena.slot_of(0, e)
                    if s >= 0:
                        np.testing.assert_array_equal(arena.read_slot(0, s), recs[e][:m.record_raw])
        finally:
            arena.close()
    np.testing.assert_array_equal(bits(outs[0]), bits(outs[1]))
    np.testing.assert_array_equal(bits(outs[1]), bits(want))
