"""Router on the device (the step before the routed-expert FFN): logits to
selected expert ids and weights as upstream build_moe_ffn computes them.

CPU: the oracle (orc_router) is pinned against a second, independent
restatement in numpy written from the same published graph (softmax in the
arm64 order with the shared expf, sigmoid, selection bias, group-limited
selection, descending top-k with ties to the lower id, SOFTMAX_WEIGHT,
norm_w, scale_w), bit for bit; the C-ABI refuses the descriptions the oracle
refuses. GPU: gx_router_forward equals the oracle bit for bit over every
gating form, expert counts with and without a tail of four, strided logits
and several layers; gx_stack_plan_run_routed (router + stack with no host
round trip) equals the host-routed plan and the oracle layer."""
import ctypes as C

import numpy as np
import pytest

SOFTMAX, SIGMOID, SOFTMAX_WEIGHT = 0, 1, 2

# (label, gating, E, k, groups, group_used, norm_w, w_scale, bias)
SCHEMES = [
    ("olmoe", SOFTMAX, 64, 8, 0, 0, False, None, False),
    ("qwen3", SOFTMAX, 128, 8, 0, 0, True, None, False),
    ("gpt-oss", SOFTMAX_WEIGHT, 128, 4, 0, 0, False, None, False),
    ("deepseek-v3", SIGMOID, 256, 8, 8, 4, True, 2.5, True),
    ("sigmoid-flat", SIGMOID, 160, 6, 0, 0, True, None, True),
    ("tail-of-four", SOFTMAX, 1001, 32, 0, 0, True, 1.5, False),
    ("max-experts", SOFTMAX, 1024, 1, 0, 0, False, None, False),
    ("groups-32", SIGMOID, 1024, 16, 32, 3, False, None, True),
]


def _desc(orc, gating, E, k, groups, group_used, norm_w, w_scale):
    return orc.RouterDesc(gating, E, k, groups, group_used, 1 if norm_w else 0, 0 if w_scale is None else 1,
                          1.0 if w_scale is None else w_scale)


def _logits(rng, rows, E):
    """N(0,1) plus the log of a Zipf(1.1) weight of a permuted rank, per row."""
    w = 1.0 / np.arange(1, E + 1) ** 1.1
    w /= w.sum()
    bias = np.log(w)[rng.permutation(E)]
    return (rng.standard_normal((rows, E)) + bias).astype(np.float32)


# ------------------------------------------------ numpy restatement (CPU)

def _np_soft_max(x, expf):
    x = np.asarray(x, np.float32)
    m = np.float32(x.max())
    e = expf((x - m).astype(np.float32))
    s = 0.0
    nc = len(x) // 4
    for c in range(nc):
        v = e[4 * c:4 * c + 4]
        s += float(np.float32(np.float32(v[0] + v[1]) + np.float32(v[2] + v[3])))
    for j in range(4 * nc, len(x)):
        s += float(e[j])
    inv = np.float32(1.0 / s)
    return (e * inv).astype(np.float32)


def _np_router(orc, gating, E, k, groups, group_used, norm_w, w_scale, logits, bias, T):
    ids = np.zeros((logits.shape[0], k), np.int32)
    wts = np.zeros((logits.shape[0], k), np.float32)
    one = np.float32(1.0)
    for row, x in enumerate(logits):
        if gating == SIGMOID:
            probs = (one / (one + orc.expf(-x))).astype(np.float32)
        elif gating == SOFTMAX:
            probs = _np_soft_max(x, orc.expf)
        else:
            probs = x.copy()
        sel = probs + bias[row // T] if bias is not None else probs.copy()
        sel = sel.astype(np.float32)
        if groups > 1:
            gs = E // groups
            g = sel.reshape(groups, gs)
            top2 = np.sort(g, axis=1)[:, -2:]
            score = (top2[:, 1] + top2[:, 0]).astype(np.float32)
            keep = np.argsort(-score, kind="stable")[:group_used]
            mask = np.zeros(groups, bool)
            mask[keep] = True
            sel = np.where(np.repeat(mask, gs), sel, np.float32(-np.inf)).astype(np.float32)
        top = np.argsort(-sel, kind="stable")[:k]
        w = probs[top].astype(np.float32)
        if gating == SOFTMAX_WEIGHT:
            w = _np_soft_max(w, orc.expf)
        if norm_w:
            s = np.float32(sum(float(v) for v in w))
            s = s if s > np.float32(6.103515625e-5) else np.float32(6.103515625e-5)
            w = (w / s).astype(np.float32)
        if w_scale is not None:
            w = (w * np.float32(w_scale)).astype(np.float32)
        ids[row] = top
        wts[row] = w
    return ids, wts


@pytest.mark.parametrize("scheme", SCHEMES, ids=[s[0] for s in SCHEMES])
def test_oracle_router_matches_numpy_restatement(orc, scheme):
    _, gating, E, k, G, gu, norm_w, w_scale, with_bias = scheme
    rng = np.random.default_rng(E * 31 + k)
    T, n_layers = 5, 2
    logits = _logits(rng, T * n_layers, E)
    bias = (0.1 * rng.standard_normal((n_layers, E))).astype(np.float32) if with_bias else None
    d = _desc(orc, gating, E, k, G, gu, norm_w, w_scale)
    ids, w = orc.router(d, logits, bias, n_layers=n_layers)
    ids2, w2 = _np_router(orc, gating, E, k, G, gu, norm_w, w_scale, logits, bias, T)
    np.testing.assert_array_equal(ids, ids2)
    np.testing.assert_array_equal(w.view(np.uint32), w2.view(np.uint32))
    if G > 1:
        gs = E // G
        for row in ids:
            assert len(set((row // gs).tolist())) <= gu


def test_oracle_router_ties_go_to_the_lower_id(orc):
    d = _desc(orc, SOFTMAX, 64, 8, 0, 0, True, None)
    ids, w = orc.router(d, np.zeros((2, 64), np.float32))
    assert ids.tolist() == [list(range(8))] * 2
    assert np.all(w == np.float32(1 / 8))
    # equal group scores: the lower groups are kept
    d = _desc(orc, SIGMOID, 64, 4, 8, 2, False, None)
    ids, _ = orc.router(d, np.zeros((1, 64), np.float32))
    assert ids.tolist() == [[0, 1, 2, 3]]


BAD = [
    (3, 64, 8, 0, 0),       # gating
    (0, 64, 0, 0, 0),       # k = 0
    (0, 64, 33, 0, 0),      # k > 32
    (0, 4, 8, 0, 0),        # k > E
    (0, 2048, 8, 0, 0),     # E > 1024
    (1, 96, 8, 7, 4),       # E % groups
    (1, 64, 8, 64, 8),      # groups > 32 (and one expert per group)
    (1, 64, 8, 8, 0),       # no group kept
    (1, 64, 8, 8, 9),       # more groups kept than exist
    (1, 64, 20, 8, 2),      # kept groups hold fewer than k experts
]


def test_router_rejects_what_the_oracle_rejects(gxlib, orc):
    from galactus_b200 import _lib as L
    lib = gxlib.lib()
    for g, E, k, G, gu in BAD:
        d = L.gx_router_desc(g, E, k, G, gu, 0, 0, 1.0)
        assert orc.lib().orc_router_valid(C.byref(orc.RouterDesc(g, E, k, G, gu, 0, 0, 1.0))) == 0
        # validated before any device work: no GPU needed
        rc = lib.gx_router_forward(C.byref(d), 8, E, None, 1, 1, 8, 8, None, None, None)
        assert rc == L.GX_ERR_INVALID, (g, E, k, G, gu)
    for _, g, E, k, G, gu, *_ in SCHEMES:
        assert orc.lib().orc_router_valid(C.byref(orc.RouterDesc(g, E, k, G, gu, 0, 0, 1.0))) == 1


# ------------------------------------------------------------------- GPU

def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.gpu
@pytest.mark.parametrize("T,n_layers,pad", [(1, 1, 0), (7, 3, 0), (64, 2, 5)])
@pytest.mark.parametrize("scheme", SCHEMES, ids=[s[0] for s in SCHEMES])
def test_router_bitwise_vs_oracle(gxlib, orc, dev, scheme, T, n_layers, pad):
    import torch
    from galactus_b200.moe import route, router_desc, device_error
    _, gating, E, k, G, gu, norm_w, w_scale, with_bias = scheme
    rng = np.random.default_rng(E + 7 * T + n_layers)
    logits = _logits(rng, T * n_layers, E)
    bias = (0.1 * rng.standard_normal((n_layers, E))).astype(np.float32) if with_bias else None
    want_ids, want_w = orc.router(_desc(orc, gating, E, k, G, gu, norm_w, w_scale), logits, bias, n_layers=n_layers)
    # strided logits rows (ld = E + pad)
    buf = torch.full((T * n_layers, E + pad), float("nan"), dtype=torch.float32, device=dev)
    buf[:, :E] = torch.from_numpy(logits)
    lg = buf[:, :E]
    bd = torch.from_numpy(bias).to(dev) if bias is not None else None
    d = router_desc(gating, E, k, groups=G, group_used=gu, norm_w=norm_w, w_scale=w_scale)
    ids, w = route(d, lg, bd, n_layers=n_layers)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), want_ids)
    np.testing.assert_array_equal(_bits(w.cpu().numpy()), _bits(want_w))
    assert device_error() == 0


@pytest.mark.gpu
def test_router_maps_ids_to_slots(gxlib, orc, dev):
    """With the arena's slot table the router also writes each id's slot; an
    expert without a slot gives -1 and the device error word, never a read."""
    import torch
    from galactus_b200.models import ModelShape
    from galactus_b200.moe import device_error, model_router, route, slot_table
    base = gxlib.MODELS["qwen3-30b"]
    m = ModelShape(**{**base.__dict__, "experts": 16, "layers": 2})
    arena = gxlib.Arena(m, capacity_bytes=m.experts * m.record * m.layers, policy=gxlib.POLICY_AUTO, max_tokens=4)
    for L in range(m.layers):
        for e in range(m.experts):
            arena.load_record(L, e, orc.synth_record(m, m.seed, L, e))
    from galactus_b200._lib import GxError, GX_ERR_STATE
    with pytest.raises(GxError) as ei:
        slot_table(arena, 0, m.layers, require_all=True)
    assert ei.value.code == GX_ERR_STATE
    stream = torch.cuda.current_stream()
    arena.warm_all(stream)
    table = slot_table(arena, 0, m.layers, require_all=True)
    tab = table.cpu().numpy()
    assert sorted(tab[0].tolist()) == list(range(m.experts))
    rng = np.random.default_rng(3)
    logits = torch.from_numpy(_logits(rng, 4 * m.layers, m.experts)).to(dev)
    slots = torch.empty((4 * m.layers, m.used), dtype=torch.int32, device=dev)
    ids, _ = route(model_router(m), logits, n_layers=m.layers, slot_table=table, slots=slots)
    torch.cuda.synchronize()
    ids_h, slots_h = ids.cpu().numpy(), slots.cpu().numpy()
    for row in range(4 * m.layers):
        assert slots_h[row].tolist() == [int(tab[row // 4, e]) for e in ids_h[row]]
    assert device_error() == 0
    # a table with a hole: the router reports it
    holes = table.clone()
    holes[:, :] = -1
    route(model_router(m), logits, n_layers=m.layers, slot_table=holes, slots=slots)
    torch.cuda.synchronize()
    assert device_error() == 1 and (slots.cpu().numpy() == -1).all()
    arena.close()


@pytest.mark.gpu
@pytest.mark.parametrize("name,T", [("qwen3-30b", 1), ("qwen3-30b", 4), ("olmoe", 2)])
def test_stack_plan_run_routed(gxlib, orc, dev, tmp_path, name, T):
    """Router + stack plan with no host round trip: the ids equal the oracle
    router's, and the outputs equal the oracle layer on those routes, bit for
    bit. A non-pinned arena is refused; with a route trace open the served
    ids are recorded."""
    import torch
    from galactus_b200._lib import GX_ERR_STATE, GxError
    from galactus_b200.models import ModelShape
    from galactus_b200.moe import StackPlan, device_error, model_router
    from galactus_b200.route_trace import close_trace, open_trace, read_trace
    base = gxlib.MODELS[name]
    m = ModelShape(**{**base.__dict__, "experts": 16, "layers": 3})
    k = m.used
    recs = [np.stack([orc.synth_record(m, m.seed, L, e) for e in range(m.experts)]) for L in range(m.layers)]

    def make_arena(slots):
        a = gxlib.Arena(m, capacity_bytes=slots * m.record * m.layers, policy=gxlib.POLICY_AUTO, max_tokens=T)
        for L in range(m.layers):
            for e in range(m.experts):
                a.load_record(L, e, recs[L][e])
        return a

    x = torch.zeros((m.layers, T, m.hidden), dtype=torch.float32, device=dev)
    w = torch.zeros((m.layers, T, k), dtype=torch.float32, device=dev)
    out = torch.zeros((m.layers, T, m.hidden), dtype=torch.float32, device=dev)
    ptr = lambda t: [t[L].data_ptr() for L in range(m.layers)]
    desc = model_router(m)
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(11 + T)

    small = make_arena(k + 2)
    plan = StackPlan(small, 0, m.layers, ptr(x), ptr(w), ptr(out), k, T)
    lg = torch.from_numpy(_logits(rng, m.layers * T, m.experts)).to(dev)
    with pytest.raises(GxError) as ei:
        plan.run_routed(desc, lg, stream=stream)
    assert ei.value.code == GX_ERR_STATE
    plan.close()
    small.close()

    arena = make_arena(m.experts)
    arena.warm_all(stream)
    plan = StackPlan(arena, 0, m.layers, ptr(x), ptr(w), ptr(out), k, T)
    ids_d = torch.empty((m.layers * T, k), dtype=torch.int32, device=dev)
    trace = tmp_path / "routes.txt"
    for step in range(4):
        logits = _logits(rng, m.layers * T, m.experts)
        xs = rng.standard_normal((m.layers, T, m.hidden)).astype(np.float32)
        x.copy_(torch.from_numpy(xs))
        out.fill_(float("nan"))
        if step == 3:
            open_trace(str(trace), arch=name)
        st = plan.run_routed(desc, torch.from_numpy(logits).to(dev), ids_out=ids_d, stream=stream)
        if step == 3:
            close_trace()
        torch.cuda.synchronize()
        assert st.hits == m.layers * T * k and st.misses == 0
        want_ids, want_w = orc.router(desc_oracle(orc, desc), logits, None, n_layers=m.layers)
        np.testing.assert_array_equal(ids_d.cpu().numpy(), want_ids)
        np.testing.assert_array_equal(_bits(w.cpu().numpy().reshape(-1, k)), _bits(want_w))
        got = out.cpu().numpy()
        for L in range(m.layers):
            want = orc.moe_layer(m, recs[L], xs[L], want_ids[L * T:(L + 1) * T], want_w[L * T:(L + 1) * T])
            np.testing.assert_array_equal(_bits(got[L]), _bits(want), err_msg=f"{name} T={T} step {step} layer {L}")
        assert device_error() == 0
    tr = read_trace(str(trace))
    assert len(tr["entries"]) == m.layers
    for L, e in enumerate(tr["entries"]):
        assert e["layer"] == L and e["ids"] == want_ids[L * T:(L + 1) * T].ravel().tolist()
        assert all(r == 1 for r in e["resident"])
    plan.close()
    arena.close()


def desc_oracle(orc, d):
    return orc.RouterDesc(d.gating, d.n_expert, d.n_expert_used, d.n_groups, d.n_group_used, d.norm_w, d.scale_w,
                          d.w_scale)
