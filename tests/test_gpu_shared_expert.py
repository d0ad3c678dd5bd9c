"""The shared expert of DeepSeek-V3-shaped layers (BASELINE cfg 5: 256 routed
IQ1_S experts plus one Q4_K shared expert): out = moe_out + shexp(x), the
upstream ggml_add(moe_out, ffn_shexp) after build_moe_ffn, bit-identical to
the oracle (routed layer, dense Q4_K FFN, one f32 add) at batch 1 and 16."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_shared_expert_bitwise(gxlib, orc, dev):
    from galactus_b200.models import ModelShape
    from galactus_b200.moe import shared_expert
    base = gxlib.MODELS["deepseek-v3"]
    m = base.with_layers(1).with_experts(24)
    k = m.used
    # the shared expert: one dense SwiGLU FFN, Q4_K gate/up/down, I = 2048
    ms = ModelShape("deepseek-v3-shared", 1, m.hidden, 1, 1, 2048, gxlib.TYPE_Q4_K, gxlib.TYPE_Q4_K, gxlib.TYPE_Q4_K,
                    seed=m.seed + 100)
    sh_rec = orc.synth_record(ms, ms.seed, 0, 0)
    sh_dev = torch.from_numpy(sh_rec).to(dev)
    sh = shared_expert(sh_dev, gxlib.TYPE_Q4_K, gxlib.TYPE_Q4_K, m.hidden, 2048)
    assert (sh.desc.off_gate, sh.desc.off_up) == (ms.off_gate, ms.off_up)
    arena = gxlib.Arena(m, capacity_bytes=m.experts * m.record, policy=gxlib.POLICY_AUTO, max_tokens=16)
    try:
        recs = np.stack([orc.synth_record(m, m.seed, 0, e) for e in range(m.experts)])
        for e in range(m.experts):
            arena.load_record(0, e, recs[e])
        rng = np.random.default_rng(77)
        stream = torch.cuda.current_stream()
        for T in (1, 16, 3):
            ids = np.stack([rng.choice(m.experts, k, replace=False) for _ in range(T)]).astype(np.int32)
            w = rng.random((T, k)).astype(np.float32)
            x = rng.standard_normal((T, m.hidden)).astype(np.float32)
            out = torch.full((T, m.hidden), float("nan"), dtype=torch.float32, device=dev)
            arena.layer_forward_shared(0, torch.from_numpy(x).to(dev), ids, torch.from_numpy(w).to(dev), sh, out,
                                       stream=stream)
            torch.cuda.synchronize()
            routed = orc.moe_layer(m, recs, x, ids, w)
            shexp = orc.moe_layer(ms, sh_rec[None], x, np.zeros((T, 1), np.int32), np.ones((T, 1), np.float32))
            want = (routed + shexp).astype(np.float32)
            np.testing.assert_array_equal(bits(out.cpu().numpy()), bits(want), err_msg=f"T={T}")
        from galactus_b200.moe import device_error
        assert device_error() == 0
    finally:
        arena.close()
