"""GGUF tier loading: a checkpoint written by gguf-py with routed-expert
tensors blk.L.ffn_{down,gate,up}_exps.weight (the synthetic model's bytes)
gives the geometry, and loaded into an arena's host tier gives records equal,
byte for byte and by FNV-1a 64, to the record layout down | gate | up."""
import ctypes as C

import numpy as np
import pytest


def _fnv1a64(data: bytes) -> int:
    h = 14695981039346656037
    for b in data:
        h = ((h ^ b) * 1099511628211) & ((1 << 64) - 1)
    return h


def _write_moe_gguf(path, m, orc, layers, first_layer=0, extra_dense=True):
    from gguf import GGMLQuantizationType, GGUFWriter
    w = GGUFWriter(str(path), "qwen3moe")
    w.add_block_count(first_layer + layers)
    w.add_expert_count(m.experts)
    w.add_expert_used_count(m.used)
    w.add_string("general.name", "synthetic-moe")
    w.add_array("tokenizer.ggml.tokens", ["a", "b", "c"])
    if extra_dense:
        w.add_tensor("token_embd.weight", np.zeros((4, m.hidden), np.float32))
    for L in range(first_layer, first_layer + layers):
        for role, t, ne0, rows, r in (("down", m.type_down, m.intermediate, m.hidden, 0),
                                      ("gate", m.type_gate, m.hidden, m.intermediate, 1),
                                      ("up", m.type_up, m.hidden, m.intermediate, 2)):
            per = np.stack([orc.synth_weights(t, ne0, rows, m.seed, (L * m.experts + e) * 3 + r)
                            for e in range(m.experts)])
            w.add_tensor(f"blk.{L}.ffn_{role}_exps.weight", per.reshape(m.experts, rows, -1),
                         raw_dtype=GGMLQuantizationType(t))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_fnv1a64_vectors(gxlib):
    lib = gxlib.lib()
    for data in (b"", b"a", b"foobar", bytes(range(256)) * 3):
        buf = C.create_string_buffer(data, len(data))
        assert lib.gx_fnv1a64(buf, len(data)) == _fnv1a64(data)
    assert lib.gx_fnv1a64(C.create_string_buffer(b"", 0), 0) == 0xcbf29ce484222325


@pytest.mark.parametrize("name", ["qwen3-30b", "olmoe"])
def test_gguf_moe_info(gxlib, orc, tmp_path, name):
    from galactus_b200 import _lib as L
    from galactus_b200.models import ModelShape
    m = ModelShape(**{**gxlib.MODELS[name].__dict__, "experts": 6, "layers": 3})
    path = tmp_path / "m.gguf"
    _write_moe_gguf(path, m, orc, layers=2, first_layer=1)
    info = L.gx_gguf_moe()
    L.check(gxlib.lib().gx_gguf_moe_info(str(path).encode(), C.byref(info)), "gx_gguf_moe_info")
    assert info.arch.decode() == "qwen3moe"
    assert (info.first_layer, info.last_layer, info.experts, info.used, info.block_count) == (1, 2, 6, m.used, 3)
    assert (info.type_gate, info.type_up, info.type_down) == (m.type_gate, m.type_up, m.type_down)
    assert (info.hidden, info.intermediate) == (m.hidden, m.intermediate)
    assert info.record_bytes == m.record and info.record_bytes_raw == m.record_raw


def test_gguf_rejects_non_gguf_and_dense(gxlib, tmp_path):
    from galactus_b200 import _lib as L
    bad = tmp_path / "x.gguf"
    bad.write_bytes(b"NOTGGUF" + bytes(64))
    info = L.gx_gguf_moe()
    assert gxlib.lib().gx_gguf_moe_info(str(bad).encode(), C.byref(info)) == L.GX_ERR_INVALID
    from gguf import GGUFWriter
    dense = tmp_path / "dense.gguf"
    w = GGUFWriter(str(dense), "llama")
    w.add_block_count(1)
    w.add_tensor("blk.0.ffn_down.weight", np.zeros((8, 32), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    assert gxlib.lib().gx_gguf_moe_info(str(dense).encode(), C.byref(info)) == L.GX_ERR_INVALID


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["qwen3-30b", "gpt-oss-120b"])
def test_gguf_loads_the_tier(gxlib, orc, dev, tmp_path, name):
    from galactus_b200.models import ModelShape
    base = gxlib.MODELS[name]
    m = ModelShape(**{**base.__dict__, "experts": base.used + 2, "layers": 2})
    path = tmp_path / "m.gguf"
    _write_moe_gguf(path, m, orc, layers=2)
    arena = gxlib.Arena(m, capacity_bytes=m.experts * m.record * m.layers, policy=gxlib.POLICY_AUTO, max_tokens=1)
    n = C.c_uint32()
    gxlib.check(gxlib.lib().gx_arena_load_gguf(arena.h, str(path).encode(), C.byref(n)), "gx_arena_load_gguf")
    assert n.value == m.experts * m.layers
    stream = torch_stream()
    arena.warm_all(stream)
    for L in range(m.layers):
        for e in range(m.experts):
            got = arena.read_slot(L, arena.slot_of(L, e))
            want = orc.synth_record(m, m.seed, L, e)
            assert np.array_equal(got[:m.record_raw], want[:m.record_raw]), (L, e)
            assert gxlib.lib().gx_fnv1a64(got.ctypes.data, m.record_raw) == _fnv1a64(want[:m.record_raw].tobytes())
    arena.close()


def torch_stream():
    import torch
    return torch.cuda.current_stream()
