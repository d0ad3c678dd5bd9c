"""TEST INFRASTRUCTURE ONLY -- Python face of the CPU oracle.

Loads oracle/liboracle.so (built by oracle/Makefile from gx_oracle.cpp) and
runs oracle/_ref/h4ref_replay (the reference's own slot policy). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module;
the product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_REPLAY = HERE / "_ref" / "h4ref_replay"
GRID_FIXTURE = HERE.parent / "tests" / "golden" / "iq1s_grid.npy"

Q8_0, Q4_K, Q6_K, Q8_K, IQ1_S, MXFP4 = 8, 12, 14, 15, 19, 39
BLOCK_BYTES = {Q8_0: 34, Q8_K: 292, Q4_K: 144, Q6_K: 210, MXFP4: 17, IQ1_S: 50}
BLOCK_ELEMS = {Q8_0: 32, Q8_K: 256, Q4_K: 256, Q6_K: 256, MXFP4: 32, IQ1_S: 256}


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


class LayerDesc(C.Structure):
    _fields_ = [("type_gate", C.c_int32), ("type_up", C.c_int32), ("type_down", C.c_int32), ("act", C.c_int32),
                ("alpha", C.c_float), ("limit", C.c_float), ("H", C.c_int64), ("I", C.c_int64),
                ("off_gate", C.c_int64), ("off_up", C.c_int64), ("record_bytes", C.c_int64), ("n_experts", C.c_int64)]


class RouterDesc(C.Structure):
    """gating (0 softmax, 1 sigmoid, 2 softmax over the selected), experts, k,
    groups, groups kept, norm_w, scale_w, w_scale (layout of gx_router_desc)."""
    _fields_ = [("gating", C.c_int32), ("n_expert", C.c_int32), ("n_expert_used", C.c_int32),
                ("n_groups", C.c_int32), ("n_group_used", C.c_int32), ("norm_w", C.c_int32),
                ("scale_w", C.c_int32), ("w_scale", C.c_float)]


_P = C.c_void_p
_I64 = C.c_int64
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        h = C.CDLL(str(LIB))
        h.orc_fp16_to_fp32.restype = C.c_float
        h.orc_fp16_to_fp32.argtypes = [C.c_uint16]
        h.orc_fp32_to_fp16.restype = C.c_uint16
        h.orc_fp32_to_fp16.argtypes = [C.c_float]
        h.orc_quantize_q8_0.argtypes = [_P, _I64, _P]
        h.orc_quantize_q8_K.argtypes = [_P, _I64, _P]
        h.orc_vec_dot.restype = C.c_float
        h.orc_vec_dot.argtypes = [C.c_int, _I64, _P, _P]
        h.orc_dequantize_row.argtypes = [C.c_int, _P, _P, _I64]
        h.orc_expf.restype = C.c_float
        h.orc_expf.argtypes = [C.c_float]
        h.orc_expf_many.argtypes = [_P, _P, _I64]
        h.orc_swiglu.argtypes = [_P, _P, _P, _I64]
        h.orc_swiglu_oai.argtypes = [_P, _P, _P, _I64, C.c_float, C.c_float]
        h.orc_combine.argtypes = [_P, _P, _P, _I64, _I64, _I64]
        h.orc_mul_mat_id.restype = C.c_int
        h.orc_mul_mat_id.argtypes = [C.c_int, _P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P, _I64,
                                     _I64, _P, C.c_int]
        h.orc_moe_layer.restype = C.c_int
        h.orc_moe_layer.argtypes = [C.POINTER(LayerDesc), _P, _P, _P, _P, _I64, _I64, _P, C.c_int]
        h.orc_set_iq1s_grid.argtypes = [_P]
        h.orc_router_valid.restype = C.c_int
        h.orc_router_valid.argtypes = [C.POINTER(RouterDesc)]
        h.orc_router.restype = C.c_int
        h.orc_router.argtypes = [C.POINTER(RouterDesc), _P, _I64, _P, _I64, _I64, _P, _P]
        h.orc_synth_normal.argtypes = [_P, _I64, C.c_uint64, C.c_uint64, C.c_float]
        h.orc_synth_weights.restype = C.c_int
        h.orc_synth_weights.argtypes = [C.c_int, _P, _I64, _I64, C.c_uint64, C.c_uint64, C.c_float]
        grid = iq1s_grid()
        h.orc_set_iq1s_grid(grid.ctypes.data)
        _lib = h
    return _lib


def iq1s_grid() -> np.ndarray:
    """int8 [2048, 8] IQ1_S codebook, from the committed fixture (made from gguf-py)."""
    g = np.load(GRID_FIXTURE)
    assert g.shape == (2048, 8) and g.dtype == np.int8
    return np.ascontiguousarray(g)


def nthreads() -> int:
    return max(1, os.cpu_count() or 1)


def row_bytes(t: int, n: int) -> int:
    return (n // BLOCK_ELEMS[t]) * BLOCK_BYTES[t]


def fp32_to_fp16(x: float) -> int:
    return lib().orc_fp32_to_fp16(x)


def quantize(vdt: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    rows = x.reshape(-1, n)
    out = np.zeros((rows.shape[0], row_bytes(vdt, n)), dtype=np.uint8)
    fn = lib().orc_quantize_q8_0 if vdt == Q8_0 else lib().orc_quantize_q8_K
    for i in range(rows.shape[0]):
        fn(rows[i].ctypes.data, n, out[i].ctypes.data)
    return out


def vec_dot(t: int, n: int, wrow: np.ndarray, yrow: np.ndarray) -> float:
    return lib().orc_vec_dot(t, n, wrow.ctypes.data, yrow.ctypes.data)


def dequantize_row(t: int, data: np.ndarray, n: int) -> np.ndarray:
    out = np.zeros(n, dtype=np.float32)
    lib().orc_dequantize_row(t, np.ascontiguousarray(data).ctypes.data, out.ctypes.data, n)
    return out


def expf(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_expf_many(x.ctypes.data, y.ctypes.data, x.size)
    return y


def act_exp_libm(on: bool) -> None:
    """Swap the exp inside the oracle's activations for the C library's expf
    (True) or back to the shared one (False)."""
    lib().orc_act_exp_libm(1 if on else 0)


def swiglu(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32); u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    lib().orc_swiglu(g.ctypes.data, u.ctypes.data, out.ctypes.data, g.size)
    return out


def swiglu_oai(g, u, alpha=1.702, limit=7.0):
    g = np.ascontiguousarray(g, dtype=np.float32); u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    lib().orc_swiglu_oai(g.ctypes.data, u.ctypes.data, out.ctypes.data, g.size, alpha, limit)
    return out


def combine(y: np.ndarray, w: np.ndarray) -> np.ndarray:
    """y [T, k, H], w [T, k] -> [T, H]"""
    y = np.ascontiguousarray(y, dtype=np.float32); w = np.ascontiguousarray(w, dtype=np.float32)
    T, k, H = y.shape
    out = np.zeros((T, H), dtype=np.float32)
    lib().orc_combine(y.ctypes.data, w.ctypes.data, out.ctypes.data, H, k, T)
    return out


def router(desc: RouterDesc, logits: np.ndarray, bias: np.ndarray | None = None,
           n_layers: int = 1) -> tuple[np.ndarray, np.ndarray]:
    """logits f32 [n_layers*T, E], bias f32 [n_layers, E] or None ->
    ids int32 [n_layers*T, k], weights f32 [n_layers*T, k]"""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, E = logits.shape
    T = rows // n_layers
    k = desc.n_expert_used
    ids = np.zeros((rows, k), np.int32)
    w = np.zeros((rows, k), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rc = lib().orc_router(C.byref(desc), logits.ctypes.data, E, None if b is None else b.ctypes.data, T, n_layers,
                          ids.ctypes.data, w.ctypes.data)
    if rc != 0:
        raise ValueError("oracle router: invalid description")
    return ids, w


def mul_mat_id(t: int, experts: np.ndarray, ne00: int, ne01: int, b: np.ndarray, ids: np.ndarray,
               nb01: int | None = None, threads: int | None = None) -> np.ndarray:
    """experts: uint8 [n_as, nb02] (row r of expert e at e*nb02 + r*nb01);
    b: f32 [T, ne11, ne00]; ids: int32 [T, k] -> f32 [T, k, ne01]"""
    experts = np.ascontiguousarray(experts, dtype=np.uint8)
    b = np.ascontiguousarray(b, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    n_as, nb02 = experts.shape
    T, ne11, _ = b.shape
    k = ids.shape[1]
    nb01 = nb01 or row_bytes(t, ne00)
    dst = np.zeros((T, k, ne01), dtype=np.float32)
    rc = lib().orc_mul_mat_id(t, experts.ctypes.data, ne00, ne01, nb01, nb02, n_as, b.ctypes.data, ne11, T,
                              ne00 * 4, ne00 * ne11 * 4, ids.ctypes.data, k, k * 4, dst.ctypes.data,
                              threads or nthreads())
    if rc != 0:
        raise ValueError("oracle mul_mat_id: expert id out of range")
    return dst


def moe_layer(model, records: np.ndarray, x: np.ndarray, ids: np.ndarray, w: np.ndarray,
              threads: int | None = None) -> np.ndarray:
    """records: uint8 [n_experts, record]; x [T, H]; ids [T, k]; w [T, k] -> [T, H]"""
    records = np.ascontiguousarray(records, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, k = ids.shape
    d = LayerDesc(model.type_gate, model.type_up, model.type_down, model.act, model.alpha, model.limit,
                  model.hidden, model.intermediate, model.off_gate, model.off_up, records.shape[1], records.shape[0])
    out = np.zeros((T, model.hidden), dtype=np.float32)
    rc = lib().orc_moe_layer(C.byref(d), records.ctypes.data, x.ctypes.data, ids.ctypes.data, w.ctypes.data, k, T,
                             out.ctypes.data, threads or nthreads())
    if rc != 0:
        raise ValueError("oracle moe_layer failed")
    return out


def synth_normal(n: int, seed: int, stream_id: int, sigma: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_synth_normal(out.ctypes.data, n, seed, stream_id, sigma)
    return out


def synth_weights(t: int, ne00: int, n_rows: int, seed: int, stream_id: int, sigma: float = 0.02) -> np.ndarray:
    out = np.zeros(row_bytes(t, ne00) * n_rows, dtype=np.uint8)
    rc = lib().orc_synth_weights(t, out.ctypes.data, ne00, n_rows, seed, stream_id, sigma)
    if rc != 0:
        raise ValueError("oracle synth_weights: bad type or size")
    return out


def synth_record(model, seed: int, layer: int, expert: int) -> np.ndarray:
    """One padded record (down | gate | up) of the synthetic model, the same
    streams the benchmark uses: stream id = (layer*experts + expert)*3 + role."""
    rec = np.zeros(model.record, dtype=np.uint8)
    base = (layer * model.experts + expert) * 3
    down = synth_weights(model.type_down, model.intermediate, model.hidden, seed, base + 0)
    gate = synth_weights(model.type_gate, model.hidden, model.intermediate, seed, base + 1)
    up = synth_weights(model.type_up, model.hidden, model.intermediate, seed, base + 2)
    rec[:down.size] = down
    rec[model.off_gate:model.off_gate + gate.size] = gate
    rec[model.off_up:model.off_up + up.size] = up
    return rec


# ------------------------------------------------------------- policy oracle

def ref_replay_available() -> bool:
    return REF_REPLAY.exists()


def ref_replay(first_layer: int, last_layer: int, experts: int, used: int, capacity_bytes: int, fraction: float,
               policy: str, batches: list[tuple[int, list[int]]], record: int = 16384):
    """Run the reference's ExpertCache/ExpertStore on a trace of micro-batches.
    Returns (quotas per layer, [(hits, evicted, slots, resident)] per batch)."""
    if not REF_REPLAY.exists():
        build()
    with tempfile.TemporaryDirectory() as td:
        prof = Path(td) / "profile.txt"
        lines = ["galactus-profile 1", "arch synthetic", f"first_layer {first_layer}", f"last_layer {last_layer}",
                 f"experts {experts}", f"used {used}", "align 16384"]
        lines += [f"layer {l} record {record} raw {record}" for l in range(first_layer, last_layer + 1)]
        lines.append("end")
        prof.write_text("\n".join(lines) + "\n")
        inp = [f"{capacity_bytes} {fraction!r} {len(batches)}"]
        for layer, ex in batches:
            inp.append(f"{layer} {len(ex)} " + " ".join(str(e) for e in ex))
        env = dict(os.environ, GALACTUS_PROFILE=str(prof), GALACTUS_H4_CACHE_POLICY=policy)
        env.pop("GALACTUS_H4_CACHE_PLAN", None)
        r = subprocess.run([str(REF_REPLAY)], input="\n".join(inp) + "\n", capture_output=True, text=True, env=env,
                           check=True, cwd=td)
    out = r.stdout.splitlines()
    quotas = [tuple(int(v) for v in tok.split(":")) for tok in out[0].split()[1:]]
    res = []
    i = 1
    while i < len(out):
        _, layer, count = out[i].split()
        count = int(count)
        acc = [tuple(int(v) for v in out[i + 1 + j].split()[1:]) for j in range(count)]
        slots = [int(v) for v in out[i + 1 + count].split()[1:]]
        resident = [int(v) for v in out[i + 2 + count].split()[1:]]
        res.append(([a[0] == 1 for a in acc], [a[2] if a[1] else -1 for a in acc], slots, resident))
        i += 3 + count
    return quotas, res
