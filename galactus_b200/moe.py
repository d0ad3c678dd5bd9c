"""Python face of the C-ABI: the slot policy, the HBM arena with its host tier,
the remap node, mul_mat_id and the MoE layer entry point.

Device buffers are passed as raw device addresses (ints) or as objects with a
``data_ptr()`` method (torch tensors); streams as cudaStream_t handles (ints).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Sequence

import numpy as np

from . import _lib as L
from .models import ModelShape


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    if isinstance(x, np.ndarray):
        return int(x.ctypes.data)
    raise TypeError(f"cannot take the address of {type(x)}")


def _stream(s) -> int:
    if s is None:
        return 0
    if isinstance(s, int):
        return s
    if hasattr(s, "cuda_stream"):
        return int(s.cuda_stream)
    raise TypeError(f"not a stream: {type(s)}")


@dataclass(frozen=True)
class LayerShape:
    hidden: int
    intermediate: int
    type_gate: int
    type_up: int
    type_down: int
    act: int = L.ACT_SWIGLU
    alpha: float = 1.702
    limit: float = 7.0

    @staticmethod
    def of(m: ModelShape) -> "LayerShape":
        return LayerShape(m.hidden, m.intermediate, m.type_gate, m.type_up, m.type_down, m.act, m.alpha, m.limit)


def record_layout(m: ModelShape) -> dict:
    return {"down": (0, m.down_bytes), "gate": (m.off_gate, m.gate_bytes), "up": (m.off_up, m.up_bytes),
            "raw": m.record_raw, "record": m.record}


def _profile(first: int, last: int, experts: int, used: int, record: Sequence[int], raw: Sequence[int]):
    n = last - first + 1
    rec = (C.c_uint64 * n)(*record)
    rraw = (C.c_uint64 * n)(*raw)
    prof = L.gx_profile(first, last, experts, used, C.cast(rec, C.POINTER(C.c_uint64)),
                        C.cast(rraw, C.POINTER(C.c_uint64)))
    return prof, (rec, rraw)


class SlotPolicy:
    """Host-only slot policy and ledger (gx_policy_*)."""

    def __init__(self, first_layer: int, last_layer: int, experts: int, used: int, record_bytes: Sequence[int],
                 capacity_bytes: int, protected_fraction: float = 0.75, policy: int = L.POLICY_AUTO,
                 plan_quotas: Sequence[int] | None = None):
        self._lib = L.lib()
        prof, self._keep = _profile(first_layer, last_layer, experts, used, record_bytes, record_bytes)
        plan = None
        if plan_quotas is not None:
            plan = (C.c_uint32 * len(plan_quotas))(*plan_quotas)
        h = C.c_void_p()
        L.check(self._lib.gx_policy_create(C.byref(prof), capacity_bytes, protected_fraction, policy,
                                           C.cast(plan, C.POINTER(C.c_uint32)) if plan is not None else None,
                                           C.byref(h)), "gx_policy_create")
        self.h = h
        self.first_layer, self.last_layer, self.experts = first_layer, last_layer, experts

    def close(self):
        if self.h:
            self._lib.gx_policy_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def quota(self, layer: int) -> tuple[int, int, int]:
        q, p, b = C.c_uint32(), C.c_uint32(), C.c_uint32()
        L.check(self._lib.gx_policy_quota(self.h, layer, C.byref(q), C.byref(p), C.byref(b)), "gx_policy_quota")
        return q.value, p.value, b.value

    def serve(self, layer: int, experts: Sequence[int]):
        n = len(experts)
        ex = (C.c_int32 * max(n, 1))(*experts)
        slots = (C.c_int32 * max(n, 1))()
        hits = (C.c_uint8 * max(n, 1))()
        ev = (C.c_int32 * max(n, 1))()
        st = L.gx_serve_stats()
        rc = self._lib.gx_policy_serve(self.h, layer, ex, n, slots, hits, ev, C.byref(st))
        L.check(rc, "gx_policy_serve")
        return list(slots[:n]), [bool(h) for h in hits[:n]], list(ev[:n]), st

    def slot_of(self, layer: int, expert: int) -> int:
        return self._lib.gx_policy_slot_of(self.h, layer, expert)

    def counters(self) -> tuple[int, int, int]:
        a, b, c = C.c_uint64(), C.c_uint64(), C.c_uint64()
        L.check(self._lib.gx_policy_counters(self.h, C.byref(a), C.byref(b), C.byref(c)))
        return a.value, b.value, c.value


class Arena:
    """HBM slot arena + pinned host tier + remap node (gx_arena_*)."""

    def __init__(self, model: ModelShape, capacity_bytes: int, *, protected_fraction: float = 0.75,
                 policy: int = L.POLICY_AUTO, device: int = 0, host_tier: bool = True, max_tokens: int = 1,
                 first_layer: int = 0, plan_quotas: Sequence[int] | None = None, host_tier_base: int = 0):
        self._lib = L.lib()
        self.model = model
        self.first_layer = first_layer
        self.last_layer = first_layer + model.layers - 1
        prof, self._keep = _profile(first_layer, self.last_layer, model.experts, model.used,
                                    [model.record] * model.layers, [model.record_raw] * model.layers)
        cfg = L.gx_arena_config()
        cfg.profile = prof
        cfg.capacity_bytes = capacity_bytes
        cfg.protected_fraction = protected_fraction
        cfg.policy = policy
        self._plan = (C.c_uint32 * len(plan_quotas))(*plan_quotas) if plan_quotas is not None else None
        cfg.plan_quotas = C.cast(self._plan, C.POINTER(C.c_uint32)) if self._plan is not None else None
        cfg.device = device
        cfg.host_tier = 1 if host_tier else 0
        cfg.max_tokens = max_tokens
        cfg.hidden = model.hidden
        cfg.intermediate = model.intermediate
        cfg.host_tier_base = host_tier_base or None
        h = C.c_void_p()
        L.check(self._lib.gx_arena_create(C.byref(cfg), C.byref(h)), "gx_arena_create")
        self.h = h
        self.desc = L.gx_layer_desc(model.type_gate, model.type_up, model.type_down, model.act, model.alpha,
                                    model.limit, model.hidden, model.intermediate, model.off_gate, model.off_up)

    def close(self):
        if getattr(self, "h", None):
            self._lib.gx_arena_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # host tier
    def host_record(self, layer: int, expert: int) -> np.ndarray:
        p = self._lib.gx_arena_host_record(self.h, layer, expert)
        if not p:
            raise L.GxError(L.GX_ERR_STATE, "gx_arena_host_record")
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(self.model.record,))

    def host_record_ptr(self, layer: int, expert: int) -> int:
        p = self._lib.gx_arena_host_record(self.h, layer, expert)
        if not p:
            raise L.GxError(L.GX_ERR_STATE, "gx_arena_host_record")
        return int(p)

    def load_record(self, layer: int, expert: int, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data, dtype=np.uint8)
        L.check(self._lib.gx_load_record(self.h, layer, expert, data.ctypes.data, data.nbytes), "gx_load_record")

    def layer_view(self, layer: int) -> tuple[int, int, int]:
        base, rec, slots = C.c_void_p(), C.c_uint64(), C.c_uint32()
        L.check(self._lib.gx_arena_layer_view(self.h, layer, C.byref(base), C.byref(rec), C.byref(slots)))
        return int(base.value or 0), rec.value, slots.value

    def read_slot(self, layer: int, slot: int, nbytes: int | None = None) -> np.ndarray:
        n = nbytes or self.model.record_raw
        out = np.empty(n, np.uint8)
        L.check(self._lib.gx_arena_read_slot(self.h, layer, slot, out.ctypes.data, n), "gx_arena_read_slot")
        return out

    def quota(self, layer: int) -> tuple[int, int, int]:
        pol = self._lib.gx_arena_policy(self.h)
        q, p, b = C.c_uint32(), C.c_uint32(), C.c_uint32()
        L.check(self._lib.gx_policy_quota(pol, layer, C.byref(q), C.byref(p), C.byref(b)))
        return q.value, p.value, b.value

    def slot_of(self, layer: int, expert: int) -> int:
        return self._lib.gx_policy_slot_of(self._lib.gx_arena_policy(self.h), layer, expert)

    def remap(self, layer: int, ids: np.ndarray, stream=None, slots: np.ndarray | None = None):
        """The remap node on a host I32 view [ne1, ne0] (numpy strides honoured)."""
        assert ids.dtype == np.int32 and ids.ndim == 2
        ne1, ne0 = ids.shape
        if slots is None:
            slots = np.zeros((ne1, ne0), dtype=np.int32)
        st = L.gx_serve_stats()
        L.check(self._lib.gx_remap_serve(self.h, layer, ids.ctypes.data, ne0, ne1, ids.strides[1], ids.strides[0],
                                         slots.ctypes.data, slots.strides[1], slots.strides[0], _stream(stream),
                                         C.byref(st)), "gx_remap_serve")
        return slots, st

    def warm_all(self, stream=None) -> None:
        L.check(self._lib.gx_arena_warm_all(self.h, _stream(stream)), "gx_arena_warm_all")

    def timing(self, enable: bool) -> None:
        L.check(self._lib.gx_arena_timing(self.h, 1 if enable else 0))

    def timing_read(self) -> tuple[float, float, int]:
        a, b, n = C.c_double(), C.c_double(), C.c_uint64()
        L.check(self._lib.gx_arena_timing_read(self.h, C.byref(a), C.byref(b), C.byref(n)), "gx_arena_timing_read")
        return a.value, b.value, n.value

    def stats(self) -> dict:
        s = L.gx_arena_stats()
        L.check(self._lib.gx_stats(self.h, C.byref(s)))
        return {k: getattr(s, k) for k, _ in s._fields_}

    def layer_forward(self, layer: int, x, ids: np.ndarray, w, out, stream=None) -> L.gx_serve_stats:
        """One MoE layer: x [T, H] f32 device, ids [T, k] int32 HOST, w [T, k] f32 device, out [T, H] device."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        T, k = ids.shape
        st = L.gx_serve_stats()
        L.check(self._lib.gx_moe_layer_forward(self.h, layer, C.byref(self.desc), _ptr(x), ids.ctypes.data, _ptr(w),
                                               k, T, _ptr(out), _stream(stream), C.byref(st)),
                "gx_moe_layer_forward")
        return st

    def layer_forward_shared(self, layer: int, x, ids: np.ndarray, w, shared: "L.gx_shared_expert", out,
                             stream=None) -> L.gx_serve_stats:
        """layer_forward plus a shared expert: out = moe_out + shexp(x)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        T, k = ids.shape
        st = L.gx_serve_stats()
        L.check(self._lib.gx_moe_layer_forward_shared(self.h, layer, C.byref(self.desc), _ptr(x), ids.ctypes.data,
                                                      _ptr(w), k, T, C.byref(shared), _ptr(out), _stream(stream),
                                                      C.byref(st)), "gx_moe_layer_forward_shared")
        return st


def shared_expert(record, type_gate: int, type_down: int, hidden: int, intermediate: int,
                  act: int = L.ACT_SWIGLU) -> L.gx_shared_expert:
    """A shared expert whose record (down | gate | up, 16-byte aligned roles)
    lies at device address `record`."""
    down = L.row_bytes(type_down, intermediate) * hidden
    gate = L.row_bytes(type_gate, hidden) * intermediate
    off_gate = (down + 15) // 16 * 16
    off_up = (off_gate + gate + 15) // 16 * 16
    d = L.gx_layer_desc(type_gate, type_gate, type_down, act, 1.702, 7.0, hidden, intermediate, off_gate, off_up)
    return L.gx_shared_expert(_ptr(record), d)


def shared_record_bytes(type_gate: int, type_down: int, hidden: int, intermediate: int) -> int:
    sh = shared_expert(0, type_gate, type_down, hidden, intermediate)
    return sh.desc.off_up + L.row_bytes(type_gate, hidden) * intermediate


class StackCall:
    """A prepared gx_moe_stack_forward call: fixed device pointers per layer,
    host routes swapped in per call (no per-layer Python work)."""

    def __init__(self, arena: "Arena", first_layer: int, n_layers: int, x_ptrs, w_ptrs, out_ptrs, k: int, T: int):
        self.arena, self.first, self.n, self.k, self.T = arena, first_layer, n_layers, k, T
        self.x = (C.c_void_p * n_layers)(*x_ptrs)
        self.w = (C.c_void_p * n_layers)(*w_ptrs)
        self.out = (C.c_void_p * n_layers)(*out_ptrs)
        self.st = L.gx_serve_stats()
        self.fn = arena._lib.gx_moe_stack_forward

    def set_pointers(self, x_ptrs=None, w_ptrs=None, out_ptrs=None):
        for arr, ptrs in ((self.x, x_ptrs), (self.w, w_ptrs), (self.out, out_ptrs)):
            if ptrs is not None:
                for i, p in enumerate(ptrs):
                    arr[i] = p

    def __call__(self, ids: np.ndarray, stream=None) -> L.gx_serve_stats:
        """ids: int32 C-contiguous [n_layers, T, k] on the host."""
        rc = self.fn(self.arena.h, self.first, self.n, C.byref(self.arena.desc), self.x, ids.ctypes.data, self.w,
                     self.k, self.T, self.out, _stream(stream), C.byref(self.st))
        if rc != L.GX_OK:
            raise L.GxError(rc, "gx_moe_stack_forward")
        return self.st


class StackPlan:
    """gx_stack_plan_*: a decode stack captured once in a CUDA graph."""

    def __init__(self, arena: "Arena", first_layer: int, n_layers: int, x_ptrs, w_ptrs, out_ptrs, k: int, T: int,
                 timing: bool = False, layerwise: bool = False):
        self.arena, self.n, self.k, self.T = arena, n_layers, k, T
        xs = (C.c_void_p * n_layers)(*x_ptrs)
        ws = (C.c_void_p * n_layers)(*w_ptrs)
        os_ = (C.c_void_p * n_layers)(*out_ptrs)
        h = C.c_void_p()
        L.check(arena._lib.gx_stack_plan_create(arena.h, first_layer, n_layers, C.byref(arena.desc), xs, ws, os_, k, T,
                                                (L.GX_PLAN_TIMING if timing else 0)
                                                | (L.GX_PLAN_LAYERWISE if layerwise else 0),
                                                C.byref(h)), "gx_stack_plan_create")
        self.h = h
        self.st = L.gx_serve_stats()
        self.fn = arena._lib.gx_stack_plan_run

    def __call__(self, ids: np.ndarray, stream=None) -> L.gx_serve_stats:
        rc = self.fn(self.h, ids.ctypes.data, _stream(stream), C.byref(self.st))
        if rc != L.GX_OK:
            raise L.GxError(rc, "gx_stack_plan_run")
        return self.st

    def run_routed(self, desc: "L.gx_router_desc", logits, bias=None, ids_out=None, stream=None) -> L.gx_serve_stats:
        """Route on the device (logits device f32 [n_layers*T, E], bias device
        f32 [n_layers, E] or None) and run the stack, no host round trip;
        the plan's weight pointers must be consecutive [T, k] slices of one
        buffer and every layer pinned."""
        ld = logits.stride(0) if hasattr(logits, "stride") else desc.n_expert
        rc = self.arena._lib.gx_stack_plan_run_routed(self.h, C.byref(desc), _ptr(logits), ld, _ptr(bias),
                                                      _ptr(ids_out), _stream(stream), C.byref(self.st))
        if rc != L.GX_OK:
            raise L.GxError(rc, "gx_stack_plan_run_routed")
        return self.st

    def info(self) -> dict:
        """Launch shape: stack_kernel (one persistent kernel) or per-layer kernels."""
        i = L.gx_stack_plan_info()
        L.check(self.arena._lib.gx_stack_plan_info_get(self.h, C.byref(i)), "gx_stack_plan_info_get")
        return {name: getattr(i, name) for name, _ in i._fields_}

    def timing(self) -> tuple[float, float]:
        """(gate/up ms, down ms) summed over layers; the stack kernel reports
        its whole duration as the first value and 0.0 as the second."""
        a, b = C.c_double(), C.c_double()
        L.check(self.arena._lib.gx_stack_plan_timing(self.h, C.byref(a), C.byref(b)), "gx_stack_plan_timing")
        return a.value, b.value

    def close(self):
        if getattr(self, "h", None):
            self.arena._lib.gx_stack_plan_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def router_desc(gating: int, n_expert: int, k: int, *, groups: int = 0, group_used: int = 0, norm_w: bool = False,
                w_scale: float | None = None) -> L.gx_router_desc:
    return L.gx_router_desc(gating, n_expert, k, groups, group_used, 1 if norm_w else 0,
                            0 if w_scale is None else 1, 1.0 if w_scale is None else w_scale)


# the router of each model family (upstream build_moe_ffn's arguments for it)
ROUTERS = {
    "olmoe-1b-7b": dict(gating=L.GX_GATING_SOFTMAX),
    "qwen3-30b-a3b": dict(gating=L.GX_GATING_SOFTMAX, norm_w=True),
    "qwen3-235b-a22b": dict(gating=L.GX_GATING_SOFTMAX, norm_w=True),
    "gpt-oss-120b": dict(gating=L.GX_GATING_SOFTMAX_WEIGHT),
    "deepseek-v3": dict(gating=L.GX_GATING_SIGMOID, groups=8, group_used=4, norm_w=True, w_scale=2.5),
}


def model_router(model) -> L.gx_router_desc:
    """The router description of a model family (softmax + renormalised top-k by default)."""
    kw = ROUTERS.get(model.name, dict(gating=L.GX_GATING_SOFTMAX, norm_w=True))
    return router_desc(n_expert=model.experts, k=model.used, **kw)


def route(desc: L.gx_router_desc, logits, bias=None, n_layers: int = 1, ids=None, weights=None,
          slot_table=None, slots=None, stream=None):
    """gx_router_forward on device tensors: logits [n_layers*T, E] -> ids i32
    and weights f32 [n_layers*T, k] (and slots through a device slot table)."""
    import torch
    rows = logits.shape[0]
    T = rows // n_layers
    k = desc.n_expert_used
    if ids is None:
        ids = torch.empty((rows, k), dtype=torch.int32, device=logits.device)
    if weights is None:
        weights = torch.empty((rows, k), dtype=torch.float32, device=logits.device)
    L.check(L.lib().gx_router_forward(C.byref(desc), _ptr(logits), logits.stride(0), _ptr(bias), T, n_layers,
                                      _ptr(ids), _ptr(weights), _ptr(slot_table), _ptr(slots), _stream(stream)),
            "gx_router_forward")
    return ids, weights


def slot_table(arena: "Arena", first_layer: int, n_layers: int, require_all: bool = False, stream=None):
    """Device i32 [n_layers, E]: the slot of every expert, -1 when not resident."""
    import torch
    t = torch.empty((n_layers, arena.model.experts), dtype=torch.int32, device="cuda")
    L.check(L.lib().gx_arena_slot_table(arena.h, first_layer, n_layers, _ptr(t), 1 if require_all else 0,
                                        _stream(stream)), "gx_arena_slot_table")
    return t


def ep_owner(placement: int, n_expert: int, world: int, expert: int) -> tuple[int, int]:
    """(rank, local id) of a global expert under an expert-parallel placement."""
    r, l = C.c_int32(), C.c_int32()
    L.check(L.lib().gx_ep_owner(placement, n_expert, world, expert, C.byref(r), C.byref(l)), "gx_ep_owner")
    return r.value, l.value


def ep_plan(placement: int, n_expert: int, world: int, ids: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-destination pair counts and the pair indices t*k+s grouped by destination."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, k = ids.shape
    counts = np.zeros(world, np.int32)
    pairs = np.zeros(T * k, np.int32)
    L.check(L.lib().gx_ep_plan(placement, n_expert, world, ids.ctypes.data, k, T, counts.ctypes.data,
                               pairs.ctypes.data), "gx_ep_plan")
    return counts, pairs


class ExpertParallel:
    """gx_ep_*: expert-parallel layer steps over an NCCL communicator.
    `arena` holds this rank's experts (local ids); `comm` is an ncclComm_t
    address, e.g. the NCCL process group's ``_comm_ptr()``."""

    def __init__(self, arena: "Arena", comm: int, rank: int, world: int, n_expert: int,
                 placement: int = L.GX_EP_MODULO):
        self.arena = arena
        h = C.c_void_p()
        L.check(arena._lib.gx_ep_init(arena.h, C.c_void_p(comm), rank, world, n_expert, placement, C.byref(h)),
                "gx_ep_init")
        self.h = h
        self.st = L.gx_serve_stats()

    def layer_forward(self, layer: int, x, ids: np.ndarray, w, out, stream=None) -> L.gx_serve_stats:
        """x [T, H] device f32, ids [T, k] HOST global expert ids, w [T, k] device, out [T, H] device."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        T, k = ids.shape
        L.check(self.arena._lib.gx_ep_layer_forward(self.h, layer, C.byref(self.arena.desc), _ptr(x), ids.ctypes.data,
                                                    _ptr(w), k, T, _ptr(out), _stream(stream), C.byref(self.st)),
                "gx_ep_layer_forward")
        return self.st

    def stack_forward(self, first_layer: int, x_ptrs, ids: np.ndarray, w_ptrs, out_ptrs, stream=None,
                      check: bool = True):
        """n consecutive layers in one step: x_ptrs / w_ptrs / out_ptrs lists of
        n device addresses ([T, H], [T, k], [T, H]); ids HOST int32 [n, T, k]
        global expert ids. Returns (status, stats); raises on error if check."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        n, T, k = ids.shape
        xs = (C.c_void_p * n)(*[_ptr(p) for p in x_ptrs])
        ws = (C.c_void_p * n)(*[_ptr(p) for p in w_ptrs])
        os_ = (C.c_void_p * n)(*[_ptr(p) for p in out_ptrs])
        rc = self.arena._lib.gx_ep_stack_forward(self.h, first_layer, n, C.byref(self.arena.desc), xs, ids.ctypes.data,
                                                 ws, k, T, os_, _stream(stream), C.byref(self.st))
        if check:
            L.check(rc, "gx_ep_stack_forward")
        return rc, self.st

    def close(self):
        if getattr(self, "h", None):
            self.arena._lib.gx_ep_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def mul_mat_id(type_: int, as_, ne00: int, ne01: int, nb01: int, nb02: int, n_as: int,
               b, ne11: int, ne12: int, nb11: int, nb12: int,
               ids, ne20: int, ne21: int, nbi1: int, dst, stream=None) -> None:
    """ggml_mul_mat_id with ggml's tensor conventions (all device addresses)."""
    L.check(L.lib().gx_mul_mat_id(type_, _ptr(as_), ne00, ne01, nb01, nb02, n_as, _ptr(b), ne11, ne12, nb11, nb12,
                                  _ptr(ids), ne20, ne21, nbi1, _ptr(dst), _stream(stream)), "gx_mul_mat_id")


def device_error() -> int:
    code = C.c_int32()
    L.check(L.lib().gx_device_error(C.byref(code)))
    return code.value
