"""Cache plans: per-layer slot quotas from measured miss curves.

Python side of gx_cache_plan_* / gx_plan_layer_quotas / gx_policy_plan_quotas
(the reference's CachePlan and plan_layer_quotas, src/h4/h4-cache-plan.hpp:
55-117). A plan's quotas go to Arena(..., plan_quotas=...).
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import _lib as L


class CachePlan:
    """A plan file in the reference's text format."""

    def __init__(self, path: str):
        h = C.c_void_p()
        L.check(L.lib().gx_cache_plan_load(str(path).encode(), C.byref(h)), f"gx_cache_plan_load({path})")
        self.h = h
        first, last, experts, used = C.c_uint32(), C.c_uint32(), C.c_uint32(), C.c_uint32()
        arch = C.create_string_buffer(128)
        L.check(L.lib().gx_cache_plan_info(h, C.byref(first), C.byref(last), C.byref(experts), C.byref(used), arch, 128))
        self.first_layer, self.last_layer = first.value, last.value
        self.experts, self.used, self.arch = experts.value, used.value, arch.value.decode()

    def curve(self, layer: int) -> np.ndarray:
        out = np.zeros(self.experts + 1, np.uint32)
        L.check(L.lib().gx_cache_plan_curve(self.h, layer, out.ctypes.data), "gx_cache_plan_curve")
        return out

    def curves(self) -> np.ndarray:
        return np.stack([self.curve(l) for l in range(self.first_layer, self.last_layer + 1)])

    def engine_quotas(self, record_bytes: Sequence[int], capacity_bytes: int, protected_fraction: float = 0.75,
                      used: int | None = None) -> np.ndarray | None:
        """The quotas the engine applies for this plan, or None when the
        uniform quota stays (other geometry, full residency)."""
        n = self.last_layer - self.first_layer + 1
        rec = (C.c_uint64 * n)(*[int(r) for r in record_bytes])
        prof = L.gx_profile(self.first_layer, self.last_layer, self.experts, used or self.used, rec, rec)
        out = np.zeros(n, np.uint32)
        rc = L.lib().gx_policy_plan_quotas(C.byref(prof), capacity_bytes, protected_fraction, self.h, out.ctypes.data)
        if rc == L.GX_ERR_STATE:
            return None
        L.check(rc, "gx_policy_plan_quotas")
        return out

    def close(self):
        if getattr(self, "h", None):
            L.lib().gx_cache_plan_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def plan_layer_quotas(curves: np.ndarray, record_bytes: Sequence[int], budget: int, floor: int,
                      ceiling: int) -> np.ndarray:
    """The reference allocator: curves [layers, len] misses at quota 0..len-1."""
    curves = np.ascontiguousarray(curves, dtype=np.uint32)
    n, m = curves.shape
    rec = np.ascontiguousarray(record_bytes, dtype=np.uint64)
    out = np.zeros(n, np.uint32)
    L.check(L.lib().gx_plan_layer_quotas(curves.ctypes.data, n, m, rec.ctypes.data, budget, floor, ceiling,
                                          out.ctypes.data), "gx_plan_layer_quotas")
    return out
