"""Route traces (GALACTUS_H4_ROUTES / gx_route_observer_*): open, close and
read the reference's "galactus.route-observer.v1" text format
(src/h4/h4-route-observer.hpp:213-262)."""
from __future__ import annotations

import ctypes as C

from . import _lib as L


def open_trace(path: str, arch: str = "unknown", entry_cap: int = 0) -> None:
    L.check(L.lib().gx_route_observer_open(str(path).encode(), arch.encode(), entry_cap), "gx_route_observer_open")


def close_trace() -> None:
    L.check(L.lib().gx_route_observer_close(), "gx_route_observer_close")


def read_trace(path: str) -> dict:
    """Header fields and entries: {layer, tokens, k, enter_ns, serve_start_ns,
    serve_end_ns, gap_ns, bytes_read, ids, resident}."""
    out: dict = {"records": {}, "entries": []}
    with open(path, encoding="utf-8") as f:
        for line in f:
            parts = line.split()
            if not parts:
                continue
            if parts[0] == "#":
                h = parts[1:]
                if not h:
                    continue
                if h[0] == "galactus.route-observer.v1":
                    out["version"] = 1
                elif h[0] == "arch":
                    out["arch"] = h[1]
                elif h[0] == "first_layer":
                    out.update(first_layer=int(h[1]), last_layer=int(h[3]), experts=int(h[5]), used=int(h[7]))
                elif h[0] == "cache_bytes":
                    out.update(cache_bytes=int(h[1]), protected=float(h[3]), quota=int(h[5]), probation=int(h[7]),
                               slots=int(h[9]))
                elif h[0] == "record":
                    out["records"][int(h[1])] = int(h[2])
                elif h[0] == "entries":
                    out.update(n_entries=int(h[1]), truncated=h[3] == "1")
            elif parts[0] == "e":
                pairs = [t.split(":") for t in parts[10:]]
                out["entries"].append({
                    "seq": int(parts[1]), "layer": int(parts[2]), "tokens": int(parts[3]), "k": int(parts[4]),
                    "enter_ns": int(parts[5]), "serve_start_ns": int(parts[6]), "serve_end_ns": int(parts[7]),
                    "gap_ns": int(parts[8]), "bytes_read": int(parts[9]),
                    "ids": [int(a) for a, _ in pairs], "resident": [int(b) for _, b in pairs]})
    return out
