#!/usr/bin/env python
"""Benchmark of the routed-expert FFN of a quantized MoE layer on B200.

One GPU (the default; the headline):
  gpt-oss-120b-shaped MoE stack -- 36 layers, hidden 2880, 128 experts, top-4,
  expert intermediate 2880, clamped SwiGLU (limit 7.0), MXFP4 experts (seed 2),
  every expert resident in HBM (61 GB slot cache). A step is one decode token
  through the 36 routed-expert layers: per layer the remap (slot policy on the
  host), gate/up + activation, down + weighted combine, all layers in one
  persistent kernel launched from a captured plan.
    value  decode tokens/s, inputs resident in HBM
    e2e    the same through the C-ABI with host buffers: per step the hidden
           states and router weights go host->device and the layer outputs
           device->host inside the timed region
  Beside it in the same JSON line (each with its own timing, outside the
  region of `value`): the same model at batches 8 and 64 and at 25 GB / 5 GB
  slot caches (steady state, misses streamed from the pinned host tier;
  expert-major waves where a batch's experts exceed the cache's batch bound),
  the Qwen3-30B-A3B Q8_0 stack (48 layers: decode, 512-token prefill, 50 % /
  25 % caches), the OLMoE-shaped single layer (512 sequential tokens, 16 of 64
  slots, LRU and SLRU) and the expert-parallel Qwen3-235B-A22B line on one GPU.

N GPUs (torchrun, one process per GPU): expert parallelism on the
Qwen3-235B-A22B shape -- hidden 4096, 128 experts, top-8, intermediate 1536,
Q4_K gate/up + Q6_K down (seed 3) -- expert e on GPU e mod N, a slot cache of
10 slots per layer per GPU (the 12 GB per-GPU cap over 94 layers), misses
streamed from each GPU's pinned host tier, each GPU serving its own decode
token per step; NCCL dispatch and combine over NVLink (gx_ep_stack_forward).
`scaling` is "weak" (tokens per GPU fixed). Rank 0 checks one layer of the
last step bit for bit against the single-GPU layer path.

Weights read per step exceed the 126 MB L2 by far, so no L2 flush is needed.
All inputs are seeded synthetic data with BASELINE's shapes and distributions.

`--impl reference` times the CPU oracle (the port of the reference's CPU
arithmetic; ggml itself is not vendored with the reference) on the same
workload and config, all host threads, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 2 ** 20
HEADLINE_MODEL = "gpt-oss-120b"
EP_MODEL = "qwen3-235b"
EP_SLOTS = 10            # 12 GB per GPU over 94 layers of 12.24 MB records
EP_LAYERS = 24           # of 94: 94 layers' host tiers (147 GB in all) exceed the box's host memory
# slot caches of the single-GPU sweeps (slots per layer, name)
SWEEPS = {"gpt-oss-120b": [(52, "25 GB"), (10, "5 GB")], "qwen3-30b": [(64, "50%"), (32, "25%")]}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default=None, help="the single-GPU headline model (default gpt-oss-120b)")
    ap.add_argument("--layers", type=int, default=0, help="fewer layers (small profiling cases only)")
    ap.add_argument("--experts", type=int, default=0,
                    help="fewer experts per layer (small profiling cases only: keeps the resident arena small "
                         "while each token still touches top-k experts per layer)")
    ap.add_argument("--headline-only", action="store_true", help="time the headline and e2e lines only (profiling)")
    ap.add_argument("--ep", action="store_true", help="the expert-parallel line alone, also on one GPU")
    ap.add_argument("--ep-model", default=EP_MODEL)
    ap.add_argument("--ep-layers", type=int, default=EP_LAYERS)
    ap.add_argument("--ep-slots", type=int, default=EP_SLOTS)
    ap.add_argument("--ep-tokens", type=int, default=1, help="decode tokens per GPU per step")
    ap.add_argument("--ep-prewarm", type=int, default=48, help="untimed steps that bring the slot caches to steady state")
    ap.add_argument("--sweep-warm", type=int, default=512, help="tokens that warm a sweep cache before timing")
    ap.add_argument("--sweep-steps", type=int, default=256, help="timed tokens of a batch-1 sweep point")
    ap.add_argument("--prefill", type=int, default=512)
    ap.add_argument("--cpu-tokens", type=int, default=2, help="tokens of the CPU baseline sample (every layer)")
    return ap.parse_args()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def pci_bus_id(torch, dev):
    """NVML's PCI bus id string of a CUDA device (CUDA and NVML orders can differ)."""
    try:
        pr = torch.cuda.get_device_properties(dev)
        return f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
    except Exception:
        return None


class ClockSampler:
    """SM clock and clock-event reasons sampled DURING the timed region: NVML
    read-only queries polled every ~2 ms from a background thread (enough
    samples even for a 20 ms region). Nothing is set."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
               "hw_power_brake": "nvmlClocksEventReasonHwPowerBrakeSlowdown"}

    def __init__(self, gpu_index: int, pci_bus_id: str | None = None):
        self.gpu = gpu_index
        self.pci = pci_bus_id
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.masks: dict[str, int] = {}
        self._stop = threading.Event()
        self.t = None
        self.nv = None

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            try:
                h = nv.nvmlDeviceGetHandleByPciBusId(self.pci) if self.pci else nv.nvmlDeviceGetHandleByIndex(self.gpu)
            except Exception:
                h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.nv, self.h = nv, h
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.masks = {k: getattr(nv, v, 0) for k, v in self.REASONS.items()}
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            time.sleep(0.01)
        except Exception:
            self.nv = None
        return self

    def _poll(self):
        nv, h = self.nv, self.h
        while not self._stop.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                     int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
            except Exception:
                return
            time.sleep(0.002)

    def __exit__(self, *a):
        self._stop.set()
        if self.t:
            self.t.join(timeout=2)
        if self.nv:
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        reasons = set()
        for _, mask in self.samples:
            for name, bit in self.masks.items():
                if bit and (mask & bit):
                    reasons.add(name)
        sm = [c for c, _ in self.samples]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvml"}


# ------------------------------------------------------------- workloads

def shaped_model(gx, name, layers=0, experts=0):
    model = gx.MODELS[name]
    if layers:
        model = model.with_layers(layers)
    if experts:
        model = model.with_experts(experts)
    return model


def wtypes(gx, model):
    tn = gx.TYPE_NAMES
    return tn[model.type_gate] if model.type_gate == model.type_down else \
        f"{tn[model.type_gate]} gate/up + {tn[model.type_down]} down"


def atypes(gx, model):
    return "/".join(sorted({"q8_0" if t in (gx.TYPE_Q8_0, gx.TYPE_MXFP4) else "q8_K"
                            for t in (model.type_gate, model.type_down)}))


def single_config(gx, model, slots="100%"):
    """Metric, config dict and dtype of a single-GPU stack line (shared by both arms)."""
    NL, H, E, k, I = model.layers, model.hidden, model.experts, model.used, model.intermediate
    metric = f"MoE-layer decode tok/s ({NL}-layer routed-expert FFN stack, full slot residency)"
    config = {"workload": f"{model.name} MoE stack, batch-1 decode, {NL} layers, H {H}, E {E}, top-{k}, I {I}, "
                          f"{wtypes(gx, model)}, slot cache {slots}", "model": model.name, "global_batch": 1,
              "seq_len": 1, "parallelism": "single",
              "l2": f"inputs larger than L2: ~{NL * k * model.record_raw / 1e9:.2f} GB of expert weights read per step "
                    f"vs 126 MB L2, no flush"}
    dtype = f"int8 dot / f32 tail ({wtypes(gx, model)} weights, {atypes(gx, model)} activations)"
    return metric, config, dtype


def ep_config(gx, model, world, T, slots):
    metric = f"MoE-layer decode tok/s, expert-parallel ({model.layers}-layer routed-expert FFN stack, " \
             f"{slots} slots per layer per GPU)"
    config = {"workload": f"{model.name} MoE stack, {T} decode token(s) per GPU, {model.layers} of 94 layers, "
                          f"H {model.hidden}, E {model.experts} (expert e on GPU e mod {world}), top-{model.used}, "
                          f"I {model.intermediate}, {wtypes(gx, model)}, {slots} slots per layer per GPU "
                          f"(12 GB cap), misses from pinned host DRAM",
              "model": model.name, "global_batch": world * T, "seq_len": 1, "parallelism": f"ep{world}",
              "experts_per_gpu": model.experts // world,
              "l2": "expert weights read per step exceed L2, no flush"}
    return metric, config


def free_pinned(torch):
    torch.cuda.synchronize()
    try:
        torch._C._host_emptyCache()
    except Exception:
        pass


def fill_tier(gx, torch, model, tier_t, dev, owned=None):
    """Generate the records of every layer on the device (the generator the
    oracle restates, byte for byte) and copy them into the pinned host tier,
    layer-major then expert (owned: global ids of this rank's experts, in
    local order)."""
    lib = gx.lib()
    E = model.experts
    owned = list(range(E)) if owned is None else owned
    n = len(owned)
    stage = torch.empty(n * model.record, dtype=torch.uint8, device=dev)
    for L in range(model.layers):
        stage.zero_()
        base = stage.data_ptr()
        for li, e in enumerate(owned):
            sid = (L * E + e) * 3
            r = base + li * model.record
            gx.check(lib.gx_synth_weights(model.type_down, r, model.intermediate, model.hidden, model.seed, sid + 0,
                                          0.02, None))
            gx.check(lib.gx_synth_weights(model.type_gate, r + model.off_gate, model.hidden, model.intermediate,
                                          model.seed, sid + 1, 0.02, None))
            gx.check(lib.gx_synth_weights(model.type_up, r + model.off_up, model.hidden, model.intermediate,
                                          model.seed, sid + 2, 0.02, None))
        tier_t[L * n * model.record:(L + 1) * n * model.record].copy_(stage)
    torch.cuda.synchronize()
    del stage


def roofline_of(gx, model, T, stack_ms):
    """The stack kernel's algorithmic bytes per launch (expert rows of every
    layer plus the inputs, activations, weights and outputs it moves) and the
    achieved GB/s."""
    H, I, k, NL = model.hidden, model.intermediate, model.used, model.layers
    rb_h = gx.row_bytes(model.type_gate, H)
    rb_i = gx.row_bytes(model.type_down, I)
    gu = k * T * 2 * I * rb_h + T * H * 4 + k * T * I * 4
    dn = k * T * H * rb_i + k * T * I * 4 + k * T * 4 + T * H * 4
    dbytes = NL * (gu + dn)
    return dbytes, dbytes / (stack_ms / 1e3) / 1e9


def timed(torch, stream, fn):
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    r = fn()
    ev1.record(stream)
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1), r


# ------------------------------------------------------------ one GPU

class Single:
    """One model on one GPU: its pinned host tier, arenas and plans."""

    def __init__(self, gx, torch, model, dev, stream, max_tokens=1):
        from galactus_b200.routing import routes
        self.gx, self.torch, self.model, self.dev, self.stream = gx, torch, model, dev, stream
        NL, E, H, k = model.layers, model.experts, model.hidden, model.used
        t0 = time.time()
        self.tier = torch.empty(NL * E * model.record, dtype=torch.uint8, pin_memory=True)
        fill_tier(gx, torch, model, self.tier, dev)
        self.tier_ptr = self.tier.data_ptr()
        self.setup_s = time.time() - t0
        self.max_tokens = max_tokens
        self.P = 64                      # distinct input rows, cycled
        self.routes = lambda n, seed, rho=0.7: routes(model, n, NL, seed=seed, rho=rho)
        self.xs = np.random.default_rng(0).standard_normal((self.P, NL, H)).astype(np.float32)
        self.x_dev = torch.from_numpy(self.xs).to(dev)
        self.out_dev = torch.empty((NL, H), dtype=torch.float32, device=dev)
        self.x_fix = torch.empty((NL, H), dtype=torch.float32, device=dev)
        self.w_fix = torch.empty((NL, k), dtype=torch.float32, device=dev)

    def arena(self, slots, max_tokens=None):
        gx, m = self.gx, self.model
        return gx.Arena(m, capacity_bytes=slots * m.record * m.layers, policy=gx.POLICY_AUTO,
                        max_tokens=max_tokens or self.max_tokens, host_tier_base=self.tier_ptr, device=self.dev.index or 0)

    def plan(self, arena, timing=False):
        from galactus_b200.moe import StackPlan
        NL, k = self.model.layers, self.model.used
        return StackPlan(arena, 0, NL, [self.x_fix[L].data_ptr() for L in range(NL)],
                         [self.w_fix[L].data_ptr() for L in range(NL)], [self.out_dev[L].data_ptr() for L in range(NL)],
                         k, 1, timing=timing)

    def run_plan(self, plan, ids_c, w_dev, t_first, n, e2e=None):
        h = m = 0
        for i in range(n):
            t = t_first + i
            s = t % self.P
            if e2e is None:
                self.x_fix.copy_(self.x_dev[s], non_blocking=True)
                self.w_fix.copy_(w_dev[t], non_blocking=True)
            else:
                h_x, h_w, h_out = e2e
                self.x_fix.copy_(h_x[s], non_blocking=True)
                self.w_fix.copy_(h_w[t], non_blocking=True)
            st = plan(ids_c[t], self.stream)
            h += st.hits
            m += st.misses
            if e2e is not None:
                e2e[2][s].copy_(self.out_dev, non_blocking=True)
        return h, m

    def close(self):
        del self.tier
        free_pinned(self.torch)


def headline(args, gx, torch, sg, dev, local):
    """value, e2e, e2e with the device router, the stack kernel's duration."""
    from galactus_b200.moe import model_router
    from galactus_b200.routing import logits
    model, stream = sg.model, sg.stream
    NL, E, H, k = model.layers, model.experts, model.hidden, model.used
    n_tok = args.warmup + args.steps
    ids_all, w_all = sg.routes(n_tok, model.seed * 1000 + 17)
    ids_c = [np.ascontiguousarray(ids_all[t][:, None, :]) for t in range(n_tok)]     # [NL, 1, k]
    w_dev = torch.from_numpy(np.ascontiguousarray(w_all)).to(dev)                   # [n_tok, NL, k]
    res = {}
    arena = sg.arena(E)
    with torch.cuda.stream(stream):
        arena.warm_all(stream)
        torch.cuda.synchronize()
        plan = sg.plan(arena)
        sg.run_plan(plan, ids_c, w_dev, 0, args.warmup)
        with ClockSampler(local, pci_bus_id(torch, dev)) as clk:
            ms, (h, m) = timed(torch, stream, lambda: sg.run_plan(plan, ids_c, w_dev, args.warmup, args.steps))
        res["ms"] = ms
        res["clocks"] = clk.summary()
        res["hit_rate"] = h / max(1, h + m)
        # e2e: host buffers, copies inside the timed region
        h_x = torch.from_numpy(sg.xs).pin_memory()
        h_w = torch.from_numpy(np.ascontiguousarray(w_all)).pin_memory()
        h_out = torch.empty((sg.P, NL, H), dtype=torch.float32).pin_memory()
        sg.run_plan(plan, ids_c, w_dev, 0, args.warmup, e2e=(h_x, h_w, h_out))
        ms_e2e, _ = timed(torch, stream, lambda: sg.run_plan(plan, ids_c, w_dev, args.warmup, args.steps,
                                                             e2e=(h_x, h_w, h_out)))
        res["e2e"] = {"value": args.steps / (ms_e2e / 1e3), "unit": "tok/s",
                      "h2d_bytes_per_step": NL * H * 4 + NL * k * 4, "d2h_bytes_per_step": NL * H * 4}
        # e2e with the router on the device: hidden states and router logits in,
        # ids, slots and weights written by the router, outputs back
        rdesc = model_router(model)
        h_lg = torch.from_numpy(logits(model, sg.P, NL, seed=model.seed * 1000 + 29, rho=0.7)).pin_memory()
        lg_fix = torch.empty((NL, E), dtype=torch.float32, device=dev)

        def routed(t_first, n):
            for i in range(n):
                s = (t_first + i) % sg.P
                sg.x_fix.copy_(h_x[s], non_blocking=True)
                lg_fix.copy_(h_lg[s], non_blocking=True)
                plan.run_routed(rdesc, lg_fix, stream=stream)
                h_out[s].copy_(sg.out_dev, non_blocking=True)

        routed(0, args.warmup)
        ms_r, _ = timed(torch, stream, lambda: routed(args.warmup, args.steps))
        res["e2e_device_router"] = {"value": args.steps / (ms_r / 1e3), "unit": "tok/s",
                                    "h2d_bytes_per_step": NL * H * 4 + NL * E * 4, "d2h_bytes_per_step": NL * H * 4}
        res["plan"] = plan.info()
        plan.close()   # one plan at a time: a tensor-core plan holds a copy of every slot
        # the stack kernel's duration: CUDA events recorded inside the graph around it
        kplan = sg.plan(arena, timing=True)
        stack_ms = 0.0
        for i in range(args.steps):
            sg.run_plan(kplan, ids_c, w_dev, args.warmup + i, 1)
            stack_ms += kplan.timing()[0]
        kplan.close()
        res["stack_ms"] = stack_ms / args.steps
    return arena, res


def batches_line(args, gx, torch, sg, arena, dev):
    """The same stack at batches of 8 and 64 decode tokens, full residency."""
    from galactus_b200.moe import StackCall, StackPlan
    model, stream = sg.model, sg.stream
    NL, H, k = model.layers, model.hidden, model.used
    out = {}
    for T in (8, 64):
        if T > sg.max_tokens:
            continue
        n = 4 + 8
        ids_all, w_all = sg.routes(n * T, model.seed * 1000 + 40 + T)
        ids = np.ascontiguousarray(ids_all.reshape(n, T, NL, k).transpose(0, 2, 1, 3))       # [n, NL, T, k]
        w = torch.from_numpy(np.ascontiguousarray(w_all.reshape(n, T, NL, k).transpose(0, 2, 1, 3))).to(dev)
        x = torch.from_numpy(np.random.default_rng(T).standard_normal((NL, T, H)).astype(np.float32)).to(dev)
        o = torch.empty((NL, T, H), dtype=torch.float32, device=dev)
        wf = torch.empty((NL, T, k), dtype=torch.float32, device=dev)
        ptr = lambda t: [t[L].data_ptr() for L in range(NL)]
        if k * T <= 64:
            runner = StackPlan(arena, 0, NL, ptr(x), ptr(wf), ptr(o), k, T)
            kind = "captured plan (persistent stack kernel)"
        else:
            runner = StackCall(arena, 0, NL, ptr(x), ptr(wf), ptr(o), k, T)
            kind = "per-layer C-ABI calls (three kernels per layer)"
        with torch.cuda.stream(stream):
            def go(a, b):
                for s in range(a, b):
                    wf.copy_(w[s], non_blocking=True)
                    runner(ids[s], stream)
            go(0, 4)
            ms, _ = timed(torch, stream, lambda: go(4, n))
        if hasattr(runner, "close"):
            runner.close()
        out[f"T{T}"] = {"tok_s": (n - 4) * T / (ms / 1e3), "ms_per_step": ms / (n - 4), "path": kind}
    return out


def sweep_line(args, gx, torch, sg, dev, points, batch):
    """Steady-state residency sweep: each cache is warmed with --sweep-warm
    routed tokens, then timed (--sweep-steps tokens at batch 1, 32 tokens at
    larger batches); hit rate and host->HBM GB/s beside tok/s. Returns the
    lines and the batch-1 traces (for the reference policy in the CPU leg)."""
    from galactus_b200.moe import StackCall
    model, stream = sg.model, sg.stream
    NL, H, k = model.layers, model.hidden, model.used
    T = batch
    lines, traces = [], []
    for slots, name in points:
        warm = max(1, args.sweep_warm // T)
        timed_n = args.sweep_steps if T == 1 else max(2, 32 // T)
        n = warm + timed_n
        ids_all, w_all = sg.routes(n * T, model.seed * 1000 + 50 + slots + T)
        ids = np.ascontiguousarray(ids_all.reshape(n, T, NL, k).transpose(0, 2, 1, 3))        # [n, NL, T, k]
        a = sg.arena(slots, max_tokens=T)
        if T == 1:
            plan = sg.plan(a)
            w_dev = torch.from_numpy(np.ascontiguousarray(w_all)).to(dev)
            ids_c = [np.ascontiguousarray(ids[s]) for s in range(n)]
            with torch.cuda.stream(stream):
                sg.run_plan(plan, ids_c, w_dev, 0, warm)
                s0 = a.stats()
                ms, (hh, mm) = timed(torch, stream, lambda: sg.run_plan(plan, ids_c, w_dev, warm, timed_n))
                s1 = a.stats()
            plan.close()
            traces.append((slots, ids))
        else:
            x = torch.from_numpy(np.random.default_rng(T).standard_normal((NL, T, H)).astype(np.float32)).to(dev)
            o = torch.empty((NL, T, H), dtype=torch.float32, device=dev)
            wf = torch.from_numpy(np.full((NL, T, k), 1.0 / k, np.float32)).to(dev)
            ptr = lambda t: [t[L].data_ptr() for L in range(NL)]
            call = StackCall(a, 0, NL, ptr(x), ptr(wf), ptr(o), k, T)
            with torch.cuda.stream(stream):
                for s in range(warm):
                    call(ids[s], stream)
                torch.cuda.synchronize()
                s0 = a.stats()

                def go():
                    hh = mm = 0
                    for s in range(warm, n):
                        st = call(ids[s], stream)
                        hh += st.hits
                        mm += st.misses
                    return hh, mm
                ms, (hh, mm) = timed(torch, stream, go)
                s1 = a.stats()
        moved = s1["bytes_h2d"] - s0["bytes_h2d"]
        lines.append({"slot_cache": name, "slots_per_layer": a.quota(0)[0], "batch": T,
                      "tok_s": timed_n * T / (ms / 1e3), "hit_rate": hh / max(1, hh + mm),
                      "h2d_gb_s": moved / (ms / 1e3) / 1e9, "h2d_ceiling_gb_s": "PCIe Gen5 x16, ~55-64",
                      "h2d_bytes_per_token": moved / (timed_n * T), "warm_tokens": warm * T,
                      "timed_tokens": timed_n * T})
        a.close()
    return lines, traces


def prefill_line(args, gx, torch, sg, arena, dev):
    from galactus_b200.moe import StackCall
    model, stream = sg.model, sg.stream
    NL, H, k = model.layers, model.hidden, model.used
    Tp = args.prefill
    pid, pw = sg.routes(Tp, 4242)
    px = torch.from_numpy(np.random.default_rng(7).standard_normal((NL, Tp, H)).astype(np.float32)).to(dev)
    pwd = torch.from_numpy(np.ascontiguousarray(pw.transpose(1, 0, 2))).to(dev)
    pout = torch.empty((NL, Tp, H), dtype=torch.float32, device=dev)
    pcall = StackCall(arena, 0, NL, [px[L].data_ptr() for L in range(NL)], [pwd[L].data_ptr() for L in range(NL)],
                      [pout[L].data_ptr() for L in range(NL)], k, Tp)
    pids = np.ascontiguousarray(pid.transpose(1, 0, 2))                      # [NL, Tp, k]
    with torch.cuda.stream(stream):
        pcall(pids, stream)
        ms, _ = timed(torch, stream, lambda: [pcall(pids, stream) for _ in range(2)])
    return {"tokens": Tp, "tok_s": Tp / (ms / 2 / 1e3), "ms": ms / 2}


def stack_line(args, gx, torch, name, dev, local, stream, extras):
    """A single-GPU line for one model: headline, e2e, roofline and, with
    extras, batches, prefill and the residency sweep."""
    model = shaped_model(gx, name, args.layers, args.experts)
    max_tokens = 64
    if extras and model.type_gate == gx.TYPE_Q8_0 and args.prefill:
        max_tokens = max(max_tokens, args.prefill)
    sg = Single(gx, torch, model, dev, stream, max_tokens=max_tokens)
    arena, res = headline(args, gx, torch, sg, dev, local)
    peak, peak_kind = measured_peaks()
    dbytes, achieved = roofline_of(gx, model, 1, res["stack_ms"])
    # DRAM traffic of one launch: the per-layer figure of an ncu capture of the
    # same kernel and row types, times the layers streamed
    traffic = None
    tensor_cores = res["plan"].get("tensor_cores", 0) if res["plan"]["stack_kernel"] else 0
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        key = "k_stack_per_layer_tma_tensor_cores" if tensor_cores == 2 else "k_stack_per_layer"
        per_layer = json.loads(tp.read_text()).get(model.name, {}).get(key)
        traffic = per_layer * model.layers if per_layer else None
    kernel = "k_stack (persistent: all layers, gate/up+act, down+combine"
    kernel += "; MXFP4 block dots on tcgen05, codes loaded by TMA)" if tensor_cores == 2 else ")"
    metric, config, dtype = single_config(gx, model)
    line = {
        "metric": metric, "value": args.steps / (res["ms"] / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": res["ms"] / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype,
        "data": f"synthetic (seeded {wtypes(gx, model)} weights; Zipf(1.1)+AR(0.7) routes; N(0,1) states)",
        "config": config, "e2e": res["e2e"], "e2e_device_router": res["e2e_device_router"],
        "gpu_launches": (1 if res["plan"]["stack_kernel"] else 3 * model.layers) * args.steps,
        "plan": res["plan"], "hit_rate": res["hit_rate"],
        "roofline": {"bound": "hbm", "kernel": kernel,
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "traffic": traffic, "algorithmic_bytes_per_launch": dbytes,
                     "avg_launch_ms": res["stack_ms"]},
        "clocks": res["clocks"], "setup_s": sg.setup_s,
    }
    traces = []
    if extras:
        line["batches"] = batches_line(args, gx, torch, sg, arena, dev)
        if model.type_gate == gx.TYPE_Q8_0 and args.prefill:
            line["prefill"] = prefill_line(args, gx, torch, sg, arena, dev)
    arena.close()
    if extras and name in SWEEPS:
        pts = SWEEPS[name]
        line["sweep"], traces = sweep_line(args, gx, torch, sg, dev, pts, 1)
        if name == "gpt-oss-120b":
            # the 5 GB cache at batches 8 and 64: more experts than slots, waves
            for T in (8, 64):
                more, _ = sweep_line(args, gx, torch, sg, dev, [pts[-1]], T)
                line["sweep"] += more
    sg.close()
    from galactus_b200.moe import device_error
    err = device_error()
    if err:
        raise RuntimeError(f"device error {err}")
    return model, line, traces


def olmoe_line(args, gx, torch, dev, stream):
    """BASELINE cfg 1 as written: one OLMoE-shaped layer, 512 sequential
    decode tokens (softmax top-8 over Zipf-biased Gaussian logits), a slot
    cache of 16 of 64 experts under LRU and under the reference's default
    SLRU (frequency victim)."""
    from galactus_b200.routing import routes
    model = gx.MODELS["olmoe"].with_layers(1)
    H, k = model.hidden, model.used
    tier = torch.empty(model.experts * model.record, dtype=torch.uint8, pin_memory=True)
    fill_tier(gx, torch, model, tier, dev)
    n = 512
    ids, w = routes(model, n, 1, seed=model.seed * 1000 + 3, rho=0.0)
    x = torch.from_numpy(np.random.default_rng(3).standard_normal((n, H)).astype(np.float32)).to(dev)
    wd = torch.from_numpy(np.ascontiguousarray(w[:, 0])).to(dev)
    out = torch.empty((n, H), dtype=torch.float32, device=dev)
    res = {"workload": "olmoe-1b-7b single MoE layer, 512 sequential decode tokens, 16 of 64 slots"}
    for pol, name in ((gx.POLICY_LRU, "lru"), (gx.POLICY_AUTO, "slru")):
        a = gx.Arena(model, capacity_bytes=16 * model.record, policy=pol, max_tokens=1, host_tier_base=tier.data_ptr(),
                     device=dev.index or 0)
        with torch.cuda.stream(stream):
            def go():
                h = m = 0
                for t in range(n):
                    st = a.layer_forward(0, x[t:t + 1], ids[t, 0][None], wd[t:t + 1], out[t:t + 1], stream)
                    h += st.hits
                    m += st.misses
                return h, m
            ms, (h, m) = timed(torch, stream, go)
            s = a.stats()
        res[name] = {"tok_s": n / (ms / 1e3), "hit_rate": h / max(1, h + m), "misses": m,
                     "h2d_gb_s": s["bytes_h2d"] / (ms / 1e3) / 1e9}
        a.close()
    del tier
    free_pinned(torch)
    return res, ids[:, 0]


def run_single(args):
    import torch

    import galactus_b200 as gx
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gx.check(gx.lib().gx_device_init(local))
    stream = torch.cuda.Stream(device=dev)
    extras = not args.headline_only
    name = args.model or HEADLINE_MODEL
    model, line, traces = stack_line(args, gx, torch, name, dev, local, stream, extras)
    cfg1_ids = None
    if extras and not (args.layers or args.experts):
        if name != "qwen3-30b":
            _, l2, _ = stack_line(args, gx, torch, "qwen3-30b", dev, local, stream, True)
            for key in ("n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline", "unit"):
                l2.pop(key, None)
            line["qwen3_30b"] = l2
        line["olmoe_single_layer"], cfg1_ids = olmoe_line(args, gx, torch, dev, stream)
        line["ep_1gpu"] = ep_measure(args, gx, torch, 1, 0, local, dev, None)
        # configs 5 and 4 as one-GPU stacks of 8 layers x 16 experts, all
        # resident (their 58- and 94-layer host tiers do not fit host memory;
        # the work per layer is the full model's)
        for key, nm in (("deepseek_v3_8x16", "deepseek-v3"), ("qwen3_235b_8x16", "qwen3-235b")):
            sub = argparse.Namespace(**{**vars(args), "layers": 8, "experts": 16})
            _, l3, _ = stack_line(sub, gx, torch, nm, dev, local, stream, False)
            for k in ("n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline", "unit"):
                l3.pop(k, None)
            line[key] = l3
    if args.cpu_tokens > 0:
        line["cpu_baseline"] = cpu_baseline_leg(args, gx, model, traces, cfg1_ids)
    print(json.dumps(line), flush=True)


# ------------------------------------------------------ expert parallelism

def ep_measure(args, gx, torch, world, rank, local, dev, comm):
    """The expert-parallel decode line (every rank runs it; rank 0's dict is printed)."""
    import torch.distributed as dist

    from galactus_b200.models import ModelShape
    from galactus_b200.moe import ExpertParallel, device_error
    from galactus_b200.routing import routes
    model = shaped_model(gx, args.ep_model, args.ep_layers, args.experts)
    E, k, H, NL, T = model.experts, model.used, model.hidden, model.layers, args.ep_tokens
    owned = [e for e in range(E) if e % world == rank]
    lm = ModelShape(**{**model.__dict__, "experts": len(owned), "used": min(k, len(owned))})
    t0 = time.time()
    tier = torch.empty(NL * len(owned) * model.record, dtype=torch.uint8, pin_memory=True)
    fill_tier(gx, torch, model, tier, dev, owned=owned)
    slots = min(args.ep_slots, len(owned))
    arena = gx.Arena(lm, capacity_bytes=slots * model.record * NL, policy=gx.POLICY_AUTO,
                     max_tokens=world * T * k, host_tier_base=tier.data_ptr(), device=local)
    setup_s = time.time() - t0
    stream = torch.cuda.Stream(device=dev)
    ep = ExpertParallel(arena, comm or 0, rank, world, E, 0)   # expert e on rank e % world
    n_steps = args.ep_prewarm + args.warmup + args.steps
    ids_all, w_all = routes(model, n_steps * T, NL, seed=model.seed * 1000 + 31 + rank, rho=0.7)
    ids_s = [np.ascontiguousarray(ids_all[s * T:(s + 1) * T].transpose(1, 0, 2)) for s in range(n_steps)]  # [NL,T,k]
    w_np = np.ascontiguousarray(w_all.reshape(n_steps, T, NL, k).transpose(0, 2, 1, 3))                   # [n,NL,T,k]
    w_dev = torch.from_numpy(w_np).to(dev)
    xs = np.random.default_rng(100 + rank).standard_normal((NL, T, H)).astype(np.float32)
    x_dev = torch.from_numpy(xs).to(dev)
    out = torch.empty((NL, T, H), dtype=torch.float32, device=dev)
    xp = [x_dev[L] for L in range(NL)]
    op = [out[L] for L in range(NL)]

    def barrier():
        if world > 1:
            dist.barrier()

    def run(a, b, e2e=None):
        h = m = 0
        for s in range(a, b):
            if e2e is not None:
                h_x, h_w, h_out, w_fix = e2e
                x_dev.copy_(h_x, non_blocking=True)
                w_fix.copy_(h_w[s], non_blocking=True)
                ws = w_fix
            else:
                ws = w_dev[s]
            _, st = ep.stack_forward(0, xp, ids_s[s], [ws[L] for L in range(NL)], op, stream)
            if e2e is not None:
                e2e[2].copy_(out, non_blocking=True)
            h += st.hits
            m += st.misses
        return h, m

    first = args.ep_prewarm + args.warmup
    with torch.cuda.stream(stream):
        run(0, first)
        torch.cuda.synchronize()
        barrier()
        s0 = arena.stats()
        with ClockSampler(local, pci_bus_id(torch, dev)) as clk:
            ms, (h, m) = timed(torch, stream, lambda: run(first, n_steps))
        s1 = arena.stats()
        # e2e: inputs from pinned host memory, outputs back, inside the timed region
        h_x = torch.from_numpy(xs).pin_memory()
        h_w = torch.from_numpy(w_np).pin_memory()
        h_out = torch.empty((NL, T, H), dtype=torch.float32).pin_memory()
        w_fix = torch.empty((NL, T, k), dtype=torch.float32, device=dev)
        barrier()
        ms_e2e, _ = timed(torch, stream, lambda: run(first, n_steps, e2e=(h_x, h_w, h_out, w_fix)))
    t = torch.tensor([ms, ms_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(t[0].item()), float(t[1].item())
    parity = None
    if rank == 0:
        parity = ep_parity_check(gx, torch, model, ids_s[n_steps - 1][0], w_dev[n_steps - 1, 0], x_dev[0], out[0],
                                 dev, stream)
    err = device_error()
    moved = s1["bytes_h2d"] - s0["bytes_h2d"]
    ep.close()
    arena.close()
    del tier
    free_pinned(torch)
    metric, config = ep_config(gx, model, world, T, slots)
    # kernels per step: the row gather, the owner's reorder in and out, per
    # layer the three layer kernels (more when a layer runs in waves: one
    # gather, three per chunk, a scatter and a combine), the scatter home and
    # one combine per layer
    launches = args.steps * (4 + NL * 4)
    return {"metric": metric, "value": world * T * args.steps / (ms / 1e3), "ms_per_step": ms / args.steps,
            "config": config, "hit_rate_rank0": h / max(1, h + m), "h2d_gb_s_rank0": moved / (ms / 1e3) / 1e9,
            "e2e": {"value": world * T * args.steps / (ms_e2e / 1e3), "unit": "tok/s",
                    "h2d_bytes_per_step": NL * T * H * 4 + NL * T * k * 4, "d2h_bytes_per_step": NL * T * H * 4},
            "gpu_launches": launches, "ep_parity": parity, "device_error": err, "clocks": clk.summary(),
            "setup_s": setup_s, "exchanges_per_step": {"header_all_to_alls": 2, "host_syncs": 2, "row_all_to_alls": 2}}


def ep_parity_check(gx, torch, model, ids, w, x, got, dev, stream):
    """Layer 0 of one step again on this GPU alone: an arena holding every
    expert the step's tokens use (records from the same generator), the
    single-GPU layer entry, bits compared."""
    from galactus_b200.models import ModelShape
    ex = sorted(set(int(e) for e in ids.ravel()))
    m1 = ModelShape(**{**model.__dict__, "layers": 1, "experts": len(ex), "used": min(model.used, len(ex))})
    lib = gx.lib()
    a = gx.Arena(m1, capacity_bytes=len(ex) * model.record, policy=gx.POLICY_AUTO, max_tokens=ids.shape[0],
                 device=dev.index or 0)
    stage = torch.empty(model.record, dtype=torch.uint8, device=dev)
    for li, e in enumerate(ex):
        stage.zero_()
        sid = (0 * model.experts + e) * 3
        r = stage.data_ptr()
        gx.check(lib.gx_synth_weights(model.type_down, r, model.intermediate, model.hidden, model.seed, sid, 0.02, None))
        gx.check(lib.gx_synth_weights(model.type_gate, r + model.off_gate, model.hidden, model.intermediate, model.seed,
                                      sid + 1, 0.02, None))
        gx.check(lib.gx_synth_weights(model.type_up, r + model.off_up, model.hidden, model.intermediate, model.seed,
                                      sid + 2, 0.02, None))
        torch.cuda.synchronize()
        a.load_record(0, li, stage.cpu().numpy())
    remap = {e: i for i, e in enumerate(ex)}
    lids = np.array([[remap[int(e)] for e in row] for row in ids], np.int32)
    ref = torch.empty_like(got)
    with torch.cuda.stream(stream):
        a.layer_forward(0, x, lids, w, ref, stream)
    torch.cuda.synchronize()
    ok = bool(torch.equal(ref.view(torch.int32), got.view(torch.int32)))
    a.close()
    return {"bitwise_equal": ok, "checked": "rank 0, layer 0 of the last step, vs the single-GPU layer path "
                                           "(itself bit-identical to the CPU oracle in the GPU tests)"}


def run_ep(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import galactus_b200 as gx
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        pg = dist.distributed_c10d._get_default_group()
        comm = pg._get_backend(dev)._comm_ptr()
    gx.check(gx.lib().gx_device_init(local))
    r = ep_measure(args, gx, torch, world, rank, local, dev, comm)
    if rank == 0:
        line = {"metric": r.pop("metric"), "value": r.pop("value"), "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r.pop("ms_per_step"),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8 dot / f32 tail (q4_K gate/up + q6_K down weights, q8_K activations)",
                "data": "synthetic (seeded weights; Zipf(1.1)+AR(0.7) routes per GPU; N(0,1) states)",
                "config": r.pop("config"), "e2e": r.pop("e2e"), **r}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------- CPU legs

def cpu_baseline_leg(args, gx, model, traces, cfg1_ids):
    """The oracle (CPU port of the reference's arithmetic) on the headline
    workload: --cpu-tokens decode tokens through EVERY layer of the stack,
    all host threads; and the reference's own slot policy (compiled from its
    sources where they lie, when present) replayed on the sweep's and cfg 1's
    traces, for its hit rate beside ours."""
    from galactus_b200.routing import routes
    from oracle import oracle as orc
    NL, H, k = model.layers, model.hidden, model.used
    n = args.cpu_tokens
    ids, w = routes(model, n, NL, seed=model.seed * 1000 + 17, rho=0.7)
    xs = np.random.default_rng(0).standard_normal((n, NL, H)).astype(np.float32)
    total = 0.0
    for t in range(n):
        for L in range(NL):
            ex = sorted(set(ids[t, L].tolist()))
            recs = np.stack([orc.synth_record(model, model.seed, L, e) for e in ex])
            remap = {e: i for i, e in enumerate(ex)}
            cid = np.array([[remap[e] for e in ids[t, L]]], np.int32)
            t0 = time.perf_counter()
            orc.moe_layer(model, recs, xs[t, L][None], cid, w[t, L][None], threads=os.cpu_count())
            total += time.perf_counter() - t0
    per_tok = total / n
    out = {"value": 1.0 / per_tok, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
           "sample": f"{n} decode token(s) x all {NL} layers of the headline workload (oracle moe_layer, "
                     f"{os.cpu_count()} threads; ggml is not vendored with the reference)"}
    if orc.ref_replay_available():
        pol = []
        for slots, ids_tr in traces:
            # [n, NL, 1, k] -> (layer, ids) batches in serving order
            batches = [(L, ids_tr[s, L].ravel().tolist()) for s in range(ids_tr.shape[0]) for L in range(NL)]
            _, res = orc.ref_replay(0, NL - 1, model.experts, k, slots * 16384 * NL, 0.75, "auto", batches)
            tail = res[args.sweep_warm * NL:]
            hits = sum(sum(hh) for hh, _, _, _ in tail)
            acc = sum(len(hh) for hh, _, _, _ in tail)
            pol.append({"slots_per_layer": slots, "reference_policy_hit_rate": hits / max(1, acc)})
        if cfg1_ids is not None:
            _, res = orc.ref_replay(0, 0, 64, 8, 16 * 16384, 0.75, "auto", [(0, r.tolist()) for r in cfg1_ids])
            hits = sum(sum(hh) for hh, _, _, _ in res)
            pol.append({"olmoe_single_layer": "slru", "reference_policy_hit_rate": hits / (len(res) * 8)})
        out["reference_policy"] = pol
    return out


def cached_record(cache, limit, key, make):
    """The record of key from a bounded LRU cache (an OrderedDict, least
    recently used first), made and inserted on a miss. The record is returned
    before any later insertion can evict it."""
    r = cache.get(key)
    if r is None:
        while len(cache) >= limit:
            cache.popitem(last=False)
        r = cache[key] = make()
    else:
        cache.move_to_end(key)
    return r


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import galactus_b200 as gx
    from galactus_b200.routing import routes
    from oracle import oracle as orc
    model = shaped_model(gx, args.model or HEADLINE_MODEL, args.layers, args.experts)
    NL, H = model.layers, model.hidden
    ids_all, w_all = routes(model, args.warmup + args.steps, NL, seed=model.seed * 1000 + 17, rho=0.7)
    xs = np.random.default_rng(0).standard_normal((8, NL, H)).astype(np.float32)
    # each step: one decode token through every layer of the stack; the
    # records are generated once (a bounded cache; the routes' locality makes
    # most of them repeat) and only the layer arithmetic is timed
    from collections import OrderedDict
    cache: OrderedDict = OrderedDict()          # least recently used first
    limit = max(64, int(8e9 // model.record))
    times = []
    for t in range(args.warmup + args.steps):
        tt = 0.0
        for L in range(NL):
            ex = sorted(set(ids_all[t, L].tolist()))
            recs = np.stack([cached_record(cache, limit, (L, e), lambda L=L, e=e: orc.synth_record(model, model.seed, L, e))
                             for e in ex])
            remap = {e: i for i, e in enumerate(ex)}
            cid = np.array([[remap[e] for e in ids_all[t, L]]], np.int32)
            t0 = time.perf_counter()
            orc.moe_layer(model, recs, xs[t % 8, L][None], cid, w_all[t, L][None], threads=os.cpu_count())
            tt += time.perf_counter() - t0
        if t >= args.warmup:
            times.append(tt)
    per_tok = sum(times) / len(times)
    v = 1.0 / per_tok
    metric, config, dtype = single_config(gx, model)
    line = {
        "impl": "reference", "metric": metric, "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_tok * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded weights; Zipf(1.1)+AR(0.7) routes; N(0,1) "
                                                     "states)", "config": config,
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"each step: 1 decode token x all {NL} layers (oracle moe_layer, "
                                   f"{os.cpu_count()} threads; ggml is not vendored with the reference)"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args)
    elif world > 1 or args.ep:
        run_ep(args)
    else:
        run_single(args)


if __name__ == "__main__":
    main()
