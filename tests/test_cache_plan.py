"""Cache plans: the plan-file parser and the quota allocator against the
reference's own code (golden vectors made by oracle/_ref/h4ref_plan, built
from src/h4/h4-cache-plan.cpp), and the engine quotas feeding the policy."""
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
REF_PLAN = HERE.parent / "oracle" / "_ref" / "h4ref_plan"


def test_allocator_matches_reference_golden(gxlib):
    from galactus_b200.cache_plan import plan_layer_quotas
    cases = json.loads((HERE / "golden" / "plan_quotas.json").read_text())
    assert len(cases) >= 30
    for i, c in enumerate(cases):
        got = plan_layer_quotas(np.array(c["curves"], np.uint32), c["record_bytes"], c["budget"], c["floor"],
                                c["ceiling"])
        assert got.tolist() == c["quotas"], f"case {i}"
        spent = sum(q * r for q, r in zip(got.tolist(), c["record_bytes"]))
        assert spent <= c["budget"]
        assert all(c["floor"] <= q <= max(c["floor"], c["ceiling"]) for q in got.tolist())


@pytest.mark.skipif(not REF_PLAN.exists(), reason="reference plan binary not built here")
def test_allocator_matches_reference_live(gxlib):
    from galactus_b200.cache_plan import plan_layer_quotas
    rng = np.random.default_rng(99)
    for _ in range(60):
        n, m = int(rng.integers(1, 12)), int(rng.integers(4, 40))
        curves = np.sort(rng.integers(0, 5000, (n, m)), axis=1)[:, ::-1].copy()
        curves[rng.random((n, m)) < 0.2] += 7   # rises
        rec = rng.integers(1, 9, n) * 16384
        floor = int(rng.integers(0, 4))
        ceiling = int(rng.integers(floor, m + 2))
        budget = int(rec.sum() * (floor + rng.integers(0, m)))
        stdin = f"Q {n} {m} {floor} {ceiling} {budget}\n" + " ".join(map(str, rec)) + "\n" + \
            "\n".join(" ".join(map(str, row)) for row in curves) + "\n"
        out = subprocess.run([str(REF_PLAN)], input=stdin, capture_output=True, text=True, check=True).stdout.split()
        if out[0] == "E":
            with pytest.raises(gxlib.GxError):
                plan_layer_quotas(curves.astype(np.uint32), rec, budget, floor, ceiling)
            continue
        got = plan_layer_quotas(curves.astype(np.uint32), rec, budget, floor, ceiling)
        assert got.tolist() == [int(v) for v in out[1:]]


def _plan_text(first, last, experts, curves, *, header="galactus-cache-plan 1", end=True, extra=""):
    lines = [header, "arch testmoe", f"first_layer {first}", f"last_layer {last}", f"experts {experts}", "used 4",
             "source synthetic.routes", "tokens 64"]
    lines += [f"curve {first + i} " + " ".join(map(str, row)) for i, row in enumerate(curves)]
    if extra:
        lines.append(extra)
    if end:
        lines.append("end")
    return "\n".join(lines) + "\n"


def test_plan_file_parse_and_reject(gxlib, tmp_path):
    from galactus_b200.cache_plan import CachePlan
    rng = np.random.default_rng(3)
    curves = [sorted(rng.integers(0, 900, 17).tolist(), reverse=True) for _ in range(5)]
    good = tmp_path / "plan.txt"
    good.write_text(_plan_text(2, 6, 16, curves))
    plan = CachePlan(str(good))
    assert (plan.first_layer, plan.last_layer, plan.experts, plan.arch) == (2, 6, 16, "testmoe")
    assert plan.curves().tolist() == curves
    bad = {
        "header": _plan_text(2, 6, 16, curves, header="galactus-cache-plan 2"),
        "no_end": _plan_text(2, 6, 16, curves, end=False),
        "short_curve": _plan_text(2, 6, 16, [curves[0][:-3]] + curves[1:]),
        "unknown_key": _plan_text(2, 6, 16, curves, extra="colour blue"),
        "count": _plan_text(2, 7, 16, curves),
        "not_contiguous": _plan_text(2, 6, 16, curves).replace("curve 4 ", "curve 5 ", 1),
    }
    for name, text in bad.items():
        f = tmp_path / f"{name}.txt"
        f.write_text(text)
        with pytest.raises(gxlib.GxError):
            CachePlan(str(f))
        if REF_PLAN.exists():
            out = subprocess.run([str(REF_PLAN)], input=f"L {f}\n", capture_output=True, text=True).stdout.split()
            assert out[0] == "E", name   # the reference rejects it too
    if REF_PLAN.exists():
        out = subprocess.run([str(REF_PLAN)], input=f"L {good}\n", capture_output=True, text=True).stdout.splitlines()
        assert out[0].split() == ["P", "2", "6", "16"]
        assert [list(map(int, l.split())) for l in out[1:]] == curves


def test_engine_quotas_feed_the_policy(gxlib, tmp_path):
    """The engine's plan: the uniform budget, floor = uniform probation + 1; the
    policy built with those quotas gives each layer its planned quota, inside
    the uniform arena."""
    from galactus_b200.cache_plan import CachePlan
    rng = np.random.default_rng(11)
    experts, used, layers = 64, 8, 12
    curves = []
    for L in range(layers):
        start = 2000 - 100 * L
        row = [int(start * (0.93 ** max(0, q - 2)) * (0.6 if L < 3 else 1.0)) for q in range(experts + 1)]
        row[0] = row[1] = row[2]
        curves.append(row)
    f = tmp_path / "p.txt"
    f.write_text(_plan_text(0, layers - 1, experts, curves))
    plan = CachePlan(str(f))
    rec = [4079616] * layers
    capacity = 16 * sum(rec)   # uniform quota 16
    q = plan.engine_quotas(rec, capacity, 0.75, used=used)
    assert q is not None and len(q) == layers
    assert int((q.astype(np.int64) * np.array(rec)).sum()) <= capacity
    assert q.tolist() != [16] * layers   # the plan moved slots
    pol = gxlib.SlotPolicy(0, layers - 1, experts, used, rec, capacity, 0.75, gxlib.POLICY_AUTO, plan_quotas=q.tolist())
    assert [pol.quota(L)[0] for L in range(layers)] == q.tolist()
    # full residency: the uniform quota stays
    assert plan.engine_quotas(rec, experts * sum(rec), 0.75, used=used) is None
