"""Route traces: the observer records every served micro-batch in the
reference's "galactus.route-observer.v1" format; the reference's own replay
tool (scripts/replay-cache.py --verify, run when GALACTUS_REFERENCE_DIR names
the reference tree) reads our trace and finds its replayed SLRU in agreement with every
residency bit and every byte."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

_REF = os.environ.get("GALACTUS_REFERENCE_DIR", "")
REPLAY = Path(_REF) / "scripts" / "replay-cache.py" if _REF else None


def _zipf_batches(rng, n_steps, layers, experts, k):
    p = 1.0 / np.arange(1, experts + 1) ** 1.1
    p /= p.sum()
    return [[rng.choice(experts, k, replace=False, p=p).astype(np.int32) for _ in range(layers)] for _ in range(n_steps)]


def test_policy_trace_matches_served_batches(gxlib, tmp_path):
    from galactus_b200.route_trace import close_trace, open_trace, read_trace
    layers, experts, used = 4, 64, 8
    rec = [4079616] * layers
    pol = gxlib.SlotPolicy(0, layers - 1, experts, used, rec, 16 * sum(rec), 0.5, gxlib.POLICY_UNIFORM)
    path = tmp_path / "routes.txt"
    open_trace(str(path), arch="olmoe")
    rng = np.random.default_rng(1)
    steps = _zipf_batches(rng, 60, layers, experts, used)
    hits_seen = []
    for step in steps:
        for L, ids in enumerate(step):
            before = [pol.slot_of(L, int(e)) >= 0 for e in ids]
            pol.serve(L, ids.tolist())
            hits_seen.append(before)
    close_trace()
    tr = read_trace(str(path))
    assert tr["version"] == 1 and tr["arch"] == "olmoe"
    assert (tr["first_layer"], tr["last_layer"], tr["experts"], tr["used"]) == (0, layers - 1, experts, used)
    assert tr["quota"] == 16 and tr["slots"] == 16 and tr["cache_bytes"] == 16 * sum(rec)
    assert tr["records"] == {L: rec[L] for L in range(layers)}
    assert tr["n_entries"] == len(tr["entries"]) == 60 * layers and not tr["truncated"]
    flat = [(L, ids) for step in steps for L, ids in enumerate(step)]
    for e, (L, ids), before in zip(tr["entries"], flat, hits_seen):
        assert e["layer"] == L and e["ids"] == ids.tolist()
        assert e["resident"] == [int(b) for b in before]
        assert e["enter_ns"] <= e["serve_start_ns"] <= e["serve_end_ns"]
    # closed: further serves are not recorded and the file stays as written
    pol.serve(0, steps[0][0].tolist())
    assert len(read_trace(str(path))["entries"]) == 60 * layers


def test_trace_cap_truncates(gxlib, tmp_path):
    from galactus_b200.route_trace import close_trace, open_trace, read_trace
    rec = [1 << 20] * 2
    pol = gxlib.SlotPolicy(0, 1, 16, 2, rec, 8 * sum(rec), 0.75, gxlib.POLICY_UNIFORM)
    path = tmp_path / "capped.txt"
    open_trace(str(path), entry_cap=5)
    for i in range(9):
        pol.serve(i % 2, [i % 16, (i + 3) % 16])
    close_trace()
    tr = read_trace(str(path))
    assert tr["n_entries"] == 5 and tr["truncated"]


@pytest.mark.skipif(REPLAY is None or not REPLAY.exists(), reason="GALACTUS_REFERENCE_DIR unset or without the replay tool")
def test_reference_replay_verifies_our_trace(gxlib, tmp_path):
    """The reference's replay-cache.py --verify replays its SLRU baseline over
    our trace: every recorded residency bit and the recorded bytes agree (the
    tool exits with an error on the first disagreement)."""
    from galactus_b200.route_trace import close_trace, open_trace
    layers, experts, used = 6, 64, 8
    rec = [4079616] * layers
    pol = gxlib.SlotPolicy(0, layers - 1, experts, used, rec, 20 * sum(rec), 0.5, gxlib.POLICY_UNIFORM)
    path = tmp_path / "routes.txt"
    open_trace(str(path), arch="olmoe")
    rng = np.random.default_rng(8)
    for step in _zipf_batches(rng, 300, layers, experts, used):
        for L, ids in enumerate(step):
            pol.serve(L, ids.tolist())
    close_trace()
    # bytes in the trace: whole records per miss, as the reference's reader counts them
    r = subprocess.run([sys.executable, str(REPLAY), "--routes", str(path), "--verify", "--policy", "slru"],
                       capture_output=True, text=True, timeout=600, cwd=str(tmp_path))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
