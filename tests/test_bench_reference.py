"""The reference arm of bench.py on the CPU: its bounded record cache keeps
every record a layer needs while it evicts, and one small run prints the
contract's line."""
import json
import subprocess
import sys
from collections import OrderedDict
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_record_cache_never_evicts_what_it_returns():
    sys.path.insert(0, str(ROOT))
    import bench
    cache = OrderedDict()
    made = []
    for step in range(50):
        keys = [(step % 7, e) for e in sorted({(step * 5 + j * 3) % 11 for j in range(4)})]
        recs = [bench.cached_record(cache, 3, k, lambda k=k: (made.append(k), k)[1]) for k in keys]
        assert recs == keys and len(cache) <= 3
    assert len(made) > 3   # evictions happened


def test_reference_arm_prints_its_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--layers", "2", "--steps", "2",
                          "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] in ("port", "reference") and line["steps"] == 2
