"""Generate the committed golden fixtures under tests/golden/.

Run in a container that has the gguf-py package (0.19.0) and, for the policy
traces, the reference tree (oracle/_ref/h4ref_replay built by oracle/Makefile):

    python tests/golden/make_golden.py

Fixtures:
  iq1s_grid.npy          int8 [2048, 8], the IQ1_S codebook read from gguf-py
  dequant_<type>.npz     random blocks and gguf-py's float dequantization of them
  q8_0_quant.npz         f32 blocks and gguf-py's Q8_0 quantization of them
  policy_traces.json     micro-batch traces and the reference policy's answers
                         (hits, evictions, slots, resident set) per batch
  plan_quotas.json       synthetic miss curves (noisy, with flat steps and
                         rises), budgets, floors, ceilings and the reference
                         allocator's quotas (oracle/_ref/h4ref_plan)
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from gguf.quants import IQ1_S, MXFP4, Q4_K, Q6_K, Q8_0  # noqa: E402

N_BLOCKS = 48


def fp16_bits(rng, n, lo, hi):
    return np.float16(rng.uniform(lo, hi, n)).view(np.uint16)


def blocks_q8_0(rng):
    b = np.zeros((N_BLOCKS, 34), np.uint8)
    b[:, 0:2] = fp16_bits(rng, N_BLOCKS, -0.05, 0.05).view(np.uint8).reshape(-1, 2)
    b[:, 2:] = rng.integers(0, 256, (N_BLOCKS, 32), dtype=np.uint8)
    return b


def blocks_q4_k(rng):
    b = rng.integers(0, 256, (N_BLOCKS, 144), dtype=np.uint8)
    b[:, 0:2] = fp16_bits(rng, N_BLOCKS, 1e-4, 0.01).view(np.uint8).reshape(-1, 2)
    b[:, 2:4] = fp16_bits(rng, N_BLOCKS, 1e-4, 0.01).view(np.uint8).reshape(-1, 2)
    return b


def blocks_q6_k(rng):
    b = rng.integers(0, 256, (N_BLOCKS, 210), dtype=np.uint8)
    b[:, 208:210] = fp16_bits(rng, N_BLOCKS, 1e-4, 0.01).view(np.uint8).reshape(-1, 2)
    return b


def blocks_mxfp4(rng):
    b = rng.integers(0, 256, (N_BLOCKS, 17), dtype=np.uint8)
    b[:, 0] = rng.integers(100, 150, N_BLOCKS, dtype=np.uint8)
    b[:3, 0] = [0, 1, 2]  # the subnormal scales of e8m0_half
    return b


def blocks_iq1_s(rng):
    b = rng.integers(0, 256, (N_BLOCKS, 50), dtype=np.uint8)
    b[:, 0:2] = fp16_bits(rng, N_BLOCKS, 1e-4, 0.01).view(np.uint8).reshape(-1, 2)
    return b


def synthetic_curve(rng, experts: int) -> list[int]:
    """Misses at quota 0..experts: a falling curve with noise, flat steps and
    occasional rises (an SLRU is not a stack algorithm); entries 0 and 1 repeat
    the value at quota 2, as the reference's plans do."""
    start = int(rng.integers(500, 3000))
    vals, v = [], float(start)
    for q in range(experts + 1):
        if q >= 3:
            v = max(0.0, v * float(rng.uniform(0.80, 1.0)) - float(rng.integers(0, 20)))
            if rng.random() < 0.15:
                v += float(rng.integers(1, 40))   # a rise
        vals.append(int(v))
    vals[0] = vals[1] = vals[2]
    return vals


def make_plan_cases() -> None:
    import subprocess
    ref = HERE.parent.parent / "oracle" / "_ref" / "h4ref_plan"
    if not ref.exists():
        print("reference plan binary absent: plan_quotas.json not regenerated")
        return
    rng = np.random.default_rng(4242)
    cases = []
    for i in range(40):
        n = int(rng.integers(1, 24))
        experts = int(rng.choice([8, 16, 32, 64, 128]))
        curves = [synthetic_curve(rng, experts) for _ in range(n)]
        rec = [int(rng.choice([16384 * int(rng.integers(50, 400)), 4079616, 5013504])) for _ in range(n)]
        floor = int(rng.integers(2, max(3, experts // 4)))
        ceiling = int(rng.choice([experts, max(floor, experts // 2)]))
        base = sum(rec) * floor
        budget = int(base + rng.uniform(-0.05, 1.5) * sum(rec) * max(1, experts // 3))
        stdin = f"Q {n} {experts + 1} {floor} {ceiling} {budget}\n" + " ".join(map(str, rec)) + "\n" + \
            "\n".join(" ".join(map(str, c)) for c in curves) + "\n"
        out = subprocess.run([str(ref)], input=stdin, capture_output=True, text=True, check=True).stdout.split()
        cases.append({"curves": curves, "record_bytes": rec, "floor": floor, "ceiling": ceiling, "budget": budget,
                      "quotas": [int(v) for v in out[1:]] if out[0] == "R" else None})
    (HERE / "plan_quotas.json").write_text(json.dumps(cases))
    print("plan_quotas.json:", len(cases), "cases,", sum(c["quotas"] is None for c in cases), "rejected")


def main() -> None:
    rng = np.random.default_rng(20261201)
    IQ1_S.init_grid()
    grid = np.asarray(IQ1_S.grid).reshape(2048, 8).astype(np.int8)
    np.save(HERE / "iq1s_grid.npy", grid)

    for name, cls, make in [("q8_0", Q8_0, blocks_q8_0), ("q4_K", Q4_K, blocks_q4_k), ("q6_K", Q6_K, blocks_q6_k),
                            ("mxfp4", MXFP4, blocks_mxfp4), ("iq1_s", IQ1_S, blocks_iq1_s)]:
        blocks = make(rng)
        expected = cls.dequantize_blocks(blocks.copy()).astype(np.float32)
        np.savez_compressed(HERE / f"dequant_{name}.npz", blocks=blocks, expected=expected)

    x = rng.standard_normal((256, 32)).astype(np.float32)
    x[0] = 0.0                                # all-zero block
    x[1, :] = np.linspace(-1, 1, 32)          # exact values
    q = Q8_0.quantize_blocks(x.copy())
    np.savez_compressed(HERE / "q8_0_quant.npz", x=x, q=q.astype(np.uint8))

    # policy traces, answered by the reference's own ExpertCache/ExpertStore
    from oracle import oracle as orc
    orc.build()
    make_plan_cases()
    if not orc.ref_replay_available():
        print("reference policy binary absent: policy_traces.json not regenerated")
        return
    cases = []
    prng = np.random.default_rng(7)
    for policy in ["uniform", "frequency", "auto", "plan"]:
        for experts, used, quota_slots, fraction, n_batches, tok in [
            (64, 8, 16, 0.75, 300, 1), (64, 8, 12, 0.5, 300, 1), (128, 8, 32, 0.75, 200, 2),
            (32, 4, 10, 0.75, 200, 1), (16, 2, 16, 0.75, 80, 2),
        ]:
            first, last = 3, 5
            layers = last - first + 1
            capacity = quota_slots * layers * 16384 + 1000
            batches = []
            zipf = 1.0 / np.arange(1, experts + 1) ** 1.1
            zipf /= zipf.sum()
            for bi in range(n_batches):
                layer = first + (bi % layers)
                ex: list[int] = []
                for _ in range(tok):
                    pick = prng.choice(experts, size=used, replace=False, p=zipf)
                    ex.extend(int(e) for e in pick)
                batches.append((layer, ex))
            # the engine refuses a micro-batch with more distinct experts than
            # min(quota, probation) of its layer: keep every batch inside it
            quotas, _ = orc.ref_replay(first, last, experts, used, capacity, fraction, policy, batches[:1])
            kept = []
            for layer, ex in batches:
                q, _, prob = quotas[layer - first]
                bound = min(q, prob)
                out, seen = [], set()
                for e in ex:
                    if e in seen or len(seen) < bound:
                        seen.add(e)
                        out.append(e)
                kept.append((layer, out))
            batches = kept
            quotas, res = orc.ref_replay(first, last, experts, used, capacity, fraction, policy, batches)
            ok = []
            for (layer, ex), r in zip(batches, res):
                ok.append({"layer": layer, "experts": ex, "hits": [int(h) for h in r[0]], "evicted": r[1],
                           "slots": r[2], "resident": r[3]})
            cases.append({"policy": policy, "first": first, "last": last, "experts": experts, "used": used,
                          "capacity": capacity, "fraction": fraction, "quotas": quotas, "batches": ok})
    (HERE / "policy_traces.json").write_text(json.dumps(cases))
    print(f"wrote {len(cases)} policy cases")


if __name__ == "__main__":
    if "--plans" in sys.argv:
        make_plan_cases()
        sys.exit(0)
    main()
