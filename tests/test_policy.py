"""The product's slot policy (gx_policy_*, host only) against the reference's
own ExpertCache/ExpertStore: the hand-worked KATs of
scripts/tests/test-replay-cache.py:70-112, the committed traces answered by
the reference binary (tests/golden/policy_traces.json), and fresh traces
replayed live through oracle/_ref/h4ref_replay when it is built."""
import json
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"
POLICY = {"auto": 0, "uniform": 1, "plan": 2, "frequency": 3}


def make_policy(gxlib, first, last, experts, used, capacity, fraction, policy, record=16384):
    return gxlib.SlotPolicy(first, last, experts, used, [record] * (last - first + 1), capacity, fraction, policy)


def test_slru_by_hand(gxlib):
    """quota 4 at 0.5: 2 protected, 2 probation; every branch fires once."""
    p = make_policy(gxlib, 0, 0, 64, 2, 4 * 16384, 0.5, POLICY["uniform"])
    assert p.quota(0) == (4, 2, 2)
    _, h, ev, _ = p.serve(0, [1])
    assert h == [False]
    _, h, _, _ = p.serve(0, [2])
    assert h == [False]
    _, h, _, _ = p.serve(0, [1])
    assert h == [True]          # second access promotes 1
    _, h, _, _ = p.serve(0, [3])
    assert h == [False]
    _, h, ev, _ = p.serve(0, [4])
    assert h == [False] and ev == [2]   # probation holds 2: oldest (2) leaves
    assert p.slot_of(0, 2) == -1 and p.slot_of(0, 1) >= 0
    _, h, _, _ = p.serve(0, [3])
    assert h == [True]
    _, h, ev, _ = p.serve(0, [4])
    assert h == [True]          # promoting 3 and 4 demotes 1 to probation
    # quota 4 never holds more than 4 keys, slots are a permutation of 0..3
    slots = [p.slot_of(0, e) for e in range(64) if p.slot_of(0, e) >= 0]
    assert sorted(slots) == sorted(set(slots)) and len(slots) <= 4


def test_segment_split_and_floor(gxlib):
    # shipped split of quota 37 at 0.75 is 27 protected and 10 probation
    p = make_policy(gxlib, 0, 0, 128, 8, 37 * 16384, 0.75, POLICY["uniform"])
    assert p.quota(0) == (37, 27, 10)
    # the probation floor (used experts) applies to auto/plan/frequency, not uniform
    p = make_policy(gxlib, 0, 0, 128, 8, 9 * 16384, 0.75, POLICY["auto"])
    q, prot, prob = p.quota(0)
    assert q == 9 and prob == 8 and prot == 1
    p = make_policy(gxlib, 0, 0, 128, 8, 9 * 16384, 0.75, POLICY["uniform"])
    assert p.quota(0) == (9, 6, 3)
    # full residency: both segments equal the quota
    p = make_policy(gxlib, 0, 0, 64, 8, 10 ** 12, 0.75, POLICY["auto"])
    assert p.quota(0) == (64, 64, 64)


def test_policy_rejects(gxlib):
    from galactus_b200 import GxError
    with pytest.raises(GxError):
        make_policy(gxlib, 0, 0, 64, 8, 16384, 0.75, 1)          # quota 1
    with pytest.raises(GxError):
        make_policy(gxlib, 0, 0, 64, 8, 10 * 16384, 1.0, 1)      # fraction outside (0,1)
    with pytest.raises(GxError):
        gxlib.SlotPolicy(0, 0, 64, 8, [1000], 10 ** 9)            # record not 16 KiB aligned
    p = make_policy(gxlib, 0, 0, 64, 8, 16 * 16384, 0.75, 1)    # probation 4
    with pytest.raises(GxError) as e:
        p.serve(0, [1, 2, 3, 4, 5])                               # 5 distinct > probation
    assert e.value.code == gxlib._lib.GX_ERR_BATCH
    with pytest.raises(GxError) as e:
        p.serve(0, [64])
    assert e.value.code == gxlib._lib.GX_ERR_DOMAIN
    # duplicates in a batch count once
    slots, hits, _, st = p.serve(0, [1, 1, 2, 2])
    assert st.distinct == 2 and slots[0] == slots[1] and hits == [False, True, False, True]


def test_full_residency_never_evicts(gxlib):
    p = make_policy(gxlib, 0, 1, 32, 4, 10 ** 12, 0.75, POLICY["auto"])
    rng = np.random.default_rng(0)
    for _ in range(500):
        layer = int(rng.integers(0, 2))
        _, _, ev, _ = p.serve(layer, rng.choice(32, 4, replace=False).tolist())
        assert ev == [-1] * 4


def test_lru_mode(gxlib):
    p = make_policy(gxlib, 0, 0, 64, 2, 4 * 16384, 0.75, 4)
    assert p.quota(0) == (4, 0, 4)
    for e in [1, 2, 3, 4]:
        p.serve(0, [e])
    p.serve(0, [1])                 # 1 becomes most recent
    _, h, ev, _ = p.serve(0, [5])   # evicts the least recent: 2
    assert h == [False] and ev == [2]
    assert p.slot_of(0, 5) == 1     # 2's slot (LIFO: released then reused)


def _check_case(gxlib, case, batches_answers):
    p = make_policy(gxlib, case["first"], case["last"], case["experts"], case["used"], case["capacity"],
                    case["fraction"], POLICY[case["policy"]])
    for layer in range(case["first"], case["last"] + 1):
        assert list(p.quota(layer)) == list(case["quotas"][layer - case["first"]])
    assert batches_answers, "an empty comparison is not a pass"
    for bi, b in enumerate(batches_answers):
        slots, hits, ev, _ = p.serve(b["layer"], b["experts"])
        where = f'{case["policy"]} e{case["experts"]} batch {bi}'
        assert [int(h) for h in hits] == b["hits"], where
        assert ev == b["evicted"], where
        assert slots == b["slots"], where
        resident = [e for e in range(case["experts"]) if p.slot_of(b["layer"], e) >= 0]
        assert resident == b["resident"], where


def test_policy_matches_reference_traces(gxlib):
    cases = json.loads((GOLD / "policy_traces.json").read_text())
    assert len(cases) == 20
    for case in cases:
        _check_case(gxlib, case, case["batches"])


def test_policy_matches_live_reference(gxlib, orc):
    if not orc.ref_replay_available():
        pytest.skip("reference policy binary not built (reference tree absent)")
    rng = np.random.default_rng(123)
    for policy in ["uniform", "frequency", "auto"]:
        experts, used, first, last = 48, 6, 0, 1
        capacity = 14 * 2 * 16384
        batches = []
        for bi in range(6000):       # enough accesses to cross the 4096-access halving
            layer = bi % 2
            n_tok = int(rng.integers(1, 3))
            ex = []
            for _ in range(n_tok):
                ex += rng.choice(experts, used, replace=False, p=None).tolist()
            batches.append((layer, ex))
        # keep batches within the probation bound of the reference engine
        quotas, _ = orc.ref_replay(first, last, experts, used, capacity, 0.75, policy, batches[:1])
        bound = min(quotas[0][0], quotas[0][2])
        trimmed = []
        for layer, ex in batches:
            out, seen = [], set()
            for e in ex:
                if e in seen or len(seen) < bound:
                    seen.add(e)
                    out.append(e)
            trimmed.append((layer, out))
        batches = trimmed
        quotas, res = orc.ref_replay(first, last, experts, used, capacity, 0.75, policy, batches)
        answers = [{"layer": l, "experts": e, "hits": [int(h) for h in r[0]], "evicted": r[1], "slots": r[2],
                    "resident": r[3]} for (l, e), r in zip(batches, res)]
        case = {"policy": policy, "first": first, "last": last, "experts": experts, "used": used,
                "capacity": capacity, "fraction": 0.75, "quotas": quotas}
        _check_case(gxlib, case, answers)
