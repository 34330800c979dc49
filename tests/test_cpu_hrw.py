"""Expert placement: our rendezvous hashing against the reference's own
plans (tests/golden/hrw_plans.json, generated from src/expert_network/hrw.py
by tests/golden/make_golden.py)."""
from __future__ import annotations

import json
import os

import pytest

from expert_sniper_b200 import hrw

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "hrw_plans.json")


def _plans():
    with open(GOLDEN) as f:
        return json.load(f)["plans"]


@pytest.mark.parametrize("case", _plans(), ids=lambda c: f"{len(c['roster'])}x{c['num_experts']}")
def test_plan_matches_reference(case):
    roster, E = case["roster"], case["num_experts"]
    assert hrw.plan(roster, E) == case["plan"]
    assert [hrw.owner(roster, e) for e in range(E)] == case["owners"]
    if "partition_node-b" in case:
        assert hrw.partition(roster, "node-b", E) == case["partition_node-b"]


def test_known_counts_128_over_8():
    counts = [len(v) for v in hrw.plan(hrw.gpu_roster(8), 128).values()]
    assert counts == [7, 20, 18, 17, 17, 11, 16, 22]
    assert hrw.plan(hrw.gpu_roster(8), 128)["gpu0"] == [13, 33, 34, 42, 64, 72, 101]


@pytest.mark.parametrize("n,E", [(2, 128), (4, 128), (8, 128), (8, 64), (8, 512), (3, 10)])
def test_bounded_plan(n, E):
    roster = hrw.gpu_roster(n)
    bp = hrw.bounded_plan(roster, E)
    cap = -(-E // n)
    assert sorted(e for v in bp.values() for e in v) == list(range(E))
    assert max(len(v) for v in bp.values()) <= cap
    # experts whose HRW owner still had room stay where plain HRW puts them
    plain = hrw.plan(roster, E)
    kept = sum(len(set(bp[r]) & set(plain[r])) for r in roster)
    assert kept >= E * 0.6


def test_owner_table_and_errors():
    roster = hrw.gpu_roster(4)
    table = hrw.owner_table(hrw.plan(roster, 64), roster, 64)
    assert min(table) == 0 and max(table) <= 3 and -1 not in table
    with pytest.raises(ValueError):
        hrw.partition(roster, "gpu9", 64)
