"""Expert placement over a GPU roster by rendezvous (highest-random-weight)
hashing.

Same rule as src/expert_network/hrw.py:11-30: the owner of expert e under a
roster is the node id n whose sha256(f"{n}:{e}") digest is byte-wise
largest. Every rank computes the same placement from the roster alone.

`bounded_plan` is a capacity-bounded variant: experts are placed in
ascending id order, each on its highest-scoring node that still has fewer
than ceil(E / N) experts. It uses the same scores (so it is still
coordination-free) and gives every node at most ceil(E / N) experts, which
bounds the per-GPU weight bytes of an expert-parallel decode step.
"""
from __future__ import annotations

import hashlib


def score(node_id: str, expert_id: int) -> bytes:
    return hashlib.sha256(f"{node_id}:{expert_id}".encode()).digest()


def owner(roster, expert_id: int) -> str:
    return max(roster, key=lambda n: score(n, expert_id))


def partition(roster, me: str, num_experts: int):
    if me not in roster:
        raise ValueError(f"{me!r} is not in the roster {list(roster)}")
    return sorted(e for e in range(num_experts) if owner(roster, e) == me)


def plan(roster, num_experts: int) -> dict:
    out = {n: [] for n in roster}
    for e in range(num_experts):
        out[owner(roster, e)].append(e)
    return out


def bounded_plan(roster, num_experts: int, capacity: int = None) -> dict:
    roster = list(roster)
    if capacity is None:
        capacity = -(-num_experts // len(roster))
    if capacity * len(roster) < num_experts:
        raise ValueError("capacity too small for the number of experts")
    out = {n: [] for n in roster}
    for e in range(num_experts):
        for n in sorted(roster, key=lambda n: score(n, e), reverse=True):
            if len(out[n]) < capacity:
                out[n].append(e)
                break
    return out


def gpu_roster(world_size: int):
    """The roster gpu0..gpu{N-1} used for one box."""
    return [f"gpu{i}" for i in range(world_size)]


def owner_table(placement: dict, roster, num_experts: int):
    """expert id -> rank index (position of its owner in the roster)."""
    rank = {n: i for i, n in enumerate(roster)}
    table = [-1] * num_experts
    for n, experts in placement.items():
        for e in experts:
            table[e] = rank[n]
    return table
