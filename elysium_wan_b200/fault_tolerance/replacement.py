"""Spare selection for a convicted slot (reference:
src/wantrain/fault_tolerance/replacement.py:28-120): prefer an identical model,
then the same device class, then any live spare; within a tier the same region
first, then the most memory; hosts remembered as dead are skipped."""

from __future__ import annotations


def find_replacement(dead, candidates: list, match: str = "any", dead_hosts: set | None = None):
    dead_hosts = dead_hosts or set()
    # A dead spare never qualifies. Hosts remembered as dead are skipped, except
    # the loopback host, which every worker of a one-machine fleet shares.
    pool = [c for c in candidates
            if c.alive and (c.host not in dead_hosts or c.host == "127.0.0.1")]
    pool = [c for c in pool if c.node_id != dead.node_id]
    if not pool:
        return None

    def tier(c):
        if c.caps.get("device_name") and c.caps.get("device_name") == dead.caps.get("device_name"):
            return 0
        if c.device_class == dead.device_class:
            return 1
        return 2

    if match == "model":
        pool = [c for c in pool if tier(c) == 0]
    elif match == "device":
        pool = [c for c in pool if tier(c) <= 1]
    if not pool:
        return None
    return min(pool, key=lambda c: (tier(c), c.region != dead.region, -(c.vram_gb or 0), c.node_id))
