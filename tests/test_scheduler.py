"""Zero-bubble solver, IWRR and partition DP.

Would fail if: a solved order dropped or duplicated an op, deadlocked,
exceeded its memory budget, ran B/W out of microbatch order, lost to 1F1B on
uniform costs, or if IWRR / the min-max partition disagreed with brute force.
"""

import itertools
import random

import pytest

from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.scheduler import partition as part
from elysium_wan_b200.scheduler.zero_bubble import (ZBConfig, iwrr, one_f_one_b, peak_memory,
                                                    simulate, zero_bubble)


def _valid(orders, p, m):
    for s, o in enumerate(orders):
        for op in "FBW":
            assert sorted(mb for x, mb in o if x == op) == list(range(m)), (s, op)
            mbs = [mb for x, mb in o if x == op]
            assert mbs == sorted(mbs)


@pytest.mark.parametrize("p,m", [(2, 4), (4, 8), (4, 16), (8, 16), (8, 64)])
@pytest.mark.parametrize("mode", ["1p", "2p"])
def test_zb_valid_and_beats_1f1b(p, m, mode):
    cfg = ZBConfig(p, m, [1.0] * p, [1.0] * p, [1.0] * p)
    sch = zero_bubble(cfg, mode)
    _valid(sch.orders, p, m)
    simulate(cfg, sch.orders)
    base = one_f_one_b(cfg)
    assert sch.makespan <= base.makespan + 1e-9
    lim = (1 if mode == "1p" else 2) * p * 1.0
    assert max(peak_memory(cfg, sch.orders)) <= lim + 1e-9


def test_zb_2p_is_nearly_bubble_free():
    p, m = 4, 16
    cfg = ZBConfig(p, m, [1.0] * p, [1.0] * p, [1.0] * p)
    sch = zero_bubble(cfg, "2p")
    assert sch.bubble_rate < 0.05


def test_zb_heterogeneous_costs_and_comm():
    rnd = random.Random(0)
    for _ in range(20):
        p = rnd.randint(2, 6)
        m = rnd.randint(p, 3 * p)
        f = [rnd.uniform(0.5, 2) for _ in range(p)]
        cfg = ZBConfig(p, m, f, [x * rnd.uniform(0.9, 1.4) for x in f],
                       [x * rnd.uniform(0.6, 1.0) for x in f], [rnd.uniform(0, 0.5) for _ in range(p - 1)])
        sch = zero_bubble(cfg, "2p")
        _valid(sch.orders, p, m)
        simulate(cfg, sch.orders)


def test_single_stage():
    cfg = ZBConfig(1, 5, [1.0], [1.0], [1.0])
    sch = zero_bubble(cfg, "1p")
    _valid(sch.orders, 1, 5)


def test_iwrr_matches_bruteforce():
    assert iwrr(6, [1, 1]) == [0, 1, 0, 1, 0, 1]
    for w in ([2, 1], [1, 3, 2], [1.5, 1.0]):
        got = iwrr(12, w)
        for i in range(1, 13):
            cnt = [got[:i].count(q) for q in range(len(w))]
            # every prefix is within one microbatch of the weighted share
            for q in range(len(w)):
                assert abs(cnt[q] - i * w[q] / sum(w)) <= 1.0 + 1e-9


def test_partition_dp_matches_bruteforce():
    rnd = random.Random(1)
    for _ in range(30):
        n = rnd.randint(3, 8)
        S = rnd.randint(1, n)
        costs = [rnd.uniform(1, 10) for _ in range(n)]
        speeds = [rnd.uniform(0.5, 2) for _ in range(S)]
        got = part.assign_layers(costs, speeds)
        best = None
        for cuts in itertools.combinations(range(1, n), S - 1):
            b = [0, *cuts, n]
            v = max(sum(costs[b[i]:b[i + 1]]) / speeds[i] for i in range(S))
            best = v if best is None else min(best, v)
        gv = max(sum(costs[a:b]) / speeds[i] for i, (a, b) in enumerate(got))
        assert abs(gv - best) < 1e-9


def test_even_partition_baseline_cut():
    cfg = make_config("gpt15b")
    p = part.even_blocks_partition(cfg, 8)
    assert p[0] == [0, 7] and p[-1] == [43, 50]
    assert all(b - a == 6 for a, b in p[1:-1])


def test_selective_recompute_rules():
    """The in-flight rule (recompute only where an order holds more than one
    microbatch between F and B; the last stage never does) and the memory
    rule (keep F's tensors where the in-flight peak of them fits)."""
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec
    from elysium_wan_b200.scheduler.zero_bubble import in_flight_peak, selective_recompute

    spec = JobSpec(model=make_config("toy", n_layer=4), stages=4, microbatches=8, mb_size=1,
                   recompute=True).finalize()
    peaks = [in_flight_peak(o[0]) for o in spec.schedule_order]
    assert peaks[-1] == 1 and peaks[0] > 1
    sel = selective_recompute(spec)
    assert sel == [p > 1 for p in peaks] and sel[-1] is False
    assert selective_recompute(spec, force={3}) is None  # every stage then recomputes
    big = selective_recompute(spec, budget_bytes=[1e18] * 4)
    assert big == [False] * 4
    assert selective_recompute(spec, budget_bytes=[0.0] * 4) is None
    spec.recompute = False
    assert selective_recompute(spec) is None
