"""JobSpec: finalize, validation, pins and JSON round trip.

Would fail if: finalize produced an order that skips or repeats an op, a
malformed partition or ownership were accepted, or pins() changed with
fields that move no bits (schedule, ownership, grad_sync).
"""

import pytest

from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.runtime.spec import JobSpec, first_pin_difference


def _spec(**kw):
    cfg = make_config("toy", n_layer=4)
    return JobSpec(model=cfg, stages=kw.pop("stages", 2), microbatches=kw.pop("microbatches", 4), **kw)


def test_finalize_defaults():
    s = _spec().finalize()
    assert s.partition[0][0] == 0 and s.partition[-1][1] == s.model.n_entries
    assert s.stage_widths == [1, 1]
    assert len(s.schedule_order) == 2


def test_wide_ownership_round_robin():
    s = _spec(stage_widths=[2, 1]).finalize()
    assert s.mb_owner[0] == [0, 1, 0, 1]
    assert s.owned(0, 1) == [1, 3]
    assert s.world_size == 3
    assert s.slot_of(2) == (1, 0)


def test_rejects_bad_partition():
    with pytest.raises(ValueError):
        _spec(partition=[[0, 2], [3, 6]]).finalize()


def test_rejects_out_of_order_w():
    s = _spec(stages=1, microbatches=2)
    s.schedule_order = [[[["F", 0], ["F", 1], ["B", 0], ["B", 1], ["W", 1], ["W", 0]]]]
    with pytest.raises(ValueError):
        s.finalize()


def test_pins_ignore_schedule_and_roundtrip():
    a = _spec().finalize()
    b = JobSpec.from_json(a.to_json()).finalize()
    assert a.pins() == b.pins()
    b.grad_sync = "nccl"
    b.reschedule()
    assert first_pin_difference(a.pins(), b.pins()) is None
    b.lr = 0.5
    assert first_pin_difference(a.pins(), b.pins()) == "lr"
