"""The benchmark's planning on CPU: every BASELINE config at 1, 2, 4 and 8 GPUs
gets a layout that uses exactly those GPUs, a contiguous cut of the whole
layer list, a schedule the spec accepts, and a memory plan that fits the
device (moments moved to the host only when the device cannot hold them).

Would fail if a config planned a layout for the wrong number of GPUs, left
an entry out of the cut, produced an order the engine refuses, or planned a
stage whose parameter state alone overflows a 178 GiB device.
"""

import argparse

import pytest

import bench

GiB = 1 << 30


def _args(config, n, **kw):
    c = bench.CONFIGS[config]
    base = dict(gpus=n, config=config, model=c["model"], metric=c["metric"],
                microbatches=c["microbatches"], mb_size=c["mb_size"], widths=None,
                widths_list=None, n_layer=None, no_w_pair=False, grad_sync="fused", warmup=3,
                steps=3)
    base.update(kw)
    return argparse.Namespace(**base)


@pytest.mark.parametrize("config", sorted(bench.CONFIGS))
@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_plan_covers_every_layer_and_fits(config, n):
    args = _args(config, n)
    try:
        spec = bench.plan_spec(args, n, 178 * GiB)
    except SystemExit as e:  # refused with the reason: only when the weights cannot fit
        assert "do not fit" in str(e) and config == "25.1b" and n <= 2, e
        return
    assert sum(spec.stage_widths) == n
    cuts = spec.partition
    assert cuts[0][0] == 0 and cuts[-1][1] == spec.model.n_entries
    assert all(a < b for a, b in cuts) and all(cuts[i][1] == cuts[i + 1][0] for i in range(len(cuts) - 1))
    assert len(spec.schedule_order) == spec.stages
    for r, w in enumerate(spec.stage_widths):
        assert len(spec.schedule_order[r]) == w
    biggest = max(bench._numel(spec.model, a, b) for a, b in cuts)
    wmin = min(spec.stage_widths)
    resident = biggest * 10 + (4 * biggest if wmin > 1 else 0)
    moments = 0 if spec.optimizer == "adamw-host" else 8 * biggest / wmin
    assert resident + moments < 178 * GiB


def test_layout_rules():
    assert bench.layout(_args("15.8b", 8), 8) == [1] * 8
    assert bench.layout(_args("0.6b", 8), 8) == [4, 4]
    assert bench.layout(_args("2.8b", 8), 8) == [2, 2, 2, 2]
    assert bench.layout(_args("0.6b", 2, widths="2"), 2) == [2]
    with pytest.raises(SystemExit):
        bench.layout(_args("0.6b", 4, widths="1,2"), 4)
    with pytest.raises(SystemExit):
        bench.layout(_args("2.8b", 6), 6)


def test_single_device_runs_w_inline_and_moments_on_host():
    spec = bench.plan_spec(_args("15.8b", 1), 1, 178 * GiB)
    assert spec.optimizer == "adamw-host"  # 15.8B of fp32 moments do not fit next to the weights
    order = spec.schedule_order[0][0]
    assert [op for op, _ in order[:3]] == ["F", "B", "W"] and not spec.w_pair
