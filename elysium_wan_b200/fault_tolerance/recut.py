"""Re-cut: move a width-1 chain's checkpoint wave to another partition.

Reference behaviour: src/wantrain/runtime/recut.py (RUNTIME-I26). Every
entry keeps its parameters, optimizer moments and buffers byte for byte; only
their place in the flat stores changes, and the new waves carry the new
partition in their pins, so a run resumed from them under the new partition
continues the uninterrupted run exactly. Unlike the reference, the stage count
may change too (the flat layouts make the mapping mechanical): an elastic
job can move from 8 stages to 6 and back at a wave.

Refused before anything is written: a wide stage, waves of different steps
or optimizer step counts, a wave whose store does not match its stage's
entries, or partitions that do not tile the same entries.
"""

from __future__ import annotations

import math

import torch

from elysium_wan_b200.fault_tolerance import checkpoint as ckpt
from elysium_wan_b200.models.gpt import entry_specs
from elysium_wan_b200.models.params import plan_layout


def stage_layout(cfg, span):
    specs = [s for e in range(*span) for s in entry_specs(cfg, e)]
    _, index, nt, numel, _ = plan_layout(specs)
    return index, nt, numel


def _check_partition(part, n_entries):
    if part[0][0] != 0 or part[-1][1] != n_entries or \
            any(part[i][1] != part[i + 1][0] for i in range(len(part) - 1)) or \
            any(a >= b for a, b in part):
        raise ValueError(f"partition {part} does not tile the {n_entries} entries contiguously")


def recut_states(states: list[dict], cfg, old: list, new: list) -> list[dict]:
    """states[r]: the wave payload of width-1 stage r under `old`; -> one
    payload per stage of `new` for the same step."""
    old = [tuple(x) for x in old]
    new = [tuple(x) for x in new]
    _check_partition(old, cfg.n_entries)
    _check_partition(new, cfg.n_entries)
    if len(states) != len(old):
        raise ValueError(f"{len(states)} waves for {len(old)} stages")
    steps = {int(s["step"]) for s in states}
    ts = {int(s["opt"]["t"]) for s in states}
    if len(steps) != 1 or len(ts) != 1:
        raise ValueError(f"waves of different steps {sorted(steps)} / optimizer steps {sorted(ts)}")
    params, moments, buffers, losses = {}, {}, {}, {}
    rng_of_entry = {}
    for r, s in enumerate(states):
        index, nt, numel = stage_layout(cfg, old[r])
        flat = s["params"]
        if flat.numel() != numel or set(s["names"]) != set(index):
            raise ValueError(f"wave r{r}: its store does not match entries {old[r]}")
        m, v = s["opt"]["m"].reshape(-1), s["opt"]["v"].reshape(-1)
        if m.numel() != nt:
            raise ValueError(f"wave r{r}: optimizer holds {m.numel()} moments, the stage {nt}")
        for name, (off, shape) in index.items():
            n = math.prod(shape)
            params[name] = flat[off:off + n]
            if off < nt:
                moments[name] = (m[off:off + n], v[off:off + n])
        buffers.update(s.get("buffers") or {})
        losses.update(s.get("losses") or {})
        for e in range(*old[r]):
            rng_of_entry[e] = s.get("rng")
    out = []
    for span in new:
        index, nt, numel = stage_layout(cfg, span)
        flat = torch.zeros(numel, dtype=torch.float32)
        m = torch.zeros(nt, dtype=torch.float32)
        v = torch.zeros(nt, dtype=torch.float32)
        for name, (off, shape) in index.items():
            n = math.prod(shape)
            flat[off:off + n] = params[name]
            if off < nt:
                m[off:off + n], v[off:off + n] = moments[name]
        mine = {k: t for k, t in buffers.items() if int(k.split(".", 1)[0]) in range(*span)}
        state = {"step": steps.copy().pop(), "params": flat, "names": list(index),
                 "opt": {"t": ts.copy().pop(), "m": m, "v": v}, "buffers": mine,
                 "losses": losses if span[1] == cfg.n_entries else {},
                 "rng": rng_of_entry.get(span[0])}
        out.append(state)
    return out


def recut(spec_old, spec_new, step: int | None = None) -> int:
    """Read spec_old's waves at `step` (default: the newest common step),
    write spec_new's waves for the same step; returns the step."""
    if any(w != 1 for w in spec_old.stage_widths) or any(w != 1 for w in spec_new.stage_widths):
        raise ValueError("re-cut moves width-1 chains only")
    if step is None:
        step = ckpt.common_step(spec_old)
        if step is None:
            raise FileNotFoundError("no common wave to re-cut")
    states = []
    for r in range(spec_old.stages):
        st, _ = ckpt.load_latest(spec_old, r, 0, step)
        states.append(st)
    for r, st in enumerate(recut_states(states, spec_old.model, spec_old.partition,
                                        spec_new.partition)):
        ckpt.commit_wave(spec_new, r, 0, step, st, replace=True)
    return step
