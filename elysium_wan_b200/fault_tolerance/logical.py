"""Logical checkpoints: a width-free, cut-free form of a run's state, and
conversion of checkpoint waves between layouts.

Reference behaviour: src/wantrain/runtime/logical_ckpt.py (`build_manifest`,
`check_manifest`, `select_wave`, `assemble`, `as_zero1`, `from_zero1`): a
layout-independent checkpoint with per-chunk sha256, and conversion between
ZeRO-1 and pieces stages. Here the flat stores make the mapping mechanical:

- `gather(spec, step)` reads every slot's wave of `step` (width-1, ZeRO-1 or
  pieces stages, any partition) and returns, per parameter name, its fp32
  master and its AdamW moments, plus the optimizer step count, buffers,
  losses and RNG state;
- `scatter(state, spec, step)` writes the waves `spec` resumes from (any
  partition, widths and shard mode): a job can change its cut, its replica
  count and ZeRO-1 <-> pieces at a wave and continue bit for bit;
- `save(state, dir)` / `load(dir)` keep the logical form on disk as three
  safetensors files (params, exp_avg, exp_avg_sq), the buffers / losses / RNG
  in the safe object codec (transport/serial.py, no pickle), and a manifest with the
  step, the recipe pins that do not name a topology, and a sha256 per file
  and per 16 MiB chunk; `load` verifies every chunk.
"""

from __future__ import annotations

import hashlib
import json
import math
import os

import torch

from elysium_wan_b200.fault_tolerance import checkpoint as ckpt
from elysium_wan_b200.models.gpt import entry_specs
from elysium_wan_b200.models.params import pieces_held, plan_layout, shard_ranges
from elysium_wan_b200.parallel.zero1 import shard_bounds
from elysium_wan_b200.transport import serial

CHUNK = 16 << 20
_TOPOLOGY_PINS = ("partition", "zero1_widths", "device_types", "stage_widths")


def _layout(cfg, span, pieces: bool):
    specs = [s for e in range(*span) for s in entry_specs(cfg, e)]
    _, index, nt, numel, nr = plan_layout(specs, replicated_first=pieces)
    return index, nt, numel, nr


def _spans(index, lo, hi):
    """(name, flat offset range ∩ [lo, hi)) of every tensor overlapping [lo, hi)."""
    for name, (off, shape) in index.items():
        n = math.prod(shape)
        a, b = max(lo, off), min(hi, off + n)
        if a < b:
            yield name, off, a, b


def gather(spec, step: int | None = None) -> dict:
    """The logical state of `spec`'s waves at `step` (default: newest common)."""
    if step is None:
        step = ckpt.common_step(spec)
        if step is None:
            raise FileNotFoundError("no common wave")
    cfg = spec.model
    params, m_all, v_all = {}, {}, {}
    buffers, losses, rng = {}, {}, {}
    ts = set()
    for r, w in enumerate(spec.stage_widths):
        pieces = spec.shard == "pieces" and w > 1
        index, nt, numel, nr = _layout(cfg, spec.partition[r], pieces)
        flat_p = torch.zeros(numel, dtype=torch.float32)
        flat_m = torch.zeros(nt, dtype=torch.float32)
        flat_v = torch.zeros(nt, dtype=torch.float32)
        for p in range(w):
            st, _ = ckpt.load_latest(spec, r, p, step)
            opt = st["opt"]
            if pieces:
                rb = shard_ranges(nr, w)[p]
                held = pieces_held(nr, nt, numel, w, p)
                mb = held[1]
                base = 0
                for lo, hi in held:
                    flat_p[lo:hi] = st["params"][base: base + hi - lo]
                    base += hi - lo
                for (lo, hi), key in ((rb, "r"), (mb, "m")):
                    flat_m[lo:hi] = opt[key]["m"].reshape(-1)
                    flat_v[lo:hi] = opt[key]["v"].reshape(-1)
                ts.add(int(opt["m"]["t"]))
            else:
                flat_p.copy_(st["params"])
                lo, hi = (0, nt) if w == 1 else shard_bounds(nt, w)[p]
                flat_m[lo:hi] = opt["m"].reshape(-1)
                flat_v[lo:hi] = opt["v"].reshape(-1)
                ts.add(int(opt["t"]))
            buffers.update(st.get("buffers") or {})
            losses.update(st.get("losses") or {})
            if p == 0:
                rng[r] = st.get("rng")
        for name, (off, shape) in index.items():
            n = math.prod(shape)
            params[name] = flat_p[off:off + n].view(shape).clone()
            if off < nt:
                m_all[name] = flat_m[off:off + n].view(shape).clone()
                v_all[name] = flat_v[off:off + n].view(shape).clone()
    if len(ts) != 1:
        raise ValueError(f"waves disagree on the optimizer step count: {sorted(ts)}")
    pins = {k: v for k, v in spec.pins().items() if k not in _TOPOLOGY_PINS}
    return {"step": step, "t": ts.pop(), "params": params, "exp_avg": m_all,
            "exp_avg_sq": v_all, "buffers": buffers, "losses": losses, "rng": rng,
            "pins": pins}


def scatter(state: dict, spec, step: int | None = None):
    """Write the waves `spec` resumes from at `step` (default: state["step"])."""
    step = state["step"] if step is None else step
    cfg = spec.model
    want = {k: v for k, v in spec.pins().items() if k not in _TOPOLOGY_PINS}
    for k in set(want) | set(state["pins"]):
        if json.dumps(want.get(k), sort_keys=True) != json.dumps(state["pins"].get(k),
                                                                 sort_keys=True):
            raise ValueError(f"pin {k!r} differs: the logical state is another recipe")
    for r, w in enumerate(spec.stage_widths):
        pieces = spec.shard == "pieces" and w > 1
        index, nt, numel, nr = _layout(cfg, spec.partition[r], pieces)
        flat_p = torch.zeros(numel, dtype=torch.float32)
        flat_m = torch.zeros(nt, dtype=torch.float32)
        flat_v = torch.zeros(nt, dtype=torch.float32)
        for name, (off, shape) in index.items():
            n = math.prod(shape)
            flat_p[off:off + n] = state["params"][name].reshape(-1)
            if off < nt:
                flat_m[off:off + n] = state["exp_avg"][name].reshape(-1)
                flat_v[off:off + n] = state["exp_avg_sq"][name].reshape(-1)
        a, b = spec.partition[r]
        bufs = {k: t for k, t in state["buffers"].items() if int(k.split(".", 1)[0]) in range(a, b)}
        first_entry_rng = next((state["rng"][k] for k in sorted(state["rng"])), None)
        for p in range(w):
            if pieces:
                rb = shard_ranges(nr, w)[p]
                held = pieces_held(nr, nt, numel, w, p)
                mb = held[1]
                params = torch.cat([flat_p[lo:hi] for lo, hi in held])
                opt = {"t": state["t"], "pieces": {"k": p, "w": w},
                       "r": {"t": state["t"], "m": flat_m[rb[0]:rb[1]].clone(),
                             "v": flat_v[rb[0]:rb[1]].clone()},
                       "m": {"t": state["t"], "m": flat_m[mb[0]:mb[1]].clone(),
                             "v": flat_v[mb[0]:mb[1]].clone()}}
            else:
                lo, hi = (0, nt) if w == 1 else shard_bounds(nt, w)[p]
                params = flat_p.clone()
                opt = {"t": state["t"], "m": flat_m[lo:hi].clone(), "v": flat_v[lo:hi].clone()}
            wave = {"step": step, "params": params, "names": list(index), "opt": opt,
                    "buffers": bufs, "losses": state["losses"] if r == spec.stages - 1 else {},
                    "rng": first_entry_rng}
            ckpt.commit_wave(spec, r, p, step, wave, replace=True)
    return step


def convert(spec_old, spec_new, step: int | None = None) -> int:
    """Re-lay `spec_old`'s waves for `spec_new` (cut, widths, shard mode)."""
    return scatter(gather(spec_old, step), spec_new)


# ------------------------------------------------------------------ on disk
def _chunks(path: str) -> list:
    out = []
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(CHUNK), b""):
            out.append(hashlib.sha256(b).hexdigest())
    return out


def save(state: dict, out: str) -> str:
    """The logical state as safetensors + a chunk-hashed manifest."""
    from elysium_wan_b200.models.hf import save_file

    os.makedirs(out, exist_ok=True)
    files = {}
    for key in ("params", "exp_avg", "exp_avg_sq"):
        path = os.path.join(out, f"{key}.safetensors")
        save_file({k: v.contiguous() for k, v in state[key].items()}, path)
        files[os.path.basename(path)] = {"sha256": ckpt._sha256(path), "chunks": _chunks(path),
                                         "size": os.path.getsize(path)}
    extra = os.path.join(out, "extra.ewbs")  # safe object codec: no pickle
    serial.save({"buffers": state["buffers"], "losses": state["losses"], "rng": state["rng"]}, extra)
    files["extra.ewbs"] = {"sha256": ckpt._sha256(extra), "chunks": _chunks(extra),
                           "size": os.path.getsize(extra)}
    man = {"step": state["step"], "t": state["t"], "pins": state["pins"], "chunk": CHUNK,
           "files": files}
    with open(os.path.join(out, "manifest.json"), "w") as f:
        json.dump(man, f, indent=1)
    return out


def load(src: str) -> dict:
    """Read and verify (every 16 MiB chunk) a logical checkpoint."""
    from elysium_wan_b200.models.hf import load_state

    with open(os.path.join(src, "manifest.json")) as f:
        man = json.load(f)
    for name, ent in man["files"].items():
        path = os.path.join(src, name)
        if os.path.getsize(path) != ent["size"] or _chunks(path) != ent["chunks"]:
            raise ValueError(f"{path}: a chunk does not match the manifest")
    extra = serial.load(os.path.join(src, "extra.ewbs"))
    return {"step": man["step"], "t": man["t"], "pins": man["pins"],
            "params": load_state(os.path.join(src, "params.safetensors")),
            "exp_avg": load_state(os.path.join(src, "exp_avg.safetensors")),
            "exp_avg_sq": load_state(os.path.join(src, "exp_avg_sq.safetensors")),
            **extra}
