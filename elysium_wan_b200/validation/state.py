"""Canonical state manifest: sha256 of every parameter, AdamW moment and the
step, keyed by full-model name, plus the loss hex strings.

Reference: src/wantrain/validation/state.py:126-404 (reference_manifest,
distributed_manifest, diff_manifests). Two runs with equal manifests hold
byte-identical training state.
"""

from __future__ import annotations

import hashlib
import json

import torch


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def store_entries(store, m=None, v=None, lo=0) -> dict:
    """Per-parameter digests of a store (and of moments given as flat tensors
    covering [lo, lo + len))."""
    out = {}
    for name in store.names():
        off, shape = store.index[name]
        n = 1
        for s in shape:
            n *= s
        ent = {"param": _sha(store.master[off: off + n])}
        if m is not None and lo <= off and off + n <= lo + m.numel():
            ent["exp_avg"] = _sha(m[off - lo: off - lo + n])
            ent["exp_avg_sq"] = _sha(v[off - lo: off - lo + n])
        out[name] = ent
    return out


def reference_manifest(oracle) -> dict:
    params = {}
    for r, m in enumerate(oracle.stages):
        # the shards' moments in order cover [0, nt): join them so a tensor
        # that straddles a shard boundary gets its moments too
        mm = torch.cat([o.m.reshape(-1).cpu() for o in oracle.opts[r]])
        vv = torch.cat([o.v.reshape(-1).cpu() for o in oracle.opts[r]])
        params.update(store_entries(m.store, mm, vv, 0))
    return {"params": params, "step": oracle.opts[0][0].t,
            "losses": {f"{s}:{mb}": float(v).hex() for s, mb, v in oracle.losses}}


def distributed_manifest(spec, step: int | None = None) -> dict:
    """The same manifest for a distributed run, read from its checkpoint waves
    at `step` (default: the newest wave every slot holds) through the logical
    form, whatever the cut, the widths and the ZeRO-1 / pieces layout."""
    from elysium_wan_b200.fault_tolerance import logical

    st = logical.gather(spec, step)
    params = {}
    for name, t in st["params"].items():
        ent = {"param": _sha(t)}
        if name in st["exp_avg"]:
            ent["exp_avg"] = _sha(st["exp_avg"][name])
            ent["exp_avg_sq"] = _sha(st["exp_avg_sq"][name])
        params[name] = ent
    return {"params": params, "step": st["t"],
            "losses": {f"{s}:{mb}": float(v).hex() for (s, mb), v in _loss_items(st["losses"])}}


def _loss_items(losses):
    out = []
    for k, v in (losses or {}).items():
        if isinstance(k, (tuple, list)):
            out.append(((int(k[0]), int(k[1])), v))
        elif isinstance(k, str) and ":" in k:
            a, b = k.split(":")
            out.append(((int(a), int(b)), v))
    return out


def write_manifest(path: str, man: dict):
    with open(path, "w") as f:
        json.dump(man, f, indent=1, sort_keys=True)


def diff_manifests(a: dict, b: dict) -> list:
    diffs = []
    for k in sorted(set(a.get("params", {})) | set(b.get("params", {}))):
        if a["params"].get(k) != b["params"].get(k):
            diffs.append(k)
    if a.get("step") != b.get("step"):
        diffs.append("step")
    return diffs
