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
        ents = store_entries(m.store)
        from elysium_wan_b200.parallel.zero1 import shard_bounds

        bounds = shard_bounds(m.store.nt, oracle.widths[r]) if oracle.widths[r] > 1 else [(0, m.store.nt)]
        for (lo, hi), o in zip(bounds, oracle.opts[r]):
            mm, vv = o.m, o.v
            sub = store_entries(m.store, mm, vv, lo)
            for k, e in sub.items():
                if "exp_avg" in e:
                    ents[k].update(e)
        params.update(ents)
    return {"params": params, "step": oracle.opts[0][0].t,
            "losses": {f"{s}:{mb}": float(v).hex() for s, mb, v in oracle.losses}}


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
