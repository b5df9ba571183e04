"""Checkpoint waves: immutable, sha256-verified per-slot snapshots.

Layout (public surface, same as the reference, src/wantrain/fault_tolerance/
checkpoint.py:1-160):
    <out_dir>/waves/<tag>/r<R>p<P>/step-<N:08d>/{state.pt, wave.json}
wave.json lists every file with its sha256 and size and is written last; the
step directory is staged under a temporary name and renamed into place, so a
wave either exists completely or not at all. At most WAVE_KEEP waves are kept
per slot. The legacy alias <tag>_ckpt_rank<R>p<P>.pt is a hard link to the
newest state.pt. `state.pt` holds {step, params, names, opt, losses, rng,
pins}.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil

import torch

WAVE_KEEP = 3


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def slot_dir(out_dir: str, tag: str, stage: int, peer: int) -> str:
    return os.path.join(out_dir, "waves", tag, f"r{stage}p{peer}")


def wave_dir(out_dir: str, tag: str, stage: int, peer: int, step: int) -> str:
    return os.path.join(slot_dir(out_dir, tag, stage, peer), f"step-{step:08d}")


def commit_wave(spec, stage: int, peer: int, step: int, state: dict, replace: bool = False) -> str:
    """Write state.pt + wave.json atomically; prune to WAVE_KEEP; refresh the
    alias. An existing wave of the step is kept, unless `replace` (re-cut
    writes the same step under a new partition): the new wave is staged
    completely, then swapped in by two renames."""
    final = wave_dir(spec.out_dir, spec.tag, stage, peer, step)
    if os.path.isdir(final) and not replace:
        return final
    tmp = final + ".staging"
    shutil.rmtree(tmp, ignore_errors=True)
    os.makedirs(tmp)
    state = dict(state)
    state["pins"] = spec.pins()
    sp = os.path.join(tmp, "state.pt")
    torch.save(state, sp)
    with open(sp, "rb") as f:
        os.fsync(f.fileno())
    files = {"state.pt": {"sha256": _sha256(sp), "size": os.path.getsize(sp)}}
    meta = {"step": step, "stage": stage, "peer": peer, "tag": spec.tag, "files": files}
    with open(os.path.join(tmp, "wave.json"), "w") as f:
        json.dump(meta, f, indent=1)
        f.flush()
        os.fsync(f.fileno())
    if os.path.isdir(final):
        old = final + ".replaced"
        shutil.rmtree(old, ignore_errors=True)
        os.rename(final, old)
        os.rename(tmp, final)
        shutil.rmtree(old, ignore_errors=True)
    else:
        os.rename(tmp, final)
    alias = os.path.join(spec.out_dir, f"{spec.tag}_ckpt_rank{stage}p{peer}.pt")
    try:
        if os.path.exists(alias):
            os.remove(alias)
        os.link(os.path.join(final, "state.pt"), alias)
    except OSError:
        pass
    prune(spec.out_dir, spec.tag, stage, peer)
    return final


def list_waves(out_dir: str, tag: str, stage: int, peer: int) -> list:
    d = slot_dir(out_dir, tag, stage, peer)
    if not os.path.isdir(d):
        return []
    out = []
    for name in os.listdir(d):
        if name.startswith("step-") and not name.endswith((".staging", ".replaced")):
            try:
                out.append(int(name[5:]))
            except ValueError:
                pass
    return sorted(out)


def prune(out_dir, tag, stage, peer, keep: int = WAVE_KEEP):
    for s in list_waves(out_dir, tag, stage, peer)[:-keep]:
        shutil.rmtree(wave_dir(out_dir, tag, stage, peer, s), ignore_errors=True)


def validate_wave(path: str) -> dict:
    """Check wave.json and every listed file's size and sha256; returns the meta."""
    meta_p = os.path.join(path, "wave.json")
    if not os.path.exists(meta_p):
        raise ValueError(f"{path}: no wave.json (incomplete wave)")
    with open(meta_p) as f:
        meta = json.load(f)
    for name, ent in meta["files"].items():
        p = os.path.join(path, name)
        if not os.path.exists(p) or os.path.getsize(p) != ent["size"]:
            raise ValueError(f"{path}: {name} missing or truncated")
        if _sha256(p) != ent["sha256"]:
            raise ValueError(f"{path}: {name} sha256 mismatch")
    return meta


def load_latest(spec, stage: int, peer: int, step: int | None = None):
    """(state, step) of the requested or newest valid wave whose pins match."""
    from elysium_wan_b200.runtime.spec import first_pin_difference

    steps = list_waves(spec.out_dir, spec.tag, stage, peer)
    if step is not None:
        steps = [s for s in steps if s == step]
    for s in reversed(steps):
        path = wave_dir(spec.out_dir, spec.tag, stage, peer, s)
        try:
            validate_wave(path)
        except ValueError:
            continue
        # the restricted unpickler: tensors and plain containers only, so a
        # wave shipped from another machine cannot run code when it is read
        state = torch.load(os.path.join(path, "state.pt"), map_location="cpu", weights_only=True)
        diff = first_pin_difference(spec.pins(), state.get("pins", {}))
        if diff is not None:
            raise ValueError(f"wave {path} was written under another recipe: pin {diff!r} differs")
        return state, s
    raise FileNotFoundError(f"no valid wave for slot r{stage}p{peer} in {spec.out_dir}")


def common_step(spec) -> int | None:
    """Newest step for which every slot holds a valid wave (the resume point)."""
    sets = []
    for r, w in enumerate(spec.stage_widths):
        for p in range(w):
            sets.append(set(list_waves(spec.out_dir, spec.tag, r, p)))
    if not sets:
        return None
    common = set.intersection(*sets)
    return max(common) if common else None


class CheckpointStore:
    """Coordinator-side store of shipped waves: files arrive under
    <root>/<run>/waves/..., are verified, and the common step across slots is
    the heal point (reference CheckpointStore, checkpoint.py:656-900)."""

    def __init__(self, root: str):
        self.root = root
        os.makedirs(root, exist_ok=True)

    def stage_part(self, rel_path: str, data: bytes) -> str:
        p = os.path.join(self.root, rel_path + ".part")
        os.makedirs(os.path.dirname(p), exist_ok=True)
        with open(p, "wb") as f:
            f.write(data)
        return p

    def commit_staged(self, rel_dir: str) -> bool:
        d = os.path.join(self.root, rel_dir)
        if not os.path.isdir(d):
            return False
        for name in os.listdir(d):
            if name.endswith(".part"):
                os.replace(os.path.join(d, name), os.path.join(d, name[:-5]))
        try:
            validate_wave(d)
        except ValueError:
            shutil.rmtree(d, ignore_errors=True)
            return False
        # Keep the newest WAVE_KEEP waves of this slot, like the workers do.
        slot = os.path.dirname(d)
        steps = sorted(int(x[5:]) for x in os.listdir(slot)
                       if x.startswith("step-") and not x.endswith(".part") and x[5:].isdigit())
        for old in steps[:-WAVE_KEEP]:
            shutil.rmtree(os.path.join(slot, f"step-{old:08d}"), ignore_errors=True)
        return True

    def common_step(self, spec) -> int | None:
        from copy import copy

        s = copy(spec)
        s.out_dir = self.root
        return common_step(s)
