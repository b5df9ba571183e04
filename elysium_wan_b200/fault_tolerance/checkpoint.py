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


def _step_of(name: str) -> int | None:
    """N of a committed wave directory name "step-<N:08d>", else None."""
    if not name.startswith("step-"):
        return None
    digits = name[5:]
    if not digits.isdigit() or len(digits) < 8:
        return None
    return int(digits)


def list_waves(out_dir: str, tag: str, stage: int, peer: int) -> list:
    """Steps of the slot's committed waves: directories named step-<N> that
    hold a wave.json (a wave is renamed into place only once it is whole, so a
    directory without wave.json is never a wave)."""
    d = slot_dir(out_dir, tag, stage, peer)
    if not os.path.isdir(d):
        return []
    out = []
    for name in os.listdir(d):
        n = _step_of(name)
        if n is not None and os.path.isfile(os.path.join(d, name, "wave.json")):
            out.append(n)
    return sorted(out)


def prune(out_dir, tag, stage, peer, keep: int = WAVE_KEEP):
    for s in list_waves(out_dir, tag, stage, peer)[:-keep]:
        shutil.rmtree(wave_dir(out_dir, tag, stage, peer, s), ignore_errors=True)


def validate_wave(path: str, step: int | None = None) -> dict:
    """Check wave.json and every listed file's size and sha256, that the
    directory holds nothing the manifest does not list, and (given `step`)
    that the manifest names that step; returns the meta."""
    meta_p = os.path.join(path, "wave.json")
    if not os.path.exists(meta_p):
        raise ValueError(f"{path}: no wave.json (incomplete wave)")
    try:
        with open(meta_p) as f:
            meta = json.load(f)
        files = dict(meta["files"])
    except (json.JSONDecodeError, KeyError, TypeError) as e:
        raise ValueError(f"{path}: unreadable wave.json ({e})") from None
    if step is not None and meta.get("step") != step:
        raise ValueError(f"{path}: wave.json names step {meta.get('step')!r}, not {step}")
    extra = sorted(set(os.listdir(path)) - set(files) - {"wave.json"})
    if extra:
        raise ValueError(f"{path}: files the manifest does not list: {extra}")
    for name, ent in files.items():
        if not safe_name(name):
            raise ValueError(f"{path}: bad file name {name!r} in wave.json")
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
            validate_wave(path, s)
        except ValueError:
            continue
        # the restricted unpickler: tensors and plain containers only, so a
        # wave shipped from another machine cannot run code when it is read
        try:
            state = torch.load(os.path.join(path, "state.pt"), map_location="cpu",
                               weights_only=True)
        except Exception as e:  # noqa: BLE001 - any failure to read means "not a checkpoint"
            raise ValueError(f"wave {path}: state.pt is not a checkpoint ({type(e).__name__})") \
                from None
        if not isinstance(state, dict):
            raise ValueError(f"wave {path}: state.pt is not a checkpoint")
        if s > spec.steps:
            raise ValueError(f"wave {path} is at step {s}, past the run's {spec.steps} steps: "
                             "resume with at least as many steps")
        diff = first_pin_difference(spec.pins(), state.get("pins", {}))
        if diff is not None:
            raise ValueError(f"wave {path} was written under another recipe: pin {diff!r} differs")
        return state, s
    raise FileNotFoundError(f"no valid wave for slot r{stage}p{peer} in {spec.out_dir}")


def drop_after(out_dir: str, tag: str, stage: int, peer: int, step: int) -> list:
    """Remove the slot's waves newer than `step` and the temporaries of a
    writer killed mid-commit. A run resumed at `step` abandoned the timeline
    those waves belong to (after a re-plan they may not even hold the same
    bits), so a later resume point must never pick one; a fresh launch passes
    -1 and keeps none. The alias follows the newest wave left. -> the steps
    removed."""
    d = slot_dir(out_dir, tag, stage, peer)
    if not os.path.isdir(d):
        return []
    gone = []
    for name in os.listdir(d):
        n = _step_of(name)
        if n is not None and n > step:
            shutil.rmtree(os.path.join(d, name), ignore_errors=True)
            gone.append(n)
        elif n is None and name.startswith("step-") and name.endswith((".staging", ".replaced")):
            shutil.rmtree(os.path.join(d, name), ignore_errors=True)
    if gone:
        alias = os.path.join(out_dir, f"{tag}_ckpt_rank{stage}p{peer}.pt")
        left = list_waves(out_dir, tag, stage, peer)
        try:
            if os.path.exists(alias):
                os.remove(alias)
            if left:
                os.link(os.path.join(wave_dir(out_dir, tag, stage, peer, left[-1]), "state.pt"),
                        alias)
        except OSError:
            pass
    return sorted(gone)


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


def safe_name(name) -> bool:
    """A plain file or directory name: no separator, no parent reference, no
    NUL, not hidden, not empty. Names arriving in control messages are used
    only if they pass."""
    return (isinstance(name, str) and 0 < len(name) <= 255 and "/" not in name
            and "\\" not in name and "\0" not in name and name not in (".", "..")
            and not name.startswith("."))


class CheckpointStore:
    """Coordinator-side store of shipped waves (reference CheckpointStore,
    src/wantrain/fault_tolerance/checkpoint.py:656-900).

    Parts arrive per slot into a staging area outside every wave directory,
    <root>/<run>/.incoming/r<R>p<P>/step-<N>/, keyed by the slot of the
    connection that sent them (never by a path from the message). When the last
    part (wave.json) arrives the staged directory is validated (every listed
    file's size and sha256, and the wave's own step, stage and peer) and only
    then renamed into <root>/<run>/waves/<tag>/r<R>p<P>/step-<N>, so a wave in
    the store is always whole: a slot that dies half-way through shipping
    leaves nothing that the resume point can pick. The heal pins its resume
    step so that pruning never removes the wave being restored."""

    def __init__(self, root: str):
        self.root = root
        self.pinned: set = set()
        os.makedirs(root, exist_ok=True)

    def _incoming(self, run_id: str, stage: int, peer: int, step: int) -> str:
        return os.path.join(self.root, run_id, ".incoming", f"r{stage}p{peer}", f"step-{step:08d}")

    @staticmethod
    def _check(run_id, stage, peer, step, name=None):
        if not safe_name(run_id):
            raise ValueError(f"bad run id {run_id!r}")
        for v in (stage, peer, step):
            if type(v) is not int or v < 0:
                raise ValueError(f"bad slot or step {v!r}")
        if name is not None and not safe_name(name):
            raise ValueError(f"bad part name {name!r}")

    def stage_part(self, run_id: str, stage: int, peer: int, step: int, name: str, data) -> str:
        """Write one shipped file of the slot's wave at `step` into staging
        (`data`: bytes, or a body the control channel streamed to a file,
        which is renamed into place)."""
        from elysium_wan_b200.transport.control import write_body

        self._check(run_id, stage, peer, step, name)
        d = self._incoming(run_id, stage, peer, step)
        os.makedirs(d, exist_ok=True)
        p = os.path.join(d, name)
        write_body(data, p)
        return p

    def commit_staged(self, run_id: str, tag: str, stage: int, peer: int, step: int) -> bool:
        """Validate the staged wave and rename it into place (False, and the
        staging removed, if it does not validate)."""
        self._check(run_id, stage, peer, step)
        if not safe_name(tag):
            raise ValueError(f"bad tag {tag!r}")
        d = self._incoming(run_id, stage, peer, step)
        if not os.path.isdir(d):
            return False
        try:
            meta = validate_wave(d)
            if (meta.get("step"), meta.get("stage"), meta.get("peer")) != (step, stage, peer):
                raise ValueError("wave.json names another slot or step")
        except (ValueError, KeyError, OSError, json.JSONDecodeError):
            shutil.rmtree(d, ignore_errors=True)
            return False
        final = wave_dir(os.path.join(self.root, run_id), tag, stage, peer, step)
        os.makedirs(os.path.dirname(final), exist_ok=True)
        if os.path.isdir(final):  # waves are immutable: the first whole copy stays
            shutil.rmtree(d, ignore_errors=True)
        else:
            os.rename(d, final)
        self._prune(os.path.dirname(final))
        return True

    def _prune(self, slot: str):
        steps = sorted(n for n in (_step_of(x) for x in os.listdir(slot)) if n is not None)
        for old in steps[:-WAVE_KEEP]:
            if old not in self.pinned:
                shutil.rmtree(os.path.join(slot, f"step-{old:08d}"), ignore_errors=True)

    def drop_after(self, run_id: str, tag: str, step: int) -> list:
        """Every slot's waves of the run newer than `step`, and the parts
        staged for them: the run resumes at `step`, so they belong to an
        abandoned timeline. A pinned wave stays. -> [(slot dir, step)]."""
        if not safe_name(run_id) or not safe_name(tag):
            raise ValueError("bad run id or tag")
        gone = []
        base = os.path.join(self.root, run_id, "waves", tag)
        for slot in sorted(os.listdir(base)) if os.path.isdir(base) else []:
            for name in os.listdir(os.path.join(base, slot)):
                n = _step_of(name)
                if n is not None and n > step and n not in self.pinned:
                    shutil.rmtree(os.path.join(base, slot, name), ignore_errors=True)
                    gone.append((slot, n))
        inc = os.path.join(self.root, run_id, ".incoming")
        for slot in sorted(os.listdir(inc)) if os.path.isdir(inc) else []:
            for name in os.listdir(os.path.join(inc, slot)):
                n = _step_of(name)
                if n is not None and n > step:
                    shutil.rmtree(os.path.join(inc, slot, name), ignore_errors=True)
        return sorted(gone)

    def common_step(self, run_id: str, spec) -> int | None:
        """The newest step every slot of `spec` holds a whole wave of in the
        run's store (the resume point of a heal)."""
        from copy import copy

        s = copy(spec)
        s.out_dir = os.path.join(self.root, run_id)
        return common_step(s)
