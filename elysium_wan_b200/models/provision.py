"""Data provisioning: a data-reading slot holds, verified, the bytes its
microbatches draw before it connects.

Reference behaviour: src/wantrain/model/provision.py (`needed_shards`,
`ensure_manifest`, `provision_slot`). Only the first stage (inputs) and the
last stage (targets) read the corpus; microbatch mb draws logical shard
mb % data_shards, so a slot needs the shards of the microbatches it owns
(and that set moves with ownership after a heal). Before connecting:

1. the manifest is made local (fetched from `dataset_source` when missing)
   and, when the spec pins one, checked against `dataset_sha256`;
2. each needed shard's bytes (its shard file, or that range of the whole
   stream) are verified against the manifest's per-shard sha256 (the whole
   stream against its sha256 when the shard counts differ);
3. missing or corrupt bytes are fetched from the source (a directory or an
   http(s) URL holding the prepared files) into a temp file, verified, and
   renamed into place;
4. with bytes missing or wrong and no source, the slot refuses, naming the
   shards.

A verified file leaves a stamp (size, mtime, digest) next to it so a restart
does not hash the corpus again; every fetched byte is checked against the
pinned manifest, so integrity never depends on the source.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import urllib.parse
import urllib.request

import numpy as np

from elysium_wan_b200.models import dataset as ds

FETCH_TIMEOUT_S = 60


class DataRefused(RuntimeError):
    """This node cannot hold the verified bytes its slot needs."""


def needed_shards(spec, stage: int, peer: int) -> list[int]:
    if not spec.dataset_path or stage not in (0, spec.stages - 1):
        return []
    n = max(1, int(spec.data_shards or 1))
    return sorted({mb % n for mb in spec.owned(stage, peer)})


def _sha(path: str, lo: int = 0, hi: int | None = None) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        f.seek(lo)
        left = (os.path.getsize(path) if hi is None else hi) - lo
        while left > 0:
            b = f.read(min(left, 1 << 20))
            if not b:
                break
            h.update(b)
            left -= len(b)
    return h.hexdigest()


def manifest_digest(dataset: str) -> str | None:
    p = ds.manifest_path(dataset)
    return ds.file_digest(p) if os.path.exists(p) else None


def _stamp_path(path: str) -> str:
    return f"{path}.verified.json"


def _verified(path: str, lo: int, hi: int, want: str) -> bool:
    """sha256 of [lo, hi) of `path` equals `want` (cached by size and mtime)."""
    if not os.path.exists(path):
        return False
    st = os.stat(path)
    key = f"{lo}:{hi}"
    stamps = {}
    try:
        with open(_stamp_path(path)) as f:
            stamps = json.load(f)
    except (OSError, ValueError):
        pass
    ent = stamps.get(key)
    if ent and ent.get("size") == st.st_size and ent.get("mtime") == st.st_mtime and \
            ent.get("sha256") == want:
        return True
    if hi > st.st_size or _sha(path, lo, hi) != want:
        return False
    stamps[key] = {"size": st.st_size, "mtime": st.st_mtime, "sha256": want}
    tmp = _stamp_path(path) + f".{os.getpid()}.tmp"
    with open(tmp, "w") as f:
        json.dump(stamps, f)
    os.replace(tmp, _stamp_path(path))
    return True


def _is_url(source: str) -> bool:
    return urllib.parse.urlparse(source).scheme in ("http", "https")


def _fetch(source: str, name: str, dest: str) -> bool:
    """Copy `name` from the source (a directory or an http(s) base URL) into
    dest via a temp file; False when the source lacks it."""
    tmp = f"{dest}.{os.getpid()}.part"
    try:
        if _is_url(source):
            url = source.rstrip("/") + "/" + urllib.parse.quote(name)
            with urllib.request.urlopen(url, timeout=FETCH_TIMEOUT_S) as r, open(tmp, "wb") as f:
                shutil.copyfileobj(r, f, 1 << 20)
        else:
            src = os.path.join(source, name)
            if not os.path.exists(src):
                return False
            shutil.copyfile(src, tmp)
        os.replace(tmp, dest)
        return True
    except OSError:
        if os.path.exists(tmp):
            os.remove(tmp)
        return False


def ensure_manifest(dataset: str, pinned: str | None = None, source: str | None = None) -> dict:
    """The local manifest, fetched when missing, checked against the pin."""
    mp = ds.manifest_path(dataset)
    if not os.path.exists(mp):
        if not source or not _fetch(source, os.path.basename(mp), mp):
            raise DataRefused(f"{mp} is missing and no dataset_source provides it")
    if pinned and ds.file_digest(mp) != pinned:
        if source and _fetch(source, os.path.basename(mp), mp) and ds.file_digest(mp) == pinned:
            pass
        else:
            raise DataRefused(f"{mp} is not the planned corpus (manifest sha256 differs from "
                              f"dataset_sha256)")
    with open(mp) as f:
        return json.load(f)


def provision(dataset: str, shards: list, n_shards: int, pinned: str | None = None,
              source: str | None = None) -> dict:
    """Verify (and fetch) the bytes of `shards`; returns a report."""
    m = ensure_manifest(dataset, pinned, source)
    isz = np.dtype(ds.DTYPES[m["dtype"]]).itemsize
    total = int(m["total_tokens"])
    per_shard = m.get("shard_sha256") if int(m.get("n_shards", 1)) == n_shards else None
    fetched, checked = [], []
    if per_shard:
        for k in shards:
            lo, hi = ds.shard_bounds(total, k, n_shards)
            want = per_shard[k]
            shard_file = f"{dataset}.shard{k}of{n_shards}"
            if _verified(shard_file, 0, (hi - lo) * isz, want) or \
                    _verified(dataset, lo * isz, hi * isz, want):
                checked.append(k)
                continue
            if source and _fetch(source, os.path.basename(shard_file), shard_file) and \
                    _verified(shard_file, 0, (hi - lo) * isz, want):
                fetched.append(k)
                continue
            if source and _fetch(source, os.path.basename(dataset), dataset) and \
                    _verified(dataset, lo * isz, hi * isz, want):
                fetched.append(k)
                continue
            raise DataRefused(f"shard {k} of {dataset} is missing or corrupt"
                              + ("" if source else "; set dataset_source to fetch it"))
    else:
        want = m.get("sha256")
        if want is None:
            raise DataRefused(f"{ds.manifest_path(dataset)} lists no sha256")
        if not _verified(dataset, 0, total * isz, want):
            if not (source and _fetch(source, os.path.basename(dataset), dataset)
                    and _verified(dataset, 0, total * isz, want)):
                raise DataRefused(f"{dataset} is missing or corrupt"
                                  + ("" if source else "; set dataset_source to fetch it"))
            fetched.append("all")
        checked = list(shards)
    return {"dataset": dataset, "shards": list(shards), "checked": checked, "fetched": fetched}


def provision_slot(spec, stage: int, peer: int) -> dict | None:
    """Provision what slot (stage, peer) reads; None when it reads nothing."""
    need = needed_shards(spec, stage, peer)
    if not need:
        return None
    return provision(spec.dataset_path, need, max(1, int(spec.data_shards or 1)),
                     spec.dataset_sha256, spec.dataset_source)
