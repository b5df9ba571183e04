"""Bitwise comparison of two loss files.

Output schema of the reference (src/wantrain/validation/compare.py:11-45):
{ok, compared, mismatches, max_abs_diff, first_mismatch}; losses are compared
as float.hex() strings, keyed by (step, mb).
"""

from __future__ import annotations

import json


def load_losses(path_or_obj) -> dict:
    d = path_or_obj
    if isinstance(path_or_obj, str):
        with open(path_or_obj) as f:
            d = json.load(f)
    return {(int(r["step"]), int(r["mb"])): r for r in d["losses"]}


def compare(a, b) -> dict:
    la, lb = load_losses(a), load_losses(b)
    keys = sorted(set(la) & set(lb))
    mism, first, max_abs = 0, None, 0.0
    for k in keys:
        ha, hb = la[k]["loss_hex"], lb[k]["loss_hex"]
        if ha != hb:
            mism += 1
            diff = abs(float.fromhex(ha) - float.fromhex(hb))
            max_abs = max(max_abs, diff)
            if first is None:
                first = {"step": k[0], "mb": k[1], "a": ha, "b": hb}
    missing = sorted(set(la) ^ set(lb))
    return {"ok": mism == 0 and not missing and len(keys) > 0, "compared": len(keys),
            "mismatches": mism, "max_abs_diff": max_abs, "first_mismatch": first,
            "missing": [list(m) for m in missing[:10]]}


def main(argv=None):
    import argparse

    ap = argparse.ArgumentParser(prog="wantrain compare")
    ap.add_argument("a")
    ap.add_argument("b")
    a = ap.parse_args(argv)
    r = compare(a.a, a.b)
    print(json.dumps(r, indent=2))
    return 0 if r["ok"] else 1
