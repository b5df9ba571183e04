"""Validate a user model source against the flat-layer-list contract
(reference: src/wantrain/validation/model_contract.py): the source defines
build(cfg) -> a flat list of layers; building twice under the same seed gives
identical parameters; each layer maps a tensor to a tensor of the next
layer's input shape; layers keep no state across calls."""

from __future__ import annotations

import torch


class _Target(dict):
    """A dict target read by attribute too (build(cfg) may use cfg.d_model)."""

    def __getattr__(self, k):
        try:
            return self[k]
        except KeyError as e:
            raise AttributeError(k) from e


def validate(source: str, target) -> dict:
    """target: a dict (or a config object; its fields are read) with an
    optional "example" input for the per-layer checks."""
    if not isinstance(target, dict):
        example = getattr(target, "example", None)
        target = dict(target.to_dict()) if hasattr(target, "to_dict") else dict(vars(target))
        if example is not None:
            target["example"] = example
    target = _Target(target)
    errors = []
    ns: dict = {}
    try:
        exec(compile(source, "<user model>", "exec"), ns)  # noqa: S102 - the contract's own input
    except Exception as e:
        return {"ok": False, "errors": [f"source does not execute: {e!r}"]}
    build = ns.get("build")
    if build is None:
        return {"ok": False, "errors": ["no build(cfg) function"]}
    torch.manual_seed(0)
    a = build(target)
    torch.manual_seed(0)
    b = build(target)
    layers_a, layers_b = list(a), list(b)
    if not layers_a:
        errors.append("build returned no layers")
    pa = [p.detach().clone() for layer in layers_a for p in getattr(layer, "parameters", lambda: [])()]
    pb = [p.detach() for layer in layers_b for p in getattr(layer, "parameters", lambda: [])()]
    if len(pa) != len(pb) or any(not torch.equal(x, y) for x, y in zip(pa, pb)):
        errors.append("two builds under one seed differ (build must not reseed or draw outside the seed)")
    x = target.get("example")
    if x is not None and not errors:
        h = torch.tensor(x)
        for i, layer in enumerate(layers_a):
            try:
                h1 = layer(h)
                h2 = layer(h)
            except Exception as e:
                errors.append(f"layer {i} raised {e!r}")
                break
            if not torch.equal(h1, h2):
                errors.append(f"layer {i} is not deterministic / keeps state across calls")
                break
            h = h1
    return {"ok": not errors, "errors": errors, "layers": len(layers_a)}
