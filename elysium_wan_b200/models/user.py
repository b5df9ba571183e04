"""User models (`arch: "user"`): the operator's own flat layer list, trained by
the same pipeline runtime, oracle and checkpoints as the built-in decoder.

Reference behaviour: src/wantrain/model/gpt.py:489-548 (`_build_user_layers`):
the source file named by `cfg.user_model` defines `build(cfg) -> list of
nn.Module`; it is executed only after its sha256 equals
`cfg.user_model_sha256` (so every stage provably runs the same code), under
the run's seed, and each stage keeps its slice of the list. The structural
contract (validation/model_contract.py) is the reference's: entry 0 maps
token ids to activations, the last entry maps activations to logits, every
layer is deterministic and stateless.

How it runs here: each entry's parameters are registered in the stage's flat
ParamStore (fp32 master, fp32 gradient, the same optimizer and checkpoint
waves), and the module's parameters become views of that store. Forward runs
the module under autograd; B asks autograd for the input gradient and the
parameter gradients (`torch.autograd.grad`) and adds the latter into the
store's gradient in microbatch order, so a user model folds exactly like the
built-in one and matches the single-device oracle bit for bit. W is part of
B (no deferred tasks). User models run on the host path (torch operators in
fp32), not on the sm_100a kernels, and their boundaries are fp32.
"""

from __future__ import annotations

import hashlib
import math
import os

import torch
import torch.nn.functional as F

_CACHE: dict = {}


def _source(cfg) -> bytes:
    path = cfg.user_model
    if not path:
        raise ValueError("arch 'user' needs user_model: a Python file defining build(cfg)")
    if not os.path.exists(path):
        raise FileNotFoundError(f"user model source {path!r} is not on this machine: ship it "
                                f"with the spec, or the stages would build different models")
    with open(path, "rb") as f:
        raw = f.read()
    want = cfg.user_model_sha256
    got = hashlib.sha256(raw).hexdigest()
    if want and got != want:
        raise ValueError(f"user model source does not match the spec: sha256 {want[:12]} "
                         f"expected, {got[:12]} here")
    return raw


def build_layers(cfg, seed: int) -> list:
    """The whole list, built on the CPU under `seed` (every stage builds it
    whole and keeps its slice, so a stage's values do not depend on the cut)."""
    raw = _source(cfg)
    key = (hashlib.sha256(raw).hexdigest(), seed, repr(sorted(cfg.to_dict().items())))
    if key not in _CACHE:
        ns: dict = {}
        # The operator's model is code by contract; it runs only after its
        # sha256 matched the spec.
        exec(compile(raw.decode(), cfg.user_model, "exec"), ns)  # noqa: S102
        build = ns.get("build")
        if build is None:
            raise ValueError(f"{cfg.user_model} defines no build(cfg)")
        state = torch.get_rng_state()
        torch.manual_seed(seed)
        try:
            layers = list(build(cfg))
        finally:
            torch.set_rng_state(state)
        if len(layers) != cfg.n_entries:
            raise ValueError(f"build(cfg) returned {len(layers)} layers; the spec declares "
                             f"n_layer {cfg.n_layer} (n_layer + 2 entries)")
        _CACHE[key] = layers
    return _CACHE[key]


def entry_specs(cfg, e: int) -> list:
    from elysium_wan_b200.models.params import ParamSpec

    mod = build_layers(cfg, 0)[e]
    # the module computes on views of the fp32 masters, so a pieces stage keeps
    # every one of them whole on each replica (each still steps only its range)
    return [ParamSpec(f"{e}.{n}", tuple(p.shape), "user", fan_in=1, matrix=p.dim() >= 2,
                      replicate=True)
            for n, p in mod.named_parameters()]


class UserLayer:
    """One entry of the user's list bound to a ParamStore."""

    def __init__(self, cfg, store, e: int, module: torch.nn.Module):
        self.cfg, self.s, self.e, self.m = cfg, store, e, module
        self.is_embed = e == 0
        self.is_head = e == cfg.n_entries - 1
        self.names = [f"{e}.{n}" for n, _ in module.named_parameters()]
        # the module's parameters become views of the store's fp32 master
        for (n, p), full in zip(list(module.named_parameters()), self.names):
            p.data = store.p(full)

    def params(self) -> list:
        return list(self.m.parameters())

    def forward(self, x, ctx: dict, targets=None):
        from elysium_wan_b200.models.gpt import Act

        with torch.enable_grad():
            if self.is_embed:
                xin = x
            else:
                h = x.x if isinstance(x, Act) else x
                if h.dim() == 2:  # a boundary arrives flat: [tokens, d] -> [batch, seq, d]
                    h = h.reshape(-1, self.cfg.seq_len, h.shape[-1])
                xin = h.detach().requires_grad_(True)
            y = self.m(xin)
            if self.is_head:
                loss = F.cross_entropy(y.reshape(-1, y.shape[-1]).float(), targets.reshape(-1))
                ctx.update(xin=xin, out=loss)
                return loss.detach()
            ctx.update(xin=xin, out=y)
        return Act(y.detach())

    def backward(self, ctx: dict, dy, wq: list):
        out, xin = ctx["out"], ctx["xin"]
        ps = self.params()
        inputs = ([] if self.is_embed else [xin]) + ps
        go = None if self.is_head else dy.reshape(out.shape)
        grads = torch.autograd.grad(out, inputs, grad_outputs=go, allow_unused=True)
        dx = None if self.is_embed else grads[0]
        for name, g in zip(self.names, grads[0 if self.is_embed else 1:]):
            if g is not None and self.s.g(name) is not None:
                self.s.g(name).add_(g)
        ctx.clear()
        return dx


def copy_initial(store, cfg, span, seed: int):
    """The built modules' initial values into the store (its fp32 master)."""
    layers = build_layers(cfg, seed)
    for e in range(*span):
        for n, p in layers[e].named_parameters():
            store.set_initial(f"{e}.{n}", p.detach().float())


def stage_modules(cfg, span, seed: int) -> list:
    """Private copies of the stage's modules (the cached list is shared)."""
    import copy

    layers = build_layers(cfg, seed)
    return [copy.deepcopy(layers[e]) for e in range(*span)]


def numel(cfg) -> int:
    return sum(math.prod(p.shape) for m in build_layers(cfg, 0) for p in m.parameters())
