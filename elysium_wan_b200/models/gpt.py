"""The built-in GPT as a flat layer list [Embed, Block x n_layer, Head] with an
explicit forward (F), input-gradient backward (B) and deferred weight-gradient
pass (W) per layer.

Reference: src/wantrain/model/gpt.py:301-557 (Embed / Block / Head, pre-LN,
learned positions, fused qkv, 4x GELU MLP with biases, untied head) and the
zero-bubble B/W split of src/wantrain/model/wgrad.py:45-303. The reference
obtains B from autograd and defers dW = dY^T X through a SplitLinear store;
here each layer writes its backward explicitly, so B is exactly the
activation-gradient chain (plus the LayerNorm / embedding parameter
gradients, which the reference also computes in B) and W is a list of GEMM
tasks that fold dW into fp32 gradients in the order they are run.

Boundary recipe: every entry boundary (the input of each block and of the
head) carries the config's boundary dtype. With fp8_e4m3_b128 the block
output is quantised in the epilogue of the fc2 GEMM (e4m3, one power-of-two
scale per 128 elements of a row) and dequantised in the prologue of the next
LayerNorm / as the residual of the next proj GEMM; gradients stay bf16 and
pass the quantiser unchanged (straight-through). The recipe is the same at
every boundary, so a run does not depend on where the model is cut.
"""

from __future__ import annotations

import torch

from elysium_wan_b200 import ops

from .config import GPTConfig
from .params import ParamSpec, ParamStore, init_params


class Act:
    """A boundary activation: a dense tensor, or an e4m3 payload with its
    1x128 scales."""

    __slots__ = ("x", "scale")

    def __init__(self, x: torch.Tensor, scale: torch.Tensor | None = None):
        self.x = x
        self.scale = scale

    @property
    def fp8(self) -> bool:
        return self.scale is not None

    @property
    def rows(self) -> int:
        return self.x.shape[0]

    def tensors(self) -> list[torch.Tensor]:
        return [self.x] if self.scale is None else [self.x, self.scale]


def entry_specs(cfg: GPTConfig, e: int) -> list[ParamSpec]:
    """Parameter specs of flat-list entry e, named like the reference's
    nn.ModuleList ("{e}.qkv.weight", ...)."""
    d, V, S, f, n = cfg.d_model, cfg.vocab_size, cfg.seq_len, cfg.ff, cfg.n_layer
    if e == 0:
        return [ParamSpec(f"{e}.tok.weight", (V, d), "embed"),
                ParamSpec(f"{e}.pos.weight", (S, d), "embed")]
    if e == n + 1:
        return [ParamSpec(f"{e}.ln_f.weight", (d,), "ones"),
                ParamSpec(f"{e}.ln_f.bias", (d,), "zeros"),
                ParamSpec(f"{e}.out.weight", (V, d), "normal", fan_in=d, matrix=True)]
    return [
        ParamSpec(f"{e}.ln1.weight", (d,), "ones"),
        ParamSpec(f"{e}.ln1.bias", (d,), "zeros"),
        ParamSpec(f"{e}.qkv.weight", (3 * d, d), "normal", fan_in=d, matrix=True),
        ParamSpec(f"{e}.qkv.bias", (3 * d,), "bias", fan_in=d),
        ParamSpec(f"{e}.proj.weight", (d, d), "normal_resid", fan_in=d, matrix=True),
        ParamSpec(f"{e}.proj.bias", (d,), "bias", fan_in=d),
        ParamSpec(f"{e}.ln2.weight", (d,), "ones"),
        ParamSpec(f"{e}.ln2.bias", (d,), "zeros"),
        ParamSpec(f"{e}.fc1.weight", (f, d), "normal", fan_in=d, matrix=True),
        ParamSpec(f"{e}.fc1.bias", (f,), "bias", fan_in=d),
        ParamSpec(f"{e}.fc2.weight", (d, f), "normal_resid", fan_in=f, matrix=True),
        ParamSpec(f"{e}.fc2.bias", (d,), "bias", fan_in=f),
    ]


class WTask:
    """One deferred weight-gradient unit: grad (+)= dY^T X and the bias row sum."""

    __slots__ = ("dy", "x", "w_grad", "b_grad", "peer")

    def __init__(self, dy, x, w_grad, b_grad=None):
        self.dy, self.x, self.w_grad, self.b_grad = dy, x, w_grad, b_grad
        self.peer = None  # ZeRO-1 owners' slots when this dW ends the replica's fold

    def run(self):
        if self.peer is not None:
            slots, lo, stride, flat_off, rank = self.peer
            ops.ext().gemm_peer_scatter(self.dy, self.x, self.w_grad, slots, lo, stride, flat_off,
                                        rank, 0)
        else:
            ops.linear_dw(self.dy, self.x, self.w_grad, accumulate=True)
        if self.b_grad is not None:
            ops.colsum(self.dy, self.b_grad, accumulate=True)
        self.dy = self.x = None

    def record_stream(self, stream):
        """Keep the inputs' memory alive until `stream` has consumed them."""
        self.dy.record_stream(stream)
        self.x.record_stream(stream)


class WExecutor:
    """Runs W tasks on a side CUDA stream so the weight-gradient GEMMs fill the
    SMs the critical-path B GEMMs leave idle (their last wave). Each submission
    waits for everything enqueued on the compute stream so far; tasks run in
    submission order, so every parameter still folds its microbatches in order.
    On CPU the tasks run inline."""

    def __init__(self, device, enabled: bool = True):
        self.cuda = torch.device(device).type == "cuda" and enabled
        self.stream = torch.cuda.Stream(device=device) if self.cuda else None

    def run(self, tasks: list):
        if not self.cuda:
            for t in tasks:
                t.run()
            return
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            for t in tasks:
                t.record_stream(self.stream)
                t.run()

    def join(self):
        if self.cuda:
            torch.cuda.current_stream().wait_stream(self.stream)


class Embed:
    def __init__(self, cfg, store: ParamStore, e: int):
        self.cfg, self.s, self.e = cfg, store, e

    def forward(self, tokens: torch.Tensor, ctx: dict) -> Act:
        c = self.cfg
        ctx["tokens"] = tokens
        out = ops.embed_fwd(tokens, self.s.p(f"{self.e}.tok.weight"),
                            self.s.p(f"{self.e}.pos.weight"), c.seq_len, c.fp8_boundary(),
                            out_dtype=torch.float32 if not tokens.is_cuda else torch.bfloat16)
        return Act(*out) if isinstance(out, tuple) else Act(out)

    def backward(self, ctx: dict, dy: torch.Tensor, wq: list):
        ops.embed_bwd(ctx["tokens"], dy, self.cfg.seq_len, self.s.g(f"{self.e}.tok.weight"),
                      self.s.g(f"{self.e}.pos.weight"))
        return None


class Block:
    def __init__(self, cfg, store: ParamStore, e: int):
        self.cfg, self.s, self.e = cfg, store, e
        self.n = lambda k: f"{e}.{k}"

    def forward(self, x: Act, ctx: dict) -> Act:
        c, s, n = self.cfg, self.s, self.n
        T = x.rows
        B, S, H, hd = T // c.seq_len, c.seq_len, c.n_head, c.head_dim
        h1, m1, r1 = ops.layernorm_fwd(x.x, x.scale, s.p(n("ln1.weight")), s.p(n("ln1.bias")), c.ln_eps)
        qkv = ops.linear_fwd(h1, s.w(n("qkv.weight")), s.p(n("qkv.bias")))
        o, lse = ops.attention_fwd(qkv, B, S, H, hd)
        x2 = ops.linear_fwd(o, s.w(n("proj.weight")), s.p(n("proj.bias")), epi="resid",
                            resid=x.x, resid_scale=x.scale)
        h2, m2, r2 = ops.layernorm_fwd(x2, None, s.p(n("ln2.weight")), s.p(n("ln2.bias")), c.ln_eps)
        g, u = ops.linear_fwd(h2, s.w(n("fc1.weight")), s.p(n("fc1.bias")), epi="gelu")
        if c.fp8_boundary():
            q, sc = ops.linear_fwd(g, s.w(n("fc2.weight")), s.p(n("fc2.bias")), epi="resid_q8",
                                   resid=x2)
            out = Act(q, sc)
        else:
            y = ops.linear_fwd(g, s.w(n("fc2.weight")), s.p(n("fc2.bias")), epi="resid", resid=x2)
            if not y.is_cuda and c.boundary_dtype == "bf16":
                y = y.to(torch.bfloat16).float()
            out = Act(y)
        ctx.update(x=x, h1=h1, m1=m1, r1=r1, qkv=qkv, o=o, lse=lse, x2=x2, h2=h2, m2=m2, r2=r2,
                   g=g, u=u)
        return out

    def backward(self, ctx: dict, dy: torch.Tensor, wq: list) -> torch.Tensor:
        c, s, n = self.cfg, self.s, self.n
        T = dy.shape[0]
        B, S, H, hd = T // c.seq_len, c.seq_len, c.n_head, c.head_dim
        x: Act = ctx["x"]
        du = ops.linear_dx(dy, s.w(n("fc2.weight")), gelu_u=ctx["u"])
        wq.append(WTask(dy, ctx["g"], s.g(n("fc2.weight")), s.g(n("fc2.bias"))))
        dh2 = ops.linear_dx(du, s.w(n("fc1.weight")))
        wq.append(WTask(du, ctx["h2"], s.g(n("fc1.weight")), s.g(n("fc1.bias"))))
        dx2 = ops.layernorm_bwd(dh2, ctx["x2"], None, ctx["m2"], ctx["r2"], s.p(n("ln2.weight")), dy,
                                s.g(n("ln2.weight")), s.g(n("ln2.bias")), accumulate=True)
        do = ops.linear_dx(dx2, s.w(n("proj.weight")))
        wq.append(WTask(dx2, ctx["o"], s.g(n("proj.weight")), s.g(n("proj.bias"))))
        dqkv = ops.attention_bwd(ctx["qkv"], ctx["o"], do, ctx["lse"], B, S, H, hd)
        dh1 = ops.linear_dx(dqkv, s.w(n("qkv.weight")))
        wq.append(WTask(dqkv, ctx["h1"], s.g(n("qkv.weight")), s.g(n("qkv.bias"))))
        dx = ops.layernorm_bwd(dh1, x.x, x.scale, ctx["m1"], ctx["r1"], s.p(n("ln1.weight")), dx2,
                               s.g(n("ln1.weight")), s.g(n("ln1.bias")), accumulate=True)
        ctx.clear()
        return dx


class Head:
    def __init__(self, cfg, store: ParamStore, e: int):
        self.cfg, self.s, self.e = cfg, store, e
        self.n = lambda k: f"{e}.{k}"

    def forward(self, x: Act, ctx: dict, targets: torch.Tensor):
        """LN_f -> logits (fp32) -> mean CE. Returns the loss (device scalar);
        the logits gradient is produced here too and kept for B/W."""
        c, s, n = self.cfg, self.s, self.n
        T = x.rows
        V = c.vocab_size
        h, m, r = ops.layernorm_fwd(x.x, x.scale, s.p(n("ln_f.weight")), s.p(n("ln_f.bias")), c.ln_eps)
        if h.is_cuda:
            ld = (V + 7) // 8 * 8
            logits = torch.empty((T, ld), dtype=torch.float32, device=h.device)[:, :V]
            ops.gemm(h, s.w(n("out.weight")), logits, ops.EPI_F32)
        else:
            logits = ops.linear_fwd(h, s.w(n("out.weight")), epi="f32")
        loss, dl = ops.cross_entropy(logits, V, targets.reshape(-1), 1.0 / T)
        del logits
        ctx.update(x=x, h=h, m=m, r=r, dl=dl)
        return loss

    def backward(self, ctx: dict, dy, wq: list) -> torch.Tensor:
        c, s, n = self.cfg, self.s, self.n
        V = c.vocab_size
        dl = ctx["dl"][:, :V]
        dh = ops.linear_dx(dl, s.w(n("out.weight")))
        wq.append(WTask(dl, ctx["h"], s.g(n("out.weight")), None))
        x: Act = ctx["x"]
        dx = ops.layernorm_bwd(dh, x.x, x.scale, ctx["m"], ctx["r"], s.p(n("ln_f.weight")), None,
                               s.g(n("ln_f.weight")), s.g(n("ln_f.bias")), accumulate=True)
        ctx.clear()
        return dx


class StageModel:
    """The entries [lo, hi) of the flat layer list on one device, with their
    parameter store. lo == 0 owns the embedding; hi == n_layer + 2 owns the head."""

    def __init__(self, cfg: GPTConfig, span: tuple[int, int], device, seed: int):
        cfg.validate()
        self.cfg = cfg
        self.lo, self.hi = span
        self.device = torch.device(device)
        if self.device.type == "cuda" and cfg.compute_dtype != "bf16":
            raise ValueError("the sm_100a kernels compute in bf16: set compute_dtype='bf16'")
        specs, entry_of = [], {}
        for e in range(self.lo, self.hi):
            for sp in entry_specs(cfg, e):
                specs.append(sp)
                entry_of[sp.name] = e
        work = torch.bfloat16 if self.device.type == "cuda" else None
        self.store = ParamStore(specs, self.device, work_dtype=work)
        init_params(self.store, seed, entry_of, cfg.init_std, cfg.n_layer, cfg.init_scheme)
        self.layers = []
        for e in range(self.lo, self.hi):
            if e == 0:
                self.layers.append(Embed(cfg, self.store, e))
            elif e == cfg.n_layer + 1:
                self.layers.append(Head(cfg, self.store, e))
            else:
                self.layers.append(Block(cfg, self.store, e))

    @property
    def first(self) -> bool:
        return self.lo == 0

    @property
    def last(self) -> bool:
        return self.hi == self.cfg.n_layer + 2

    def forward(self, inp, targets=None, keep: str = "all"):
        """F of one microbatch. inp: token ids (first stage) or an Act.
        keep="all" saves every layer's context for B; keep="inputs" saves only
        each layer's input (per-layer recompute in B). Returns (output Act or
        loss, per-layer saved state)."""
        saved = []
        h = inp
        for layer in self.layers:
            ctx: dict = {}
            x_in = h
            if isinstance(layer, Head):
                h = layer.forward(h, ctx, targets)
            else:
                h = layer.forward(h, ctx)
            if keep == "all" or isinstance(layer, (Head, Embed)):
                saved.append(("ctx", ctx))
            else:
                ctx.clear()
                saved.append(("input", x_in))
        return h, saved

    def backward(self, saved, dy, wq: list, run_w_inline: bool = False, w_exec=None):
        """B of one microbatch: returns the input gradient (None on the first
        stage) and appends the deferred W tasks, last layer first. Layers saved
        as inputs are re-run forward just before their backward. With
        run_w_inline each layer's W tasks run right after its B (same fold
        order per parameter: one contribution per microbatch)."""
        g = dy
        for layer, (kind, obj) in zip(reversed(self.layers), reversed(saved)):
            if kind == "input":
                ctx: dict = {}
                layer.forward(obj, ctx)
            else:
                ctx = obj
            tasks: list = [] if run_w_inline else wq
            g = layer.backward(ctx, g, tasks)
            if run_w_inline:
                if w_exec is not None:
                    w_exec(tasks)
                else:
                    for t in tasks:
                        t.run()
        return g
