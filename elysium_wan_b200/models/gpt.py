"""The built-in GPT as a flat layer list [Embed, Block x n_layer, Head] with an
explicit forward (F), input-gradient backward (B) and deferred weight-gradient
pass (W) per layer.

Reference: src/wantrain/model/gpt.py:301-557 (Embed / Block / Head, pre-LN,
learned positions, fused qkv, 4x GELU MLP with biases, untied head), the
generalized block of src/wantrain/model/arch.py:1-270 (RMSNorm, SwiGLU, RoPE,
GQA, no bias, tied embeddings; MoE in moe.py) and the
zero-bubble B/W split of src/wantrain/model/wgrad.py:45-303. The reference
obtains B from autograd and defers dW = dY^T X through a SplitLinear store;
here each layer writes its backward explicitly, so B is exactly the
activation-gradient chain (plus the LayerNorm / embedding parameter
gradients, which the reference also computes in B) and W is a list of GEMM
tasks that fold dW into fp32 gradients in the order they are run.

Boundary recipe: every entry boundary (the input of each block and of the
head) carries the config's boundary dtype. With an fp8 recipe
(fp8_e4m3_b128 / fp8_e5m2_b128) the block output is quantised in the
epilogue of the fc2 GEMM (one power-of-two scale per 128 elements of a row)
and dequantised in the prologue of the next LayerNorm / as the residual of
the next proj GEMM; with fp16 the same epilogue writes fp16 and the same two
readers widen it; gradients stay in the compute dtype and pass the boundary
unchanged (straight-through). The recipe is the same at every boundary
(the embedding's output included), so a run does not depend on where the
model is cut.
"""

from __future__ import annotations

import torch

from elysium_wan_b200 import ops

from .config import GPTConfig
from .params import ParamSpec, ParamStore, init_params


class Act:
    """A boundary activation: a dense tensor (bf16 / fp16 on the GPU, fp32 on
    the host path), or an fp8 payload (e4m3 / e5m2) with its 1x128 scales."""

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


def uses_general_arch(cfg: GPTConfig) -> bool:
    """Any non-default knob selects the generalized block (the reference's
    dispatch in src/wantrain/model/gpt.py:470-476), whose parameter names
    follow src/wantrain/model/arch.py (mlp.fc1, mlp.gate, q / kv, ...)."""
    return (cfg.norm != "layernorm" or cfg.mlp != "gelu" or cfg.pos != "learned"
            or cfg.n_kv_head is not None or not cfg.bias or cfg.tie_embeddings
            or cfg.d_ff is not None or cfg.moe_experts > 0)


def _linear(name, out_f, in_f, bias, resid=False, pack=False):
    """pack: the partner listed next is read together with this one (its
    weight after this weight, its bias after this bias)."""
    w = ParamSpec(f"{name}.weight", (out_f, in_f), "normal_resid" if resid else "normal",
                  fan_in=in_f, matrix=True, pack=pack)
    return [w], ([ParamSpec(f"{name}.bias", (out_f,), "bias", fan_in=in_f, pack=pack)]
                 if bias else [])


def _norm_specs(name, d, layernorm):
    out = [ParamSpec(f"{name}.weight", (d,), "ones")]
    if layernorm:
        out.append(ParamSpec(f"{name}.bias", (d,), "zeros"))
    return out


LORA_TARGETS = {
    "attn": ("qkv", "q", "kv", "proj"),
    "attn_mlp": ("qkv", "q", "kv", "proj", "gate", "up", "down", "fc1", "fc2"),
    "all": ("qkv", "q", "kv", "proj", "gate", "up", "down", "fc1", "fc2", "out"),
}


def entry_specs(cfg: GPTConfig, e: int) -> list[ParamSpec]:
    """Specs of entry e; with LoRA (lora_rank > 0) every base tensor is frozen
    and each targeted linear gains a trainable adapter `{linear}.A.weight`
    (r x in, kaiming-uniform from its own positional stream) and
    `{linear}.B.weight` (out x r, zeros), declared after the entry's base
    tensors so the base init is the same as without LoRA (reference:
    src/wantrain/model/lora.py)."""
    if cfg.arch == "user":
        from elysium_wan_b200.models import user

        return user.entry_specs(cfg, e)
    base = _base_specs(cfg, e)
    if not cfg.lora_rank:
        return base
    want = LORA_TARGETS[cfg.lora_targets]
    out, adapters = [], []
    for sp in base:
        out.append(ParamSpec(sp.name, sp.shape, sp.init, sp.fan_in, sp.matrix, sp.pack,
                             frozen=True, replicate=sp.replicate))
        stem = sp.name[:-len(".weight")] if sp.name.endswith(".weight") else None
        if sp.matrix and stem and stem.split(".")[-1] in want:
            o, i = sp.shape
            # the merge W + s B A reads the adapters' fp32 masters: a pieces
            # stage keeps them whole on every replica
            adapters += [ParamSpec(f"{stem}.A.weight", (cfg.lora_rank, i), "lora_a", fan_in=i,
                                   matrix=True, replicate=True),
                         ParamSpec(f"{stem}.B.weight", (o, cfg.lora_rank), "zeros", fan_in=cfg.lora_rank,
                                   matrix=True, replicate=True)]
    return out + adapters


class LoraWTask:
    """W of a frozen linear with an adapter y += s * (x A^T) B^T:
    dA += s (dY B)^T X and dB += s dY^T (X A^T); four skinny GEMMs instead of
    the full dY^T X."""

    __slots__ = ("dy", "x", "a", "b", "ga", "gb", "scale", "peer")

    def __init__(self, dy, x, a, b, ga, gb, scale):
        self.dy, self.x, self.a, self.b, self.ga, self.gb = dy, x, a, b, ga, gb
        self.scale = scale
        self.peer = None

    def run(self):
        u = ops.linear_dx(self.dy, self.b)
        u.mul_(self.scale)
        ops.linear_dw(u, self.x, self.ga, accumulate=True)
        t = ops.linear_fwd(self.x, self.a)
        t.mul_(self.scale)
        ops.linear_dw(self.dy, t, self.gb, accumulate=True)
        self.dy = self.x = None

    def record_stream(self, stream):
        self.dy.record_stream(stream)
        self.x.record_stream(stream)


def w_tasks(store, dy, x, wnames: list, bnames: list | None, scale: float = 1.0) -> list:
    """The W tasks of a linear, or of linears that share their input and sit
    back to back (q with kv, gate with up; dy then holds their output columns
    side by side): one dY^T X task for a trainable base, adapter tasks for a
    frozen base with LoRA, nothing for a frozen base without one."""
    gw = store.gj(wnames) if len(wnames) > 1 else store.g(wnames[0])
    if gw is not None:
        gb = None
        if bnames:
            gb = store.gj(bnames) if len(bnames) > 1 else store.g(bnames[0])
        return [WTask(dy, x, gw, gb)]
    out, col = [], 0
    for wn in wnames:
        rows = store.index[wn][1][0]
        stem = wn[:-len(".weight")]
        a = f"{stem}.A.weight"
        if a in store.index:
            d = dy if len(wnames) == 1 else dy[:, col:col + rows]
            out.append(LoraWTask(d, x, store.w(a), store.w(f"{stem}.B.weight"), store.g(a),
                                 store.g(f"{stem}.B.weight"), scale))
        col += rows
    return out


def _base_specs(cfg: GPTConfig, e: int) -> list[ParamSpec]:
    """Parameter specs of flat-list entry e, named like the reference's
    nn.ModuleList ("{e}.qkv.weight", ...). Matrices one GEMM reads as one
    operand (q with kv, gate with up) are listed back to back, then their
    biases, so the store holds each group contiguously."""
    d, V, S, f, n = cfg.d_model, cfg.vocab_size, cfg.seq_len, cfg.ff, cfg.n_layer
    if e == 0:
        out = [ParamSpec(f"{e}.tok.weight", (V, d), "embed")]
        if cfg.pos == "learned":
            out.append(ParamSpec(f"{e}.pos.weight", (S, d), "embed"))
        return out
    ln = cfg.norm == "layernorm"
    if e == n + 1:
        out = _norm_specs(f"{e}.ln_f", d, ln)
        if not cfg.tie_embeddings:
            out.append(ParamSpec(f"{e}.out.weight", (V, d), "normal", fan_in=d, matrix=True))
        return out
    if not uses_general_arch(cfg):
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
    b = cfg.bias
    out = _norm_specs(f"{e}.ln1", d, ln)
    if cfg.kv_heads == cfg.n_head:
        w, bb = _linear(f"{e}.qkv", 3 * d, d, b)
        out += w + bb
    else:
        wq, bq = _linear(f"{e}.q", d, d, b, pack=True)
        wkv, bkv = _linear(f"{e}.kv", 2 * cfg.kv_heads * cfg.head_dim, d, b)
        out += wq + wkv + bq + bkv
    w, bb = _linear(f"{e}.proj", d, d, b, resid=True)
    out += w + bb + _norm_specs(f"{e}.ln2", d, ln)
    if cfg.is_moe_layer(e):
        from .moe import moe_specs

        return out + moe_specs(cfg, e)
    if cfg.mlp == "gelu":
        w1, b1 = _linear(f"{e}.mlp.fc1", f, d, b)
        w2, b2 = _linear(f"{e}.mlp.fc2", d, f, b, resid=True)
        return out + w1 + b1 + w2 + b2
    wg, bg = _linear(f"{e}.mlp.gate", f, d, b, pack=True)
    wu, bu = _linear(f"{e}.mlp.up", f, d, b)
    wd, bd = _linear(f"{e}.mlp.down", d, f, b, resid=True)
    return out + wg + wu + bg + bu + wd + bd


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
                                        rank, 0, None, None)
        else:
            ops.linear_dw(self.dy, self.x, self.w_grad, accumulate=True)
        if self.b_grad is not None:
            ops.colsum(self.dy, self.b_grad, accumulate=True)
        self.dy = self.x = None

    def record_stream(self, stream):
        """Keep the inputs' memory alive until `stream` has consumed them."""
        self.dy.record_stream(stream)
        self.x.record_stream(stream)


class PairWTask:
    """The W of one linear for two microbatches of a slot (its owned
    microbatches 2k and 2k + 1): dW (+)= dY1^T X1 + dY2^T X2 in one GEMM over
    both token sets, then the bias row sums in microbatch order. A ZeRO-1 peer
    scatter on the second (the replica's last) runs on the paired GEMM too."""

    __slots__ = ("t1", "t2")

    def __init__(self, t1: WTask, t2: WTask):
        self.t1, self.t2 = t1, t2

    def run(self):
        t1, t2 = self.t1, self.t2
        if t2.peer is not None:
            slots, lo, stride, flat_off, rank = t2.peer
            ops.ext().gemm_peer_scatter(t1.dy, t1.x, t2.w_grad, slots, lo, stride, flat_off, rank,
                                        0, t2.dy, t2.x)
        else:
            ops.linear_dw_pair(t1.dy, t1.x, t2.dy, t2.x, t2.w_grad, accumulate=True)
        if t2.b_grad is not None:
            ops.colsum(t1.dy, t2.b_grad, accumulate=True)
            ops.colsum(t2.dy, t2.b_grad, accumulate=True)
        t1.dy = t1.x = t2.dy = t2.x = None

    def record_stream(self, stream):
        self.t1.record_stream(stream)
        self.t2.record_stream(stream)


def pair_w_tasks(first: list, second: list) -> list:
    """The W tasks of two microbatches of a slot, paired linear by linear where
    both are plain dW tasks of the same gradient (same shapes); any other task
    (adapters, expert GEMMs with different token counts, ...) runs unpaired in
    microbatch order, which is the fold the oracle declares for it too."""
    if len(first) != len(second):
        return list(first) + list(second)
    out, tail = [], []
    for a, b in zip(first, second):
        if (type(a) is WTask and type(b) is WTask and a.peer is None
                and a.w_grad.data_ptr() == b.w_grad.data_ptr() and a.w_grad.shape == b.w_grad.shape
                and a.dy.shape[1:] == b.dy.shape[1:] and a.x.shape[1:] == b.x.shape[1:]
                and (a.b_grad is None) == (b.b_grad is None)):
            out.append(PairWTask(a, b))
        else:
            out.append(a)
            tail.append(b)
    # unpaired second-microbatch tasks after every first-microbatch task: each
    # gradient still folds microbatch 2k before 2k + 1
    return out + tail


class WExecutor:
    """Runs W tasks on a side CUDA stream so the weight-gradient GEMMs fill the
    SMs the critical-path B GEMMs leave idle (their last wave). Each submission
    waits for everything enqueued on the compute stream so far; tasks run in
    submission order, so every parameter still folds its microbatches in order.
    On CPU the tasks run inline."""

    def __init__(self, device, enabled: bool = True):
        self.cuda = torch.device(device).type == "cuda" and enabled
        self.stream = torch.cuda.Stream(device=device) if self.cuda else None

    def run(self, tasks: list, timing: bool = False):
        """Enqueue `tasks`; with `timing`, returns (start, end) CUDA events
        recorded around them on the side stream (the W work's device time)."""
        if not self.cuda:
            for t in tasks:
                t.run()
            return None
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            e0 = e1 = None
            if timing:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record()
            for t in tasks:
                t.record_stream(self.stream)
                t.run()
            if timing:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record()
        return (e0, e1) if timing else None

    def join(self):
        if self.cuda:
            torch.cuda.current_stream().wait_stream(self.stream)


class Embed:
    is_embed, is_head = True, False
    def __init__(self, cfg, store: ParamStore, e: int):
        self.cfg, self.s, self.e = cfg, store, e
        self.has_pos = cfg.pos == "learned"

    def forward(self, tokens: torch.Tensor, ctx: dict) -> Act:
        c = self.cfg
        ctx["tokens"] = tokens
        wpe = self.s.p(f"{self.e}.pos.weight") if self.has_pos else None
        out = ops.embed_fwd(tokens, self.s.p(f"{self.e}.tok.weight"), wpe, c.seq_len,
                            ops.q8_dtype(c.boundary_dtype),
                            out_dtype=ops.act_dtype(c.boundary_dtype, tokens.is_cuda))
        return Act(*out) if isinstance(out, tuple) else _boundary_out(c, out)

    def backward(self, ctx: dict, dy: torch.Tensor, wq: list):
        dwte = self.s.g(f"{self.e}.tok.weight")
        if dwte is None:  # frozen table (LoRA): nothing to accumulate
            return None
        dwpe = self.s.g(f"{self.e}.pos.weight") if self.has_pos else None
        ops.embed_bwd(ctx["tokens"], dy, self.cfg.seq_len, dwte, dwpe)
        return None


_HOST_ROUND = {"bf16": torch.bfloat16, "fp16": torch.float16}


def _boundary_out(cfg, y) -> Act:
    """A dense entry output in the boundary dtype: on the GPU the producing
    kernel already wrote it; the host path keeps fp32 holding the recipe's
    rounding (bf16 or fp16)."""
    if not y.is_cuda and cfg.boundary_dtype in _HOST_ROUND:
        y = y.to(_HOST_ROUND[cfg.boundary_dtype]).float()
    return Act(y)


class Block:
    """One decoder block. Default knobs: the built-in GPT block (pre-LN,
    fused qkv, 4x GELU MLP with biases). Otherwise the generalized block:
    LayerNorm or RMSNorm, q / kv projections for grouped-query attention,
    rotary positions on q and k, GELU or SwiGLU MLP or the MoE block, biases
    optional."""

    def __init__(self, cfg, store: ParamStore, e: int):
        self.cfg, self.s, self.e = cfg, store, e
        self.n = lambda k: f"{e}.{k}"
        n = self.n
        gen = uses_general_arch(cfg)
        self.lora_s = cfg.lora_alpha / cfg.lora_rank if cfg.lora_rank else 1.0
        self.rms = cfg.norm == "rmsnorm"
        self.eps = cfg.norm_eps
        self.bias = cfg.bias
        if cfg.kv_heads == cfg.n_head:
            self.qkv_w, self.qkv_b = [n("qkv.weight")], [n("qkv.bias")]
        else:
            self.qkv_w, self.qkv_b = [n("q.weight"), n("kv.weight")], [n("q.bias"), n("kv.bias")]
        self.moe = None
        if cfg.is_moe_layer(e):
            from .moe import MoEMLP

            self.moe = MoEMLP(cfg, store, e)
            self.mlp = "moe"
        elif not gen:
            self.mlp = "gelu"
            self.up_w, self.up_b = [n("fc1.weight")], [n("fc1.bias")]
            self.dn_w, self.dn_b = n("fc2.weight"), n("fc2.bias")
        elif cfg.mlp == "gelu":
            self.mlp = "gelu"
            self.up_w, self.up_b = [n("mlp.fc1.weight")], [n("mlp.fc1.bias")]
            self.dn_w, self.dn_b = n("mlp.fc2.weight"), n("mlp.fc2.bias")
        else:
            self.mlp = "swiglu"
            self.up_w = [n("mlp.gate.weight"), n("mlp.up.weight")]
            self.up_b = [n("mlp.gate.bias"), n("mlp.up.bias")]
            self.dn_w, self.dn_b = n("mlp.down.weight"), n("mlp.down.bias")

    # parameter accessors (biases None when the block has none)
    def _w(self, names):
        return self.s.wj(names) if len(names) > 1 else self.s.w(names[0])

    def _bp(self, names):
        if not self.bias:
            return None
        return self.s.pj(names) if len(names) > 1 else self.s.p(names[0])

    def _bg(self, names):
        if not self.bias:
            return None
        return self.s.gj(names) if len(names) > 1 else self.s.g(names[0])

    def _gw(self, names):
        return self.s.gj(names) if len(names) > 1 else self.s.g(names[0])

    def _bn(self, names):
        return names if self.bias else None

    def _norm(self, x, xs, which):
        s, n = self.s, self.n
        beta = None if self.rms else s.p(n(f"{which}.bias"))
        return ops.layernorm_fwd(x, xs, s.p(n(f"{which}.weight")), beta, self.eps)

    def _norm_bwd(self, dy, x, xs, m, r, which, dres):
        s, n = self.s, self.n
        dg = s.g(n(f"{which}.weight"))
        dbeta = None if self.rms else s.g(n(f"{which}.bias"))
        if dg is None:  # frozen norm: its gradient goes to a scratch nobody reads
            d = x.shape[1]
            dg = s.sink(2 * d)[:d]
            dbeta = None if self.rms else s.sink(2 * d)[d:]
        return ops.layernorm_bwd(dy, x, xs, m, r, s.p(n(f"{which}.weight")), dres, dg, dbeta,
                                 accumulate=True)

    def forward(self, x: Act, ctx: dict) -> Act:
        c, s, n = self.cfg, self.s, self.n
        T = x.rows
        B, S, H, hd = T // c.seq_len, c.seq_len, c.n_head, c.head_dim
        h1, m1, r1 = self._norm(x.x, x.scale, "ln1")
        qkv = ops.linear_fwd(h1, self._w(self.qkv_w), self._bp(self.qkv_b))
        if c.pos == "rope":
            ops.rope(qkv, S, c.d_model + c.kv_heads * hd, hd, c.rope_theta)
        o, lse = ops.attention_fwd(qkv, B, S, H, hd, c.kv_heads)
        x2 = ops.linear_fwd(o, s.w(n("proj.weight")), self._bp([n("proj.bias")]), epi="resid",
                            resid=x.x, resid_scale=x.scale)
        h2, m2, r2 = self._norm(x2, None, "ln2")
        ctx.update(x=x, h1=h1, m1=m1, r1=r1, qkv=qkv, o=o, lse=lse, x2=x2, h2=h2, m2=m2, r2=r2)
        q8 = ops.q8_dtype(c.boundary_dtype)
        out_dt = ops.act_dtype(c.boundary_dtype, x2.is_cuda)
        if self.mlp == "moe":
            y = self.moe.forward(h2, ctx)
            out = ops.residual_add(x2, y)  # x2 + y in the compute dtype
            if q8 is not None:
                return Act(*ops.quant_q8(out, q8))
            if out.is_cuda and out.dtype != out_dt:
                out = out.to(out_dt)
            return _boundary_out(c, out)
        if self.mlp == "gelu":
            g, u = ops.linear_fwd(h2, self._w(self.up_w), self._bp(self.up_b), epi="gelu")
            ctx.update(g=g, u=u)
            hin = g
        else:
            gu = ops.linear_fwd(h2, self._w(self.up_w), self._bp(self.up_b))
            hin = ops.swiglu_fwd(gu)
            ctx.update(gu=gu, g=hin)
        bdn = self._bp([self.dn_b])
        if q8 is not None:
            q, sc = ops.linear_fwd(hin, s.w(self.dn_w), bdn, epi="resid_q8", resid=x2, q8=q8)
            return Act(q, sc)
        y = ops.linear_fwd(hin, s.w(self.dn_w), bdn, epi="resid", resid=x2, out_dtype=out_dt)
        return _boundary_out(c, y)

    def backward(self, ctx: dict, dy: torch.Tensor, wq: list) -> torch.Tensor:
        c, s, n = self.cfg, self.s, self.n
        T = dy.shape[0]
        B, S, H, hd = T // c.seq_len, c.seq_len, c.n_head, c.head_dim
        x: Act = ctx["x"]
        if self.mlp == "moe":
            dh2 = self.moe.backward(ctx, dy, wq)
        elif self.mlp == "gelu":
            du = ops.linear_dx(dy, s.w(self.dn_w), gelu_u=ctx["u"])
            wq += w_tasks(s, dy, ctx["g"], [self.dn_w], self._bn([self.dn_b]), self.lora_s)
            dh2 = ops.linear_dx(du, self._w(self.up_w))
            wq += w_tasks(s, du, ctx["h2"], self.up_w, self._bn(self.up_b), self.lora_s)
        else:
            dh = ops.linear_dx(dy, s.w(self.dn_w))
            wq += w_tasks(s, dy, ctx["g"], [self.dn_w], self._bn([self.dn_b]), self.lora_s)
            dgu = ops.swiglu_bwd(dh, ctx["gu"])
            del dh
            dh2 = ops.linear_dx(dgu, self._w(self.up_w))
            wq += w_tasks(s, dgu, ctx["h2"], self.up_w, self._bn(self.up_b), self.lora_s)
        dx2 = self._norm_bwd(dh2, ctx["x2"], None, ctx["m2"], ctx["r2"], "ln2", dy)
        do = ops.linear_dx(dx2, s.w(n("proj.weight")))
        wq += w_tasks(s, dx2, ctx["o"], [n("proj.weight")], self._bn([n("proj.bias")]),
                      self.lora_s)
        dqkv = ops.attention_bwd(ctx["qkv"], ctx["o"], do, ctx["lse"], B, S, H, hd, c.kv_heads)
        if c.pos == "rope":
            ops.rope(dqkv, S, c.d_model + c.kv_heads * hd, hd, c.rope_theta, inverse=True)
        dh1 = ops.linear_dx(dqkv, self._w(self.qkv_w))
        wq += w_tasks(s, dqkv, ctx["h1"], self.qkv_w, self._bn(self.qkv_b), self.lora_s)
        dx = self._norm_bwd(dh1, x.x, x.scale, ctx["m1"], ctx["r1"], "ln1", dx2)
        ctx.clear()
        return dx


class Head:
    is_embed, is_head = False, True
    def __init__(self, cfg, store: ParamStore, e: int):
        self.cfg, self.s, self.e = cfg, store, e
        self.n = lambda k: f"{e}.{k}"
        self.rms = cfg.norm == "rmsnorm"
        # A tied head reads (and adds its gradient into) the embedding table.
        self.out = "0.tok.weight" if cfg.tie_embeddings else f"{e}.out.weight"

    def forward(self, x: Act, ctx: dict, targets: torch.Tensor):
        """LN_f -> logits (fp32) -> mean CE. Returns the loss (device scalar);
        the logits gradient is produced here too and kept for B/W."""
        c, s, n = self.cfg, self.s, self.n
        T = x.rows
        V = c.vocab_size
        beta = None if self.rms else s.p(n("ln_f.bias"))
        h, m, r = ops.layernorm_fwd(x.x, x.scale, s.p(n("ln_f.weight")), beta, c.norm_eps)
        if h.is_cuda:
            # fused logits GEMM + cross-entropy: no fp32 logits in memory
            loss, dl = ops.head_ce(h, s.w(self.out), targets, V, 1.0 / T)
        else:
            logits = ops.linear_fwd(h, s.w(self.out), epi="f32")
            loss, dl = ops.cross_entropy(logits, V, targets.reshape(-1), 1.0 / T)
            del logits
        ctx.update(x=x, h=h, m=m, r=r, dl=dl)
        return loss

    def backward(self, ctx: dict, dy, wq: list) -> torch.Tensor:
        c, s, n = self.cfg, self.s, self.n
        V = c.vocab_size
        dl = ctx["dl"][:, :V]
        dh = ops.linear_dx(dl, s.w(self.out))
        scale = c.lora_alpha / c.lora_rank if c.lora_rank else 1.0
        if c.tie_embeddings:
            if not c.lora_rank or c.lora_targets == "all":
                wq.append(WTask(dl, ctx["h"], s.tied_grad, None))
        else:
            wq += w_tasks(s, dl, ctx["h"], [self.out], None, scale)
        x: Act = ctx["x"]
        dg = s.g(n("ln_f.weight"))
        dbeta = None if self.rms else s.g(n("ln_f.bias"))
        if dg is None:
            d = x.x.shape[1]
            dg = s.sink(2 * d)[:d]
            dbeta = None if self.rms else s.sink(2 * d)[d:]
        dx = ops.layernorm_bwd(dh, x.x, x.scale, ctx["m"], ctx["r"], s.p(n("ln_f.weight")), None,
                               dg, dbeta, accumulate=True)
        ctx.clear()
        return dx


class StageModel:
    """The entries [lo, hi) of the flat layer list on one device, with their
    parameter store. lo == 0 owns the embedding; hi == n_layer + 2 owns the head."""

    def __init__(self, cfg: GPTConfig, span: tuple[int, int], device, seed: int,
                 shard: tuple | None = None):
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
        # Tied embeddings: the head's stage without the table holds a relay copy
        # of it (not trained here: stage 0 sends the updated values each step);
        # it draws the same init stream as the table (entry 0, index 0).
        self.tied = cfg.tie_embeddings and self.hi == cfg.n_entries
        if self.tied and self.lo > 0:
            V, d = cfg.vocab_size, cfg.d_model
            specs.append(ParamSpec("0.tok.weight", (V, d), "embed", fan_in=d, matrix=True,
                                   frozen=True))
            entry_of["0.tok.weight"] = 0
        # CPU stores read the master directly unless a working copy must differ
        # from it (LoRA's merged weights) or hold more than it (pieces).
        work = torch.bfloat16 if self.device.type == "cuda" else (
            torch.float32 if cfg.lora_rank or shard is not None else None)
        if cfg.lora_rank and cfg.moe_experts:
            raise NotImplementedError("LoRA over MoE blocks is not built")
        if cfg.lora_rank and self.device.type == "cuda" and cfg.lora_rank % 8:
            raise ValueError("lora_rank must be a multiple of 8 on the GPU kernels")
        if cfg.arch == "user" and self.device.type != "cpu":
            raise ValueError("user models run on the host path (device cpu)")
        self.store = ParamStore(specs, self.device, work_dtype=work, shard=shard)
        if cfg.arch == "user":
            from elysium_wan_b200.models import user

            user.copy_initial(self.store, cfg, span, seed)
        else:
            init_params(self.store, seed, entry_of, cfg.init_std, cfg.n_layer, cfg.init_scheme,
                        first_of_entry={"0.tok.weight": 0} if self.tied and self.lo > 0 else None)
        # The head's gradient of a tied table accumulates apart from the
        # embedding's (its own fold, microbatch order); before the optimizer the
        # table's gradient becomes (embedding part) + (head part) on every cut.
        self.store.tied_grad = (torch.zeros((cfg.vocab_size, cfg.d_model), dtype=torch.float32,
                                            device=self.device) if self.tied else None)
        # adapted linears: (base weight, A, B)
        self.adapters = [(n[:-len(".A.weight")] + ".weight", n, n[:-len(".A.weight")] + ".B.weight")
                         for n in self.store.names() if n.endswith(".A.weight")]
        self.after_step()
        self.layers = []
        if cfg.arch == "user":
            from elysium_wan_b200.models import user

            mods = user.stage_modules(cfg, span, seed)
            self.layers = [user.UserLayer(cfg, self.store, e, m)
                           for e, m in zip(range(self.lo, self.hi), mods)]
            return
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

    def zero_grad(self):
        self.store.zero_grad()
        if self.store.tied_grad is not None:
            self.store.tied_grad.zero_()

    def fold_tied(self, head_part=None):
        """Table gradient += the head's part (its own, or one received from the
        head's stage). Called once per step, after every microbatch."""
        g = self.store.g("0.tok.weight")
        if g is None:
            return
        g.add_(self.store.tied_grad if head_part is None else head_part)

    def set_tied_table(self, values):
        """The relay copy takes stage 0's updated table (and its working copy)."""
        s = self.store
        s.p("0.tok.weight").copy_(values)
        s.w("0.tok.weight").copy_(values)

    def after_step(self):
        """Refresh what depends on the trained tensors: with LoRA, the working
        copy of each adapted base becomes W + (alpha / r) B A (computed in
        fp32, rounded once), so forward and input-gradient GEMMs run the
        merged weight unchanged."""
        if not self.adapters:
            return
        s, c = self.store, self.cfg
        scale = c.lora_alpha / c.lora_rank
        with torch.no_grad():
            for w, a, b in self.adapters:
                merged = s.p(w) + scale * (s.p(b) @ s.p(a))
                s.w(w).copy_(merged)

    def moe_blocks(self) -> list:
        """The MoE MLPs of this stage, in entry order."""
        return [l.moe for l in self.layers if isinstance(l, Block) and l.moe is not None]

    def take_moe_records(self) -> list:
        """Pop every MoE record of the step, sorted by (layer, call order)."""
        out = []
        for m in self.moe_blocks():
            out += m.take_records()
        return out

    def moe_bias_update(self, counts: dict, global_tokens: int):
        """Selection-bias update after the optimizer step; counts maps the
        entry index to the global batch's int64 expert counts."""
        for m in self.moe_blocks():
            if m.e in counts:
                m.bias_update(counts[m.e], global_tokens)

    def buffers(self) -> dict:
        """Non-trained state a checkpoint carries (MoE selection biases)."""
        return {f"{m.p}.sel_bias": m.sel_bias for m in self.moe_blocks()}

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
            if getattr(layer, "is_head", False):
                h = layer.forward(h, ctx, targets)
            else:
                h = layer.forward(h, ctx)
            if keep == "all" or getattr(layer, "is_head", False) or getattr(layer, "is_embed", False):
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
                ctx: dict = {"_recompute": True}
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
