"""The exact mixture-of-experts block with an explicit forward and backward.

Reference: src/wantrain/model/arch.py:279-763 (MoEMLP, moe_select,
moe_forward, the written folds of _Fanout / _Dispatch / _Combine, the aux
injection and moe_bias_update). The function is the same; here F, B and W are
written out, so the expert dW GEMMs join the deferred W queue like every
other linear:

- router logits in the compute dtype (the bf16 tcgen05 GEMM with an fp32
  output) or in fp32 (`moe_router_dtype`);
- scores softmax | softmax_k | sigmoid in fp32; selection on fp32 keys by a
  stable descending sort (never top-k), group-limited when moe_groups > 1,
  then the k chosen experts in ascending index per token;
- weights = the score at the selected experts (never the selection bias),
  optionally renormalised by a left fold in ascending expert order, times
  moe_scale;
- dispatch: slots sorted by (expert, token), one gather; each expert runs
  exactly once on exactly its rows (zero rows included) as a SwiGLU of
  GEMMs; combine is the left fold over ascending expert index of w * Y in
  fp32; a shared expert (optionally sigmoid-gated) adds on top;
- aux terms (load-balance lbl, router z-loss) act per layer and microbatch:
  their coefficient is injected as their gradient, their values are
  recorded with the int64 expert counts;
- the selection-bias update after the optimizer step moves each bias by
  exactly +gamma, -gamma or 0 from integer counts of the global batch.

Every fold that the reference writes as a left fold is a left fold here, in
the same order, so a run is deterministic; the gradient of x is the left fold
of its consumers' gradients in the order router, dispatch, shared expert,
shared gate.
"""

from __future__ import annotations

from typing import NamedTuple

import torch

from elysium_wan_b200 import ops

from .params import ParamSpec


class MoERecord(NamedTuple):
    layer: int
    aux: dict  # {"lbl": float hex, "z": float hex}
    counts: torch.Tensor  # int64 (E,), sums to T * k


def moe_specs(cfg, e: int) -> list[ParamSpec]:
    """Parameters of the MoE MLP of entry e, named like the reference's
    module tree (router, experts.i.{gate,up,down}, shared_expert,
    shared_expert_gate)."""
    d, E, f = cfg.d_model, cfg.moe_experts, cfg.moe_width
    p = f"{e}.mlp"
    clamped = cfg.moe_expert == "swiglu_clamped"
    # the router's fp32 master is read directly (fp32 router logits), so a
    # pieces stage keeps it whole on every replica
    out = [ParamSpec(f"{p}.router.weight", (E, d), "normal", fan_in=d, matrix=True,
                     replicate=True)]
    if cfg.moe_router_bias:
        out.append(ParamSpec(f"{p}.router.bias", (E,), "bias", fan_in=d))

    def expert(name, width, bias):
        sp = [ParamSpec(f"{name}.gate.weight", (width, d), "normal", fan_in=d, matrix=True,
                        pack=True),
              ParamSpec(f"{name}.up.weight", (width, d), "normal", fan_in=d, matrix=True)]
        if bias:
            sp += [ParamSpec(f"{name}.gate.bias", (width,), "bias", fan_in=d, pack=True),
                   ParamSpec(f"{name}.up.bias", (width,), "bias", fan_in=d)]
        sp.append(ParamSpec(f"{name}.down.weight", (d, width), "normal_resid", fan_in=width,
                            matrix=True))
        if bias:
            sp.append(ParamSpec(f"{name}.down.bias", (d,), "bias", fan_in=width))
        return sp

    for i in range(E):
        out += expert(f"{p}.experts.{i}", f, clamped)
    if cfg.moe_shared_d_ff:
        out += expert(f"{p}.shared_expert", cfg.moe_shared_d_ff, False)
        if cfg.moe_shared_gate == "sigmoid":
            out.append(ParamSpec(f"{p}.shared_expert_gate.weight", (1, d), "normal", fan_in=d))
    return out


def _stable_desc(key: torch.Tensor) -> torch.Tensor:
    return torch.sort(key, dim=-1, descending=True, stable=True).indices


def moe_select(key: torch.Tensor, k: int, groups: int = 1, topk_groups: int = 1) -> torch.Tensor:
    """(T, E) fp32 keys -> (T, k) selected experts, ascending per token.

    With groups, a group's key is the sum of its two largest keys; the
    topk_groups groups first in a stable descending sort are eligible, and the
    first k of the stable descending order restricted to them are taken. A NaN
    key is fatal."""
    if bool(torch.isnan(key).any()):
        raise ValueError("MoE selection: a NaN router key is fatal")
    T, E = key.shape
    order = _stable_desc(key)
    if groups > 1:
        kg = key.view(T, groups, E // groups)
        top2 = torch.sort(kg, dim=-1, descending=True, stable=True).values[..., :2]
        chosen = _stable_desc(top2[..., 0] + top2[..., 1])[:, :topk_groups]
        allowed = torch.zeros(T, groups, dtype=torch.uint8, device=key.device)
        allowed.scatter_(1, chosen, 1)
        allowed = allowed.repeat_interleave(E // groups, dim=1)
        # eligible experts first, keeping the key order within each class
        order = order.gather(1, _stable_desc(allowed.gather(1, order)))
    return torch.sort(order[:, :k], dim=-1).values


def _left_fold(cols):
    acc = cols[0]
    for c in cols[1:]:
        acc = acc + c
    return acc


class MoEMLP:
    def __init__(self, cfg, store, e: int):
        self.cfg, self.s, self.e = cfg, store, e
        self.p = f"{e}.mlp"
        self.E, self.k = cfg.moe_experts, cfg.moe_top_k
        self.clamped = cfg.moe_expert == "swiglu_clamped"
        self.sel_bias = torch.zeros(self.E, dtype=torch.float32, device=store.device)
        self.records: list[MoERecord] = []

    # --------------------------------------------------------------- helpers
    def _n(self, k):
        return f"{self.p}.{k}"

    def _expert_names(self, name):
        gu = [f"{name}.gate.weight", f"{name}.up.weight"]
        gub = [f"{name}.gate.bias", f"{name}.up.bias"]
        return gu, gub, f"{name}.down.weight", f"{name}.down.bias"

    def _swiglu_fwd(self, x, name, bias):
        s = self.s
        gu_w, gu_b, dn_w, dn_b = self._expert_names(name)
        gu = ops.linear_fwd(x, s.wj(gu_w), s.pj(gu_b) if bias else None)
        if self.clamped and bias:
            h = self._clamped_act(gu)
        else:
            h = ops.swiglu_fwd(gu)
        y = ops.linear_fwd(h, s.w(dn_w), s.p(dn_b) if bias else None)
        return y, gu, h

    def _clamped_act(self, gu):
        """(u + 1) * g * sigmoid(alpha g) with g <= limit, |u| <= limit."""
        c = self.cfg
        f = gu.shape[1] // 2
        g = gu[:, :f].float().clamp(max=c.moe_limit)
        u = gu[:, f:].float().clamp(min=-c.moe_limit, max=c.moe_limit)
        return ((u + 1) * (g * torch.sigmoid(g * c.moe_alpha))).to(gu.dtype)

    def _clamped_bwd(self, dh, gu):
        c = self.cfg
        f = gu.shape[1] // 2
        g0, u0 = gu[:, :f].float(), gu[:, f:].float()
        g = g0.clamp(max=c.moe_limit)
        u = u0.clamp(min=-c.moe_limit, max=c.moe_limit)
        sg = torch.sigmoid(g * c.moe_alpha)
        act = g * sg
        d = dh.float()
        dg = d * (u + 1) * (sg + g * c.moe_alpha * sg * (1 - sg)) * (g0 <= c.moe_limit)
        du = d * act * ((u0 >= -c.moe_limit) & (u0 <= c.moe_limit))
        return torch.cat([dg, du], dim=1).to(gu.dtype)

    def _swiglu_bwd(self, dy, x, gu, h, name, bias, wq):
        from .gpt import WTask

        s = self.s
        gu_w, gu_b, dn_w, dn_b = self._expert_names(name)
        dh = ops.linear_dx(dy, s.w(dn_w))
        wq.append(WTask(dy, h, s.g(dn_w), s.g(dn_b) if bias else None))
        dgu = self._clamped_bwd(dh, gu) if (self.clamped and bias) else ops.swiglu_bwd(dh, gu)
        dx = ops.linear_dx(dgu, s.wj(gu_w))
        wq.append(WTask(dgu, x, s.gj(gu_w), s.gj(gu_b) if bias else None))
        return dx

    def _router_logits(self, x):
        s, c = self.s, self.cfg
        w = self._n("router.weight")
        b = s.p(self._n("router.bias")) if c.moe_router_bias else None
        if c.moe_router_dtype == "fp32" or not x.is_cuda or self.E % 8:
            lf = x.float() @ s.p(w).t()
            return lf + b if b is not None else lf
        return ops.linear_fwd(x, s.w(w), b, epi="f32")

    # --------------------------------------------------------------- forward
    def forward(self, x: torch.Tensor, ctx: dict) -> torch.Tensor:
        """x: the normalised block input [T, d] (compute dtype). Returns the
        MLP output [T, d] (compute dtype, before the residual add)."""
        c, E, k = self.cfg, self.E, self.k
        T, d = x.shape
        lf = self._router_logits(x).float()
        if c.moe_score == "sigmoid":
            sc = torch.sigmoid(lf)
            q = sc / sc.sum(-1, keepdim=True)
        else:
            sc = torch.softmax(lf, -1)
            q = sc
        if c.moe_select == "logit":
            key = lf
        elif c.moe_select == "score":
            key = sc
        else:
            key = sc + self.sel_bias
        sel = moe_select(key, k, c.moe_groups, c.moe_topk_groups)
        if c.moe_score == "softmax_k":
            p = torch.softmax(lf.gather(1, sel), -1)
        else:
            p = sc.gather(1, sel)
        den = None
        if c.moe_norm:
            den = _left_fold(p.unbind(1)) + c.moe_norm_eps
            pn = p / den[:, None]
        else:
            pn = p
        w = pn * c.moe_scale

        flat_e = sel.reshape(-1)
        flat_t = torch.arange(T, device=x.device).repeat_interleave(k)
        perm = torch.sort(flat_e * T + flat_t, stable=True).indices
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(T * k, device=x.device)
        pos = inv.view(T, k)
        counts = torch.bincount(flat_e, minlength=E)
        src = flat_t[perm]
        xd = x.index_select(0, src)
        w_perm = None
        xd_in = xd
        if c.moe_apply == "input":
            w_perm = w.reshape(-1).index_select(0, perm)
            xd = (xd.float() * w_perm[:, None]).to(x.dtype)
        cnt = counts.tolist()
        Ys, saved, off = [], [], 0
        for i, ci in enumerate(cnt):
            if ci == 0:
                saved.append(None)
                continue
            rows = xd[off:off + ci]
            y, gu, h = self._swiglu_fwd(rows, self._n(f"experts.{i}"), self.clamped)
            Ys.append(y)
            saved.append((rows, gu, h))
            off += ci
        Y = torch.cat(Ys, 0) if Ys else x.new_zeros((0, d))
        Ysl = Y.index_select(0, pos.reshape(-1)).view(T, k, d).float()
        if c.moe_apply == "input":
            out = _left_fold([Ysl[:, j] for j in range(k)])
        else:
            out = _left_fold([w[:, j, None] * Ysl[:, j] for j in range(k)])
        sh = None
        if c.moe_shared_d_ff:
            ys, gu_s, h_s = self._swiglu_fwd(x, self._n("shared_expert"), False)
            ysf = ys.float()
            zg = None
            if c.moe_shared_gate == "sigmoid":
                zg = x.float() @ self.s.p(self._n("shared_expert_gate.weight")).t()
                out = out + torch.sigmoid(zg) * ysf
            else:
                out = out + ysf
            sh = (gu_s, h_s, ysf, zg)
        y_out = out.to(x.dtype)

        # aux values (recorded once per microbatch: not on a recompute pass)
        cf = counts.to(torch.float32)
        if c.moe_lbl_scope == "layer":
            lbl = (E / (T * T * k)) * (cf * q.sum(0)).sum()
            cs = None
        else:
            S = c.seq_len
            b = T // S
            cs = torch.nn.functional.one_hot(sel.view(b, S * k), E).sum(1).to(torch.float32)
            lbl = ((E / (S * S * k)) * (cs * q.view(b, S, E).sum(1)).sum(-1)).mean()
        lse = torch.logsumexp(lf, -1)
        z = (lse * lse).mean()
        if not ctx.get("_recompute"):
            self.records.append(MoERecord(self.e, {"lbl": float(lbl).hex(), "z": float(z).hex()},
                                          counts.detach().cpu()))
        ctx["moe"] = dict(x=x, lf=lf, sc=sc, q=q, sel=sel, p=p, den=den, w=w, perm=perm, pos=pos,
                          src=src, cnt=cnt, saved=saved, Ysl=Ysl, xd_in=xd_in, w_perm=w_perm,
                          sh=sh, cs=cs, lse=lse)
        return y_out

    # --------------------------------------------------------------- backward
    def backward(self, ctx: dict, dy: torch.Tensor, wq: list) -> torch.Tensor:
        """dy: gradient of the MLP output [T, d]. Returns d(x) in the
        compute dtype; appends the expert / shared / router W tasks."""
        from .gpt import WTask

        c, E, k, s = self.cfg, self.E, self.k, self.s
        m = ctx.pop("moe")
        x, lf, sc, sel, w, perm, pos = (m[n] for n in ("x", "lf", "sc", "sel", "w", "perm", "pos"))
        T, d = x.shape
        g = dy.float()
        cdt = x.dtype

        # shared expert and its gate
        dx_sh = dx_gate = None
        if m["sh"] is not None:
            gu_s, h_s, ysf, zg = m["sh"]
            if zg is not None:
                gate = torch.sigmoid(zg)
                dys = (gate * g).to(cdt)
                dzg = (g * ysf).sum(-1, keepdim=True) * gate * (1 - gate)
                gw = self._n("shared_expert_gate.weight")
                dx_gate = dzg @ s.p(gw)
                s.g(gw).add_(dzg.t() @ x.float())
            else:
                dys = g.to(cdt)
            dx_sh = self._swiglu_bwd(dys, x, gu_s, h_s, self._n("shared_expert"), False, wq).float()

        # combine
        Ysl = m["Ysl"]
        if c.moe_apply == "input":
            dYsl = g[:, None, :].expand(T, k, d)
            dw = None
        else:
            dYsl = w[..., None] * g[:, None, :]
            dw = (g[:, None, :] * Ysl).sum(-1)
        dY = dYsl.reshape(T * k, d).to(cdt).index_select(0, perm)

        # experts, each once on its rows, in expert order
        dxd_parts, off = [], 0
        for i, ci in enumerate(m["cnt"]):
            if ci == 0:
                continue
            rows, gu, h = m["saved"][i]
            dxd_parts.append(self._swiglu_bwd(dY[off:off + ci], rows, gu, h,
                                              self._n(f"experts.{i}"), self.clamped, wq))
            off += ci
        dxd = torch.cat(dxd_parts, 0) if dxd_parts else x.new_zeros((0, d))
        if c.moe_apply == "input":
            w_perm = m["w_perm"]
            dw_perm = (dxd.float() * m["xd_in"].float()).sum(-1)
            dxd = (dxd.float() * w_perm[:, None]).to(cdt)
            dw = dw_perm.index_select(0, pos.reshape(-1)).view(T, k)
        # dispatch: a token's k slot gradients folded in ascending expert order
        G = dxd.float().index_select(0, pos.reshape(-1)).view(T, k, d)
        dx_disp = _left_fold([G[:, j] for j in range(k)])

        # weights -> scores -> router logits
        dpn = dw * c.moe_scale
        if c.moe_norm:
            D, p = m["den"], m["p"]
            dp = dpn / D[:, None] - ((dpn * p).sum(-1) / (D * D))[:, None]
        else:
            dp = dpn
        dlf = torch.zeros_like(lf)
        if c.moe_score == "softmax_k":
            p = m["p"]
            dsel = p * (dp - (dp * p).sum(-1, keepdim=True))
            dlf.scatter_(1, sel, dsel)
            dq = self._dq(m, T)
            if dq is not None:
                qq = torch.softmax(lf, -1)
                dlf = dlf + qq * (dq - (dq * qq).sum(-1, keepdim=True))
        else:
            ds = torch.zeros_like(lf).scatter_(1, sel, dp)
            dq = self._dq(m, T)
            if c.moe_score == "softmax":
                if dq is not None:
                    ds = ds + dq
                dlf = sc * (ds - (ds * sc).sum(-1, keepdim=True))
            else:
                if dq is not None:
                    tot = sc.sum(-1, keepdim=True)
                    ds = ds + dq / tot - (dq * sc).sum(-1, keepdim=True) / (tot * tot)
                dlf = ds * sc * (1 - sc)
        if c.moe_z_coef:
            dlf = dlf + c.moe_z_coef * (2.0 / T) * m["lse"][:, None] * torch.softmax(lf, -1)

        # router
        rw = self._n("router.weight")
        rb = s.g(self._n("router.bias")) if c.moe_router_bias else None
        if c.moe_router_dtype == "fp32" or not x.is_cuda or E % 8:
            dx_r = dlf @ s.p(rw)
            s.g(rw).add_(dlf.t() @ x.float())
            if rb is not None:
                rb.add_(dlf.sum(0))
        else:
            dl16 = dlf.to(cdt)
            dx_r = ops.linear_dx(dl16, s.w(rw)).float()
            wq.append(WTask(dl16, x, s.g(rw), rb))
        dx = dx_r + dx_disp
        if dx_sh is not None:
            dx = dx + dx_sh
        if dx_gate is not None:
            dx = dx + dx_gate
        return dx.to(cdt)

    def _dq(self, m, T):
        """Gradient the load-balance term injects into q (None without it)."""
        c, E, k = self.cfg, self.E, self.k
        if not c.moe_lbl_coef:
            return None
        cf = torch.bincount(m["sel"].reshape(-1), minlength=E).to(torch.float32)
        if c.moe_lbl_scope == "layer":
            return (c.moe_lbl_coef * E / (T * T * k)) * cf[None, :].expand(T, E)
        S = c.seq_len
        b = T // S
        per = (c.moe_lbl_coef * E / (S * S * k) / b) * m["cs"]  # (b, E)
        return per[:, None, :].expand(b, S, E).reshape(T, E)

    # --------------------------------------------------------------- bias update
    def bias_update(self, counts: torch.Tensor, global_tokens: int):
        """sel_bias += gamma * sign(T_g k - E c_i) with the global batch's
        int64 counts; the sign is taken in integers (0 on equality)."""
        c, E, k = self.cfg, self.E, self.k
        if not isinstance(counts, torch.Tensor) or counts.dtype != torch.int64 or \
                tuple(counts.shape) != (E,):
            raise ValueError(f"MoE layer {self.e}: counts must be int64 of shape ({E},)")
        if bool((counts < 0).any()) or int(counts.sum()) != global_tokens * k:
            raise ValueError(f"MoE layer {self.e}: counts are negative or do not sum to "
                             f"T_g*k={global_tokens * k}")
        gamma = float(c.moe_bias_rate)
        if gamma == 0:
            return
        sgn = torch.sign(global_tokens * k - E * counts).to(self.sel_bias.device)
        moved = self.sel_bias + sgn.to(torch.float32) * gamma
        self.sel_bias.copy_(torch.where(sgn == 0, self.sel_bias, moved))

    def take_records(self) -> list:
        out, self.records = self.records, []
        return out
