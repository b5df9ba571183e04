"""Plain torch-autograd restatement (fp32) of the generalized decoder block:
RMSNorm / LayerNorm, q / kv grouped-query attention with adjacent-pair RoPE,
GELU or SwiGLU MLP, optional biases, tied embeddings, and the MoE MLP (router
scores, stable selection, renormalisation, combine, shared expert, aux terms
added to the loss). Used only as a test oracle for the explicit F / B / W
code in elysium_wan_b200.models."""

import math

import torch
import torch.nn.functional as F


def _norm(cfg, x, P, name):
    w = P[f"{name}.weight"]
    if cfg.norm == "layernorm":
        return F.layer_norm(x, (x.shape[-1],), w, P[f"{name}.bias"], cfg.ln_eps)
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + cfg.rms_eps) * w


def _lin(x, P, name, bias):
    y = x @ P[f"{name}.weight"].t()
    return y + P[f"{name}.bias"] if bias else y


def _rope(x, S, theta):
    """x: (B, heads, S, hd); rotates pairs (2i, 2i+1) by pos * theta^(-2i/hd)."""
    hd = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    ang = torch.outer(torch.arange(S, dtype=torch.float64), inv)
    c, s = torch.cos(ang).float(), torch.sin(ang).float()
    x1, x2 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1).flatten(-2)


def _swiglu(x, P, name, bias, cfg=None, clamped=False):
    g, u = _lin(x, P, f"{name}.gate", bias), _lin(x, P, f"{name}.up", bias)
    if clamped:
        g = g.clamp(max=cfg.moe_limit)
        u = u.clamp(min=-cfg.moe_limit, max=cfg.moe_limit)
        return _lin((u + 1) * (g * torch.sigmoid(g * cfg.moe_alpha)), P, f"{name}.down", bias)
    return _lin(F.silu(g) * u, P, f"{name}.down", bias)


def _select(key, k, groups, topk_groups):
    T, E = key.shape
    order = torch.sort(key, dim=-1, descending=True, stable=True).indices
    if groups > 1:
        kg = key.view(T, groups, E // groups)
        top2 = torch.sort(kg, dim=-1, descending=True, stable=True).values[..., :2]
        chosen = torch.sort(top2[..., 0] + top2[..., 1], dim=-1, descending=True,
                            stable=True).indices[:, :topk_groups]
        allowed = torch.zeros(T, groups, dtype=torch.uint8).scatter_(1, chosen, 1)
        allowed = allowed.repeat_interleave(E // groups, dim=1)
        order = order.gather(1, torch.sort(allowed.gather(1, order), dim=-1, descending=True,
                                           stable=True).indices)
    return torch.sort(order[:, :k], dim=-1).values


def _moe(cfg, x, P, e, sel_bias):
    """Returns (out, aux loss) of the MoE MLP on x (T, d)."""
    E, k = cfg.moe_experts, cfg.moe_top_k
    T = x.shape[0]
    p = f"{e}.mlp"
    lf = _lin(x, P, f"{p}.router", cfg.moe_router_bias)
    if cfg.moe_score == "sigmoid":
        sc = torch.sigmoid(lf)
        q = sc / sc.sum(-1, keepdim=True)
    else:
        sc = torch.softmax(lf, -1)
        q = sc
    key = {"logit": lf, "score": sc, "score_bias": sc + sel_bias}[cfg.moe_select].detach()
    sel = _select(key, k, cfg.moe_groups, cfg.moe_topk_groups)
    pw = torch.softmax(lf.gather(1, sel), -1) if cfg.moe_score == "softmax_k" else sc.gather(1, sel)
    if cfg.moe_norm:
        pw = pw / (pw.sum(-1, keepdim=True) + cfg.moe_norm_eps)
    w = pw * cfg.moe_scale
    out = torch.zeros_like(x)
    clamped = cfg.moe_expert == "swiglu_clamped"
    for i in range(E):
        for j in range(k):
            rows = (sel[:, j] == i).nonzero().reshape(-1)
            if rows.numel() == 0:
                continue
            xin = x[rows]
            if cfg.moe_apply == "input":
                xin = xin * w[rows, j, None]
            y = _swiglu(xin, P, f"{p}.experts.{i}", clamped, cfg, clamped)
            if cfg.moe_apply != "input":
                y = w[rows, j, None] * y
            out = out.index_add(0, rows, y)
    if cfg.moe_shared_d_ff:
        ys = _swiglu(x, P, f"{p}.shared_expert", False)
        if cfg.moe_shared_gate == "sigmoid":
            ys = torch.sigmoid(x @ P[f"{p}.shared_expert_gate.weight"].t()) * ys
        out = out + ys
    counts = torch.bincount(sel.reshape(-1), minlength=E).float()
    if cfg.moe_lbl_scope == "layer":
        lbl = (E / (T * T * k)) * (counts * q.sum(0)).sum()
    else:
        S = cfg.seq_len
        b = T // S
        cs = F.one_hot(sel.view(b, S * k), E).sum(1).float()
        lbl = ((E / (S * S * k)) * (cs * q.view(b, S, E).sum(1)).sum(-1)).mean()
    z = (torch.logsumexp(lf, -1) ** 2).mean()
    return out, cfg.moe_lbl_coef * lbl + cfg.moe_z_coef * z


def ref_loss_general(cfg, P: dict, idx, tgt, sel_biases=None):
    B, S = idx.shape
    d, H, Hk, hd = cfg.d_model, cfg.n_head, cfg.kv_heads, cfg.head_dim
    T = B * S
    x = P["0.tok.weight"][idx.reshape(-1)]
    if cfg.pos == "learned":
        x = x + P["0.pos.weight"][torch.arange(T) % S]
    aux = 0.0
    for e in range(1, cfg.n_layer + 1):
        h = _norm(cfg, x, P, f"{e}.ln1")
        if Hk == H:
            qkv = _lin(h, P, f"{e}.qkv", cfg.bias)
            q, kk, v = qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:]
        else:
            q = _lin(h, P, f"{e}.q", cfg.bias)
            kv = _lin(h, P, f"{e}.kv", cfg.bias)
            kk, v = kv[:, :Hk * hd], kv[:, Hk * hd:]
        q = q.view(B, S, H, hd).transpose(1, 2)
        kk = kk.view(B, S, Hk, hd).transpose(1, 2)
        v = v.view(B, S, Hk, hd).transpose(1, 2)
        if cfg.pos == "rope":
            q, kk = _rope(q, S, cfg.rope_theta), _rope(kk, S, cfg.rope_theta)
        kk = kk.repeat_interleave(H // Hk, dim=1)
        v = v.repeat_interleave(H // Hk, dim=1)
        att = (q @ kk.transpose(-2, -1)) / math.sqrt(hd)
        att = att.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
        o = (torch.softmax(att, -1) @ v).transpose(1, 2).reshape(T, d)
        x = x + _lin(o, P, f"{e}.proj", cfg.bias)
        h2 = _norm(cfg, x, P, f"{e}.ln2")
        if cfg.is_moe_layer(e):
            sb = sel_biases[e] if sel_biases else torch.zeros(cfg.moe_experts)
            y, a = _moe(cfg, h2, P, e, sb)
            aux = aux + a
        elif cfg.mlp == "gelu":
            y = _lin(F.gelu(_lin(h2, P, f"{e}.mlp.fc1", cfg.bias)), P, f"{e}.mlp.fc2", cfg.bias)
        else:
            y = _swiglu(h2, P, f"{e}.mlp", cfg.bias)
        x = x + y
    e = cfg.n_layer + 1
    h = _norm(cfg, x, P, f"{e}.ln_f")
    wout = P["0.tok.weight"] if cfg.tie_embeddings else P[f"{e}.out.weight"]
    ce = F.cross_entropy(h @ wout.t(), tgt.reshape(-1))
    return ce, aux
