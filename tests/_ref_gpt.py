"""Plain torch-autograd restatement of the built-in GPT (fp32), used only as a
test oracle for the explicit F/B/W implementation in elysium_wan_b200.models."""

import math

import torch
import torch.nn.functional as F


def ref_loss(cfg, P: dict, idx, tgt):
    """P maps the flat-list parameter names ("{e}.qkv.weight", ...) to tensors."""
    B, S = idx.shape
    d, H = cfg.d_model, cfg.n_head
    hd = d // H
    x = P["0.tok.weight"][idx.reshape(-1)] + P["0.pos.weight"][torch.arange(B * S) % S]
    for e in range(1, cfg.n_layer + 1):
        g = lambda k: P[f"{e}.{k}"]
        h = F.layer_norm(x, (d,), g("ln1.weight"), g("ln1.bias"), cfg.ln_eps)
        qkv = h @ g("qkv.weight").t() + g("qkv.bias")
        q, k, v = qkv.view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)
        att = (q @ k.transpose(-2, -1)) / math.sqrt(hd)
        att = att.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
        o = (torch.softmax(att, -1) @ v).transpose(1, 2).reshape(B * S, d)
        x = x + o @ g("proj.weight").t() + g("proj.bias")
        h2 = F.layer_norm(x, (d,), g("ln2.weight"), g("ln2.bias"), cfg.ln_eps)
        u = h2 @ g("fc1.weight").t() + g("fc1.bias")
        x = x + F.gelu(u) @ g("fc2.weight").t() + g("fc2.bias")
    e = cfg.n_layer + 1
    h = F.layer_norm(x, (d,), P[f"{e}.ln_f.weight"], P[f"{e}.ln_f.bias"], cfg.ln_eps)
    logits = h @ P[f"{e}.out.weight"].t()
    return F.cross_entropy(logits, tgt.reshape(-1))
