"""An example user model for `arch: "user"`: token + position embedding,
n_layer residual tanh-MLP blocks, a LayerNorm + linear head (build(cfg) -> n_layer + 2 modules)."""

import torch
from torch import nn


class Embed(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.tok = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.pos = nn.Parameter(torch.randn(cfg.seq_len, cfg.d_model) * 0.02)

    def forward(self, idx):
        return self.tok(idx) + self.pos[: idx.shape[1]]


class Block(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.ln = nn.LayerNorm(cfg.d_model)
        self.fc = nn.Linear(cfg.d_model, 2 * cfg.d_model)
        self.proj = nn.Linear(2 * cfg.d_model, cfg.d_model)

    def forward(self, x):
        return x + self.proj(torch.tanh(self.fc(self.ln(x))))


class Head(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.ln = nn.LayerNorm(cfg.d_model)
        self.out = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)

    def forward(self, x):
        return self.out(self.ln(x))


def build(cfg):
    return [Embed(cfg)] + [Block(cfg) for _ in range(cfg.n_layer)] + [Head(cfg)]
