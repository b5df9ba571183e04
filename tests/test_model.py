"""The explicit F / B / W split of the GPT equals autograd, and a model cut
into stages computes exactly what the whole model computes.

Would fail if: a backward formula, a deferred W task, the bias / LayerNorm /
embedding gradient folds, or the per-entry deterministic initialisation were
wrong, or if cutting the flat layer list changed any value.
"""

import torch

from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.models.gpt import StageModel

from ._ref_gpt import ref_loss


def _run(models, idx, tgt):
    """F through every stage, B back, then every W task in order."""
    wqs = [[] for _ in models]
    ctxs = []
    h = idx
    for m in models:
        out, c = m.forward(h, targets=tgt if m.last else None)
        ctxs.append(c)
        h = out
    loss = h
    dy = None
    for i in range(len(models) - 1, -1, -1):
        dy = models[i].backward(ctxs[i], dy, wqs[i])
    for wq in wqs:
        for t in wq:
            t.run()
    return loss


def test_fbw_matches_autograd():
    torch.manual_seed(0)
    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    m = StageModel(cfg, (0, cfg.n_entries), "cpu", seed=3)
    idx = torch.randint(0, cfg.vocab_size, (2, cfg.seq_len))
    tgt = torch.randint(0, cfg.vocab_size, (2, cfg.seq_len))
    m.store.zero_grad()
    loss = _run([m], idx, tgt)
    P = {n: m.store.p(n).detach().clone().requires_grad_(True) for n in m.store.names()}
    ref = ref_loss(cfg, P, idx, tgt)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 1e-5
    for n in m.store.names():
        g = m.store.g(n)
        r = P[n].grad
        err = ((g - r).norm() / (r.norm() + 1e-12)).item()
        assert err < 1e-4, (n, err)


def test_cut_model_is_identical_to_whole():
    cfg = make_config("toy", n_layer=3, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    whole = StageModel(cfg, (0, cfg.n_entries), "cpu", seed=11)
    parts = [StageModel(cfg, (0, 2), "cpu", seed=11), StageModel(cfg, (2, 4), "cpu", seed=11),
             StageModel(cfg, (4, cfg.n_entries), "cpu", seed=11)]
    for p in parts:
        for n in p.store.names():
            assert torch.equal(p.store.p(n), whole.store.p(n)), n
    idx = torch.randint(0, cfg.vocab_size, (2, cfg.seq_len))
    tgt = torch.randint(0, cfg.vocab_size, (2, cfg.seq_len))
    for st in [whole] + parts:
        st.store.zero_grad()
    l1 = _run([whole], idx, tgt)
    l2 = _run(parts, idx, tgt)
    assert l1.item().hex() == l2.item().hex()
    for p in parts:
        for n in p.store.names():
            assert torch.equal(p.store.g(n), whole.store.g(n)), n


def test_fp8_boundary_cpu_roundtrip():
    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=128, n_head=4, seq_len=16,
                      boundary_dtype="fp8_e4m3_b128")
    m = StageModel(cfg, (0, cfg.n_entries), "cpu", seed=5)
    idx = torch.randint(0, cfg.vocab_size, (1, cfg.seq_len))
    tgt = torch.randint(0, cfg.vocab_size, (1, cfg.seq_len))
    m.store.zero_grad()
    loss = _run([m], idx, tgt)
    assert torch.isfinite(loss)
    assert m.store.grad.abs().sum() > 0
