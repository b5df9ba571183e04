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
    if models[0].cfg.tie_embeddings:  # the step's tied fold (engine: before the optimizer)
        models[0].fold_tied(models[-1].store.tied_grad if len(models) > 1 else None)
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


def _general_check(cfg, seed=3, tol=2e-4, B=2):
    from ._ref_general import ref_loss_general

    torch.manual_seed(0)
    m = StageModel(cfg, (0, cfg.n_entries), "cpu", seed=seed)
    idx = torch.randint(0, cfg.vocab_size, (B, cfg.seq_len))
    tgt = torch.randint(0, cfg.vocab_size, (B, cfg.seq_len))
    m.store.zero_grad()
    loss = _run([m], idx, tgt)
    P = {n: m.store.p(n).detach().clone().requires_grad_(True) for n in m.store.names()}
    ce, aux = ref_loss_general(cfg, P, idx, tgt)
    (ce + aux).backward()
    assert abs(loss.item() - ce.item()) < 1e-5
    for n in m.store.names():
        g, r = m.store.g(n), P[n].grad
        if r is None:
            r = torch.zeros_like(g)
        err = ((g - r).norm() / (r.norm() + 1e-12)).item()
        assert err < tol or (g - r).abs().max().item() < 1e-7, (n, err)
    return m


def test_llama_block_matches_autograd():
    """RMSNorm, q / kv grouped-query attention with RoPE, SwiGLU, no bias."""
    cfg = make_config("llama_tiny", n_layer=2, vocab_size=97, d_model=64, n_head=4, n_kv_head=2,
                      seq_len=16)
    m = _general_check(cfg)
    assert "1.q.weight" in m.store.names() and "1.mlp.gate.weight" in m.store.names()
    assert "0.pos.weight" not in m.store.names()


def test_general_block_variants_match_autograd():
    """LayerNorm + GELU + learned positions with biases under the general
    names, full multi-head rope, tied embeddings."""
    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                      d_ff=96)
    m = _general_check(cfg)
    assert "1.mlp.fc1.weight" in m.store.names()
    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                      norm="rmsnorm", pos="rope", mlp="swiglu", bias=True, tie_embeddings=True)
    m = _general_check(cfg)
    assert "3.out.weight" not in m.store.names()


def test_moe_block_matches_autograd():
    cfg = make_config("moe_tiny", n_layer=2, vocab_size=97, d_model=64, n_head=4, n_kv_head=2,
                      seq_len=16, moe_experts=4, moe_top_k=2, moe_d_ff=32, moe_shared_d_ff=32,
                      moe_layers=[1])
    m = _general_check(cfg)
    recs = m.take_moe_records()
    assert [r.layer for r in recs] == [2] and int(recs[0].counts.sum()) == 2 * 16 * 2


def test_moe_variants_match_autograd():
    base = dict(n_layer=1, vocab_size=97, d_model=64, n_head=4, n_kv_head=2, seq_len=16,
                moe_experts=4, moe_d_ff=32, moe_shared_d_ff=0)
    for extra in (dict(moe_score="sigmoid", moe_norm=True, moe_norm_eps=1e-6, moe_top_k=2,
                       moe_lbl_scope="sequence"),
                  dict(moe_score="softmax_k", moe_top_k=2, moe_router_bias=True,
                       moe_select="logit"),
                  dict(moe_apply="input", moe_top_k=1, moe_shared_d_ff=32,
                       moe_shared_gate="none"),
                  dict(moe_groups=2, moe_topk_groups=1, moe_top_k=2, moe_scale=2.0),
                  dict(moe_expert="swiglu_clamped", moe_top_k=2, moe_limit=0.5)):
        cfg = make_config("moe_tiny", **{**base, **extra})
        _general_check(cfg)


def test_moe_bias_update_moves_by_gamma():
    cfg = make_config("moe_tiny", n_layer=1, moe_experts=4, moe_top_k=1, moe_bias_rate=0.1,
                      moe_select="score_bias")
    m = StageModel(cfg, (0, cfg.n_entries), "cpu", seed=1)
    blk = m.moe_blocks()[0]
    m.moe_bias_update({1: torch.tensor([1, 3, 2, 2], dtype=torch.int64)}, 8)
    # T k = 8, E c = 4, 12, 8, 8 -> signs +, -, 0, 0
    assert blk.sel_bias.tolist() == [0.1, -0.1, 0.0, 0.0] or \
        torch.allclose(blk.sel_bias, torch.tensor([0.1, -0.1, 0.0, 0.0]))
    import pytest

    with pytest.raises(ValueError):
        m.moe_bias_update({1: torch.tensor([1, 1, 1, 1], dtype=torch.int64)}, 8)


def test_lora_adapters_match_autograd():
    """LoRA: base frozen (no gradient, no optimizer state), adapters trained;
    the forward runs W + (alpha/r) B A and the adapter gradients equal
    autograd through that merge."""
    import dataclasses

    from ._ref_general import ref_loss_general

    for targets in ("attn", "all"):
        cfg = make_config("llama_tiny", n_layer=2, vocab_size=97, d_model=64, n_head=4,
                          n_kv_head=2, seq_len=16, lora_rank=4, lora_alpha=8.0,
                          lora_targets=targets)
        m = StageModel(cfg, (0, cfg.n_entries), "cpu", seed=3)
        st = m.store
        torch.manual_seed(1)
        for n in st.names():  # B starts at zero; give it values so both paths are exercised
            if n.endswith(".B.weight"):
                st.p(n).normal_(0, 0.05)
        st.sync_work()
        m.after_step()
        assert st.nt < st.numel and st.grad.numel() == st.nt
        assert st.g("1.q.weight") is None and st.g("1.q.A.weight") is not None
        idx = torch.randint(0, 97, (2, 16))
        tgt = torch.randint(0, 97, (2, 16))
        st.zero_grad()
        loss = _run([m], idx, tgt)
        P = {n: st.p(n).detach().clone().requires_grad_(n.endswith((".A.weight", ".B.weight")))
             for n in st.names()}
        eff = dict(P)
        s = cfg.lora_alpha / cfg.lora_rank
        for w, a, b in m.adapters:
            eff[w] = P[w] + s * (P[b] @ P[a])
        base_cfg = dataclasses.replace(cfg, lora_rank=0)
        ce, _ = ref_loss_general(base_cfg, eff, idx, tgt)
        ce.backward()
        assert abs(loss.item() - ce.item()) < 1e-5
        for n in st.names():
            if n.endswith((".A.weight", ".B.weight")):
                g, r = st.g(n), P[n].grad
                err = ((g - r).norm() / (r.norm() + 1e-12)).item()
                assert err < 2e-4, (targets, n, err)
        if targets == "all":
            assert "3.out.A.weight" in st.names()
