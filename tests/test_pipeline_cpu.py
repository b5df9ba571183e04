"""Multi-process pipelines over gloo on CPU are bit-identical to the
single-device oracle (losses compared as float.hex()).

Would fail if: a stage routed a boundary to the wrong peer, the schedule
reordered a fold, the ZeRO-1 reduce-scatter / all-gather or the declared
fold tree drifted from the oracle, or recompute changed a value.
"""

import os

import pytest
import torch

from elysium_wan_b200.launch.local import run_and_compare
from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.runtime.spec import JobSpec


def _cfg(**kw):
    return make_config("toy", n_layer=4, vocab_size=97, d_model=128, n_head=4, seq_len=16, **kw)


CASES = {
    "chain2": dict(stages=2),
    # AdamW moments in host memory (streamed through the device on a GPU)
    "host_adamw_wide_1_2": dict(stages=2, stage_widths=[1, 2], optimizer="adamw-host"),
    # Width-1 stages fold the W of microbatches 2k and 2k + 1 with one GEMM;
    # 5 microbatches leave the last one unpaired; the wide stage does not pair.
    "w_pair_chain3": dict(stages=3, w_pair=True, microbatches=5),
    "w_pair_wide_1_2": dict(stages=2, stage_widths=[1, 2], w_pair=True),
    "chain3_fp8_recompute": dict(stages=3, recompute=True, model_kw=dict(boundary_dtype="fp8_e4m3_b128")),
    # The other boundary rungs: fp16 (host path rounds to fp16 at every entry
    # boundary) and block-scaled e5m2, the latter on a wide stage.
    "chain2_fp16": dict(stages=2, model_kw=dict(boundary_dtype="fp16")),
    "e5m2_wide_1_2": dict(stages=2, stage_widths=[1, 2], model_kw=dict(boundary_dtype="fp8_e5m2_b128")),
    "wide_2_1": dict(stages=2, stage_widths=[2, 1]),
    # Uneven peers: each peer of the wide stages runs its own lane order
    # (solved per peer, chosen because the slot simulation finds it faster).
    "lanes_2_2": dict(stages=2, stage_widths=[2, 2], peer_weights=[[1.0, 2.0], [1.0, 2.0]],
                      microbatches=6, zb_mem_mode="2p"),
    "wide_1_2": dict(stages=2, stage_widths=[1, 2]),
    # Llama block (RMSNorm, GQA, RoPE, SwiGLU, no bias) cut over 2 stages.
    "llama_chain2": dict(stages=2, model_kw=dict(norm="rmsnorm", mlp="swiglu", pos="rope",
                                                 bias=False, n_kv_head=2)),
    # Pieces (FSDP-like): the wide stage holds each matrix's fp32 master and
    # moments once, gathers the working copy; same bits as ZeRO-1.
    "pieces_1_2": dict(stages=2, stage_widths=[1, 2], shard="pieces"),
    "pieces_3_llama": dict(stages=2, stage_widths=[3, 1], shard="pieces",
                           model_kw=dict(norm="rmsnorm", mlp="swiglu", pos="rope", bias=False,
                                         n_kv_head=2)),
    # LoRA over the Llama block: frozen base, adapters trained, wide stage.
    "lora_wide_1_2": dict(stages=2, stage_widths=[1, 2],
                          model_kw=dict(norm="rmsnorm", mlp="swiglu", pos="rope", bias=False,
                                        n_kv_head=2, lora_rank=8, lora_targets="attn_mlp")),
    # Pieces under LoRA (the frozen base held whole by every replica, the
    # adapters replicated for the merge) and under MoE (the fp32 router
    # replicated, the experts sharded).
    "pieces_lora_1_2": dict(stages=2, stage_widths=[1, 2], shard="pieces",
                            model_kw=dict(norm="rmsnorm", mlp="swiglu", pos="rope", bias=False,
                                          n_kv_head=2, lora_rank=8, lora_targets="attn")),
    "pieces_moe_2_1": dict(stages=2, stage_widths=[2, 1], shard="pieces",
                           model_kw=dict(norm="rmsnorm", mlp="swiglu", pos="rope", bias=False,
                                         moe_experts=4, moe_top_k=2, moe_d_ff=64,
                                         moe_shared_d_ff=64, moe_select="score_bias",
                                         moe_bias_rate=0.01, moe_lbl_coef=0.01)),
    # MoE block with a selection bias that moves every step, recompute, a
    # wide second stage (counts summed over its replicas).
    "moe_wide_1_2": dict(stages=2, stage_widths=[1, 2], recompute=True,
                         model_kw=dict(norm="rmsnorm", mlp="swiglu", pos="rope", bias=False,
                                       moe_experts=4, moe_top_k=2, moe_d_ff=64,
                                       moe_shared_d_ff=64, moe_select="score_bias",
                                       moe_bias_rate=0.01, moe_lbl_coef=0.01, moe_z_coef=0.001)),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_pipeline_bitwise_vs_oracle(tmp_path, name):
    kw = dict(CASES[name])
    mk = kw.pop("model_kw", {})
    port = 29700 + 17 * sorted(CASES).index(name) + (os.getpid() % 50) * 3
    m = kw.pop("microbatches", 4)
    spec = JobSpec(model=_cfg(**mk), microbatches=m, mb_size=2, steps=2, out_dir=str(tmp_path),
                   port_base=port, backend="gloo", **kw)
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    assert r["compared"] == 2 * m


def test_w_pair_changes_the_fold_only_as_declared():
    """Pairing is a declared recipe: the first forward is the same, the folded
    gradients (another fp32 sum order) and so the updated weights are not,
    and it is a pin."""
    from elysium_wan_b200.validation.reference import Oracle

    base = dict(model=_cfg(), stages=2, microbatches=4, mb_size=2, steps=2)
    a = JobSpec(**base).finalize()
    b = JobSpec(**base, w_pair=True).finalize()
    oa, ob = Oracle(a), Oracle(b)
    assert [v.hex() for _, v in oa.step(0)] == [v.hex() for _, v in ob.step(0)]
    assert any(not torch.equal(x.store.master, y.store.master)
               for x, y in zip(oa.stages, ob.stages))
    assert "w_pair" in b.pins() and "w_pair" not in a.pins()


def test_tied_embeddings_across_a_cut_equal_one_stage(tmp_path):
    """A tied table split from its head by a cut (relay copy on the last
    stage, head gradient sent to stage 0, updated table sent back) gives the
    same losses as the single-device oracle, and the oracle of a 3-stage cut
    equals the oracle of one stage: the tied fold does not depend on the cut."""
    from elysium_wan_b200.validation.reference import Oracle

    mk = dict(norm="rmsnorm", mlp="swiglu", pos="rope", bias=False, tie_embeddings=True)
    port = 34000 + (os.getpid() % 300) * 9
    spec = JobSpec(model=_cfg(**mk), stages=3, microbatches=4, mb_size=2, steps=2,
                   out_dir=str(tmp_path), port_base=port, backend="gloo")
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    one = JobSpec(model=_cfg(**mk), stages=1, microbatches=4, mb_size=2, steps=2,
                  out_dir=str(tmp_path / "one")).finalize()
    o1, o3 = Oracle(one), Oracle(spec)
    for step in range(2):
        a = [v.hex() for _, v in o1.step(step)]
        b = [v.hex() for _, v in o3.step(step)]
        assert a == b


def test_pieces_layout_holds_one_range_and_resumes(tmp_path):
    """A pieces replica holds the non-matrix tensors and 1/w of the matrices in
    fp32; a run checkpointed and resumed in the pieces layout continues the
    uninterrupted run bit for bit."""
    import json

    from elysium_wan_b200.launch.local import run_local
    from elysium_wan_b200.models.gpt import StageModel

    cfg = _cfg()
    full = StageModel(cfg, (0, 3), "cpu", seed=1)
    parts = [StageModel(cfg, (0, 3), "cpu", seed=1, shard=(k, 3)) for k in range(3)]
    st = parts[0].store
    assert st.master.numel() < full.store.master.numel() / 2
    with pytest.raises(KeyError):
        parts[0].store.p("2.fc2.weight")  # a matrix held by another replica
    for k, p in enumerate(parts):  # every replica's working copy is the full model
        assert torch.equal(p.store.w("1.qkv.weight"), full.store.w("1.qkv.weight"))
    port = 35000 + (os.getpid() % 300) * 11

    def spec(steps, out, resume=False, dp=0):
        return JobSpec(model=cfg, stages=2, stage_widths=[2, 1], shard="pieces", microbatches=4,
                       mb_size=2, steps=steps, out_dir=str(out), ckpt_every=1, resume=resume,
                       port_base=port + dp, backend="gloo").finalize()

    a = run_local(spec(3, tmp_path / "a"), timeout=300)
    run_local(spec(2, tmp_path / "b", dp=3), timeout=300)
    b = run_local(spec(3, tmp_path / "b", resume=True, dp=6), timeout=300)
    with open(a) as f:
        la = {(r["step"], r["mb"]): r["loss_hex"] for r in json.load(f)["losses"]}
    with open(b) as f:
        lb = {(r["step"], r["mb"]): r["loss_hex"] for r in json.load(f)["losses"]}
    assert all(lb[k] == v for k, v in la.items() if k[0] == 2)


def _user_cfg(n_layer=4):
    import hashlib

    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "data", "user_mlp_model.py")
    sha = hashlib.sha256(open(src, "rb").read()).hexdigest()
    return make_config("toy", n_layer=n_layer, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                       arch="user", user_model=src, user_model_sha256=sha)


@pytest.mark.parametrize("stages,widths,shard", [(2, None, "zero1"), (3, [1, 2, 1], "zero1"),
                                                (2, [2, 1], "pieces")])
def test_user_model_pipeline_bitwise_vs_oracle(tmp_path, stages, widths, shard):
    """arch "user": the operator's own flat module list (sha256-pinned source)
    cut over stages, a wide stage among them (ZeRO-1, or pieces: every
    replica keeps the fp32 masters the module computes on), equals the oracle
    bit for bit."""
    port = 35500 + stages * 13 + 5 * (shard == "pieces") + (os.getpid() % 200) * 7
    kw = {"stage_widths": widths, "shard": shard} if widths else {}
    spec = JobSpec(model=_user_cfg(), stages=stages, microbatches=4, mb_size=2, steps=2,
                   out_dir=str(tmp_path), port_base=port, backend="gloo", **kw)
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    assert r["compared"] == 8


def test_user_model_source_is_pinned(tmp_path):
    from elysium_wan_b200.models.gpt import StageModel

    cfg = _user_cfg()
    bad = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                      arch="user", user_model=cfg.user_model, user_model_sha256="0" * 64)
    with pytest.raises(ValueError, match="does not match"):
        StageModel(bad, (0, bad.n_entries), "cpu", 1)
    wrong_depth = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                              arch="user", user_model=cfg.user_model)
    m = StageModel(wrong_depth, (0, 2), "cpu", 1)  # no sha pinned: accepted, builds 6 entries
    assert len(m.layers) == 2


def test_user_model_contract_refuses_a_stateful_layer(tmp_path):
    src = tmp_path / "bad_model.py"
    src.write_text(
        "import torch\nfrom torch import nn\n"
        "class E(nn.Module):\n"
        "    def __init__(s, c):\n        super().__init__(); s.t = nn.Embedding(c.vocab_size, c.d_model)\n"
        "    def forward(s, i):\n        return s.t(i)\n"
        "class Noisy(nn.Module):\n"
        "    def __init__(s, c):\n        super().__init__(); s.l = nn.Linear(c.d_model, c.d_model); s.n = 0\n"
        "    def forward(s, x):\n        s.n += 1\n        return s.l(x) * s.n\n"
        "class H(nn.Module):\n"
        "    def __init__(s, c):\n        super().__init__(); s.o = nn.Linear(c.d_model, c.vocab_size)\n"
        "    def forward(s, x):\n        return s.o(x)\n"
        "def build(c):\n    return [E(c), Noisy(c), H(c)]\n")
    cfg = make_config("toy", n_layer=1, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                      arch="user", user_model=str(src))
    with pytest.raises(ValueError, match="contract"):
        JobSpec(model=cfg, stages=1, microbatches=2, mb_size=1).finalize()


@pytest.mark.parametrize("shard", ["zero1", "pieces"])
def test_final_training_state_is_byte_identical_to_the_oracle(tmp_path, shard):
    """Beyond the losses: every fp32 master weight, AdamW moment and the step
    count of the pipeline's final waves (read back through the logical form)
    hash to the oracle's manifest."""
    import json

    from elysium_wan_b200.validation.state import diff_manifests, distributed_manifest

    port = 36200 + 31 * (shard == "pieces") + (os.getpid() % 200) * 7
    spec = JobSpec(model=_cfg(), stages=2, stage_widths=[1, 2], shard=shard, microbatches=4,
                   mb_size=2, steps=2, ckpt_every=2, out_dir=str(tmp_path), port_base=port,
                   backend="gloo")
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    spec.finalize()
    got = distributed_manifest(spec, 2)
    with open(tmp_path / "reference_state.json") as f:
        ref = json.load(f)
    assert diff_manifests(ref, got) == []
    assert len(got["params"]) == len(ref["params"]) > 10
    assert all("exp_avg" in e for e in got["params"].values())
    assert got["losses"] == {k: v for k, v in ref["losses"].items() if k.startswith(("0:", "1:"))}
