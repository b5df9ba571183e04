"""Hugging Face checkpoints: the validating safetensors reader / writer and
digest, and importers whose models compute what transformers computes.

Would fail if: the reader accepted a header whose offsets do not match its
shapes, the Llama import permuted q / k rows into the wrong rotary order,
a GQA / tied / GPT-2 mapping were wrong, or the engine's Llama block (RMSNorm,
RoPE, GQA, SwiGLU) differed from transformers' LlamaForCausalLM."""

import json
import os
import struct

import pytest
import torch

from elysium_wan_b200.models import hf
from elysium_wan_b200.models.gpt import StageModel

transformers = pytest.importorskip("transformers")


def _logits(model, idx):
    """Engine logits (fp32, CPU): run the stages up to the head's GEMM."""
    from elysium_wan_b200 import ops

    ctx = {}
    h = model.layers[0].forward(idx, ctx)
    for layer in model.layers[1:-1]:
        h = layer.forward(h, {})
    head = model.layers[-1]
    beta = None if head.rms else model.store.p(head.n("ln_f.bias"))
    y, _, _ = ops.layernorm_fwd(h.x, None, model.store.p(head.n("ln_f.weight")), beta,
                                model.cfg.norm_eps)
    return y @ model.store.p(head.out).t()


def _save_hf(m, tmp_path):
    d = tmp_path / "ckpt"
    d.mkdir()
    hf.save_file({k: v for k, v in m.state_dict().items()}, str(d / "model.safetensors"))
    with open(d / "config.json", "w") as fh:
        json.dump(m.config.to_dict(), fh)
    return str(d)


@pytest.mark.parametrize("kv,tied", [(2, False), (4, True)])
def test_llama_import_matches_transformers(tmp_path, kv, tied):
    torch.manual_seed(0)
    c = transformers.LlamaConfig(vocab_size=97, hidden_size=64, intermediate_size=96,
                                 num_hidden_layers=2, num_attention_heads=4,
                                 num_key_value_heads=kv, max_position_embeddings=32,
                                 rms_norm_eps=1e-6, rope_theta=10000.0,
                                 tie_word_embeddings=tied)
    ref = transformers.LlamaForCausalLM(c).eval()
    path = _save_hf(ref, tmp_path)
    cfg, state = hf.import_checkpoint(path, seq_len=16)
    assert cfg.n_kv_head == kv and cfg.tie_embeddings == tied
    m = StageModel(cfg, (0, cfg.n_entries), "cpu", seed=0)
    hf.load_into(m, state)
    idx = torch.randint(0, 97, (2, 16))
    with torch.no_grad():
        want = ref(idx).logits.reshape(32, 97)
    got = _logits(m, idx)
    assert (got - want).abs().max().item() < 1e-4


def test_gpt2_import_matches_transformers(tmp_path):
    torch.manual_seed(1)
    c = transformers.GPT2Config(vocab_size=97, n_positions=32, n_embd=64, n_layer=2, n_head=4)
    ref = transformers.GPT2LMHeadModel(c).eval()
    path = _save_hf(ref, tmp_path)
    cfg, state = hf.import_checkpoint(path, seq_len=16)
    m = StageModel(cfg, (0, cfg.n_entries), "cpu", seed=0)
    hf.load_into(m, state)
    idx = torch.randint(0, 97, (2, 16))
    with torch.no_grad():
        want = ref(idx).logits.reshape(32, 97)
    assert (_logits(m, idx) - want).abs().max().item() < 2e-4


def test_reader_validates_and_digest(tmp_path):
    f = str(tmp_path / "a.safetensors")
    t = {"x": torch.arange(6, dtype=torch.float32).reshape(2, 3), "y": torch.ones(4, dtype=torch.bfloat16)}
    hf.save_file(t, f)
    back = hf.load_state(f)
    assert torch.equal(back["x"], t["x"]) and torch.equal(back["y"], t["y"])
    d1 = hf.checkpoint_digest(f)
    t["x"][0, 0] = 7
    hf.save_file(t, f)
    assert hf.checkpoint_digest(f) != d1
    # a header whose offsets do not match the shape is refused before reading
    bad = str(tmp_path / "bad.safetensors")
    h = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 8]}}).encode()
    with open(bad, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(ValueError):
        hf.read_header(bad)
    with pytest.raises(FileNotFoundError):
        hf.index(str(tmp_path / "empty_dir_that_does_not_exist"))


def test_import_cli_and_training_from_checkpoint(tmp_path):
    """import-hf writes a spec pinned to the checkpoint's digest; a local run
    initialised from it starts from the imported weights and equals the
    oracle bit for bit."""
    from elysium_wan_b200 import cli
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.runtime.spec import JobSpec

    torch.manual_seed(2)
    c = transformers.LlamaConfig(vocab_size=97, hidden_size=64, intermediate_size=96,
                                 num_hidden_layers=2, num_attention_heads=4,
                                 num_key_value_heads=2, max_position_embeddings=32)
    path = _save_hf(transformers.LlamaForCausalLM(c), tmp_path)
    out = str(tmp_path / "spec.json")
    assert cli.main(["import-hf", "--path", path, "--out", out, "--seq-len", "16",
                     "--stages", "2"]) == 0
    spec = JobSpec.load(out)
    assert spec.init_sha256 == hf.checkpoint_digest(path)
    assert spec.pins()["init_sha256"] == spec.init_sha256
    spec.microbatches, spec.mb_size, spec.steps = 2, 2, 2
    spec.out_dir = str(tmp_path / "run")
    spec.port_base = 32000 + os.getpid() % 300 * 7
    spec.schedule_order = None
    spec.mb_owner = None
    r = run_and_compare(spec.finalize(), timeout=240)
    assert r["ok"], r
