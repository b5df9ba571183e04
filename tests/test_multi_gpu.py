"""Multi-GPU pipeline over NCCL is bit-identical to the single-GPU oracle
running the same sm_100a kernels (needs >= 2 GPUs; skipped otherwise).

Would fail if: NCCL routing between stages, the fp8 boundary payload, the
stage cut or the schedule changed any loss bit against the oracle, or if the
point-to-point communicators deadlocked (bounded by the process-group and
test timeouts).
"""

import pytest
import torch

from elysium_wan_b200.launch.local import run_and_compare
from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.runtime.spec import JobSpec

pytestmark = pytest.mark.gpu


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("stages,boundary", [(2, "fp8_e4m3_b128"), (2, "bf16"), (4, "fp8_e4m3_b128"),
                                             (1, "fp16"), (1, "fp8_e5m2_b128"), (2, "fp16"),
                                             (2, "fp8_e5m2_b128")])
def test_nccl_pipeline_bitwise_vs_oracle(tmp_path, stages, boundary):
    _need(stages)
    cfg = make_config("gpt15b", n_layer=max(4, stages), d_model=512, n_head=4, seq_len=256, vocab_size=4096,
                      boundary_dtype=boundary)
    spec = JobSpec(model=cfg, stages=stages, microbatches=6, mb_size=2, steps=2, device="cuda",
                   backend="nccl", out_dir=str(tmp_path),
                   port_base=29950 + 7 * stages + len(boundary))
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    assert r["compared"] == 12


@pytest.mark.parametrize("widths,sync", [([2], "fused"), ([2], "nccl"), ([1, 2], "fused")])
def test_zero1_wide_stage_bitwise_vs_oracle(tmp_path, widths, sync):
    """ZeRO-1 wide stages: the fused path (dW epilogue scatters into the owners'
    slots over NVLink, AdamW pushes the updated shard to every replica) and the
    NCCL library path both match the oracle's declared fold bit for bit."""
    _need(sum(widths))
    cfg = make_config("gpt15b", n_layer=2, d_model=512, n_head=4, seq_len=256, vocab_size=4096,
                      boundary_dtype="bf16")
    spec = JobSpec(model=cfg, stages=len(widths), stage_widths=widths, microbatches=4, mb_size=2,
                   steps=3, device="cuda", backend="nccl", grad_sync=sync, out_dir=str(tmp_path),
                   port_base=29970 + sum(widths) + len(sync))
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    assert r["compared"] == 12


@pytest.mark.parametrize("stages", [1, 2])
def test_w_pair_bitwise_vs_oracle(tmp_path, stages):
    """Paired weight-gradient folds (one GEMM for microbatches 2k and 2k + 1,
    5 microbatches so the last runs alone) on the GPU kernels: the pipeline
    equals the oracle, which pairs the same way."""
    _need(stages)
    cfg = make_config("gpt15b", n_layer=2, d_model=512, n_head=4, seq_len=256, vocab_size=4096,
                      boundary_dtype="fp8_e4m3_b128")
    spec = JobSpec(model=cfg, stages=stages, microbatches=5, mb_size=2, steps=2, device="cuda",
                   backend="nccl", w_pair=True, out_dir=str(tmp_path), port_base=29990 + stages)
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    assert r["compared"] == 10


def test_gpt2p8b_shape_4x2_zero1_320_losses_bitwise(tmp_path):
    """The 2.8B GPT's layer shape (d 2560, 32 heads of 80, MLP 10240, seq 2048,
    vocab 50257, bf16) at reduced depth as BASELINE's 4 stages x 2 ZeRO-1
    replicas with the fused gradient exchange: 32 microbatches of 2 sequences
    for 10 steps, all 320 losses equal to the single-GPU oracle bit for bit."""
    _need(8)
    cfg = make_config("gpt2_8b", n_layer=4)
    spec = JobSpec(model=cfg, stages=4, stage_widths=[2, 2, 2, 2], microbatches=32, mb_size=2,
                   steps=10, device="cuda", backend="nccl", grad_sync="fused", lr=1e-4,
                   out_dir=str(tmp_path), port_base=29940)
    r = run_and_compare(spec, timeout=900)
    assert r["ok"], r
    assert r["compared"] == 320
