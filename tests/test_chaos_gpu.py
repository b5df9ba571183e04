"""A GPU rank that leaves between steps: the coordinator convicts its slot,
heals onto a spare, and every stage relaunches on fresh NCCL communicators
from the newest common checkpoint wave; the losses stay bitwise equal to the
single-GPU oracle.

The failure is made on the host: one worker's stage process exits right
after a step (EWB_TEST_LEAVE_AFTER_STEP), with its kernels and collectives
complete; the surviving rank is stopped by the coordinator's abort. NVLS is
off for NCCL (a rank that dies bound to an NVLink multicast object has
faulted other ranks' GPUs on this pool) and the pipeline uses NCCL point-to-
point only. Would fail if conviction, the heal, the fresh process groups or
the resume changed any loss bit.
"""

import os

import pytest
import torch

from elysium_wan_b200.control.coordinator import Job
from elysium_wan_b200.launch.cluster import LocalCluster
from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.runtime.spec import JobSpec
from elysium_wan_b200.validation.compare import compare
from elysium_wan_b200.validation.reference import run_baseline

pytestmark = pytest.mark.gpu


@pytest.mark.timeout(600)
def test_rank_leaving_between_steps_heals_onto_fresh_nccl_groups(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = make_config("gpt15b", n_layer=2, d_model=512, n_head=4, seq_len=256, vocab_size=4096,
                      boundary_dtype="bf16")
    spec = JobSpec(model=cfg, stages=2, microbatches=4, mb_size=2, steps=8, device="cuda",
                   backend="nccl", ckpt_every=2, tag="leave", lr=1e-4)
    base = {"NCCL_NVLS_ENABLE": "0", "TORCH_SYMM_MEM_DISABLE_MULTICAST": "1"}
    # workers register in order: 0 (GPU 0) and 1 (GPU 1) hold the two slots,
    # 2 (GPU 1) is the spare; worker 1's stage leaves after step 4, and the
    # spare takes its slot on the same GPU
    env = [dict(base), dict(base, EWB_TEST_LEAVE_AFTER_STEP="4"), dict(base)]
    args = [["--device", "cuda:0"], ["--device", "cuda:1"], ["--device", "cuda:1"]]
    cl = LocalCluster(str(tmp_path / "cl"), ["a"] * 3, device="cuda", worker_env=env,
                      worker_args=args, stage_timeout_s=60.0, sequential=True)
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert res.ok, res.why
    assert res.heals == 1 and res.attempts == 2, (res.heals, res.attempts)
    ref = JobSpec.from_dict(spec.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 32, r
