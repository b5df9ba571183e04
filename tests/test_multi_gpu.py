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


@pytest.mark.parametrize("stages,boundary", [(2, "fp8_e4m3_b128"), (2, "bf16"), (4, "fp8_e4m3_b128")])
def test_nccl_pipeline_bitwise_vs_oracle(tmp_path, stages, boundary):
    _need(stages)
    cfg = make_config("gpt15b", n_layer=max(4, stages), d_model=512, n_head=4, seq_len=256, vocab_size=4096,
                      boundary_dtype=boundary)
    spec = JobSpec(model=cfg, stages=stages, microbatches=6, mb_size=2, steps=2, device="cuda",
                   backend="nccl", out_dir=str(tmp_path), port_base=29950 + stages)
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    assert r["compared"] == 12
