"""One tiny forward + backward + optimizer step of the flagship GPT on cuda:0,
through the sm_100a kernels (the graft entry's smoke())."""

from __future__ import annotations

import torch


def run_smoke(device: str = "cuda:0") -> dict:
    from elysium_wan_b200 import ops
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.engine import StageEngine
    from elysium_wan_b200.runtime.spec import JobSpec

    ops.ext()
    cfg = make_config("gpt15b", n_layer=2, d_model=256, n_head=2, seq_len=256, vocab_size=1024)
    spec = JobSpec(model=cfg, stages=1, microbatches=2, mb_size=1, steps=1, device=device,
                   backend="nccl").finalize()
    eng = StageEngine(spec, 0, 0, None, device)
    n0 = ops.launch_count()
    res = eng.run_step(0)
    torch.cuda.synchronize()
    launches = ops.launch_count() - n0
    status = ops.ext().status_read_clear()
    losses = [v for _, v in res]
    if status != 0 or not all(torch.isfinite(torch.tensor(losses))):
        raise RuntimeError(f"smoke failed: status={status} losses={losses}")
    out = {"losses": losses, "kernel_launches": launches}
    print(out, flush=True)
    return out


if __name__ == "__main__":
    run_smoke()
