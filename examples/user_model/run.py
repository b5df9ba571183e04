"""Train a user model (arch "user") as a 2-stage pipeline on this machine and
compare every loss with the single-device oracle:

    python examples/user_model/run.py [--stages 2 --steps 3]

The model file is pinned by its sha256 in the spec, so every stage provably
builds the same code; the spec's finalize checks the layer contract."""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def main(argv=None) -> int:
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    ap = argparse.ArgumentParser()
    ap.add_argument("--stages", type=int, default=2)
    ap.add_argument("--steps", type=int, default=3)
    a = ap.parse_args(argv)
    src = os.path.join(HERE, "model.py")
    sha = hashlib.sha256(open(src, "rb").read()).hexdigest()
    cfg = make_config("toy", n_layer=4, vocab_size=256, d_model=64, n_head=4, seq_len=32,
                      arch="user", user_model=src, user_model_sha256=sha)
    spec = JobSpec(model=cfg, stages=a.stages, microbatches=4, mb_size=2, steps=a.steps,
                   backend="gloo", out_dir=tempfile.mkdtemp(prefix="user_model_"))
    r = run_and_compare(spec, timeout=300)
    print(r)
    return 0 if r["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
