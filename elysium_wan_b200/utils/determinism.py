"""Numeric pins (reference: src/wantrain/runtime/determinism.py:28-139).

The sm_100a kernels are deterministic by construction (no atomics, fixed tile
orders, fixed reduction trees). The CPU plumbing path runs torch ops, which
need the usual pins: deterministic algorithms, no TF32, one intra-op thread,
a fixed cuBLAS workspace config for the rare library call.
"""

from __future__ import annotations

import os
import random

import numpy as np
import torch

PINNED_ENV = {"CUBLAS_WORKSPACE_CONFIG": ":4096:8", "OMP_NUM_THREADS": "1",
              "MKL_NUM_THREADS": "1"}


def pinned_env(base: dict | None = None) -> dict:
    env = dict(base if base is not None else os.environ)
    env.update(PINNED_ENV)
    return env


def setup_determinism(seed: int = 0):
    for k, v in PINNED_ENV.items():
        os.environ.setdefault(k, v)
    random.seed(seed)
    np.random.seed(seed % (2 ** 32))
    torch.manual_seed(seed)
    torch.use_deterministic_algorithms(True, warn_only=True)
    # Deterministic mode NaN-fills every torch.empty; the kernels here write
    # every element they later read, so that fill is pure overhead.
    torch.utils.deterministic.fill_uninitialized_memory = False
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_num_threads(1)


def check_determinism() -> dict:
    return {"threads": torch.get_num_threads(),
            "deterministic": torch.are_deterministic_algorithms_enabled(),
            "tf32": torch.backends.cuda.matmul.allow_tf32}


def float_hex(x: float) -> str:
    return float(x).hex()
