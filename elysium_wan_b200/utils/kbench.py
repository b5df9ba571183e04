"""Kernel micro-benchmarks on the model's shapes, timed with CUDA events.

    python -m elysium_wan_b200.utils.kbench [--model gpt15b] [--iters 20]

For each GEMM of a transformer block (forward, B-pass dX, W-pass dW) it times
the tcgen05 kernel and cuBLAS (torch.matmul) on the same operands and prints
TFLOP/s and the fraction of the measured bf16 peak (MEASURED_PEAKS.json).
Inputs are larger than L2 is not guaranteed for every shape, so each timed
iteration is preceded by a 256 MiB L2 flush.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from elysium_wan_b200 import ops

SHAPES = {
    "gpt15b": dict(T=2048, d=5120, f=20480),
    "gpt0_6b": dict(T=8192, d=1536, f=6144),
    "gpt2_8b": dict(T=4096, d=2560, f=10240),
    "gpt25b": dict(T=2048, d=5888, f=23552),
}


def _peak():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f).get("bf16_tflops", 1590.0)
    except OSError:
        return 1590.0


def time_fn(fn, iters, flush):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gpt15b", choices=sorted(SHAPES))
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    s = SHAPES[a.model]
    T, d, f = s["T"], s["d"], s["f"]
    dev = torch.device("cuda:0")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    peak = _peak()
    rows = []
    for name, N, K in [("qkv", 3 * d, d), ("proj", d, d), ("fc1", f, d), ("fc2", d, f)]:
        x = (torch.randn(T, K, device=dev) * 0.5).to(torch.bfloat16)
        w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
        dy = (torch.randn(T, N, device=dev) * 0.1).to(torch.bfloat16)
        out = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
        dx = torch.empty(T, K, dtype=torch.bfloat16, device=dev)
        gw = torch.zeros(N, K, device=dev)
        flops = 2.0 * T * N * K
        cases = {
            "fwd": (lambda: ops.gemm(x, w, out, ops.EPI_BF16), lambda: torch.matmul(x, w.t())),
            "dx": (lambda: ops.gemm(dy, w, dx, ops.EPI_BF16, b_mn=True), lambda: torch.matmul(dy, w)),
            "dw": (lambda: ops.gemm(dy, x, gw, ops.EPI_ACC_F32, a_mn=True, b_mn=True, beta=1.0),
                   lambda: torch.matmul(dy.t(), x)),
        }
        for kind, (ours, lib) in cases.items():
            t_o = time_fn(ours, a.iters, flush)
            t_l = time_fn(lib, a.iters, flush)
            r = dict(gemm=name, kind=kind, M=T if kind != "dw" else N, N=N if kind != "dw" else K,
                     K=K if kind != "dw" else T, ms=round(t_o, 4), cublas_ms=round(t_l, 4),
                     tflops=round(flops / t_o / 1e9, 1), cublas_tflops=round(flops / t_l / 1e9, 1),
                     frac_of_measured=round(flops / t_o / 1e9 / peak, 3))
            rows.append(r)
            print(json.dumps(r), flush=True)
    if a.json:
        with open(a.json, "w") as fh:
            json.dump(rows, fh, indent=1)


if __name__ == "__main__":
    main()
