"""Kernel micro-benchmarks on the model's shapes, timed with CUDA events.

    python -m elysium_wan_b200.utils.kbench [--model gpt15b] [--iters 20] [--attn]

For each GEMM of a transformer block (forward, B-pass dX, W-pass dW) it times
the tcgen05 kernel and cuBLAS (torch.matmul) on the same operands and prints
TFLOP/s and the fraction of the measured bf16 peak (MEASURED_PEAKS.json).
With --attn it times causal attention forward and backward on one
microbatch of the model (batch 1, its heads and head size) against PyTorch's
scaled_dot_product_attention pinned to the flash backend (the reference's op,
src/wantrain/model/gpt.py:374-386) on the same q, k, v.
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


ATTN = {"gpt15b": (40, 128), "gpt0_6b": (12, 128), "gpt2_8b": (32, 80), "gpt25b": (46, 128)}


def attn_rows(model: str, iters: int, flush, peak: float) -> list:
    """Our causal attention fwd / bwd vs SDPA (flash) on one 2048-token sequence."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    H, hd = ATTN[model]
    S, B = 2048, 1
    dev = flush.device
    qkv = (torch.randn(B * S, 3 * H * hd, device=dev) * 0.5).to(torch.bfloat16)
    dout = (torch.randn(B * S, H * hd, device=dev) * 0.1).to(torch.bfloat16)
    o, lse = ops.attention_fwd(qkv, B, S, H, hd)
    q, k, v = [t.view(B, S, H, hd).transpose(1, 2).contiguous().requires_grad_(True)
               for t in qkv.split(H * hd, dim=1)]
    do4 = dout.view(B, S, H, hd).transpose(1, 2).contiguous()
    # causal: half the S x S score matrix; fwd 2 GEMMs, bwd 5 (incl. the recomputed S)
    f_fwd = 2 * 2.0 * B * H * S * S * hd / 2
    f_bwd = 5 * 2.0 * B * H * S * S * hd / 2

    def sdpa_fwd():
        with sdpa_kernel(SDPBackend.FLASH_ATTENTION):
            return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)

    y = sdpa_fwd()

    def sdpa_bwd():
        torch.autograd.grad(y, (q, k, v), do4, retain_graph=True)

    rows = []
    for kind, ours, lib, flops in (
            ("attn_fwd", lambda: ops.attention_fwd(qkv, B, S, H, hd), sdpa_fwd, f_fwd),
            ("attn_bwd", lambda: ops.attention_bwd(qkv, o, dout, lse, B, S, H, hd), sdpa_bwd, f_bwd)):
        t_o = time_fn(ours, iters, flush)
        t_l = time_fn(lib, iters, flush)
        r = dict(op=kind, B=B, S=S, H=H, hd=hd, ms=round(t_o, 4), sdpa_flash_ms=round(t_l, 4),
                 tflops=round(flops / t_o / 1e9, 1), sdpa_tflops=round(flops / t_l / 1e9, 1),
                 frac_of_measured=round(flops / t_o / 1e9 / peak, 3),
                 speedup_vs_sdpa=round(t_l / t_o, 3))
        rows.append(r)
        print(json.dumps(r), flush=True)
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gpt15b", choices=sorted(SHAPES))
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", default=None)
    ap.add_argument("--attn", action="store_true", help="attention vs SDPA flash instead of GEMMs")
    a = ap.parse_args(argv)
    if a.attn:
        dev = torch.device("cuda:0")
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        rows = attn_rows(a.model, a.iters, flush, _peak())
        if a.json:
            with open(a.json, "w") as fh:
                json.dump(rows, fh, indent=1)
        return
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
