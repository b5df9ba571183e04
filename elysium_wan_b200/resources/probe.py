"""Capability probe of a worker (reference: src/wantrain/resources/probe.py).

Reports device class, memory, compute capability, SM count and (when
benchmarking) a measured bf16 GEMM rate and host-to-device bandwidth. On a
B200 the GEMM rate comes from this package's own tcgen05 kernel.
"""

from __future__ import annotations

import os
import platform
import time


def device_class(name: str) -> str:
    n = name.lower()
    for key in ("b200", "h100", "a100", "l40", "4090", "3090"):
        if key in n:
            return key
    return "cpu" if not n else n.split()[-1]


def measure(device: str = "cpu", bench: bool = False) -> dict:
    out = {"device": device, "hostname": platform.node(), "cpus": os.cpu_count()}
    try:
        import psutil

        out["host_mem_gb"] = round(psutil.virtual_memory().total / 2 ** 30, 1)
    except Exception:
        pass
    if not device.startswith("cuda"):
        out.update(device_class="cpu", vram_gb=out.get("host_mem_gb"), cc=None)
        return out
    import torch

    d = torch.device(device)
    p = torch.cuda.get_device_properties(d)
    out.update(device_name=p.name, device_class=device_class(p.name),
               vram_gb=round(p.total_memory / 2 ** 30, 1), cc=f"{p.major}.{p.minor}",
               sms=p.multi_processor_count)
    if bench:
        out["tflops_bf16"] = round(bench_tflops(d), 1)
        out["h2d_gbs"] = round(bench_h2d(d), 1)
    return out


def bench_tflops(d, n: int = 8192, iters: int = 10) -> float:
    import torch

    from elysium_wan_b200 import ops

    a = torch.randn(n, n, device=d).to(torch.bfloat16)
    b = torch.randn(n, n, device=d).to(torch.bfloat16)
    c = torch.empty(n, n, device=d, dtype=torch.bfloat16)
    for _ in range(3):
        ops.gemm(a, b, c)
    torch.cuda.synchronize(d)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        ops.gemm(a, b, c)
    e1.record()
    torch.cuda.synchronize(d)
    return 2 * n ** 3 * iters / (e0.elapsed_time(e1) / 1e3) / 1e12


def bench_h2d(d, nbytes: int = 1 << 30) -> float:
    import torch

    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    g = torch.empty(nbytes, dtype=torch.uint8, device=d)
    g.copy_(h, non_blocking=True)
    torch.cuda.synchronize(d)
    t = time.perf_counter()
    g.copy_(h, non_blocking=True)
    torch.cuda.synchronize(d)
    return nbytes / (time.perf_counter() - t) / 1e9
