"""The fused ZeRO-1 exchange kernels against their NVLink roofline and against
the NCCL library path they replace, one process per GPU.

    python -m torch.distributed.run --nnodes 1 --nproc-per-node 2 \\
        --master-addr 127.0.0.1 --master-port 29655 -m elysium_wan_b200.utils.peerbench

Cases at the fc1 shape of the 15.8B layer (dW [20480 x 5120] from 2048 tokens):

* fold_local: the dW GEMM folding into the local fp32 partial (no exchange);
* fold_peer: the same GEMM with the kEpiAccF32Peer epilogue, which stores
  local partial + tile straight into the owners' slots over NVLink;
* fold_nccl: the local fold followed by an NCCL reduce-scatter of the partial
  (the library path);
* push_fused: zero1_adamw_push over this rank's shard (AdamW on the owner,
  fp32 master and bf16 working copy stored into every replica);
* push_nccl: AdamW on the shard, then NCCL all-gathers of the fp32 master
  and the bf16 working copy.

Each figure is the max over ranks of CUDA-event time per launch (after
warm-up, a barrier and a synchronize on both sides). Roofline of a fused
case: the slower of its FLOPs at the measured bf16 peak and its NVLink bytes
per rank at the measured 770 GB/s peer-copy rate.
"""

from __future__ import annotations

import datetime
import json
import os

import torch
import torch.distributed as dist

from elysium_wan_b200 import ops
from elysium_wan_b200.parallel.fused import _symm
from elysium_wan_b200.parallel.zero1 import shard_bounds

PEER_GBS = 770.0  # measured peer-copy rate per direction on this pool's B200s


def _peak_tflops() -> float:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def _time(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(iters: int = 10) -> None:
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    rank, w = dist.get_rank(), dist.get_world_size()
    group = dist.group.WORLD
    dev = torch.device("cuda", local)
    torch.manual_seed(rank)
    T, F, D = 2048, 20480, 5120
    n = F * D
    dy = (torch.randn(T, F, device=dev) * 0.1).to(torch.bfloat16)
    x = (torch.randn(T, D, device=dev) * 0.5).to(torch.bfloat16)
    grad = torch.zeros(F, D, device=dev)
    bounds = shard_bounds(n, w)
    lo_list = [b[0] for b in bounds] + [n]
    S = max(h - l for l, h in bounds)
    lo, hi = bounds[rank]
    slots, h_slots = _symm(w * S, torch.float32, dev, group)
    slot_ptrs = list(h_slots.buffer_ptrs)
    master, h_master = _symm(n, torch.float32, dev, group)
    work, h_work = _symm(n, torch.bfloat16, dev, group)
    master.normal_()
    work.copy_(master)
    m = torch.zeros(hi - lo, device=dev)
    v = torch.zeros_like(m)
    g = torch.randn(hi - lo, device=dev) * 1e-3
    shard_out = torch.empty(S, device=dev)
    ext = ops.ext()
    peak = _peak_tflops()
    flops = 2.0 * T * F * D
    fold_bytes = n * 4 * (w - 1) / w  # each rank's partial leaves for the other owners
    push_bytes = (hi - lo) * 6 * (w - 1)  # fp32 master + bf16 copy to every other replica
    steps = [0]

    def push_fused():
        steps[0] += 1
        ext.zero1_adamw_push(master, m, v, g, lo, hi - lo, list(h_master.buffer_ptrs),
                             list(h_work.buffer_ptrs), 1e-4, 0.9, 0.95, 1e-8, 0.0, steps[0])

    flat_m = master
    flat_w = work

    def push_nccl():
        steps[0] += 1
        ops.adamw(flat_m[lo:hi], m, v, g, flat_w[lo:hi], 1e-4, 0.9, 0.95, 1e-8, 0.0, steps[0])
        if (hi - lo) == S and n == S * w:
            dist.all_gather_into_tensor(flat_m, flat_m[lo:hi], group=group)
            dist.all_gather_into_tensor(flat_w, flat_w[lo:hi], group=group)

    rows = {}
    rows["fold_local"] = _time(lambda: ops.linear_dw(dy, x, grad, accumulate=True), iters)
    rows["fold_peer"] = _time(lambda: ext.gemm_peer_scatter(dy, x, grad, slot_ptrs, lo_list, S, 0,
                                                            rank, 0, None, None), iters)

    def fold_nccl():
        ops.linear_dw(dy, x, grad, accumulate=True)
        if n == S * w:
            dist.reduce_scatter_tensor(shard_out, grad.view(-1), group=group)

    rows["fold_nccl"] = _time(fold_nccl, iters)
    rows["push_fused"] = _time(push_fused, iters)
    rows["push_nccl"] = _time(push_nccl, iters)
    st = ext.status_read_clear()
    if rank == 0:
        roof_fold = max(flops / (peak * 1e12), fold_bytes / (PEER_GBS * 1e9)) * 1e3
        roof_push = push_bytes / (PEER_GBS * 1e9) * 1e3
        out = {"world": w, "shape": f"dW [{F} x {D}] from {T} tokens", "status_word": st,
               "peak_bf16_tflops": peak, "peer_gbs": PEER_GBS,
               "fold_nvlink_mb_per_rank": round(fold_bytes / 1e6, 1),
               "push_nvlink_mb_per_rank": round(push_bytes / 1e6, 1)}
        for k, t in rows.items():
            out[f"{k}_ms"] = round(t, 4)
        out["fold_peer_roofline_ms"] = round(roof_fold, 4)
        out["fold_peer_frac_of_roofline"] = round(roof_fold / rows["fold_peer"], 3)
        out["push_fused_roofline_ms"] = round(roof_push, 4)
        out["push_fused_frac_of_roofline"] = round(roof_push / rows["push_fused"], 3)
        out["fold_peer_vs_nccl"] = round(rows["fold_nccl"] / rows["fold_peer"], 3)
        out["push_fused_vs_nccl"] = round(rows["push_nccl"] / rows["push_fused"], 3)
        print(json.dumps(out), flush=True)
    dist.barrier()
    del h_slots, h_master, h_work
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
