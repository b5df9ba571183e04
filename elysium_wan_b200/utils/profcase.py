"""One hot op at the 15.8B shapes, a few times: the small case an Nsight
Compute capture targets (one kernel, one to three launches, a few GB).

    python -m elysium_wan_b200.utils.profcase --op gemm_fwd [--iters 3]

Ops: gemm_fwd (qkv projection), gemm_dx (fc1 input gradient), gemm_dw (fc1
weight gradient fold), gemm_dw_pair (the same for two microbatches in one launch), gemm_resid (out projection + residual), gemm_fc2 (fc2 +
residual), gemm_dgelu (fc2 input gradient x GELU'), gemm_q8 (fc2 with the fp8 boundary epilogue),
attn_fwd, attn_bwd, ln_fwd, ln_bwd, ce, adamw, embed_bwd, head_gemm (the 50257-way
logits GEMM, fp32 out), head_lse (the fused logits GEMM + cross-entropy: LSE epilogue and
finalize), head_fwd (LN + fused logits / CE of the head entry), head_bwd
(its forward, backward and W).
"""

from __future__ import annotations

import argparse
import json
import time

import torch

from elysium_wan_b200 import ops

T, D, F, H, V = 2048, 5120, 20480, 40, 50257
BN = 0  # GEMM tile width (0: the launcher's choice)


def _bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def build(op):
    """Returns (fn, flops, bytes) for one launch of the op."""
    if op == "gemm_fwd":
        x, w, b = _bf(T, D), _bf(3 * D, D, scale=0.02), torch.zeros(3 * D, device="cuda")
        out = torch.empty(T, 3 * D, dtype=torch.bfloat16, device="cuda")
        return (lambda: ops.gemm(x, w, out, ops.EPI_BF16, bias=b, bn=BN)), 2.0 * T * 3 * D * D, None
    if op == "gemm_dx":
        dy, w = _bf(T, F), _bf(F, D, scale=0.02)
        out = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
        return (lambda: ops.gemm(dy, w, out, ops.EPI_BF16, b_mn=True, bn=BN)), 2.0 * T * F * D, None
    if op == "gemm_resid":  # attention out projection + residual (N = 5120)
        x, w, r = _bf(T, D), _bf(D, D, scale=0.02), _bf(T, D)
        b = torch.zeros(D, device="cuda")
        out = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
        return (lambda: ops.gemm(x, w, out, ops.EPI_RESID, bias=b, resid=r, bn=BN)), \
            2.0 * T * D * D, None
    if op == "gemm_fc2":  # fc2 forward + residual (N = 5120, K = 20480)
        g, w, r = _bf(T, F), _bf(D, F, scale=0.02), _bf(T, D)
        b = torch.zeros(D, device="cuda")
        out = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
        return (lambda: ops.gemm(g, w, out, ops.EPI_RESID, bias=b, resid=r, bn=BN)), \
            2.0 * T * F * D, None
    if op == "gemm_dgelu":  # fc2 input gradient with the GELU derivative (N = 20480)
        dy, w, u = _bf(T, D), _bf(D, F, scale=0.02), _bf(T, F)
        out = torch.empty(T, F, dtype=torch.bfloat16, device="cuda")
        return (lambda: ops.gemm(dy, w, out, ops.EPI_DGELU, b_mn=True, aux=u, bn=BN)), \
            2.0 * T * F * D, None
    if op == "gemm_dw":
        dy, x = _bf(T, F), _bf(T, D)
        g = torch.zeros(F, D, device="cuda")
        return (lambda: ops.linear_dw(dy, x, g, accumulate=True)), 2.0 * T * F * D, None
    if op == "gemm_dw_pair":  # the same fold for two microbatches in one launch
        dy1, x1, dy2, x2 = _bf(T, F), _bf(T, D), _bf(T, F), _bf(T, D)
        g = torch.zeros(F, D, device="cuda")
        return (lambda: ops.linear_dw_pair(dy1, x1, dy2, x2, g, accumulate=True)), \
            2.0 * 2 * T * F * D, None
    if op == "gemm_q8":
        g, w, r = _bf(T, F), _bf(D, F, scale=0.02), _bf(T, D)
        b = torch.zeros(D, device="cuda")
        return (lambda: ops.linear_fwd(g, w, b, epi="resid_q8", resid=r)), 2.0 * T * F * D, None
    if op in ("attn_fwd", "attn_bwd"):
        qkv = _bf(T, 3 * D)
        o, lse = ops.attention_fwd(qkv, 1, T, H, D // H)
        flops_f = 4.0 * T * T * D / 2
        if op == "attn_fwd":
            return (lambda: ops.attention_fwd(qkv, 1, T, H, D // H)), flops_f, None
        do = _bf(T, D)
        return (lambda: ops.attention_bwd(qkv, o, do, lse, 1, T, H, D // H)), 2.5 * flops_f, None
    if op in ("ln_fwd1", "ln_bwd1"):  # one microbatch (2048 rows)
        x = _bf(T, D)
        gam, bet = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
        if op == "ln_fwd1":
            return (lambda: ops.layernorm_fwd(x, None, gam, bet)), None, T * D * 4
        y, m, r = ops.layernorm_fwd(x, None, gam, bet)
        dy = _bf(T, D)
        dg, db = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
        return (lambda: ops.layernorm_bwd(dy, x, None, m, r, gam, dy, dg, db, True)), None, T * D * 8
    if op in ("ln_fwd", "ln_bwd"):
        x = _bf(8 * T, D)
        gam, bet = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
        if op == "ln_fwd":
            return (lambda: ops.layernorm_fwd(x, None, gam, bet)), None, 8 * T * D * 4
        y, m, r = ops.layernorm_fwd(x, None, gam, bet)
        dy = _bf(8 * T, D)
        dg, db = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
        return (lambda: ops.layernorm_bwd(dy, x, None, m, r, gam, dy, dg, db, True)), None, 8 * T * D * 8
    if op == "head_gemm":
        h, w = _bf(T, D), _bf(V, D, scale=0.02)
        ld = (V + 7) // 8 * 8
        logits = torch.empty((T, ld), dtype=torch.float32, device="cuda")[:, :V]
        return (lambda: ops.gemm(h, w, logits, ops.EPI_F32)), 2.0 * T * V * D, None
    if op in ("head_fwd", "head_bwd"):
        from elysium_wan_b200.models.config import make_config
        from elysium_wan_b200.models.gpt import Act, StageModel

        cfg = make_config("gpt15b", n_layer=1)
        m = StageModel(cfg, (cfg.n_entries - 1, cfg.n_entries), "cuda", seed=1)
        head = m.layers[-1]
        q, sc = ops.quant_e4m3(_bf(T, D).float())
        tgt = torch.randint(0, V, (1, T), device="cuda")
        if op == "head_fwd":
            return (lambda: head.forward(Act(q, sc), {}, tgt)), 2.0 * T * V * D, None
        ctx: dict = {}

        def fb():
            head.forward(Act(q, sc), ctx, tgt)
            wq: list = []
            head.backward(ctx, None, wq)
            for t in wq:
                t.run()
        return fb, 3 * 2.0 * T * V * D, None
    if op == "head_lse":  # the fused head: logits GEMM with the LSE epilogue, then finalize
        h, w = _bf(T, D), _bf(V, D, scale=0.02)
        tgt = torch.randint(0, V, (T,), device="cuda")
        return (lambda: ops.head_ce(h, w, tgt, V, 1.0 / T)), 2.0 * T * V * D, None
    if op == "ce":
        ld = (V + 7) // 8 * 8
        logits = torch.randn(T, ld, device="cuda")[:, :V]
        tgt = torch.randint(0, V, (T,), device="cuda")
        return (lambda: ops.cross_entropy(logits, V, tgt, 1.0 / T)), None, T * V * 6
    if op == "adamw":
        n = 1 << 26  # 64 M parameters: 1.2 GB of state, ten times L2
        p, g = torch.randn(n, device="cuda"), torch.randn(n, device="cuda")
        m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
        pb = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        return (lambda: ops.adamw(p, m, v, g, pb, 1e-4, 0.9, 0.95, 1e-8, 0.0, 1)), None, n * 30
    if op == "embed_bwd":
        idx = torch.randint(0, V, (1, T), device="cuda")
        dx = _bf(T, D)
        dwte, dwpe = torch.zeros(V, D, device="cuda"), torch.zeros(T, D, device="cuda")
        return (lambda: ops.embed_bwd(idx, dx, T, dwte, dwpe)), None, None
    raise ValueError(op)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", required=True)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--time", action="store_true", help="also print CUDA-event timing (no profiler)")
    ap.add_argument("--bn", type=int, default=0, help="GEMM tile width 128/192/256 (0: auto)")
    ap.add_argument("--no-split", action="store_true", help="no K-split of a GEMM's last wave")
    a = ap.parse_args(argv)
    global BN
    BN = a.bn
    if a.no_split:
        ops.ext().set_gemm_split(False)
    torch.manual_seed(0)
    fn, flops, nbytes = build(a.op)
    fn()
    torch.cuda.synchronize()
    if a.time:
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        ts = []
        for _ in range(10):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = sorted(ts)[len(ts) // 2]
        out = {"op": a.op, "ms": round(ms, 4)}
        if a.bn:
            out["bn"] = a.bn
        if a.no_split:
            out["split"] = False
        if flops:
            out["tflops"] = round(flops / ms / 1e9, 1)
        if nbytes:
            out["gbs"] = round(nbytes / ms / 1e6, 1)
        print(json.dumps(out), flush=True)
    for _ in range(a.iters):
        fn()
    torch.cuda.synchronize()
    time.sleep(0.01)


if __name__ == "__main__":
    main()
