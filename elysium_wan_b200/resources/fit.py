"""Fit check: build the stage's real slice, hold the schedule's peak number of
in-flight microbatches, run B/W and an optimizer step, report the allocator
peak (reference: src/wantrain/resources/fit.py, WT_FIT)."""

from __future__ import annotations

import torch


def peak_pending(order) -> int:
    live, peak = 0, 0
    for op, _ in order:
        live += 1 if op == "F" else (-1 if op == "W" else 0)
        peak = max(peak, live)
    return peak


def measure(spec, stage: int, device: str = "cpu") -> dict:
    from elysium_wan_b200.models.data import make_batch
    from elysium_wan_b200.runtime.engine import StageEngine

    dev = torch.device(device if device != "cuda" else "cuda:0")
    if dev.type == "cuda":
        torch.cuda.reset_peak_memory_stats(dev)
    eng = StageEngine(spec, stage, 0, None, dev)
    opt = eng.opt
    if eng.pieces:
        # the two range optimizers of replica 0 of a pieces stage
        from elysium_wan_b200.parallel.pieces import Pieces

        pc = Pieces(eng, None)
        opt = _Both(pc.opt_r, pc.opt_m)
    elif opt is None:
        # A wide stage: one replica's ZeRO-1 shard of the moments.
        from elysium_wan_b200.parallel.zero1 import shard_bounds
        from elysium_wan_b200.runtime import optim

        st_ = eng.store
        lo, hi = shard_bounds(st_.nt, eng.width)[0]
        opt = optim.build(spec.optimizer, st_.master[lo:hi], st_.grad[lo:hi],
                          st_.work[lo:hi] if st_.work is not None else None, spec.lr,
                          spec.adamw)
    # what the stage holds before any microbatch: parameters, gradients, moments
    base = torch.cuda.memory_allocated(dev) if dev.type == "cuda" else 0
    k = peak_pending(spec.schedule_order[stage][0])
    ok = True
    try:
        saved = []
        for mb in range(k):
            if eng.first:
                x, t = make_batch(spec.data_seed, 0, mb, spec.mb_size, spec.model.seq_len,
                                  spec.model.vocab_size)
                inp = x.to(dev)
            else:
                from elysium_wan_b200.models.gpt import Act

                T = spec.mb_size * spec.model.seq_len
                dt = torch.bfloat16 if dev.type == "cuda" else torch.float32
                inp = Act(torch.zeros(T, spec.model.d_model, dtype=dt, device=dev))
                t = torch.zeros(spec.mb_size, spec.model.seq_len, dtype=torch.long)
            out, st = eng.model.forward(inp, t.to(dev) if eng.last else None,
                                        keep="inputs" if eng.recompute else "all")
            saved.append(st)
        opt.step()
    except torch.cuda.OutOfMemoryError:
        ok = False
    peak = torch.cuda.max_memory_allocated(dev) if dev.type == "cuda" else 0
    return {"fits": ok, "peak_bytes": int(peak), "base_bytes": int(base), "in_flight": k,
            "params": int(eng.store.numel)}


class _Both:
    def __init__(self, *opts):
        self.opts = opts

    def step(self):
        for o in self.opts:
            o.step()
