"""Single-device oracle: the same recipe, the same kernels, the same folds.

Reference: run_baseline (src/wantrain/validation/reference.py:189-362). Here
the oracle builds one StageModel per pipeline stage on ONE device and runs the
microbatches through them in index order; per stage it keeps one fp32 partial
gradient per ZeRO-1 replica (the replica that owns the microbatch at that
step: `spec.owner_at`, which follows a re-plan's ownership changes) and folds
the partials in rank order before AdamW, which is the declared `dp_tree` fold
of the distributed run. Cutting the model into stages changes no value (the
boundary recipe is applied at every block boundary), so a stage-count change
never changes the oracle.

Writes {tag}_losses.json ({"losses": [{step, mb, loss_hex, loss}]}),
{tag}_state.json (the canonical state manifest) and {tag}_timing.json.
"""

from __future__ import annotations

import json
import os
import time

import torch

from elysium_wan_b200.models.data import make_batch
from elysium_wan_b200.models.gpt import StageModel, pair_w_tasks
from elysium_wan_b200.parallel.zero1 import fold_tree, shard_bounds
from elysium_wan_b200.runtime import optim
from elysium_wan_b200.utils.determinism import float_hex, setup_determinism


class Oracle:
    def __init__(self, spec, device=None):
        self.spec = spec
        self.device = torch.device(device or spec.device)
        self.stages = [StageModel(spec.model, tuple(rng), self.device, spec.init_seed)
                       for rng in spec.partition]
        from elysium_wan_b200.models.hf import init_from_spec

        for m in self.stages:
            init_from_spec(m, spec)
        self.widths = list(spec.stage_widths)
        # the declared weight-gradient pairing of width-1 stages (spec.w_pair)
        self.w_pair = [bool(spec.w_pair) and w == 1 for w in self.widths]
        self.w_stash: list = [None] * len(self.widths)
        self.partials = []
        self.opts = []
        for r, m in enumerate(self.stages):
            st = m.store
            w = self.widths[r]
            self.partials.append([torch.zeros_like(st.grad) for _ in range(w)] if w > 1 else None)
            if w == 1:
                self.opts.append([optim.build(spec.optimizer, st.master[:st.nt], st.grad,
                                              st.work[:st.nt] if st.work is not None else None,
                                              spec.lr, spec.adamw)])
            else:
                os_ = []
                self._grad_shards = getattr(self, "_grad_shards", {})
                for k, (lo, hi) in enumerate(shard_bounds(st.nt, w)):
                    work = st.work[lo:hi] if st.work is not None else None
                    os_.append(optim.build(spec.optimizer, st.master[lo:hi], st.grad[lo:hi], work,
                                           spec.lr, spec.adamw))
                self.opts.append(os_)
        self.losses: list = []

    def step(self, step: int) -> list:
        spec = self.spec
        for m in self.stages:
            m.zero_grad()
        for part in self.partials:
            if part is not None:
                for p in part:
                    p.zero_()
        out = []
        owners = spec.owner_at(step)  # a re-plan may have moved microbatches between replicas
        for mb in range(spec.microbatches):
            x, t = make_batch(spec.data_seed, step, mb, spec.mb_size, spec.model.seq_len,
                              spec.model.vocab_size, dataset=spec.dataset_path,
                              data_shards=spec.data_shards)
            x, t = x.to(self.device), t.to(self.device)
            # Route each stage's gradient into the partial of the replica owning mb.
            saved_grads = []
            for r, m in enumerate(self.stages):
                if self.partials[r] is not None:
                    saved_grads.append(m.store.grad)
                    m.store.grad = self.partials[r][owners[r][mb]]
            ctxs, h = [], x
            for m in self.stages:
                h, c = m.forward(h, t if m.last else None)
                ctxs.append(c)
            loss = h
            dy = None
            tasks_all = []
            for r in range(len(self.stages) - 1, -1, -1):
                tasks: list = []
                dy = self.stages[r].backward(ctxs[r], dy, tasks)
                tasks_all.append(tasks)
            for k, tasks in enumerate(tasks_all):
                r = len(self.stages) - 1 - k
                if self.w_pair[r]:  # microbatch 2k waits for 2k + 1; one fold per pair
                    if mb % 2 == 0 and mb + 1 < spec.microbatches:
                        self.w_stash[r] = tasks
                        continue
                    if mb % 2 == 1:
                        tasks = pair_w_tasks(self.w_stash[r], tasks)
                        self.w_stash[r] = None
                for tk in tasks:
                    tk.run()
            i = 0
            for r, m in enumerate(self.stages):
                if self.partials[r] is not None:
                    m.store.grad = saved_grads[i]
                    i += 1
            out.append((mb, loss))
        if spec.model.tie_embeddings:  # table gradient = embedding part + head part
            self.stages[0].fold_tied(self.stages[-1].store.tied_grad)
        for r, m in enumerate(self.stages):
            if self.partials[r] is not None:
                for lo, hi in shard_bounds(m.store.nt, self.widths[r]):
                    m.store.grad[lo:hi] = fold_tree([p[lo:hi] for p in self.partials[r]])
            for o in self.opts[r]:
                o.step()
            if self.partials[r] is not None:
                m.store.sync_work()
            m.after_step()
        if spec.model.tie_embeddings and len(self.stages) > 1:
            self.stages[-1].set_tied_table(self.stages[0].store.p("0.tok.weight"))
        # MoE: the global batch's expert counts drive the selection-bias update.
        tokens = spec.microbatches * spec.mb_size * spec.model.seq_len
        for m in self.stages:
            if m.moe_blocks():
                counts: dict = {}
                for rec in m.take_moe_records():
                    counts[rec.layer] = counts.get(rec.layer, 0) + rec.counts
                m.moe_bias_update(counts, tokens)
        vals = torch.stack([l.reshape(()) for _, l in out]).float().cpu().tolist()
        res = [(mb, v) for (mb, _), v in zip(out, vals)]
        for mb, v in res:
            self.losses.append((step, mb, v))
        return res


def loss_records(losses) -> list:
    return [{"step": s, "mb": m, "loss_hex": float_hex(v), "loss": v} for s, m, v in losses]


def run_baseline(spec, tag: str = "reference", device=None) -> str:
    setup_determinism(spec.init_seed)
    o = Oracle(spec, device)
    timings = []
    for step in range(spec.steps):
        if o.device.type == "cuda":
            torch.cuda.synchronize(o.device)
        t0 = time.perf_counter()
        res = o.step(step)
        if o.device.type == "cuda":
            torch.cuda.synchronize(o.device)
        dt = time.perf_counter() - t0
        tokens = spec.microbatches * spec.mb_size * spec.model.seq_len
        timings.append({"step": step, "wall_s": round(dt, 4), "tokens": tokens,
                        "tok_s": round(tokens / dt, 1)})
        print(f"WT_METRIC {json.dumps({'step': step, 'loss': res[-1][1], 'tok_s': timings[-1]['tok_s']})}",
              flush=True)
    os.makedirs(spec.out_dir, exist_ok=True)
    from elysium_wan_b200.validation.state import reference_manifest, write_manifest

    write_manifest(os.path.join(spec.out_dir, f"{tag}_state.json"), reference_manifest(o))
    path = os.path.join(spec.out_dir, f"{tag}_losses.json")
    with open(path, "w") as f:
        json.dump({"losses": loss_records(o.losses)}, f, indent=2)
    steady = timings[1:] or timings
    with open(os.path.join(spec.out_dir, f"{tag}_timing.json"), "w") as f:
        json.dump({"steps": timings,
                   "steady_tok_s": round(sum(t["tokens"] for t in steady) /
                                         max(1e-9, sum(t["wall_s"] for t in steady)), 1),
                   "total_wall_s": round(sum(t["wall_s"] for t in timings), 2)}, f, indent=2)
    return path


def main(argv=None):
    import argparse

    from elysium_wan_b200.runtime.spec import JobSpec

    ap = argparse.ArgumentParser(prog="wantrain reference")
    ap.add_argument("--spec", required=True)
    ap.add_argument("--tag", default="reference")
    a = ap.parse_args(argv)
    spec = JobSpec.load(a.spec).finalize()
    print(run_baseline(spec, a.tag))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
