"""The stage engine: executes one slot's zero-bubble order per step.

Reference: StageRuntime (src/wantrain/runtime/stage.py:193-3985): per step it
walks schedule_order[stage][peer], runs F / B / W, routes activations and
gradients to the neighbouring stages, folds gradients in microbatch order and
steps AdamW. Here the data plane is torch.distributed (NCCL over NVLink on the
GPU, gloo on CPU), every op is a short sequence of sm_100a kernels on the
compute stream, receives are posted one op ahead so NCCL moves the next input
while the current op computes, and W folds dW straight into the fp32
gradient in the GEMM epilogue (the order of W ops is the fold order, and the
spec checks it is ascending).

Per-op device time comes from CUDA events (busy fraction per stage); the
`WT_TELEM` summary keeps the reference's schema (runtime/telemetry.py).
"""

from __future__ import annotations

import os
import time

import torch

from elysium_wan_b200.models.data import make_batch
from elysium_wan_b200.models.gpt import Act, StageModel, WExecutor, pair_w_tasks
from elysium_wan_b200.parallel.p2p import dbg
from elysium_wan_b200.runtime import optim
from elysium_wan_b200.runtime.telemetry import parse_sim_slow


class StageEngine:
    def __init__(self, spec, stage: int, peer: int, comm=None, device=None):
        self.spec, self.stage, self.peer = spec, stage, peer
        self.device = torch.device(device or spec.device_for(stage, peer))
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        width = spec.stage_widths[stage]
        self.pieces = spec.shard == "pieces" and width > 1
        self.model = StageModel(spec.model, tuple(spec.partition[stage]), self.device, spec.init_seed,
                                shard=(peer, width) if self.pieces else None)
        from elysium_wan_b200.models.hf import init_from_spec

        init_from_spec(self.model, spec)
        self.store = self.model.store
        self.comm = comm
        self.order = [(op, int(mb)) for op, mb in spec.schedule_order[stage][peer]]
        self.recompute = spec.recomputes(stage)
        st = self.store
        # The optimizer covers the trainable region [0, nt) (all of it unless
        # LoRA froze the base).
        # (The pieces layout builds its two range optimizers when the comm attaches.)
        # A wide stage's ZeRO-1 layer builds the optimizer of its own shard when
        # the comm attaches (whole-stage moments would double its memory).
        self.width = spec.stage_widths[stage]
        self.opt = None if (self.pieces or self.width > 1) else optim.build(
            spec.optimizer, st.master[:st.nt], st.grad,
            st.work[:st.nt] if st.work is not None else None, spec.lr, spec.adamw)
        self.step_done = 0
        self.losses: list = []  # (step, mb, float)
        self.events: list = []  # per-op (op, mb, start_event, end_event)
        self.timing = spec.device_for(stage, peer).startswith("cuda")
        # NVTX range per F / B / W op (EWB_NVTX=1), for external timeline tools.
        self.nvtx = self.timing and os.environ.get("EWB_NVTX") == "1"
        self.telemetry: list = []
        self._host_x = None

        slow = parse_sim_slow()
        self.sim_slow = slow.get((stage, peer), slow.get(stage, (1.0, 0)))
        self.w_pair = bool(spec.w_pair) and spec.stage_widths[stage] == 1
        # W fill (reference RUNTIME-I27, src/wantrain/runtime/stage.py:3353-3373):
        # on host devices a receive that is late runs deferred W tasks, one
        # layer's at a time, instead of idling; on a GPU the side stream
        # already overlaps W with the wait.
        self.fill_w = bool(spec.schedule_fill) and self.device.type != "cuda" and not self.w_pair
        self.w_filled = 0  # W tasks run while a receive was pending (last step)
        self._w_seq: list = []
        self._w_pos = 0
        self._w_done: set = set()
        self._w_stash = None
        side = os.environ.get("EWB_W_STREAM", "1") == "1"
        self.wexec = WExecutor(self.device, enabled=side)
        self.phase: dict = {}
        # Marker lines (WT_*) go to stdout, where a stage's agent reads them.
        self.log = lambda line: print(line, flush=True)
        self.zero1 = None
        if comm is not None:
            self.attach_comm(comm)

    def attach_comm(self, comm):
        """Bind the stage channels (after warm_kernels, before the first step)."""
        self.comm = comm
        if self.width > 1 and self.zero1 is None:
            if self.pieces:
                from elysium_wan_b200.parallel.pieces import Pieces

                self.zero1 = Pieces(self, comm)
            elif self.spec.grad_sync == "fused" and self.device.type == "cuda" and \
                    not self.spec.model.lora_rank and self.spec.backend == "nccl":
                from elysium_wan_b200.parallel.fused import FusedZero1

                self.zero1 = FusedZero1(self, comm)
            else:
                from elysium_wan_b200.parallel.zero1 import Zero1

                self.zero1 = Zero1(self, comm)

    def _await(self, handle, wq: dict, step: int):
        """Wait for a receive. While it is pending (host devices), run the
        deferred W tasks of the next W op in the order, one task (one layer's
        weight gradients) at a time, once its B is done: W work still runs in
        the order's sequence, so every parameter folds its contributions in the
        same order and no bit changes; the W op itself later runs what is
        left."""
        comm = self.comm
        marks = self.zero1 is not None and hasattr(self.zero1, "mark")  # W routed by the exchange
        if self.fill_w and not marks and hasattr(comm, "ready"):
            seq = self._w_seq
            while not comm.ready(handle):
                while self._w_pos < len(seq) and seq[self._w_pos] in self._w_done:
                    self._w_pos += 1
                if self._w_pos == len(seq):
                    break
                mb = seq[self._w_pos]
                tasks = wq.get(mb)
                if not tasks:  # its B has not run yet
                    break
                t0 = time.perf_counter()
                tasks.pop(0).run()
                if not tasks:
                    self._w_done.add(mb)
                self.w_filled += 1
                self.events.append(("W", mb, t0, time.perf_counter()))
        return comm.wait(handle)

    def _run_w(self, tasks: list, mb: int):
        if self.zero1 is not None and hasattr(self.zero1, "mark"):
            self.zero1.mark(tasks, mb)
        if self.w_pair:
            # microbatch 2k waits for 2k + 1; the pair runs as one fold
            if mb % 2 == 0 and mb + 1 < self.spec.microbatches:
                self._w_stash = (mb, tasks)
                return
            if mb % 2 == 1:
                first_mb, first = self._w_stash
                if first_mb != mb - 1:
                    raise RuntimeError(f"W of microbatch {mb} without that of {mb - 1}")
                self._w_stash = None
                tasks = pair_w_tasks(first, tasks)
        # On the side stream the W op's device time is bracketed there (the
        # compute stream only enqueues it), so busy counts the W GEMMs too.
        ev = self.wexec.run(tasks, timing=self.timing)
        if ev is not None:
            self.events.append(("W", mb, ev[0], ev[1]))

    @property
    def first(self) -> bool:
        return self.model.first

    @property
    def last(self) -> bool:
        return self.model.last

    # ----------------------------------------------------------------- data
    def _stage_batches(self, step: int, mbs: list) -> dict:
        """The step's token ids and targets, generated on the host (the data
        rule is a CPU generator), written into pinned staging buffers that are
        allocated once, and copied to the device in one transfer each.

        No pinned allocation ever happens inside a step: allocating pinned
        memory can wait on the whole device, and a device-wide wait while a
        receive from a neighbouring stage is pending deadlocks the pipeline."""
        s = self.spec
        shape = (len(mbs), s.mb_size, s.model.seq_len)
        if self._host_x is None or self._host_x.shape != shape:
            pin = self.device.type == "cuda"
            self._host_x = torch.empty(shape, dtype=torch.int64, pin_memory=pin)
            self._host_t = torch.empty(shape, dtype=torch.int64, pin_memory=pin)
            self._dev_x = torch.empty(shape, dtype=torch.int64, device=self.device)
            self._dev_t = torch.empty(shape, dtype=torch.int64, device=self.device)
        for i, mb in enumerate(mbs):
            x, t = make_batch(s.data_seed, step, mb, s.mb_size, s.model.seq_len, s.model.vocab_size,
                              dataset=s.dataset_path, data_shards=s.data_shards)
            self._host_x[i].copy_(x)
            self._host_t[i].copy_(t)
        if self.device.type == "cuda":
            self._dev_x.copy_(self._host_x, non_blocking=True)
            self._dev_t.copy_(self._host_t, non_blocking=True)
            xs, ts = self._dev_x, self._dev_t
        else:
            xs, ts = self._host_x.clone(), self._host_t.clone()
        return {mb: (xs[i], ts[i]) for i, mb in enumerate(mbs)}

    def warm_kernels(self):
        """Run one F, B and W on a dummy microbatch so every kernel of the
        stage is loaded and configured before the first NCCL operation (module
        loading and first-launch set-up must not happen while a receive is
        pending). Touches only gradients, which every step zeroes."""
        s = self.spec
        T = s.mb_size * s.model.seq_len
        x = torch.zeros((s.mb_size, s.model.seq_len), dtype=torch.int64, device=self.device)
        if self.first:
            inp = x
        else:
            from elysium_wan_b200 import ops

            cuda = self.device.type == "cuda"
            z = torch.zeros((T, s.model.d_model), dtype=ops.act_dtype(s.model.boundary_dtype, cuda),
                            device=self.device)
            q8 = ops.q8_dtype(s.model.boundary_dtype)
            inp = Act(*ops.quant_q8(z, q8)) if q8 is not None else Act(z)
        out, st = self.model.forward(inp, x if self.last else None)
        dt = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        dy = None if self.last else torch.zeros((T, s.model.d_model), dtype=dt, device=self.device)
        tasks: list = []
        self.model.backward(st, dy, tasks)
        for t in tasks:
            t.run()
        self.model.zero_grad()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    # ----------------------------------------------------------------- one step
    def run_step(self, step: int) -> list:
        """Execute this slot's order for `step`; returns [(mb, loss)] on the
        last stage (floats after one device->host read), else []."""
        spec = self.spec
        comm = self.comm
        self.model.zero_grad()
        f_mbs = [mb for op, mb in self.order if op == "F"]
        b_mbs = [mb for op, mb in self.order if op == "B"]
        batches = self._stage_batches(step, f_mbs) if (self.first or self.last) else {}
        act_q: dict = {}
        grad_q: dict = {}
        fi = bi = 0
        if not self.first:
            act_q[f_mbs[0]] = comm.irecv_act(f_mbs[0])
        if not self.last:
            grad_q[b_mbs[0]] = comm.irecv_grad(b_mbs[0])
        saved: dict = {}
        wq: dict = {}
        sends: list = []
        dev_losses: list = []
        ev = self.timing
        self.events = []
        inline_done: set = set()
        self.w_filled = 0
        self._w_seq = [m for o, m in self.order if o == "W"]
        self._w_pos = 0
        self._w_done: set = set()
        keep = "inputs" if self.recompute else "all"
        for idx, (op, mb) in enumerate(self.order):
            if op == "W" and mb in inline_done:
                continue
            dbg(f"stage {self.stage} op {op}{mb} start")
            e0 = None

            def mark():
                # The op's start event goes after its input receive, so waiting
                # on a peer counts as idle, not busy.
                nonlocal e0
                if ev:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                else:
                    e0 = time.perf_counter()
                if self.nvtx:
                    torch.cuda.nvtx.range_push(f"{op}{mb}")

            if op == "F":
                if self.first:
                    inp = batches[mb][0]
                else:
                    inp = comm.as_act(self._await(act_q.pop(mb), wq, step))
                fi += 1
                if not self.first and fi < len(f_mbs):
                    act_q[f_mbs[fi]] = comm.irecv_act(f_mbs[fi])
                tgt = batches[mb][1] if self.last else None
                mark()
                out, st = self.model.forward(inp, tgt, keep=keep)
                saved[mb] = st
                if self.last:
                    dev_losses.append((mb, out))
                else:
                    sends += comm.send_act(mb, out)
            elif op == "B":
                st = saved.pop(mb)
                if self.last:
                    dy = None
                else:
                    dy = self._await(grad_q.pop(mb), wq, step)[0]
                    bi += 1
                    if bi < len(b_mbs):
                        grad_q[b_mbs[bi]] = comm.irecv_grad(b_mbs[bi])
                # A W that directly follows its own B runs layer by layer inside
                # B, releasing each layer's W inputs at once (same fold order).
                inline = (not self.w_pair and idx + 1 < len(self.order)
                          and self.order[idx + 1] == ("W", mb))
                tasks: list = []
                mark()
                dx = self.model.backward(st, dy, tasks, run_w_inline=inline,
                                         w_exec=lambda ts, m=mb: self._run_w(ts, m))
                if inline:
                    inline_done.add(mb)
                    self._w_done.add(mb)
                else:
                    wq[mb] = tasks
                if not self.first:
                    sends += comm.send_grad(mb, dx)
            else:  # W
                mark()
                self._run_w(wq.pop(mb, []), mb)
                self._w_done.add(mb)
            if self.nvtx:
                torch.cuda.nvtx.range_pop()
            if ev and not (op == "W" and self.wexec.cuda):
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record()
                self.events.append((op, mb, e0, e1))
            elif not ev and e0 is not None:
                # host device: the op ran synchronously; the timing-only seam
                # stretches it by the stage's factor (never what it computes)
                t1 = time.perf_counter()
                factor, from_step = self.sim_slow
                if factor > 1.0 and step >= from_step:
                    time.sleep((factor - 1.0) * (t1 - e0))
                    t1 = time.perf_counter()
                self.events.append((op, mb, e0, t1))
        dbg(f"stage {self.stage} ops done; waiting {len(sends)} sends")
        self.wexec.join()
        if ev:
            e_ops = torch.cuda.Event(enable_timing=True)
            e_ops.record()
        for w in sends:
            w.wait()
        if comm is not None:
            comm.flush()
        self._tied_fold()
        if self.zero1 is not None:
            self.zero1.sync_and_step()
        else:
            self._promote_moments()
            self.opt.step()
        self._tied_relay()
        self.model.after_step()
        self._moe_after_step()
        if ev:
            e_opt = torch.cuda.Event(enable_timing=True)
            e_opt.record()
            self.phase = {"first": self.events[0][2] if self.events else None, "ops_end": e_ops,
                          "opt_end": e_opt}
        self.step_done = step + 1
        out = []
        if self.last and dev_losses:
            vals = torch.stack([l.reshape(()) for _, l in dev_losses]).float().cpu().tolist()
            out = [(mb, v) for (mb, _), v in zip(dev_losses, vals)]
            for mb, v in out:
                self.losses.append((step, mb, v))
        return out

    def _promote_moments(self):
        """Before the third optimizer step of a stage whose AdamW moments live
        in host memory, move as long a prefix of them onto the device as the
        first two steps' peak leaves room for (the card's memory less the peak
        reserved by the caching allocator and a margin of 3% of the card, at
        least 2 GiB). WANTRAIN_OPT_RESIDENT=off keeps every moment on the host.
        The update is the same kernel on the same values, so bits do not change
        (reference: _promote_moments, src/wantrain/runtime/stage.py:3124)."""
        self._opt_steps = getattr(self, "_opt_steps", 0) + 1
        if self._opt_steps != 3 or not isinstance(self.opt, optim.HostAdamW) or \
                self.device.type != "cuda" or os.environ.get("WANTRAIN_OPT_RESIDENT") == "off":
            return
        total = torch.cuda.get_device_properties(self.device).total_memory
        peak = torch.cuda.max_memory_reserved(self.device)
        room = total - peak - max(2 << 30, int(0.03 * total))
        moved = self.opt.promote(room) if room > 0 else 0
        self.log(f"WT_OPT resident bytes={moved} elements={self.opt.resident}/"
                 f"{self.opt.p.numel()} room={room} peak={peak}")

    def _tied_fold(self):
        """Tied embeddings: the table's gradient becomes (embedding part) +
        (head part); across a cut the head's stage sends its part to stage 0."""
        if not self.spec.model.tie_embeddings:
            return
        if self.first and self.last:
            self.model.fold_tied()
        elif self.last:
            self.comm.tied_send(self.store.tied_grad)
        elif self.first:
            buf = torch.empty_like(self.store.p("0.tok.weight"))
            self.comm.tied_recv(buf)
            self.model.fold_tied(buf)

    def _tied_relay(self):
        """After the optimizer, stage 0 sends the updated table to the head's
        stage, whose relay copy (and working copy) take it."""
        if not self.spec.model.tie_embeddings or (self.first and self.last):
            return
        if self.first:
            self.comm.tied_send(self.store.p("0.tok.weight"))
        elif self.last:
            buf = torch.empty_like(self.store.p("0.tok.weight"))
            self.comm.tied_recv(buf)
            self.model.set_tied_table(buf)

    def _moe_after_step(self):
        """MoE bookkeeping after the optimizer step: the step's int64 expert
        counts per layer (integer sums, exact in any order; summed over the
        stage's replicas), the selection-bias update from them, and the aux
        values for telemetry."""
        if not self.model.moe_blocks():
            return
        recs = self.model.take_moe_records()
        E = self.spec.model.moe_experts
        layers = [m.e for m in self.model.moe_blocks()]
        counts = torch.zeros((len(layers), E), dtype=torch.int64)
        for r in recs:
            counts[layers.index(r.layer)] += r.counts
        if self.width > 1 and getattr(self.comm, "mesh", None) is not None:
            self.comm.mesh.all_reduce_sum(counts)  # the sealed mesh of the TCP plane
        elif self.width > 1 and self.comm is not None and getattr(self.comm, "g_stage", None):
            import torch.distributed as dist

            dev_counts = counts.to(self.device)
            dist.all_reduce(dev_counts, group=self.comm.g_stage)
            counts = dev_counts.cpu()
        tokens = self.spec.microbatches * self.spec.mb_size * self.spec.model.seq_len
        self.model.moe_bias_update({e: counts[i] for i, e in enumerate(layers)}, tokens)
        self.moe_aux = [(r.layer, r.aux) for r in recs]

    def phase_ms(self) -> dict:
        """{ops_ms, opt_ms} of the last step (after a synchronize)."""
        p = self.phase
        if not p or p.get("first") is None:
            return {}
        return {"ops_ms": round(p["first"].elapsed_time(p["ops_end"]), 2),
                "opt_ms": round(p["ops_end"].elapsed_time(p["opt_end"]), 2)}

    def op_times_ms(self) -> list:
        """[(op, mb, start_ms, dur_ms)] of the last step (after a synchronize)."""
        if not self.events:
            return []
        base = self.events[0][2]
        if isinstance(base, float):  # host clock (CPU stages)
            out = [(op, mb, (a - base) * 1e3, (b - a) * 1e3) for op, mb, a, b in self.events]
        else:
            out = [(op, mb, base.elapsed_time(a), a.elapsed_time(b)) for op, mb, a, b in self.events]
        return sorted(out, key=lambda x: x[2])

    # ----------------------------------------------------------------- state
    def state_dict(self) -> dict:
        # every tensor is a copy (a wave is written while the next step runs)
        return {"step": self.step_done, "params": self.store.master.detach().to("cpu", copy=True),
                "names": self.store.names(), "opt": self.opt.state_dict(),
                "losses": {f"{s}:{m}": v for s, m, v in self.losses},
                "buffers": {k: v.detach().to("cpu", copy=True)
                            for k, v in self.model.buffers().items()},
                "rng": torch.get_rng_state()}

    def load_state_dict(self, sd: dict):
        self.store.master.copy_(sd["params"].to(self.store.master.device))
        self.store.sync_work()
        if self.pieces and self.zero1 is not None:
            self.zero1._all_gather()  # the other replicas' matrix ranges of the working copy
        self.model.after_step()
        self.opt.load_state_dict(sd["opt"])
        for k, v in self.model.buffers().items():
            if k in sd.get("buffers", {}):
                v.copy_(sd["buffers"][k].to(v.device))
        self.step_done = int(sd["step"])
        self.losses = [(int(k.split(":")[0]), int(k.split(":")[1]), float(v))
                       for k, v in sd.get("losses", {}).items()]
        if "rng" in sd:
            torch.set_rng_state(sd["rng"])


def wall() -> float:
    return time.perf_counter()
