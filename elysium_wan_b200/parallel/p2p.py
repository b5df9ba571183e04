"""Stage-to-stage channels of the pipeline over torch.distributed.

One process per slot (stage, peer); ranks are stage-major. Activations go
forward and input gradients backward on two separate process groups, so the
two directions own separate NCCL communicators and streams and never
serialise behind each other (a recv posted for a gradient cannot block an
activation send on the same pair). Between any two slots, messages of one
direction are exchanged in increasing microbatch order on both sides, which
is what NCCL's and gloo's per-pair FIFO matching needs.

On GPUs the backend is NCCL over NVLink / NVSwitch (the reference's framed TCP
data plane, src/wantrain/transport/framing.py, has no counterpart on one box).
On CPU the backend is gloo, optionally behind a WAN shim that delays and paces
each send (reference: src/wantrain/transport/shim.py:164-247): one-way latency
plus serialisation at the link rate, seeded jitter.
"""

from __future__ import annotations

import os
import queue
import random
import sys
import threading
import time

_DEBUG = os.environ.get("EWB_DEBUG") == "1"


def dbg(msg: str):
    """Opt-in trace of communication steps (EWB_DEBUG=1) to stderr."""
    if _DEBUG:
        print(f"[ewb {time.monotonic():.3f} pid {os.getpid()}] {msg}", file=sys.stderr, flush=True)

import torch
import torch.distributed as dist

from elysium_wan_b200.models.gpt import Act


class _Shim:
    """Sender-side WAN emulation for one outgoing link: a FIFO worker thread
    that sleeps latency + bytes/rate (+ jitter) and then sends."""

    def __init__(self, link: dict, tag: str = "run"):
        from elysium_wan_b200.transport.pacer import link_buckets

        self.lat = float(link.get("latency_ms", 0.0)) / 1000.0
        self.rate = float(link.get("bw_mbps", 0.0)) * 1e6 / 8.0
        self.jit = float(link.get("jitter_ms", 0.0)) / 1000.0
        self.rng = random.Random(int(link.get("jitter_seed", 0)))
        # shared budgets (a NIC, a site pair's uplink) this link's frames cross
        self.budgets = link_buckets(link, tag)
        self.q: queue.Queue = queue.Queue()
        self.busy_until = 0.0
        self.err: Exception | None = None
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    @property
    def active(self) -> bool:
        return self.lat > 0 or self.rate > 0 or bool(self.budgets)

    def submit(self, fn, nbytes: int):
        self.q.put((fn, nbytes, time.monotonic()))

    def _loop(self):
        while True:
            item = self.q.get()
            if item is None:
                return
            fn, nbytes, t_in = item
            try:
                start = max(self.busy_until, t_in)
                ser = nbytes / self.rate if self.rate > 0 else 0.0
                end = start + ser
                # the frame crosses every shared budget at once: it has left
                # when the slowest of them has carried it
                for b in self.budgets:
                    end = max(end, b.reserve(nbytes))
                self.busy_until = end
                jit = self.rng.uniform(0, self.jit) if self.jit > 0 else 0.0
                due = self.busy_until + self.lat + jit
                d = due - time.monotonic()
                if d > 0:
                    time.sleep(d)
                fn()
            except Exception as e:  # surfaced on the next flush
                self.err = e
            finally:
                self.q.task_done()

    def flush(self):
        self.q.join()
        if self.err is not None:
            raise self.err

    def close(self):
        self.q.put(None)


class PipeComm:
    def __init__(self, spec, stage: int, peer: int, device: torch.device, timeout_s: float = 300.0):
        self.spec, self.stage, self.peer, self.device = spec, stage, peer, torch.device(device)
        self.rank = spec.rank_of(stage, peer)
        world = spec.world_size
        # One group per pipeline hop and direction (the ranks of stages j and
        # j+1). With NCCL's eager initialisation every group owns one
        # communicator and one stream and runs its point-to-point ops in issue
        # order; separate groups keep a middle stage's receive from upstream,
        # send downstream, and the two gradient directions independent.
        # Every rank creates every group in the same order.
        self.hop_fwd, self.hop_bwd = [], []
        for j in range(spec.stages - 1):
            ranks = [spec.rank_of(j, p) for p in range(spec.stage_widths[j])] + \
                    [spec.rank_of(j + 1, q) for q in range(spec.stage_widths[j + 1])]
            self.hop_fwd.append(dist.new_group(ranks) if world > 1 else None)
            self.hop_bwd.append(dist.new_group(ranks) if world > 1 else None)
        self.g_stage = None
        for r, w in enumerate(spec.stage_widths):
            g = dist.new_group([spec.rank_of(r, q) for q in range(w)]) if world > 1 else None
            if r == stage:
                self.g_stage = g
        # Tied embeddings across a cut: stage 0 and the head's stage exchange
        # the head's table gradient and the updated table once per step.
        self.g_tied = None
        if spec.model.tie_embeddings and spec.stages > 1 and world > 1:
            a, b = spec.rank_of(0, 0), spec.rank_of(spec.stages - 1, 0)
            g = dist.new_group([a, b])
            if self.rank in (a, b):
                self.g_tied = g
            self.tied_peer = b if self.rank == a else a
        cfg = spec.model
        self.T = spec.mb_size * cfg.seq_len
        self.d = cfg.d_model
        self.cuda = self.device.type == "cuda"
        from elysium_wan_b200 import ops

        self.q8 = ops.q8_dtype(cfg.boundary_dtype)  # fp8 boundary: its dtype, else None
        self.fp8 = self.q8 is not None
        self.act_dtype = ops.act_dtype(cfg.boundary_dtype, self.cuda)  # dense boundary activations
        self.grad_dtype = torch.bfloat16 if self.cuda else torch.float32  # boundary gradients
        link = spec.links[stage] if stage < len(spec.links) else {}
        back = spec.links[stage - 1] if stage > 0 and stage - 1 < len(spec.links) else {}
        from elysium_wan_b200.transport.pacer import pair_link, reverse_link

        # one pacer per direction serves every peer of the neighbour stage:
        # its receiver's budgets apply when that stage has one peer
        def dst(r):
            return (r, 0) if 0 <= r < spec.stages and spec.stage_widths[r] == 1 else None

        link = pair_link(spec, link, (stage, peer), dst(stage + 1))
        back = pair_link(spec, reverse_link(back), (stage, peer), dst(stage - 1))

        self.shim_next = _Shim(link, spec.tag) if not self.cuda else None
        self.shim_prev = _Shim(back, spec.tag) if not self.cuda else None
        self.bytes_sent = 0
        self.frames = 0
        if world > 1:
            self._init_pairs()

    # groups this slot uses
    @property
    def g_act_in(self):
        return self.hop_fwd[self.stage - 1]

    @property
    def g_act_out(self):
        return self.hop_fwd[self.stage]

    @property
    def g_grad_in(self):
        return self.hop_bwd[self.stage]

    @property
    def g_grad_out(self):
        return self.hop_bwd[self.stage - 1]

    def _init_pairs(self):
        """Create every communicator up front, in one global order.

        A communicator is built on the first operation of its group and that
        build blocks until every member joins; built lazily, stage r's early
        gradient receive (hop r backward) would wait for stage r+1 while stage
        r+1 waits for stage r's activation (hop r forward): a deadlock. Here
        every rank walks the same list of (group, sender, receiver) and
        exchanges one element on each entry it belongs to; the earliest
        unfinished entry always has both of its ranks ready, so the walk
        cannot deadlock."""
        spec = self.spec
        steps = []
        for j in range(spec.stages - 1):
            for group in (self.hop_fwd[j], self.hop_bwd[j]):
                for p in range(spec.stage_widths[j]):
                    for q in range(spec.stage_widths[j + 1]):
                        steps.append((group, spec.rank_of(j, p), spec.rank_of(j + 1, q)))
        t = torch.zeros(1, dtype=torch.float32, device=self.device)
        for i, (group, a, b) in enumerate(steps):
            if self.rank == a:
                dbg(f"rank {self.rank} init pair {i}: send to {b}")
                dist.send(t, b, group=group)
            elif self.rank == b:
                dbg(f"rank {self.rank} init pair {i}: recv from {a}")
                dist.recv(t, a, group=group)
        dbg(f"rank {self.rank} init pairs done")
        if self.g_stage is not None and self.spec.stage_widths[self.stage] > 1:
            dist.barrier(group=self.g_stage)
        if self.cuda:
            torch.cuda.synchronize(self.device)

    # ----------------------------------------------------------------- routing
    def next_rank(self, mb: int) -> int:
        s = self.stage + 1
        return self.spec.rank_of(s, self.spec.mb_owner[s][mb])

    def prev_rank(self, mb: int) -> int:
        s = self.stage - 1
        return self.spec.rank_of(s, self.spec.mb_owner[s][mb])

    # ----------------------------------------------------------------- buffers
    def _act_buffers(self):
        if self.fp8:
            return [torch.empty((self.T, self.d), dtype=torch.uint8, device=self.device),
                    torch.empty((self.T, self.d // 128), dtype=torch.float32, device=self.device)]
        return [torch.empty((self.T, self.d), dtype=self.act_dtype, device=self.device)]

    def _grad_buffer(self):
        return torch.empty((self.T, self.d), dtype=self.grad_dtype, device=self.device)

    # ----------------------------------------------------------------- sends
    def _send(self, tensors, dst, group, shim):
        nbytes = sum(t.numel() * t.element_size() for t in tensors)
        self.bytes_sent += nbytes
        self.frames += 1
        if shim is not None and shim.active:
            held = [t.clone() for t in tensors]

            def go():
                for t in held:
                    dist.send(t, dst, group=group)

            shim.submit(go, nbytes)
            return []
        return [dist.isend(t, dst, group=group) for t in tensors]

    def send_act(self, mb: int, act: Act):
        dbg(f"rank {self.rank} send act mb {mb} -> {self.next_rank(mb)}")
        ts = act.tensors()
        if self.fp8:
            ts = [ts[0].view(torch.uint8), ts[1]]
        return self._send([t.contiguous() for t in ts], self.next_rank(mb), self.g_act_out,
                          self.shim_next)

    def send_grad(self, mb: int, g: torch.Tensor):
        dbg(f"rank {self.rank} send grad mb {mb} -> {self.prev_rank(mb)}")
        g = g.to(self.grad_dtype).contiguous()
        return self._send([g], self.prev_rank(mb), self.g_grad_out, self.shim_prev)

    # ----------------------------------------------------------------- receives
    def irecv_act(self, mb: int):
        bufs = self._act_buffers()
        src = self.prev_rank(mb)
        dbg(f"rank {self.rank} post recv act mb {mb} <- {src}")
        works = [dist.irecv(b, src, group=self.g_act_in) for b in bufs]
        return bufs, works

    def irecv_grad(self, mb: int):
        buf = self._grad_buffer()
        dbg(f"rank {self.rank} post recv grad mb {mb} <- {self.next_rank(mb)}")
        return [buf], [dist.irecv(buf, self.next_rank(mb), group=self.g_grad_in)]

    @staticmethod
    def wait(handle):
        bufs, works = handle
        for w in works:
            w.wait()
        return bufs

    @staticmethod
    def ready(handle) -> bool:
        """Whether a posted receive has completed (never blocks)."""
        return all(w.is_completed() for w in handle[1])

    def as_act(self, bufs) -> Act:
        if self.fp8:
            return Act(bufs[0].view(self.q8), bufs[1])
        return Act(bufs[0])

    def tied_send(self, t):
        dist.send(t.contiguous(), self.tied_peer, group=self.g_tied)

    def tied_recv(self, buf):
        dist.recv(buf, self.tied_peer, group=self.g_tied)

    def flush(self):
        for s in (self.shim_next, self.shim_prev):
            if s is not None:
                s.flush()

    def close(self):
        for s in (self.shim_next, self.shim_prev):
            if s is not None:
                s.close()
