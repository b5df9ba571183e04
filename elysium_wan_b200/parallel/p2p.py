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

import queue
import random
import threading
import time

import torch
import torch.distributed as dist

from elysium_wan_b200.models.gpt import Act


class _Shim:
    """Sender-side WAN emulation for one outgoing link: a FIFO worker thread
    that sleeps latency + bytes/rate (+ jitter) and then sends."""

    def __init__(self, link: dict):
        self.lat = float(link.get("latency_ms", 0.0)) / 1000.0
        self.rate = float(link.get("bw_mbps", 0.0)) * 1e6 / 8.0
        self.jit = float(link.get("jitter_ms", 0.0)) / 1000.0
        self.rng = random.Random(int(link.get("jitter_seed", 0)))
        self.q: queue.Queue = queue.Queue()
        self.busy_until = 0.0
        self.err: Exception | None = None
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    @property
    def active(self) -> bool:
        return self.lat > 0 or self.rate > 0

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
                self.busy_until = start + ser
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
        ranks = list(range(world))
        # Every rank creates the same groups in the same order.
        self.g_fwd = dist.new_group(ranks) if world > 1 else None
        self.g_bwd = dist.new_group(ranks) if world > 1 else None
        self.g_stage = None
        for r, w in enumerate(spec.stage_widths):
            g = dist.new_group([spec.rank_of(r, q) for q in range(w)]) if world > 1 else None
            if r == stage:
                self.g_stage = g
        cfg = spec.model
        self.T = spec.mb_size * cfg.seq_len
        self.d = cfg.d_model
        self.cuda = self.device.type == "cuda"
        self.fp8 = cfg.fp8_boundary()
        self.act_dtype = torch.bfloat16 if self.cuda else torch.float32
        link = spec.links[stage] if stage < len(spec.links) else {}
        back = spec.links[stage - 1] if stage > 0 and stage - 1 < len(spec.links) else {}
        self.shim_next = _Shim(link) if not self.cuda else None
        self.shim_prev = _Shim(back) if not self.cuda else None
        self.bytes_sent = 0
        self.frames = 0

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
        return torch.empty((self.T, self.d), dtype=self.act_dtype, device=self.device)

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
        ts = act.tensors()
        if self.fp8:
            ts = [ts[0].view(torch.uint8), ts[1]]
        return self._send([t.contiguous() for t in ts], self.next_rank(mb), self.g_fwd,
                          self.shim_next)

    def send_grad(self, mb: int, g: torch.Tensor):
        g = g.to(self.act_dtype).contiguous()
        return self._send([g], self.prev_rank(mb), self.g_bwd, self.shim_prev)

    # ----------------------------------------------------------------- receives
    def irecv_act(self, mb: int):
        bufs = self._act_buffers()
        src = self.prev_rank(mb)
        works = [dist.irecv(b, src, group=self.g_fwd) for b in bufs]
        return bufs, works

    def irecv_grad(self, mb: int):
        buf = self._grad_buffer()
        return [buf], [dist.irecv(buf, self.next_rank(mb), group=self.g_bwd)]

    @staticmethod
    def wait(handle):
        bufs, works = handle
        for w in works:
            w.wait()
        return bufs

    def as_act(self, bufs) -> Act:
        if self.fp8:
            return Act(bufs[0].view(torch.float8_e4m3fn), bufs[1])
        return Act(bufs[0])

    def flush(self):
        for s in (self.shim_next, self.shim_prev):
            if s is not None:
                s.flush()

    def close(self):
        for s in (self.shim_next, self.shim_prev):
            if s is not None:
                s.close()
