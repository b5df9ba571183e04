"""AdamW over a stage's flat parameter store (or a ZeRO-1 shard of it).

"adamw": fp32 moments on the device, one fused kernel per step that also
writes the bf16 working copy. "adamw-host": the moments live in pinned host
memory and stream through the device in chunks on a copy stream, double
buffered, through the same kernel (elementwise, so the bits equal "adamw").
Reference: src/wantrain/runtime/optim.py:45-369 (torch AdamW and HostAdamW).
"""

from __future__ import annotations

import torch

from elysium_wan_b200 import ops

HOST_CHUNK = 64 << 20  # elements per streamed chunk (256 MB of fp32 per tensor)


class DeviceAdamW:
    def __init__(self, master, grad, work, lr, adamw: dict):
        self.p, self.g, self.work = master, grad, work
        self.m = torch.zeros_like(master)
        self.v = torch.zeros_like(master)
        self.lr = lr
        self.b1, self.b2 = adamw["betas"]
        self.eps = adamw["eps"]
        self.wd = adamw["weight_decay"]
        self.t = 0

    def step(self):
        self.t += 1
        ops.adamw(self.p, self.m, self.v, self.g, self.work, self.lr, self.b1, self.b2, self.eps,
                  self.wd, self.t)

    def state_dict(self):
        return {"t": self.t, "m": self.m.detach().cpu(), "v": self.v.detach().cpu()}

    def load_state_dict(self, sd):
        self.t = int(sd["t"])
        self.m.copy_(sd["m"].to(self.m.device))
        self.v.copy_(sd["v"].to(self.v.device))


class HostAdamW(DeviceAdamW):
    """Moments in pinned host memory, streamed through two device staging
    buffers: chunk i computes while chunk i+1 loads and chunk i-1 stores."""

    def __init__(self, master, grad, work, lr, adamw: dict, chunk: int = HOST_CHUNK):
        self.p, self.g, self.work = master, grad, work
        self.lr = lr
        self.b1, self.b2 = adamw["betas"]
        self.eps = adamw["eps"]
        self.wd = adamw["weight_decay"]
        self.t = 0
        n = master.numel()
        pin = master.is_cuda
        self.m = torch.zeros(n, dtype=torch.float32, pin_memory=pin)
        self.v = torch.zeros(n, dtype=torch.float32, pin_memory=pin)
        self.chunk = min(chunk, n)
        if pin:
            dev = master.device
            self.stage = [(torch.empty(self.chunk, device=dev), torch.empty(self.chunk, device=dev))
                          for _ in range(2)]
            # Loads and stores on separate streams so the two copy engines run
            # host->device and device->host at the same time.
            self.copy = torch.cuda.Stream(device=dev)
            self.copy_out = torch.cuda.Stream(device=dev)

    def step(self):
        self.t += 1
        if not self.p.is_cuda:
            ops.adamw(self.p, self.m, self.v, self.g, self.work, self.lr, self.b1, self.b2,
                      self.eps, self.wd, self.t)
            return
        n = self.p.numel()
        comp = torch.cuda.current_stream(self.p.device)
        loaded = [torch.cuda.Event(), torch.cuda.Event()]
        computed = [torch.cuda.Event(), torch.cuda.Event()]
        stored = [None, None]
        starts = list(range(0, n, self.chunk))

        def load(i):
            b = i % 2
            lo = starts[i]
            hi = min(n, lo + self.chunk)
            with torch.cuda.stream(self.copy):
                if stored[b] is not None:
                    self.copy.wait_event(stored[b])
                self.stage[b][0][: hi - lo].copy_(self.m[lo:hi], non_blocking=True)
                self.stage[b][1][: hi - lo].copy_(self.v[lo:hi], non_blocking=True)
                loaded[b].record(self.copy)

        load(0)
        for i, lo in enumerate(starts):
            b = i % 2
            hi = min(n, lo + self.chunk)
            if i + 1 < len(starts):
                load(i + 1)
            comp.wait_event(loaded[b])
            mm, vv = self.stage[b][0][: hi - lo], self.stage[b][1][: hi - lo]
            work = self.work[lo:hi] if self.work is not None else None
            ops.adamw(self.p[lo:hi], mm, vv, self.g[lo:hi], work, self.lr, self.b1, self.b2,
                      self.eps, self.wd, self.t)
            computed[b].record(comp)
            with torch.cuda.stream(self.copy_out):
                self.copy_out.wait_event(computed[b])
                self.m[lo:hi].copy_(mm, non_blocking=True)
                self.v[lo:hi].copy_(vv, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.copy_out)
                stored[b] = ev
        for ev in stored:
            if ev is not None:
                comp.wait_event(ev)

    def state_dict(self):
        return {"t": self.t, "m": self.m.clone(), "v": self.v.clone()}

    def load_state_dict(self, sd):
        self.t = int(sd["t"])
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])


def build(name: str, master, grad, work, lr, adamw: dict):
    if name == "adamw":
        return DeviceAdamW(master, grad, work, lr, adamw)
    if name == "adamw-host":
        return HostAdamW(master, grad, work, lr, adamw)
    raise ValueError(f"unknown optimizer {name!r}")
