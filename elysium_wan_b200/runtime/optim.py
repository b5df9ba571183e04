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
        # copies on every device: a wave is written while the next step runs
        return {"t": self.t, "m": self.m.detach().to("cpu", copy=True),
                "v": self.v.detach().to("cpu", copy=True)}

    def load_state_dict(self, sd):
        self.t = int(sd["t"])
        self.m.copy_(sd["m"].to(self.m.device))
        self.v.copy_(sd["v"].to(self.v.device))


class HostAdamW(DeviceAdamW):
    """Moments in pinned host memory, streamed through two device staging
    buffers: chunk i computes while chunk i+1 loads and chunk i-1 stores.

    Partial residency (`promote`): the moments of the first `resident`
    elements can move to the device when memory allows; those elements update
    in place with one kernel launch and only the rest cross PCIe. The same
    kernel runs on the same values wherever the moments live, so the bits do
    not change (reference: HostAdamW.promote, src/wantrain/runtime/optim.py:208,
    which moves whole parameters; here the resident part is a prefix of the
    flat store)."""

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
        self.resident = 0  # elements whose moments live on the device
        self.m_dev = self.v_dev = None
        if pin:
            dev = master.device
            self.stage = [(torch.empty(self.chunk, device=dev), torch.empty(self.chunk, device=dev))
                          for _ in range(2)]
            # Loads and stores on separate streams so the two copy engines run
            # host->device and device->host at the same time.
            self.copy = torch.cuda.Stream(device=dev)
            self.copy_out = torch.cuda.Stream(device=dev)

    def promote(self, budget_bytes: int) -> int:
        """Move the moments of a longer prefix onto the device, within
        `budget_bytes` more device memory (8 bytes per element). -> bytes moved."""
        if not self.p.is_cuda:
            return 0
        n = self.p.numel()
        want = min(n, self.resident + max(0, int(budget_bytes)) // 8)
        if want < n:
            want -= want % 64
        if want <= self.resident:
            return 0
        old = self.resident
        dev = self.p.device
        m_dev = torch.empty(want, dtype=torch.float32, device=dev)
        v_dev = torch.empty(want, dtype=torch.float32, device=dev)
        if old:
            m_dev[:old].copy_(self.m_dev)
            v_dev[:old].copy_(self.v_dev)
        m_dev[old:].copy_(self.m[old:want])
        v_dev[old:].copy_(self.v[old:want])
        torch.cuda.synchronize(dev)
        self.m_dev, self.v_dev, self.resident = m_dev, v_dev, want
        return 8 * (want - old)

    def _sync_host(self):
        """The device-resident prefix back into the host copies (the state)."""
        if self.resident:
            self.m[:self.resident].copy_(self.m_dev)
            self.v[:self.resident].copy_(self.v_dev)

    def step(self):
        self.t += 1
        if not self.p.is_cuda:
            ops.adamw(self.p, self.m, self.v, self.g, self.work, self.lr, self.b1, self.b2,
                      self.eps, self.wd, self.t)
            return
        n = self.p.numel()
        R = self.resident
        if R:
            work = self.work[:R] if self.work is not None else None
            ops.adamw(self.p[:R], self.m_dev, self.v_dev, self.g[:R], work, self.lr, self.b1,
                      self.b2, self.eps, self.wd, self.t)
        if R >= n:
            return
        comp = torch.cuda.current_stream(self.p.device)
        loaded = [torch.cuda.Event(), torch.cuda.Event()]
        computed = [torch.cuda.Event(), torch.cuda.Event()]
        stored = [None, None]
        starts = list(range(R, n, self.chunk))
        # The loads read host moments that the previous step's stores wrote on
        # the other copy stream; the compute stream waited for those stores at
        # the end of that step, so ordering the loads after it orders them
        # after the stores.
        self.copy.wait_stream(comp)

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
        self._sync_host()
        return {"t": self.t, "m": self.m.clone(), "v": self.v.clone()}

    def load_state_dict(self, sd):
        self.t = int(sd["t"])
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        if self.resident:
            self.m_dev.copy_(self.m[:self.resident])
            self.v_dev.copy_(self.v[:self.resident])


def build(name: str, master, grad, work, lr, adamw: dict):
    if name == "adamw":
        return DeviceAdamW(master, grad, work, lr, adamw)
    if name == "adamw-host":
        return HostAdamW(master, grad, work, lr, adamw)
    raise ValueError(f"unknown optimizer {name!r}")
