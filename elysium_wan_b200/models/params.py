"""Flat parameter store of one stage.

All parameters of a stage live in one contiguous fp32 master buffer (each
tensor starts on a 256-byte boundary so any view can be a TMA operand), with a
matching fp32 gradient buffer and, on the GPU, a bf16 working copy that the
GEMMs read. One flat buffer per stage makes the optimizer one kernel, a ZeRO-1
shard one contiguous slice, and a checkpoint one tensor.

The reference keeps fp32 nn.Parameters and casts them to bf16 per use under
autocast (src/wantrain/model/wgrad.py:257-265; 31% of block F time on H100 per
benchmarks/wan/runs/2026-10-13-h100/REPORT.md:116-121); here the cast happens
once per step, fused into the AdamW kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

ALIGN = 64  # elements (256 bytes of fp32)


@dataclass
class ParamSpec:
    name: str
    shape: tuple
    init: str  # "normal" | "normal_resid" | "embed" | "bias" | "zeros" | "ones"
    fan_in: int = 1
    matrix: bool = False  # read by a GEMM (needs the bf16 working copy)
    pack: bool = False  # the next tensor follows with no alignment gap (read as one operand)
    frozen: bool = False  # not trained: no gradient, no optimizer state (LoRA base)
    # pieces layout: every replica holds this matrix's fp32 master whole (a
    # kernel reads it in fp32, or another tensor is computed from it)
    replicate: bool = False


def plan_layout(specs: list[ParamSpec], replicated_first: bool = False):
    """(ordered specs, {name: (offset, shape)}, nt, numel, nr) of a flat store:
    trainable tensors first, each on an ALIGN boundary unless its predecessor
    packs it, frozen tensors after nt. With `replicated_first` (the pieces
    layout) the trainable tensors every replica holds whole (norms, biases,
    tables, and matrices marked `replicate`) come before the sharded
    matrices; nr is where the sharded matrices start."""
    train = [s for s in specs if not s.frozen]
    if replicated_first:
        train = [s for s in train if not _sharded(s)] + [s for s in train if _sharded(s)]
    ordered = train + [s for s in specs if s.frozen]
    index: dict[str, tuple[int, tuple]] = {}
    off, nt, nr = 0, None, None
    for s in ordered:
        if s.frozen and nt is None:
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            nt = max(off, ALIGN)
            off = nt
        if replicated_first and _sharded(s) and nr is None:
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            nr = off
        index[s.name] = (off, tuple(s.shape))
        n = math.prod(s.shape)
        off += n if s.pack else (n + ALIGN - 1) // ALIGN * ALIGN
    numel = max(off, ALIGN)
    nt = numel if nt is None else nt
    return ordered, index, nt, numel, (nt if nr is None else nr)


def _sharded(s: ParamSpec) -> bool:
    """Whether the pieces layout splits this tensor's fp32 master over the
    replicas (a trainable matrix nobody reads in fp32)."""
    return s.matrix and not s.frozen and not s.replicate


def pieces_held(nr: int, nt: int, numel: int, w: int, k: int) -> list:
    """[(flat lo, flat hi)] of the store that replica k of a width-w pieces
    stage holds in fp32, in the order its master buffer keeps them: the
    replicated region [0, nr), its range of the sharded matrices, and the
    frozen region [nt, numel) (not trained, read by every replica)."""
    lo, hi = [(nr + a, nr + b) for a, b in shard_ranges(nt - nr, w)][k]
    return [(0, nr), (lo, hi), (nt, numel)]


def shard_ranges(n: int, w: int) -> list:
    """w contiguous [lo, hi) ranges of n elements, boundaries on ALIGN."""
    per = (n + w - 1) // w
    per = (per + ALIGN - 1) // ALIGN * ALIGN
    return [(min(n, k * per), min(n, (k + 1) * per)) for k in range(w)]


class ParamStore:
    """Trainable tensors first, frozen ones after: the gradient buffer and the
    optimizer cover only [0, nt).

    `shard=(k, w)` is the pieces layout of replica k of a width-w stage: the
    replicated tensors [0, nr) keep a full fp32 master, the sharded matrices
    [nr, nt) keep only their k-th contiguous range [mlo, mhi) in fp32, and the
    frozen tensors [nt, numel) are held whole after them (the bf16 working
    copy stays whole; the replicas all-gather it after every step)."""

    def __init__(self, specs: list[ParamSpec], device: torch.device, work_dtype=None,
                 shard: tuple | None = None):
        self.declared = list(specs)  # declaration order (fixes each tensor's init stream)
        self.device = torch.device(device)
        self.specs, self.index, self.nt, self.numel, self.nr = plan_layout(
            specs, replicated_first=shard is not None)
        self.frozen = {s.name for s in self.specs if s.frozen}
        self.shard = shard
        if shard is not None:
            k, w = shard
            self.mbounds = [(self.nr + lo, self.nr + hi)
                            for lo, hi in shard_ranges(self.nt - self.nr, w)]
            self.held = pieces_held(self.nr, self.nt, self.numel, w, k)
            self.mlo, self.mhi = self.held[1]
            held = sum(hi - lo for lo, hi in self.held)
        else:
            self.mlo = self.mhi = self.nr
            self.held = [(0, self.numel)]
            held = self.numel
        self.master = torch.zeros(held, dtype=torch.float32, device=self.device)
        self.grad = torch.zeros(self.nt, dtype=torch.float32, device=self.device)
        self._sink = None
        self.tied_grad = None
        self.work_dtype = work_dtype
        self.work = (torch.zeros(self.numel, dtype=work_dtype, device=self.device)
                     if work_dtype is not None else None)

    def names(self) -> list[str]:
        return [s.name for s in self.specs]

    def _view(self, buf, name):
        off, shape = self.index[name]
        return buf[off: off + math.prod(shape)].view(shape)

    def p(self, name):
        """fp32 master view (in the pieces layout: a replicated or frozen
        tensor, or a matrix that lies wholly inside this replica's range)."""
        if self.shard is None:
            return self._view(self.master, name)
        off, shape = self.index[name]
        n = math.prod(shape)
        base = 0
        for lo, hi in self.held:
            if lo <= off and off + n <= hi:
                o = base + off - lo
                return self.master[o: o + n].view(shape)
            base += hi - lo
        raise KeyError(f"{name}: its fp32 master is held by another replica (pieces layout)")

    def holds(self, name) -> bool:
        try:
            self.p(name)
            return True
        except KeyError:
            return False

    def master_ranges(self) -> list:
        """[(flat lo, flat hi, master view)] of what this store holds in fp32."""
        out, base = [], 0
        for lo, hi in self.held:
            out.append((lo, hi, self.master[base: base + hi - lo]))
            base += hi - lo
        return out

    def set_initial(self, name, value):
        """Initial values of one tensor: the held part of the fp32 master and
        the whole working copy."""
        off, shape = self.index[name]
        n = math.prod(shape)
        flat = value.reshape(-1)
        for lo, hi, view in self.master_ranges():
            a, b = max(lo, off), min(hi, off + n)
            if a < b:
                view[a - lo: b - lo].copy_(flat[a - off: b - off])
        if self.work is not None:
            self.work[off: off + n].copy_(flat)

    def w(self, name):
        """Compute-dtype view (bf16 working copy on the GPU, the master on CPU)."""
        return self._view(self.work if self.work is not None else self.master, name)

    def g(self, name):
        """fp32 gradient view; None for a frozen tensor."""
        if name in self.frozen:
            return None
        return self._view(self.grad, name)

    def sink(self, n: int):
        """A scratch fp32 buffer of n elements for gradients a kernel must
        write but nobody reads (a frozen norm's)."""
        if self._sink is None or self._sink.numel() < n:
            self._sink = torch.zeros(n, dtype=torch.float32, device=self.device)
        return self._sink[:n]

    def joint_offset(self, names) -> int | None:
        """Offset of `names` when they sit back to back in the store (same
        trailing shape), so one GEMM can treat them as one matrix; else None."""
        off0, shape0 = self.index[names[0]]
        off = off0
        for n in names:
            o, shp = self.index[n]
            if o != off or tuple(shp[1:]) != tuple(shape0[1:]):
                return None
            off += math.prod(shp)
        return off0

    def _joint(self, buf, names):
        off = self.joint_offset(names)
        if off is None:
            raise ValueError(f"{names} are not contiguous in the store")
        rows = sum(self.index[n][1][0] for n in names)
        tail = tuple(self.index[names[0]][1][1:])
        return buf[off: off + rows * math.prod(tail)].view((rows,) + tail)

    def pj(self, names):
        """fp32 master view of adjacent parameters as one tensor (rows stacked)."""
        return self._joint(self.master, names)

    def wj(self, names):
        return self._joint(self.work if self.work is not None else self.master, names)

    def gj(self, names):
        if any(n in self.frozen for n in names):
            return None
        return self._joint(self.grad, names)

    def zero_grad(self):
        self.grad.zero_()

    def sync_work(self):
        """Working copy of what this store holds in fp32 (in the pieces layout
        the other replicas' matrix ranges arrive by all-gather)."""
        if self.work is None:
            return
        for lo, hi, view in self.master_ranges():
            if hi <= lo:
                continue
            if self.master.is_cuda and self.work.dtype == torch.bfloat16:
                from elysium_wan_b200 import ops

                ops.ext().cast_bf16(view, self.work[lo:hi])
            else:
                self.work[lo:hi].copy_(view)

    def state_dict(self) -> dict:
        return {name: self.p(name).detach().cpu().clone() for name in self.names()}

    def load_state_dict(self, sd: dict):
        for name in self.names():
            self.p(name).copy_(sd[name].to(self.device))
        self.sync_work()


def init_params(store: ParamStore, seed: int, entry_of: dict, std: float, n_layer: int,
                scheme: str = "gpt2", first_of_entry: dict | None = None):
    """Deterministic init: parameter j of entry e draws from its own generator
    seeded by (seed, e, j), so a stage initialises only its own slice and gets
    the same values as the single-device oracle on the same device type."""
    dev = store.device
    per_entry_count: dict[int, int] = {}
    for s in store.declared:
        e = entry_of[s.name]
        if first_of_entry and s.name in first_of_entry:
            j = first_of_entry[s.name]  # a copy of another stage's tensor: its stream
        else:
            j = per_entry_count.get(e, 0)
            per_entry_count[e] = j + 1
        gen = torch.Generator(device=dev)
        gen.manual_seed((seed * 1_000_003 + e * 7919 + j) % (2**63 - 1))
        direct = store.shard is None
        v = store.p(s.name) if direct else torch.empty(s.shape, dtype=torch.float32, device=dev)
        if s.init == "zeros":
            v.zero_()
        elif s.init == "ones":
            v.fill_(1.0)
        elif s.init == "lora_a":  # kaiming-uniform on the adapter's A, B starts at zero
            b = math.sqrt(6.0 / max(1, s.fan_in))
            v.copy_(torch.rand(s.shape, generator=gen, device=dev) * (2 * b) - b)
        elif scheme == "torch_default":
            if s.init == "embed":
                v.copy_(torch.randn(s.shape, generator=gen, device=dev))
            else:  # nn.Linear weight and bias: U(-1/sqrt(fan_in), 1/sqrt(fan_in))
                b = 1.0 / math.sqrt(max(1, s.fan_in))
                v.copy_(torch.rand(s.shape, generator=gen, device=dev) * (2 * b) - b)
        elif s.init == "bias":
            v.zero_()
        else:  # gpt2: N(0, std), residual projections scaled by 1/sqrt(2 n_layer)
            sd = std / math.sqrt(2.0 * n_layer) if s.init == "normal_resid" else std
            v.copy_(torch.randn(s.shape, generator=gen, device=dev) * sd)
        if not direct:
            store.set_initial(s.name, v)
    store.sync_work()
