"""ZeRO-1 for a wide stage: replica k owns a contiguous slice (shard k) of the
stage's flat fp32 parameters and their AdamW moments.

Declared gradient fold (the spec's `fold = "dp_tree"`, a recipe pin): each
replica folds the microbatches it owns in index order into a local fp32
partial (the W GEMM epilogue accumulates in place), then the owner of shard k
sums the replicas' partials of that shard in rank order:
    g[k] = ((p_0[k] + p_1[k]) + p_2[k]) + ...
The single-device oracle computes exactly this tree, so losses match bit for
bit. (The reference instead streams every microbatch's gradient to the owner
and left-folds all M in index order, src/wantrain/runtime/stage.py:3160-3244;
that order cannot be pre-summed per replica, hence the declared tree.)

After the owner's AdamW step the updated fp32 shards are all-gathered and
every replica refreshes its bf16 working copy.

This module is the library path (NCCL all_to_all + all_gather on GPUs, gloo
on CPU). The fused path that does the reduce-scatter from inside the W GEMM
epilogue over peer memory lives in parallel/fused.py and produces the same
bits.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from elysium_wan_b200.runtime import optim

ALIGN = 64


def shard_bounds(n: int, w: int) -> list:
    """[(lo, hi)] of w contiguous shards of n elements, boundaries on 64."""
    per = (n + w - 1) // w
    per = (per + ALIGN - 1) // ALIGN * ALIGN
    return [(min(n, k * per), min(n, (k + 1) * per)) for k in range(w)]


def all_to_all(comm, group, recv, send):
    """Equal-split all-to-all among a stage's replicas: over the sealed mesh
    of the TCP data plane when the stage has one, else the process group."""
    mesh = getattr(comm, "mesh", None)
    if mesh is not None:
        mesh.all_to_all_single(recv, send)
    else:
        dist.all_to_all_single(recv, send, group=group)


def all_gather(comm, group, out, mine):
    mesh = getattr(comm, "mesh", None)
    if mesh is not None:
        mesh.all_gather_into_tensor(out, mine)
    else:
        dist.all_gather_into_tensor(out, mine, group=group)


def fold_tree(partials: list) -> torch.Tensor:
    """The declared fold: copy of the first partial, then += in rank order."""
    acc = partials[0].clone()
    for p in partials[1:]:
        acc += p
    return acc


class Zero1:
    def __init__(self, engine, comm):
        self.e = engine
        self.comm = comm
        st = engine.store
        self.w = engine.width
        self.k = engine.peer
        self.n = st.nt  # the trainable region
        self.bounds = shard_bounds(self.n, self.w)
        lo, hi = self.bounds[self.k]
        self.lo, self.hi = lo, hi
        self.group = comm.g_stage if comm is not None else None
        spec = engine.spec
        # The optimizer holds moments of this replica's shard only.
        work = st.work[lo:hi] if st.work is not None else None
        engine.opt = optim.build(spec.optimizer, st.master[lo:hi], self._gshard(), work, spec.lr,
                                 spec.adamw)
        self._grad_shard = None

    def _gshard(self):
        # Placeholder view; replaced each step by the folded shard.
        self._g = torch.zeros(self.hi - self.lo, dtype=torch.float32, device=self.e.store.grad.device)
        return self._g

    def reduce_scatter_ordered(self):
        """Owner k receives every replica's partial of shard k and folds them in rank order."""
        st = self.e.store
        g = st.grad
        maxlen = max(h - l for l, h in self.bounds)
        send = torch.zeros(self.w * maxlen, dtype=torch.float32, device=g.device)
        for q, (l, h) in enumerate(self.bounds):
            send[q * maxlen: q * maxlen + (h - l)] = g[l:h]
        recv = torch.empty_like(send)
        all_to_all(self.comm, self.group, recv, send)
        parts = [recv[q * maxlen: q * maxlen + (self.hi - self.lo)] for q in range(self.w)]
        self._g.copy_(fold_tree(parts))

    def all_gather_params(self):
        st = self.e.store
        maxlen = max(h - l for l, h in self.bounds)
        mine = torch.zeros(maxlen, dtype=torch.float32, device=st.master.device)
        mine[: self.hi - self.lo] = st.master[self.lo:self.hi]
        out = torch.empty(self.w * maxlen, dtype=torch.float32, device=st.master.device)
        all_gather(self.comm, self.group, out, mine)
        for q, (l, h) in enumerate(self.bounds):
            if q != self.k:
                st.master[l:h] = out[q * maxlen: q * maxlen + (h - l)]
        st.sync_work()

    def sync_and_step(self):
        self.reduce_scatter_ordered()
        self.e.opt.step()
        self.all_gather_params()
