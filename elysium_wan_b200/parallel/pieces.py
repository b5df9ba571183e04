"""Pieces: FSDP-like sharding of a wide stage (`shard: "pieces"`).

Reference behaviour: src/wantrain/runtime/pieces.py and stage.py:846-1130
(each replica owns a piece of every tensor: its fp32 master, AdamW moments
and gradient fold; per-unit update and gather). Here the store's pieces
layout (models/params.py) puts the replicated tensors (norms, biases,
embedding tables, and the small matrices read in fp32: an fp32 MoE router,
LoRA adapters, which the merged weight is computed from) first and the
sharded matrices after them; replica k holds:

- the fp32 master of the replicated region in full (its kernels read fp32),
  but steps only its k-th range of it;
- the fp32 master and the AdamW moments of only its k-th range of the
  sharded region (the bulk of the parameters);
- the frozen tensors (a LoRA base) whole, untouched by the exchange;
- the whole bf16 working copy, which the GEMMs read.

A step: the replicas' fp32 gradient partials (each replica folds its own
microbatches in order) go to the owners, which fold them in rank order (the
declared `dp_tree` fold, the same as ZeRO-1); each owner steps AdamW on its
two ranges (writing their bf16 cast); then the non-matrix ranges are
all-gathered in fp32 and the matrix ranges in bf16. AdamW is elementwise and
the fold is per element, so the bits equal ZeRO-1's and the single-device
oracle's; what changes is memory (4 bytes per matrix parameter are held once
per stage, not once per replica) and traffic (the matrices move as bf16).
"""

from __future__ import annotations

import torch

from elysium_wan_b200.models.params import shard_ranges
from elysium_wan_b200.parallel.zero1 import all_gather, all_to_all, fold_tree
from elysium_wan_b200.runtime import optim


class Pieces:
    def __init__(self, engine, comm):
        st = engine.store
        if st.shard is None:
            raise ValueError("the stage was not built in the pieces layout")
        self.e, self.comm = engine, comm
        self.group = comm.g_stage if comm is not None else None
        self.w, self.k = engine.width, engine.peer
        spec = engine.spec
        self.rb = shard_ranges(st.nr, self.w)  # non-matrix ranges (flat)
        self.mb = st.mbounds                   # matrix ranges (flat)
        self.r_lo, self.r_hi = self.rb[self.k]
        self.m_lo, self.m_hi = st.mlo, st.mhi
        # One flat list of owned elements per replica: its non-matrix range,
        # then its matrix range (the gradient partials travel in this order).
        self.own = [(self.rb[q], self.mb[q]) for q in range(self.w)]
        self.S = max((r[1] - r[0]) + (m[1] - m[0]) for r, m in self.own)
        n_r, n_m = self.r_hi - self.r_lo, self.m_hi - self.m_lo
        dev = st.grad.device
        self.g = torch.zeros(n_r + n_m, dtype=torch.float32, device=dev)
        work = st.work
        self.opt_r = optim.build(spec.optimizer, st.master[self.r_lo:self.r_hi], self.g[:n_r],
                                 work[self.r_lo:self.r_hi] if work is not None else None,
                                 spec.lr, spec.adamw)
        self.opt_m = optim.build(spec.optimizer, st.master[st.nr:st.nr + n_m], self.g[n_r:],
                                 work[self.m_lo:self.m_hi] if work is not None else None,
                                 spec.lr, spec.adamw)
        engine.opt = self

    # ---------------------------------------------------------------- step
    def _reduce_scatter(self):
        g = self.e.store.grad
        send = torch.zeros(self.w * self.S, dtype=torch.float32, device=g.device)
        for q, ((rl, rh), (ml, mh)) in enumerate(self.own):
            base = q * self.S
            send[base: base + rh - rl] = g[rl:rh]
            send[base + rh - rl: base + rh - rl + mh - ml] = g[ml:mh]
        recv = torch.empty_like(send)
        all_to_all(self.comm, self.group, recv, send)
        n = self.g.numel()
        self.g.copy_(fold_tree([recv[q * self.S: q * self.S + n] for q in range(self.w)]))

    def _all_gather(self):
        st = self.e.store
        # non-matrix ranges in fp32 (every replica keeps the region whole)
        per = max(h - l for l, h in self.rb)
        if per > 0:
            mine = torch.zeros(per, dtype=torch.float32, device=st.master.device)
            mine[: self.r_hi - self.r_lo] = st.master[self.r_lo:self.r_hi]
            out = torch.empty(self.w * per, dtype=torch.float32, device=st.master.device)
            all_gather(self.comm, self.group, out, mine)
            for q, (l, h) in enumerate(self.rb):
                if q != self.k:
                    st.master[l:h] = out[q * per: q * per + h - l]
        # matrix ranges as the working copy (bf16 on the GPU)
        per = max(h - l for l, h in self.mb)
        if st.work is not None and per > 0:
            mine = torch.zeros(per, dtype=st.work.dtype, device=st.work.device)
            mine[: self.m_hi - self.m_lo] = st.work[self.m_lo:self.m_hi]
            out = torch.empty(self.w * per, dtype=st.work.dtype, device=st.work.device)
            all_gather(self.comm, self.group, out, mine)
            for q, (l, h) in enumerate(self.mb):
                if q != self.k:
                    st.work[l:h] = out[q * per: q * per + h - l]
        # the replicated region's working copy follows its fp32 master
        if st.work is not None and st.nr > 0:
            st.work[:st.nr].copy_(st.master[:st.nr])

    def sync_and_step(self):
        self._reduce_scatter()
        self.opt_r.step()
        self.opt_m.step()
        self._all_gather()

    # ---------------------------------------------------------------- state
    def state_dict(self):
        return {"t": self.opt_m.t, "pieces": {"k": self.k, "w": self.w},
                "r": self.opt_r.state_dict(), "m": self.opt_m.state_dict()}

    def load_state_dict(self, sd):
        if sd.get("pieces", {}).get("w") != self.w:
            raise ValueError("a pieces wave resumes at the width it was written at")
        self.opt_r.load_state_dict(sd["r"])
        self.opt_m.load_state_dict(sd["m"])
