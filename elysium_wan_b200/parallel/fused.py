"""ZeRO-1 with the collectives fused into the kernels, over NVLink peer memory.

Same declared fold and same bits as parallel/zero1.py (the NCCL library
path): replica r folds its own microbatches into a local fp32 partial in
microbatch order; the owner of shard k sums the replicas' partials of shard k
in rank order; the owner steps AdamW on its shard; every replica then holds
the updated fp32 master and bf16 working copy. What changes is how the bytes
move (BASELINE north star items 1 and 2):

  * reduce-scatter: the dW GEMM of each weight for a replica's LAST owned
    microbatch does not write its local gradient; its epilogue adds the tile
    to the local partial and stores the result straight into the owner's slot
    (peer memory, kEpiAccF32Peer in csrc/gemm.cu), so the transfer overlaps
    the GEMM tile by tile. Gradients the GEMMs do not produce (LayerNorm,
    biases, embeddings) are pushed by a copy kernel.
  * all-gather: the owner's AdamW kernel writes each updated fp32 value and
    its bf16 copy into every replica's master / working copy (peer stores),
    so the parameters cross NVLink once, inside the optimizer pass. (The
    reference moves PARAMS frames after its step; fusing the gather into the
    first forward GEMM instead would re-read every weight tile over NVLink
    once per M-tile of that GEMM.)
  * synchronisation: a one-element NCCL all-reduce on the stage group after
    the scatter and after the push (stream-ordered; no kernel spins on a peer).

Peer memory is PyTorch symmetric memory (IPC-mapped, multicast disabled:
only plain peer loads and stores are used).
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from elysium_wan_b200 import ops
from elysium_wan_b200.parallel.zero1 import shard_bounds

os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")


def _symm(n, dtype, device, group):
    import torch.distributed._symmetric_memory as symm

    try:
        symm.enable_symm_mem_for_group(group.group_name)
    except Exception:
        pass
    t = symm.empty(n, dtype=dtype, device=device)
    h = symm.rendezvous(t, group)
    return t, h


class FusedZero1:
    def __init__(self, engine, comm):
        self.e = engine
        st = engine.store
        self.group = comm.g_stage
        self.w = engine.width
        self.k = engine.peer
        self.n = st.numel
        self.bounds = shard_bounds(self.n, self.w)
        self.lo_list = [b[0] for b in self.bounds] + [self.n]
        self.lo, self.hi = self.bounds[self.k]
        dev = st.master.device
        self.S = max(h - l for l, h in self.bounds)
        # Master and working copy move into symmetric memory (values kept).
        m_sym, self.h_master = _symm(self.n, torch.float32, dev, self.group)
        w_sym, self.h_work = _symm(self.n, torch.bfloat16, dev, self.group)
        m_sym.copy_(st.master)
        w_sym.copy_(st.work)
        st.master, st.work = m_sym, w_sym
        self.slots, self.h_slots = _symm(self.w * self.S, torch.float32, dev, self.group)
        self.slot_ptrs = list(self.h_slots.buffer_ptrs)
        self.master_ptrs = list(self.h_master.buffer_ptrs)
        self.work_ptrs = list(self.h_work.buffer_ptrs)
        spec = engine.spec
        self.lr = spec.lr
        self.b1, self.b2 = spec.adamw["betas"]
        self.eps = spec.adamw["eps"]
        self.wd = spec.adamw["weight_decay"]
        self.t = 0
        self.m = torch.zeros(self.hi - self.lo, dtype=torch.float32, device=dev)
        self.v = torch.zeros_like(self.m)
        self.g = torch.zeros_like(self.m)
        # Flat ranges the fused GEMM epilogue does not cover.
        ranges = []
        for s in st.specs:
            if not s.matrix:
                off, shape = st.index[s.name]
                n = 1
                for x in shape:
                    n *= x
                ranges += [off, off + n]
        self.ranges = torch.tensor(ranges or [0, 0], dtype=torch.int64, device=dev)
        self.sync_t = torch.zeros(1, dtype=torch.float32, device=dev)
        # Last microbatch this replica owns: its W tasks scatter to the owners.
        self.last_mb = max(spec.owned(engine.stage, engine.peer))
        engine.opt = self  # checkpointing reads the shard state through this object
        dist.barrier(group=self.group)

    # ----------------------------------------------------------------- W hook
    def mark(self, tasks, mb):
        """Route the dW GEMMs of the last owned microbatch through the owners' slots."""
        if mb != self.last_mb:
            return
        base = self.e.store.grad.data_ptr()
        for t in tasks:
            flat_off = (t.w_grad.data_ptr() - base) // 4
            t.peer = (self.slot_ptrs, self.lo_list, self.S, flat_off, self.k)

    # ----------------------------------------------------------------- step end
    def _sync(self):
        dist.all_reduce(self.sync_t, group=self.group)

    def sync_and_step(self):
        st = self.e.store
        ops.ext().zero1_push_partials(st.grad, self.ranges, self.slot_ptrs, self.lo_list, self.S,
                                      self.k)
        self._sync()
        ops.ext().zero1_fold_slots(self.slots, self.S, self.w, self.hi - self.lo, self.g)
        self.t += 1
        ops.ext().zero1_adamw_push(st.master, self.m, self.v, self.g, self.lo, self.hi - self.lo,
                                   self.master_ptrs, self.work_ptrs, self.lr, self.b1, self.b2,
                                   self.eps, self.wd, self.t)
        self._sync()

    # ----------------------------------------------------------------- state
    def step(self):  # the engine calls sync_and_step; kept for the optimizer interface
        self.sync_and_step()

    def state_dict(self):
        return {"t": self.t, "m": self.m.detach().to("cpu", copy=True),
                "v": self.v.detach().to("cpu", copy=True)}

    def load_state_dict(self, sd):
        self.t = int(sd["t"])
        self.m.copy_(sd["m"].to(self.m.device))
        self.v.copy_(sd["v"].to(self.v.device))
