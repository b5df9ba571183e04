"""Verify before fold: which contributions get recomputed by an auditor, what
one wrong answer costs a node, and a fold that never takes an unverified
contribution.

Behaviour follows the reference's policy (src/wantrain/fault_tolerance/
audit.py; a library there too, not wired into a run), written here as three
small pieces:

- `digest(tensors)`: an exact commitment (sha256 over each tensor's shape,
  dtype and bytes, in order). Runs are bitwise deterministic per declared
  device map, so equality of digests is the whole test; there is no tolerance
  band for a forger to hide in.
- `AuditPolicy`: adaptive replication after BOINC (Anderson 2019,
  arXiv:1903.01699). A node is replicated on every item until it has passed
  `warmup` audits; after that the probability halves every `half_life`
  passed audits and never drops below `floor` (a veteran can turn). Which
  items are drawn comes from HMAC-SHA256 of a secret seed, so the audited
  node cannot predict the sample and anyone can re-derive it once the seed
  is revealed; `absolute_every` forces one audit per that many of a node's
  items whatever the draw. One mismatch bans the node (with exact digests an
  honest node never misses), and every verdict goes to a public ledger.
- `GatedFold`: the ordered fold of a fixed set of microbatch contributions
  (ascending index: the first one assigned, each next one added in fp32).
  A contribution added unverified is held in quarantine and blocks the fold
  of every later index until it is released or replaced by the auditor's
  recomputation, so an attacked fleet's result equals the honest fleet's
  bit for bit.
"""

from __future__ import annotations

import hashlib
import hmac
import math
from dataclasses import dataclass

import torch


def digest(tensors) -> str:
    """sha256 over (shape, dtype, bytes) of each tensor, in order."""
    if isinstance(tensors, torch.Tensor):
        tensors = [tensors]
    h = hashlib.sha256()
    for t in tensors:
        c = t.detach().contiguous().cpu()
        h.update(repr((tuple(c.shape), str(c.dtype))).encode())
        h.update(c.reshape(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


@dataclass(frozen=True)
class Verdict:
    node: str
    step: int
    mb: int
    ok: bool
    claimed: str      # the digest the worker committed to
    recomputed: str   # the digest the auditor produced


@dataclass
class _Standing:
    passed: int = 0      # audits passed
    failed: int = 0
    banned: bool = False
    since_audit: int = 0  # items since this node's last audit


class AuditPolicy:
    def __init__(self, seed: bytes, warmup: int = 16, floor: float = 0.02, half_life: int = 32,
                 absolute_every: int = 0):
        if not 0.0 < floor <= 1.0 or half_life <= 0 or warmup < 0 or absolute_every < 0:
            raise ValueError("need 0 < floor <= 1, half_life > 0, warmup >= 0, "
                             "absolute_every >= 0")
        self.seed = bytes(seed)
        self.warmup, self.floor, self.half_life = int(warmup), float(floor), int(half_life)
        self.absolute_every = int(absolute_every)
        self.standing: dict = {}
        self.ledger: list = []

    def _s(self, node) -> _Standing:
        return self.standing.setdefault(node, _Standing())

    def replication_p(self, node) -> float:
        """Probability that one of the node's items is recomputed."""
        s = self._s(node)
        if s.banned or s.passed < self.warmup:
            return 1.0
        return max(self.floor, math.pow(0.5, (s.passed - self.warmup) / self.half_life))

    def _draw(self, node, step: int, mb: int) -> float:
        mac = hmac.new(self.seed, f"{node}|{step}|{mb}".encode(), hashlib.sha256).digest()
        return int.from_bytes(mac[:8], "big") / 2.0 ** 64

    def replicate(self, node, step: int, mb: int) -> bool:
        """Whether item (step, mb) of `node` is recomputed by an auditor."""
        s = self._s(node)
        p = self.replication_p(node)
        forced = self.absolute_every and s.since_audit + 1 >= self.absolute_every
        hit = p >= 1.0 or bool(forced) or self._draw(node, step, mb) < p
        s.since_audit = 0 if hit else s.since_audit + 1
        return hit

    def record(self, node, step: int, mb: int, claimed: str, recomputed: str) -> bool:
        """An auditor's result; -> whether the node's answer was right. One
        wrong answer bans the node."""
        ok = claimed == recomputed
        s = self._s(node)
        if ok:
            s.passed += 1
        else:
            s.failed += 1
            s.banned = True
        self.ledger.append(Verdict(node, int(step), int(mb), ok, claimed, recomputed))
        return ok

    def banned(self, node) -> bool:
        return self._s(node).banned

    def reveal(self) -> bytes:
        """The seed, published when the audit window closes."""
        return self.seed


class GatedFold:
    """Ordered fold over microbatch indices `mbs` (ascending) with a
    quarantine gate; tensors are folded in fp32 (the first assigned)."""

    def __init__(self, mbs):
        self.order = sorted(int(m) for m in mbs)
        self.pos = 0          # contributions folded so far
        self.held: dict = {}  # mb -> (tensors, verified)
        self.acc = None

    def add(self, mb: int, tensors, verified: bool = True):
        mb = int(mb)
        if mb not in self.order or mb in self.held or self.order.index(mb) < self.pos:
            raise ValueError(f"microbatch {mb} is not expected here")
        self.held[mb] = ([t.detach() for t in tensors], bool(verified))
        self._advance()

    def release(self, mb: int):
        """The auditor agreed: the quarantined contribution may fold."""
        tensors, _ = self.held[int(mb)]
        self.held[int(mb)] = (tensors, True)
        self._advance()

    def reject(self, mb: int, replacement):
        """The auditor disagreed: its recomputation folds in the place of the
        quarantined contribution."""
        if int(mb) not in self.held:
            raise ValueError(f"microbatch {mb} was never added")
        self.held[int(mb)] = ([t.detach() for t in replacement], True)
        self._advance()

    def _advance(self):
        while self.pos < len(self.order):
            mb = self.order[self.pos]
            got = self.held.get(mb)
            if got is None or not got[1]:
                return  # missing, or in quarantine: everything after waits
            tensors = got[0]
            if self.acc is None:
                self.acc = [t.to(torch.float32).clone() for t in tensors]
            else:
                for a, t in zip(self.acc, tensors):
                    a.add_(t.to(torch.float32))
            del self.held[mb]
            self.pos += 1

    def complete(self) -> bool:
        return self.pos == len(self.order)

    def result(self) -> list:
        if not self.complete():
            waiting = [m for m in self.order[self.pos:] if m in self.held]
            raise RuntimeError(f"fold incomplete at index {self.pos}: quarantine or missing "
                               f"contributions ({waiting} held)")
        return self.acc
