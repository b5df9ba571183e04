"""Verify-before-fold audit policy (reference: src/wantrain/fault_tolerance/audit.py,
a library there too, not wired into the run): a digest per gradient
contribution, replication of a fraction of microbatches on a second peer,
adaptive: the fraction rises after a mismatch and decays while results agree
(BOINC-style)."""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import torch


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


@dataclass
class AuditPolicy:
    rate: float = 0.05
    min_rate: float = 0.01
    max_rate: float = 1.0
    decay: float = 0.9
    mismatches: dict = field(default_factory=dict)

    def should_replicate(self, step: int, mb: int) -> bool:
        h = int(hashlib.sha256(f"{step}:{mb}".encode()).hexdigest()[:8], 16) / 0xFFFFFFFF
        return h < self.rate

    def record(self, peer, agreed: bool):
        if agreed:
            self.rate = max(self.min_rate, self.rate * self.decay)
        else:
            self.mismatches[peer] = self.mismatches.get(peer, 0) + 1
            self.rate = self.max_rate

    def quarantined(self, peer) -> bool:
        return self.mismatches.get(peer, 0) >= 2
