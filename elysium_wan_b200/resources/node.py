"""What the scheduler knows about a node (reference: src/wantrain/resources/node.py)."""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class NodeInfo:
    node_id: str
    name: str
    host: str = "127.0.0.1"
    region: str = "default"
    device: str = "cpu"
    device_class: str = "cpu"
    vram_gb: float | None = None
    tflops_bf16: float | None = None
    caps: dict = field(default_factory=dict)
    alive: bool = True

    def memory_bytes(self) -> float | None:
        """Device memory in bytes, or None when the node never measured it."""
        return None if not self.vram_gb else float(self.vram_gb) * 2**30

    def speed(self) -> float:
        """Relative compute speed (measured dense bf16 TFLOP/s; 1.0 unknown)."""
        return float(self.tflops_bf16) if self.tflops_bf16 else 1.0

    @staticmethod
    def from_caps(node_id: str, caps: dict) -> "NodeInfo":
        return NodeInfo(node_id=node_id, name=caps.get("name", node_id), host=caps.get("host", "127.0.0.1"),
                        region=caps.get("region", "default"), device=caps.get("device", "cpu"),
                        device_class=caps.get("device_class", "cpu"), vram_gb=caps.get("vram_gb"),
                        tflops_bf16=caps.get("tflops_bf16"), caps=dict(caps))


def mixed_fleet(nodes: list) -> str | None:
    """A fleet mixing device types (cpu with cuda) cannot be bit-compared with
    one oracle: refused with a reason (None when the fleet is uniform)."""
    kinds = {("cuda" if n.device.startswith("cuda") else n.device) for n in nodes}
    if len(kinds) > 1:
        return f"mixed device types {sorted(kinds)}: one job runs on one device type"
    return None
