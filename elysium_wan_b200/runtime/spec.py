"""JobSpec: the single JSON object that determines a run.

Field names follow the reference (src/wantrain/runtime/spec.py:51-171) so a
wantrain spec loads unchanged; `finalize()` derives the partition, stage
widths, microbatch ownership (IWRR) and the zero-bubble order, and validates
them; `pins()` lists the fields a checkpoint's bytes depend on.

B200 additions: `backend` (nccl on GPUs, gloo / tcp on CPU), `zb_mem_mode`,
`fold` (the declared ZeRO-1 gradient fold, a recipe pin) and `grad_sync`
(how wide stages move gradients: "fused" in-kernel peer stores or "nccl";
both produce the same bits, so it is not a pin).
"""

from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field
from typing import Any

from elysium_wan_b200.models.config import GPTConfig

OPS = ("F", "B", "W")
ADAMW: dict[str, Any] = {"betas": [0.9, 0.95], "eps": 1e-8, "weight_decay": 0.0}
OPTIMIZERS = ("adamw", "adamw-host")
BACKENDS = ("nccl", "gloo", "tcp")
FOLDS = ("dp_tree",)
PACINGS = ("link", "shared")
EMISSION_ORDERS = ("store", "forward")


@dataclass
class LinkCfg:
    latency_ms: float = 0.0
    bw_mbps: float = 0.0
    jitter_ms: float = 0.0
    jitter_seed: int = 0
    # Shared budgets (transport/pacer.py), off when the key is empty: the
    # sender's NIC, the site pair's uplink in this direction, the receiver's NIC.
    egress_key: str = ""
    egress_mbps: float = 0.0
    uplink_key: str = ""
    uplink_mbps: float = 0.0
    ingress_key: str = ""
    ingress_mbps: float = 0.0


@dataclass
class JobSpec:
    # ------------------------------------------------------------- recipe
    model: GPTConfig = field(default_factory=GPTConfig)
    init_seed: int = 1234
    data_seed: int = 5678
    lr: float = 1e-3
    optimizer: str = "adamw"
    adamw: dict = field(default_factory=lambda: dict(ADAMW))
    device: str = "cpu"
    devices: list | None = None
    dataset_path: str | None = None
    dataset_sha256: str | None = None
    data_shards: int = 1
    dataset_source: str | None = None
    # initial weights from a checkpoint (a Hugging Face directory of
    # config.json + safetensors) instead of the seeded init; its digest pins it
    init_from: str | None = None
    init_sha256: str | None = None
    steps: int = 8
    microbatches: int = 8
    mb_size: int = 4
    recompute: bool = False
    recompute_stages: list | None = None
    # ------------------------------------------------------------- checkpoints
    ckpt_every: int = 0
    resume: bool = False
    resume_step: int | None = None
    # ------------------------------------------------------------- topology
    stages: int = 2
    stage_widths: list | None = None
    partition: list | None = None
    peer_weights: list | None = None
    mb_owner: list | None = None
    # The ownership earlier steps ran under, oldest first: [until_step,
    # mb_owner] means steps before until_step used that mb_owner (a re-plan
    # moved microbatches between the replicas of a wide stage at a wave). The
    # declared dp_tree fold of a step follows the ownership it ran under, so
    # the oracle reads it (`owner_at`).
    ownership_log: list = field(default_factory=list)
    stream_grads: bool = False
    # ------------------------------------------------------------- schedule
    schedule_order: list | None = None
    schedule_fill: bool = True
    zb_mem_mode: str = "auto"  # auto | 1p | 2p | given
    stage_costs: list | None = None  # measured [F, B, W] seconds per stage (profiled)
    # ------------------------------------------------------------- transport
    backend: str = "gloo"
    port_base: int = 29000
    host: str = "127.0.0.1"
    p2p_streams: int = 1
    # TCP sender fragment sizing (reference field names): a frame is cut into
    # fragments spread over the flows; with adapt_budget_ms > 0 the fragment
    # size halves (not below frag_min_bytes) while a fragment takes longer
    # than the budget to send and doubles back after 8 frames well under it.
    adapt_budget_ms: float = 0.0
    frag_min_bytes: int = 4096
    endpoints: list | None = None
    trusted_peers: list | None = None
    slot_peers: list | None = None
    dial_timeout_s: float = 0.0
    wire_codec: str = "raw"
    links: list = field(default_factory=list)
    # Shared WAN pacing, the reference's spec fields: with pacing "shared"
    # every connection also draws on its sender's NIC egress budget
    # (peer_egress_mbps[stage][peer]), its receiver's NIC ingress budget
    # (peer_ingress_mbps) and, between two sites (sites[stage][peer]), the
    # uplink of that direction (uplink_mbps["a->b"]), each a token bucket
    # that every connection of the host shares (transport/pacer.py).
    # Shim settings of the links among a wide stage's replicas (the TCP
    # plane's mesh): per stage {"p>q": link}; filled by placement from the
    # nodes' emulation profiles. This engine's own field.
    mesh_links: list | None = None
    pacing: str = "link"
    peer_egress_mbps: list | None = None
    peer_ingress_mbps: list | None = None
    sites: list | None = None
    uplink_mbps: dict | None = None
    # ------------------------------------------------------------- wide stages
    wire: str = "fp32"
    # Per stage, the order W emits its deferred gradients ("store" or
    # "forward"; the reference's field). Accepted and checked; this engine
    # folds each element in microbatch order whatever the emission order, so
    # it moves no bit and no byte.
    emission_order: list | None = None
    # Reference fields this engine does not take: explicit piece boundaries
    # (pieces here are cut over the flat store) and the device classes of an
    # arch "hf" job. Only None is accepted.
    piece_bounds: list | None = None
    device_classes: list | None = None
    shard: str = "zero1"
    fold: str = "dp_tree"
    grad_sync: str = "fused"  # fused | nccl
    # Width-1 stages fold the weight gradients of microbatches 2k and 2k + 1
    # with one GEMM over both token sets (half the fp32 read-modify-write of
    # the gradient); a recipe choice, so a pin.
    w_pair: bool = False
    # ------------------------------------------------------------- output
    out_dir: str = "runs"
    tag: str = "run"

    # ------------------------------------------------------------- derived
    @property
    def world_size(self) -> int:
        return sum(self.stage_widths or [1] * self.stages)

    def slots(self) -> list:
        """[(stage, peer)] in rank order: stage-major."""
        return [(r, p) for r, w in enumerate(self.stage_widths) for p in range(w)]

    def rank_of(self, stage: int, peer: int) -> int:
        return sum(self.stage_widths[:stage]) + peer

    def slot_of(self, rank: int) -> tuple[int, int]:
        return self.slots()[rank]

    def owned(self, rank: int, peer: int) -> list:
        """Microbatches slot (stage `rank`, `peer`) computes, ascending."""
        return [mb for mb, p in enumerate(self.mb_owner[rank]) if p == peer]

    def owner_at(self, step: int) -> list:
        """The mb_owner table step `step` ran (or runs) under."""
        for until, owners in self.ownership_log:
            if step < int(until):
                return owners
        return self.mb_owner

    def device_for(self, stage: int, peer: int = 0) -> str:
        if self.devices is not None:
            return self.devices[stage][peer]
        return self.device

    def recomputes(self, stage: int) -> bool:
        if self.recompute_stages is None:
            return bool(self.recompute)
        return bool(self.recompute_stages[stage])

    def finalize(self) -> "JobSpec":
        from elysium_wan_b200.scheduler import partition as part
        from elysium_wan_b200.scheduler.zero_bubble import iwrr
        from elysium_wan_b200.scheduler.planner import default_schedule

        self.model.validate()
        if self.optimizer not in OPTIMIZERS:
            raise ValueError(f"optimizer {self.optimizer!r} is not one of {OPTIMIZERS}")
        if self.backend not in BACKENDS:
            raise ValueError(f"backend {self.backend!r} is not one of {BACKENDS}")
        if self.fold not in FOLDS:
            raise ValueError(f"fold {self.fold!r} is not one of {FOLDS}")
        if self.shard not in ("zero1", "pieces"):
            raise ValueError(f"shard {self.shard!r} is not one of ('zero1', 'pieces')")
        if self.partition is None:
            try:
                self.partition = part.even_blocks_partition(self.model, self.stages)
            except ValueError:
                self.partition = part.proportional_partition(self.model, [1.0] * self.stages)
        self.partition = [list(map(int, r)) for r in self.partition]
        if len(self.partition) != self.stages:
            raise ValueError("partition needs one [start, end) per stage")
        prev = 0
        for a, b in self.partition:
            if a != prev or b <= a:
                raise ValueError(f"partition must tile the layer list contiguously: {self.partition}")
            prev = b
        if prev != self.model.n_entries:
            raise ValueError(f"partition ends at {prev}, the model has {self.model.n_entries} entries")
        if not self.links:
            self.links = [asdict(LinkCfg()) for _ in range(self.stages)]
        if self.stage_widths is None:
            self.stage_widths = [1] * self.stages
        if len(self.stage_widths) != self.stages:
            raise ValueError("stage_widths needs one entry per stage")
        if self.recompute_stages is not None and len(self.recompute_stages) != self.stages:
            raise ValueError("recompute_stages must name every stage")
        if self.peer_weights is None:
            self.peer_weights = [[1.0] * w for w in self.stage_widths]
        if [len(w) for w in self.peer_weights] != list(self.stage_widths):
            raise ValueError("peer_weights must have the shape of stage_widths")
        if self.mb_owner is None:
            self.mb_owner = [iwrr(self.microbatches, w) for w in self.peer_weights]
        for r, row in enumerate(self.mb_owner):
            if len(row) != self.microbatches or not all(0 <= p < self.stage_widths[r] for p in row):
                raise ValueError(f"mb_owner[{r}] must map every microbatch to a peer of stage {r}")
        last = 0
        for entry in self.ownership_log:
            until, owners = int(entry[0]), entry[1]
            if until <= last or len(owners) != self.stages or any(
                    len(row) != self.microbatches or
                    not all(0 <= int(p) < self.stage_widths[r] for p in row)
                    for r, row in enumerate(owners)):
                raise ValueError("ownership_log entries are [until_step, mb_owner] with rising "
                                 "steps and tables of this spec's shape")
            last = until
        if self.model.tie_embeddings and self.stages > 1 and \
                (self.stage_widths[0] != 1 or self.stage_widths[-1] != 1):
            raise NotImplementedError("a tied table across a cut needs width-1 first and last "
                                      "stages")
        if self.model.arch == "user":
            self._check_user_model()
        if self.emission_order is None:
            self.emission_order = ["store"] * self.stages
        if len(self.emission_order) != self.stages or \
                any(o not in EMISSION_ORDERS for o in self.emission_order):
            raise ValueError(f"emission_order must list one of {EMISSION_ORDERS} per stage")
        if self.piece_bounds is not None or self.device_classes is not None:
            raise NotImplementedError("piece_bounds and device_classes are not taken: pieces are "
                                      "cut over the flat store, and arch hf is not built")
        if self.pacing not in PACINGS:
            raise ValueError(f"pacing {self.pacing!r} is not one of {PACINGS}")
        if self.pacing == "shared":
            self._check_shared_pacing()
        if self.schedule_order is None:
            self.schedule_order = default_schedule(self)
        self._check_schedule_order()
        if self.recompute and self.recompute_stages is None and \
                os.environ.get("WANTRAIN_SELECTIVE_RECOMPUTE") == "on":
            from elysium_wan_b200.scheduler.zero_bubble import selective_recompute

            sel = selective_recompute(self)
            if sel is not None:
                self.recompute_stages = sel
        if self.resume_step is not None and not self.resume:
            raise ValueError("resume_step needs resume")
        return self

    def _check_shared_pacing(self):
        """pacing "shared": a positive egress and ingress rate and a site name
        for every slot, and an uplink rate for both directions of every pair
        of different sites that a connection of this run crosses."""
        import math

        def grid(name):
            v = getattr(self, name)
            if not isinstance(v, list) or [len(row) if isinstance(row, list) else -1
                                           for row in v] != list(self.stage_widths):
                raise ValueError(f"pacing='shared' needs {name}[stage][peer] for every slot")
            return v

        for name in ("peer_egress_mbps", "peer_ingress_mbps"):
            for r, row in enumerate(grid(name)):
                for p, x in enumerate(row):
                    if not (isinstance(x, (int, float)) and math.isfinite(x) and x > 0):
                        raise ValueError(f"pacing='shared': {name}[{r}][{p}]={x!r} is not > 0")
        sites = grid("sites")
        for r, row in enumerate(sites):
            for p, x in enumerate(row):
                if not isinstance(x, str) or not x or "->" in x or ">" in x:
                    raise ValueError(f"pacing='shared': sites[{r}][{p}]={x!r} is not a site name")
        up = self.uplink_mbps if isinstance(self.uplink_mbps, dict) else {}
        pairs = set()
        for r in range(self.stages):
            for p in range(self.stage_widths[r]):
                peers = [(r, q) for q in range(self.stage_widths[r]) if q != p]
                if r + 1 < self.stages:
                    peers += [(r + 1, q) for q in range(self.stage_widths[r + 1])]
                for r2, q in peers:
                    a, b = sites[r][p], sites[r2][q]
                    if a != b:
                        pairs |= {(a, b), (b, a)}
        if self.model.tie_embeddings and self.stages > 1:
            a, b = sites[0][0], sites[-1][0]
            if a != b:
                pairs |= {(a, b), (b, a)}
        for a, b in sorted(pairs):
            x = up.get(f"{a}->{b}")
            if not (isinstance(x, (int, float)) and math.isfinite(x) and x > 0):
                raise ValueError(f"pacing='shared': uplink_mbps[{a + '->' + b!r}] is missing or "
                                 "not > 0")

    def _check_user_model(self):
        """The structural contract of a user model (validation/model_contract.py):
        deterministic build under one seed, stateless deterministic layers."""
        from elysium_wan_b200.models.user import _source
        from elysium_wan_b200.validation.model_contract import validate

        raw = _source(self.model)  # checks the sha256 pin
        target = self.model.to_dict()
        target["example"] = [[i % self.model.vocab_size for i in range(self.model.seq_len)]]
        r = validate(raw.decode(), target)
        if not r["ok"]:
            raise ValueError("user model breaks the contract: " + "; ".join(r["errors"]))
        if r["layers"] != self.model.n_entries:
            raise ValueError(f"user model has {r['layers']} layers, the spec declares "
                             f"{self.model.n_entries} (n_layer + 2)")

    def reschedule(self) -> "JobSpec":
        self.mb_owner = None
        self.schedule_order = None
        return self.finalize()

    def _check_schedule_order(self):
        if len(self.schedule_order) != self.stages:
            raise ValueError("schedule_order needs every stage")
        for r, per_peer in enumerate(self.schedule_order):
            if len(per_peer) != self.stage_widths[r]:
                raise ValueError(f"schedule_order[{r}] needs every peer")
            for p, order in enumerate(per_peer):
                want = self.owned(r, p)
                seen = {op: [] for op in OPS}
                for op, mb in order:
                    if op not in OPS:
                        raise ValueError(f"unknown op {op!r}")
                    seen[op].append(int(mb))
                for op in OPS:
                    if sorted(seen[op]) != want:
                        raise ValueError(f"slot ({r}, {p}): {op} must cover exactly its microbatches")
                # Gradients fold in microbatch order: B and W of a slot run ascending.
                for op in ("B", "W"):
                    if seen[op] != sorted(seen[op]):
                        raise ValueError(f"slot ({r}, {p}): {op} must run in microbatch order")

    def pins(self) -> dict:
        """Fields a checkpoint's bytes depend on; a resume must match them.
        Not pins: ownership, schedule, endpoints, devices, steps, out_dir,
        grad_sync (who computes what and how bytes move never changes a bit)."""
        pins = {
            "model": self.model.to_dict(),
            "init_seed": self.init_seed,
            "data_seed": self.data_seed,
            "dataset_path": self.dataset_path,
            "data_shards": self.data_shards,
            "microbatches": self.microbatches,
            "mb_size": self.mb_size,
            "lr": self.lr,
            "adamw": self.adamw,
            "wire_codec": self.wire_codec,
            "recompute": self.recompute,
            "partition": self.partition,
            "device_types": [sorted({self.device_for(r, p).split(":")[0] for p in range(w)})
                             for r, w in enumerate(self.stage_widths)],
            "zero1_widths": self.stage_widths,
            "fold": self.fold,
        }
        if self.optimizer != "adamw":
            pins["optimizer"] = self.optimizer
        if self.w_pair:
            pins["w_pair"] = True
        if self.dataset_sha256:
            pins["dataset_sha256"] = self.dataset_sha256
        if self.init_from:
            pins["init_sha256"] = self.init_sha256
        return json.loads(json.dumps(pins))

    def to_dict(self) -> dict:
        d = asdict(self)
        d["model"] = self.model.to_dict()
        return d

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), indent=2)

    @staticmethod
    def from_dict(d: dict) -> "JobSpec":
        d = dict(d)
        d["model"] = GPTConfig.from_dict(d.get("model", {}))
        known = set(JobSpec.__dataclass_fields__)
        return JobSpec(**{k: v for k, v in d.items() if k in known})

    @staticmethod
    def from_json(s: str) -> "JobSpec":
        return JobSpec.from_dict(json.loads(s))

    @staticmethod
    def load(path: str) -> "JobSpec":
        with open(path) as f:
            return JobSpec.from_json(f.read())


def first_pin_difference(want: dict, have: dict) -> str | None:
    for k in list(want) + [k for k in have if k not in want]:
        a, b = want.get(k), have.get(k)
        if a == b and (k in want) == (k in have):
            continue
        if isinstance(a, dict) and isinstance(b, dict):
            return f"{k}.{first_pin_difference(a, b)}"
        return k
    return None
