"""The TCP data plane: stage-to-stage channels for runs across machines.

Reference behaviour: the framed, sealed TCP data plane of
src/wantrain/runtime/stage.py (per-hop flows, fragment reassembly, END
half-close) over transport/framing.py and transport/secure.py. Same interface
as parallel/p2p.PipeComm, so the engine does not know which plane it runs on:

- every slot listens on its endpoint (spec.endpoints[stage][peer] =
  [host, data_port, bind_port], else spec.host : port_base + 1000 + rank);
  the lower stage dials each slot of the next stage with `p2p_streams`
  flows, says HELLO, and every flow is sealed after an identity handshake
  (ed25519 + X25519, transport/identity.py), admission by `trusted_peers`;
- a boundary tensor leaves through the spec's wire codec (raw, planes,
  f32_planes, fp8_planes; the e4m3_b128 pair as one PLANES payload), cut into
  one fragment per flow, and is reassembled by concatenation: codecs and
  fragments never change a bit;
- one sender thread per destination slot keeps sends asynchronous (flush()
  waits for them), one reader thread per flow files whole frames by
  (type, microbatch); a WAN shim per outgoing link can pace and delay sends
  for experiments (latency, rate, jitter).

The replicas of a wide stage are joined by sealed links of their own (a
full mesh: each replica dials the higher-numbered ones), over which the
ZeRO-1 / pieces exchange runs (`StageMesh`: the partials' scatter to their
owners, the updated shards' gather, integer sums such as MoE expert counts);
the first and last stages of a tied-embedding run get a sealed link for the
table relay. So every byte between machines crosses the sealed plane; the
gloo group is kept only for process-group plumbing.

Device tensors cross through host memory (a device->host copy before the
send, a host->device copy after the receive).
"""

from __future__ import annotations

import collections
import queue
import socket
import threading
import time

import torch

from elysium_wan_b200.models.gpt import Act
from elysium_wan_b200.transport.pacer import pair_link, reverse_link
from elysium_wan_b200.transport import framing
from elysium_wan_b200.transport.framing import BWD, END, FWD, GRADS, HELLO, PARAMS, TIED

# The `mb` field of a mesh frame names the exchange it belongs to (its `chunk`
# field names the sending replica).
MESH_SCATTER, MESH_GATHER, MESH_SUM = 0, 1, 2


def slot_endpoint(spec, stage: int, peer: int) -> tuple[str, int]:
    if spec.endpoints:
        host, port = spec.endpoints[stage][peer][0], int(spec.endpoints[stage][peer][1])
        return host, port
    return spec.host, spec.port_base + 1000 + spec.rank_of(stage, peer)


class _Inbox:
    def __init__(self):
        self.cv = threading.Condition()
        self.q: dict = collections.defaultdict(collections.deque)
        self.err: Exception | None = None

    def put(self, key, frame):
        with self.cv:
            self.q[key].append(frame)
            self.cv.notify_all()

    def fail(self, e):
        with self.cv:
            if self.err is None:
                self.err = e
            self.cv.notify_all()

    def get(self, key, timeout):
        end = time.monotonic() + timeout
        with self.cv:
            while not self.q[key]:
                if self.err is not None:
                    raise ConnectionError(f"peer connection lost: {self.err}")
                left = end - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"no frame {key} within {timeout:.0f}s")
                self.cv.wait(min(left, 1.0))
            return self.q[key].popleft()


class _Link:
    """The flows to one neighbour slot and the thread that sends on them."""

    def __init__(self, comm, socks, link_cfg: dict, wire_codec: str | None = None):
        from elysium_wan_b200.parallel.p2p import _Shim

        self.comm, self.socks = comm, socks
        self.wire_codec = wire_codec or comm.wire_codec
        self.frag_size = 0  # 0: one fragment per flow; else the adapted fragment size
        self.clean = 0
        self.q: queue.Queue = queue.Queue()
        self.err: Exception | None = None
        self.shim = _Shim(link_cfg or {}, comm.spec.tag)
        # what this link has sent: whole frames, payload bytes, and the time
        # its sender spent on them (pacing included) -> per-hop telemetry
        self.stats = {"frames": 0, "bytes": 0, "busy_ms": 0.0}
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    def submit(self, item):
        self.q.put(item)

    def _send_frame(self, ftype, step, mb, tensors):
        c = self.comm
        # an fp8 boundary is the (codes, scales) pair: one frame, one payload
        payload_t = tuple(tensors) if len(tensors) > 1 else tensors[0]
        codec_id, payload, shape = framing.encode_tensor(payload_t, self.wire_codec)
        if self.frag_size:
            # adapted size: fragments taken round-robin by the flows
            n = max(1, -(-len(payload) // self.frag_size))
            frags = [payload[i * self.frag_size:(i + 1) * self.frag_size] for i in range(n)] or [b""]
        else:
            frags = framing.fragments(payload, len(self.socks))
        t0 = time.monotonic()
        for i, part in enumerate(frags):
            framing.send_frame(self.socks[i % len(self.socks)], ftype, step, mb, part, chunk=c.peer,
                               codec_id=codec_id, shape=shape, frag_idx=i, frag_cnt=len(frags))
        self._adapt((time.monotonic() - t0) / len(frags), len(frags[0]), len(payload))
        return len(payload)

    def _adapt(self, per_frag_s: float, size: int, total: int):
        """Fragment-size adaptation (reference: the sender loop of
        src/wantrain/runtime/stage.py:2032-2105, semantics only): a fragment
        slower than the budget halves the size, down to frag_min_bytes; eight
        frames in a row under a quarter of it double the size back, up to
        whole frames (the flows' default split)."""
        spec = self.comm.spec
        budget = float(spec.adapt_budget_ms) / 1e3
        if budget <= 0 or total <= 0:
            return
        floor = max(1, int(spec.frag_min_bytes))
        if per_frag_s > budget and size > floor:
            self.frag_size = max(floor, size // 2)
            self.clean = 0
        elif per_frag_s < budget / 4 and self.frag_size:
            self.clean += 1
            if self.clean >= 8:
                self.frag_size = self.frag_size * 2 if self.frag_size * 2 < total else 0
                self.clean = 0

    def _loop(self):
        while True:
            item = self.q.get()
            try:
                if item is None:
                    return
                ftype, step, mb, tensors = item
                nbytes = sum(t.numel() * t.element_size() for t in tensors)
                t0 = time.monotonic()
                if self.shim.active:
                    self.shim.submit(lambda: self._send_frame(ftype, step, mb, tensors), nbytes)
                    self.shim.flush()
                else:
                    self._send_frame(ftype, step, mb, tensors)
                st = self.stats
                st["frames"], st["bytes"] = st["frames"] + 1, st["bytes"] + nbytes
                st["busy_ms"] += (time.monotonic() - t0) * 1e3
            except Exception as e:  # surfaced on the next flush / send
                self.err = e
            finally:
                self.q.task_done()

    def flush(self):
        self.q.join()
        if self.err is not None:
            raise ConnectionError(f"peer connection lost: {self.err}")

    def close(self):
        try:
            self.flush()
            for s in self.socks:
                framing.send_end(s)
        except (OSError, ConnectionError):
            pass
        self.q.put(None)
        self.shim.close()


class TcpPipeComm:
    def __init__(self, spec, stage: int, peer: int, device, timeout_s: float = 300.0,
                 key_path: str | None = None):
        from elysium_wan_b200.transport import identity

        self.spec, self.stage, self.peer = spec, stage, peer
        self.device = torch.device(device)
        self.rank = spec.rank_of(stage, peer)
        self.timeout = timeout_s
        self.wire_codec = spec.wire_codec if spec.wire_codec != "native" else "raw"
        # The wide-stage exchange and the tied relay run on this plane's own
        # sealed links (StageMesh, the tied link); no process group carries
        # their bytes.
        self.g_stage = None
        cfg = spec.model
        self.T, self.d = spec.mb_size * cfg.seq_len, cfg.d_model
        self.cuda = self.device.type == "cuda"
        from elysium_wan_b200 import ops

        self.q8 = ops.q8_dtype(cfg.boundary_dtype)  # fp8 boundary: its dtype, else None
        self.fp8 = self.q8 is not None
        self.act_dtype = ops.act_dtype(cfg.boundary_dtype, self.cuda)  # dense boundary activations
        self.grad_dtype = torch.bfloat16 if self.cuda else torch.float32  # boundary gradients
        self.key = identity.load_or_create_key(key_path)
        self.trusted = spec.trusted_peers
        self.inbox = _Inbox()
        self.readers: list = []
        self.next_links: dict = {}  # peer of stage + 1 -> _Link
        self.prev_links: dict = {}  # peer of stage - 1 -> _Link
        self.mesh = None            # StageMesh of a wide stage
        self.tied_link = None       # the table relay's link (first <-> last stage)
        self.tied_seq = 0
        self.sent = collections.Counter()
        self.bytes_sent = 0
        self.frames = 0
        self.peers_seen: dict = {}
        self.tuning: dict = {}
        self._connect()

    # ----------------------------------------------------------------- setup
    def _seal(self, sock, role):
        from elysium_wan_b200.transport import identity, secure

        sock.settimeout(self.timeout)
        sess = identity.authenticate(sock, self.key, role, identity.P2P_DOMAIN,
                                     trusted_peers=self.trusted)
        sock.settimeout(None)
        return secure.SecureSocket(sock, sess)

    def _connect(self):
        spec, S = self.spec, self.spec.stages
        flows = max(1, int(spec.p2p_streams))
        width = spec.stage_widths[self.stage]
        n_prev = spec.stage_widths[self.stage - 1] * flows if self.stage > 0 else 0
        # a wide stage's mesh: the lower-numbered replicas dial this one
        n_mesh = self.peer if width > 1 else 0
        tied = bool(spec.model.tie_embeddings) and S > 1
        n_tied = 1 if tied and self.stage == S - 1 else 0
        n_in = n_prev + n_mesh + n_tied
        lsock = None
        if n_in:
            host, port = slot_endpoint(spec, self.stage, self.peer)
            bind = spec.endpoints[self.stage][self.peer][2] if spec.endpoints and \
                len(spec.endpoints[self.stage][self.peer]) > 2 and \
                spec.endpoints[self.stage][self.peer][2] else port
            lsock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
            lsock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            from elysium_wan_b200.transport import tuning

            self.tuning = tuning.tune(lsock)  # accepted flows inherit it
            lsock.bind(("0.0.0.0" if host not in ("127.0.0.1", "localhost") else host, int(bind)))
            lsock.listen(n_in + 4)
        accepted: dict = collections.defaultdict(dict)
        mesh_in: dict = {}
        tied_in: list = []
        acc_err: list = []

        def accept_all():
            try:
                lsock.settimeout(self.timeout)
                for _ in range(n_in):
                    c, _ = lsock.accept()
                    c.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
                    sc = self._seal(c, "listener")
                    hello = framing.recv_frame(sc)
                    if hello.type != HELLO:
                        raise framing.FrameError("expected HELLO")
                    h = hello.obj()
                    kind = h.get("link", "chain")
                    if kind == "mesh" and h.get("stage") == self.stage and \
                            0 <= int(h["peer"]) < self.peer and int(h["peer"]) not in mesh_in:
                        mesh_in[int(h["peer"])] = sc
                    elif kind == "tied" and n_tied and h.get("stage") == 0 and not tied_in:
                        tied_in.append(sc)
                    elif kind == "chain" and h.get("stage") == self.stage - 1:
                        accepted[int(h["peer"])][int(h["flow"])] = sc
                    else:
                        raise framing.FrameError(f"unexpected HELLO {h}")
                    self.peers_seen[f"{h['stage']}:{h['peer']}"] = sc.peer
            except Exception as e:
                acc_err.append(e)

        t_acc = threading.Thread(target=accept_all, daemon=True) if n_in else None
        if t_acc:
            t_acc.start()
        if self.stage + 1 < S:
            for q in range(spec.stage_widths[self.stage + 1]):
                host, port = slot_endpoint(spec, self.stage + 1, q)
                socks = []
                for f in range(flows):
                    s = self._dial(host, port)
                    sc = self._seal(s, "dialer")
                    framing.send_frame(sc, HELLO, 0, 0, {"stage": self.stage, "peer": self.peer,
                                                          "flow": f})
                    self.peers_seen[f"{self.stage + 1}:{q}"] = sc.peer
                    socks.append(sc)
                link = spec.links[self.stage] if self.stage < len(spec.links) else {}
                link = pair_link(spec, link, (self.stage, self.peer), (self.stage + 1, q))
                self.next_links[q] = _Link(self, socks, link)
                self._start_readers(socks)
        # the exchange runs on a lossless codec whatever the boundary's
        exch = "raw" if self.wire_codec == "raw" else "planes"
        mesh_out = {}
        for q in range(self.peer + 1, width) if width > 1 else ():
            sc = self._dial_sealed(self.stage, q, {"link": "mesh"})
            mesh_out[q] = sc
        tied_out = None
        if tied and self.stage == 0 and self.peer == 0:
            tied_out = self._dial_sealed(S - 1, 0, {"link": "tied"})
        if t_acc:
            t_acc.join(self.timeout + 5)
            lsock.close()
            if acc_err:
                raise ConnectionError(f"data plane accept failed: {acc_err[0]}")
            back = spec.links[self.stage - 1] if self.stage - 1 < len(spec.links) else {}
            for p in range(spec.stage_widths[self.stage - 1]) if self.stage > 0 else ():
                socks = [accepted[p][f] for f in range(flows)]
                cfg = pair_link(spec, reverse_link(back), (self.stage, self.peer),
                                (self.stage - 1, p))
                self.prev_links[p] = _Link(self, socks, cfg)
                self._start_readers(socks)
        if width > 1:
            links = {}
            for q, sc in sorted({**mesh_in, **mesh_out}.items()):
                own = (spec.mesh_links[self.stage] or {}).get(f"{self.peer}>{q}", {}) \
                    if spec.mesh_links else {}
                cfg = pair_link(spec, own, (self.stage, self.peer), (self.stage, q))
                links[q] = _Link(self, [sc], cfg, wire_codec=exch)
                self._start_readers([sc], key=lambda f: ("mesh", f.type, f.mb, f.chunk))
            if sorted(links) != [q for q in range(width) if q != self.peer]:
                raise ConnectionError(f"stage mesh incomplete: links to {sorted(links)}")
            self.mesh = StageMesh(self, links)
        sc = tied_out or (tied_in[0] if tied_in else None)
        if sc is not None:
            other = (S - 1, 0) if self.stage == 0 else (0, 0)
            cfg = pair_link(spec, {}, (self.stage, self.peer), other)
            self.tied_link = _Link(self, [sc], cfg, wire_codec=exch)
            self._start_readers([sc], key=lambda f: ("tied", f.type))

    def _dial_sealed(self, stage: int, peer: int, hello: dict):
        """One sealed flow to slot (stage, peer), announced by a HELLO."""
        host, port = slot_endpoint(self.spec, stage, peer)
        sc = self._seal(self._dial(host, port), "dialer")
        framing.send_frame(sc, HELLO, 0, 0, dict(hello, stage=self.stage, peer=self.peer, flow=0))
        self.peers_seen[f"{stage}:{peer}"] = sc.peer
        return sc

    def _dial(self, host, port):
        from elysium_wan_b200.transport import tuning

        end = time.monotonic() + self.timeout
        while True:
            try:
                s, applied = tuning.connect(host, port, 5.0)
                self.tuning = applied
                return s
            except OSError:
                if time.monotonic() > end:
                    raise
                time.sleep(0.05)

    def _start_readers(self, socks, key=None):
        """One reader thread per flow of a link. A frame's fragments travel on
        different flows (one each), so the link's flows share one reassembler.
        `key(frame)` files a whole frame in the inbox (default: type and
        microbatch)."""
        re = framing.Reassembler()
        lock = threading.Lock()
        key = key or (lambda f: (f.type, f.mb))

        def loop(sock):
            try:
                while True:
                    f = framing.recv_frame(sock)
                    if f.type == END:
                        return
                    with lock:
                        whole = re.push(f)
                    if whole is not None:
                        self.inbox.put(key(whole), whole)
            except Exception as e:
                self.inbox.fail(e)

        for sock in socks:
            t = threading.Thread(target=loop, args=(sock,), daemon=True)
            t.start()
            self.readers.append(t)

    # ----------------------------------------------------------------- routing
    def next_peer(self, mb: int) -> int:
        return self.spec.mb_owner[self.stage + 1][mb]

    def prev_peer(self, mb: int) -> int:
        return self.spec.mb_owner[self.stage - 1][mb]

    # ----------------------------------------------------------------- sends
    def _host(self, t):
        return t.detach().to("cpu", copy=True).contiguous()

    def send_act(self, mb: int, act: Act):
        if act.fp8:
            ts = [self._host(act.x), self._host(act.scale)]
        else:
            ts = [self._host(act.x.to(self.act_dtype))]
        self._enqueue(self.next_links[self.next_peer(mb)], FWD, mb, ts)
        return []

    def send_grad(self, mb: int, g: torch.Tensor):
        self._enqueue(self.prev_links[self.prev_peer(mb)], BWD, mb,
                      [self._host(g.to(self.grad_dtype))])
        return []

    def _enqueue(self, link, ftype, mb, tensors):
        if link.err is not None:
            raise ConnectionError(f"peer connection lost: {link.err}")
        step = self.sent[(ftype, mb)]
        self.sent[(ftype, mb)] += 1
        self.bytes_sent += sum(t.numel() * t.element_size() for t in tensors)
        self.frames += 1
        link.submit((ftype, step, mb, tensors))

    # ----------------------------------------------------------------- receives
    def irecv_act(self, mb: int):
        return (FWD, mb)

    def irecv_grad(self, mb: int):
        return (BWD, mb)

    def ready(self, handle) -> bool:
        """Whether the frame a receive waits for has arrived (never blocks)."""
        with self.inbox.cv:
            return bool(self.inbox.q[handle]) or self.inbox.err is not None

    def wait(self, handle):
        f = self.inbox.get(handle, self.timeout)
        t = f.tensor()
        if isinstance(t, tuple):
            return [t[0].to(self.device), t[1].to(self.device)]
        return [t.to(self.device)]

    def as_act(self, bufs) -> Act:
        if self.fp8:
            return Act(bufs[0].view(self.q8), bufs[1])
        return Act(bufs[0])

    def tied_send(self, t):
        """The table relay over its sealed link (fp32, lossless codec)."""
        self.tied_seq += 1
        self._enqueue(self.tied_link, TIED, 0, [self._host(t.float())])

    def tied_recv(self, buf):
        f = self.inbox.get(("tied", TIED), self.timeout)
        buf.copy_(f.tensor().view_as(buf).to(buf.device))

    def link_stats(self) -> dict:
        """Cumulative per-link send statistics, labelled by direction and
        peer (next<q>, prev<p>, mesh<q>, tied)."""
        out = {f"next{q}": dict(l.stats) for q, l in self.next_links.items()}
        out.update({f"prev{p}": dict(l.stats) for p, l in self.prev_links.items()})
        if self.mesh is not None:
            out.update({f"mesh{q}": dict(l.stats) for q, l in self.mesh.links.items()})
        if self.tied_link is not None:
            out["tied"] = dict(self.tied_link.stats)
        return out

    def _links(self) -> list:
        out = list(self.next_links.values()) + list(self.prev_links.values())
        out += list(self.mesh.links.values()) if self.mesh is not None else []
        return out + ([self.tied_link] if self.tied_link is not None else [])

    def flush(self):
        for link in self._links():
            link.flush()

    def close(self):
        for link in self._links():
            link.close()


class StageMesh:
    """The ZeRO-1 / pieces exchange of a wide stage over its sealed mesh
    links; the same calls, equal splits and results as the torch.distributed
    collectives it replaces on this plane (every part is exact: the links
    carry fp32 and int64 losslessly, and sums run in rank order)."""

    def __init__(self, comm, links: dict):
        self.comm, self.links = comm, links
        self.k = comm.peer
        self.w = len(links) + 1

    def _send(self, q: int, ftype: int, kind: int, t):
        self.comm._enqueue(self.links[q], ftype, kind, [self.comm._host(t)])

    def _recv(self, q: int, ftype: int, kind: int):
        return self.comm.inbox.get(("mesh", ftype, kind, q), self.comm.timeout).tensor()

    def all_to_all_single(self, recv, send):
        """Part q of `send` goes to replica q; part q of `recv` comes from it."""
        n = send.numel() // self.w
        for q in self.links:
            self._send(q, GRADS, MESH_SCATTER, send[q * n:(q + 1) * n])
        recv[self.k * n:(self.k + 1) * n].copy_(send[self.k * n:(self.k + 1) * n])
        for q in sorted(self.links):
            recv[q * n:(q + 1) * n].copy_(self._recv(q, GRADS, MESH_SCATTER).reshape(-1))

    def all_gather_into_tensor(self, out, mine):
        n = mine.numel()
        for q in self.links:
            self._send(q, PARAMS, MESH_GATHER, mine)
        out[self.k * n:(self.k + 1) * n].copy_(mine.reshape(-1))
        for q in sorted(self.links):
            out[q * n:(q + 1) * n].copy_(
                self._recv(q, PARAMS, MESH_GATHER).reshape(-1).to(out.dtype))

    def all_reduce_sum(self, t):
        """t (in place) = the replicas' t summed in rank order."""
        for q in self.links:
            self._send(q, GRADS, MESH_SUM, t)
        parts = {q: self._recv(q, GRADS, MESH_SUM).view_as(t).to(t.device)
                 for q in sorted(self.links)}
        parts[self.k] = t.clone()
        acc = parts[0].clone()
        for q in range(1, self.w):
            acc += parts[q]
        t.copy_(acc)
