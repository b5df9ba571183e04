"""Writing every byte of a buffer through a socket the kernel may briefly
refuse.

A send the kernel refuses for lack of buffer space (ENOBUFS: many workers on
one host can exhaust its socket buffers) or would block on (EAGAIN /
EWOULDBLOCK) wrote nothing, so the same remaining bytes are offered again
after a backoff that starts at 1 ms and doubles up to 100 ms. A send that
makes no progress for 5 s raises its last error, and any other error raises at
once: the peer is then lost as before (the reference's record-layer rule,
src/wantrain/transport/secure.py:97-106, `sendmsg_all`). The native frame
writer (`_wire.send_frame`) follows the same rule in C++.

`WANTRAIN_TEST_ENOBUFS="N"` (N >= 2, the reference's seam) refuses every N-th
send attempt of a sealed socket with ENOBUFS before it reaches the kernel:
timing only, the same bytes leave in the same order, later.
"""

from __future__ import annotations

import errno
import os
import time

RETRY_BUDGET_S = 5.0
RETRY_FIRST_S = 0.001
RETRY_MAX_S = 0.1
TRANSIENT = frozenset({errno.ENOBUFS, errno.EAGAIN, errno.EWOULDBLOCK})


def enobufs_every(value: str | None = None) -> int:
    """The test seam's N (0 when unset)."""
    value = os.environ.get("WANTRAIN_TEST_ENOBUFS", "") if value is None else value
    if value == "":
        return 0
    if not value.isdigit() or int(value) < 2:
        raise ValueError(f"WANTRAIN_TEST_ENOBUFS: {value!r} is not an integer >= 2")
    return int(value)


def send_all(sock, data, before=None) -> None:
    """Write every byte of `data` through `sock` (anything with `send`), in
    order, exactly once; `before()` runs ahead of every attempt (the seam)."""
    view = memoryview(data).cast("B")
    off, n = 0, len(view)
    delay, stalled_since = RETRY_FIRST_S, None
    while off < n:
        try:
            if before is not None:
                before()
            sent = sock.send(view[off:])
        except OSError as e:
            if e.errno not in TRANSIENT:
                raise
            now = time.monotonic()
            if stalled_since is None:
                stalled_since = now
            elif now - stalled_since >= RETRY_BUDGET_S:
                raise
            time.sleep(delay)
            delay = min(2 * delay, RETRY_MAX_S)
            continue
        delay, stalled_since = RETRY_FIRST_S, None
        off += sent
