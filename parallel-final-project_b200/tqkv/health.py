"""Host-side liveness of the ranks of a multi-GPU decode.

In the NVLink exchange (tqkv.peer) every rank's combine kernel waits, bounded
at about a second, for every other rank's records of the current step.  A
rank that has died or stopped stepping would make the others' combines time
out step after step, each leaving an error code in the device flag and a
meaningless O.  StepMonitor catches that on the host, between steps, before
any kernel of the next step is launched:

    monitor.start()                       # every rank is set up
    for step in range(n):
        monitor.wait_peers(step - 1)      # every peer finished the previous step
        exchange.publish(...); exchange.combine(out)
        torch.cuda.current_stream().synchronize()
        monitor.finished(step)

Each rank posts the last step it finished to a key-value store (the process
group's TCPStore, or any torch.distributed.Store); wait_peers polls the
peers' keys and raises PeerFailure when one has not caught up within the
deadline.  A rank that fails on its own (an exception) posts that with
failed(), so that the others stop at once rather than at the deadline.  No
GPU is involved, so all of this is exercised on CPU ranks
(tests/test_health_gloo.py).
"""
from __future__ import annotations

import time
from typing import Optional


class PeerFailure(RuntimeError):
    """A peer rank stopped stepping (`last_step` is the last step it posted,
    -1 if none) or reported a failure (`reason`)."""

    def __init__(self, rank: int, last_step: int, reason: Optional[str], waited_s: float):
        self.rank, self.last_step, self.reason, self.waited_s = rank, last_step, reason, waited_s
        what = f"reported failure: {reason}" if reason is not None else \
            f"no progress past step {last_step} for {waited_s:.2f} s"
        super().__init__(f"rank {rank} {what}")


class StepMonitor:
    def __init__(self, store, rank: int, world: int, deadline_s: float = 10.0,
                 prefix: str = "tqkv/health", poll_s: float = 0.002):
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside world {world}")
        self.store, self.rank, self.world = store, rank, world
        self.deadline_s, self.poll_s, self.prefix = deadline_s, poll_s, prefix

    def _key(self, kind: str, r: int) -> str:
        return f"{self.prefix}/{kind}/{r}"

    def _read(self, kind: str, r: int) -> Optional[str]:
        key = self._key(kind, r)
        if not self.store.check([key]):
            return None
        return self.store.get(key).decode()

    def start(self, timeout_s: float = 120.0) -> None:
        """Barrier before the first step, so that set-up time (which differs
        between ranks) does not count against the step deadline.  Raises
        PeerFailure naming a rank that has not arrived after `timeout_s`."""
        self.store.set(self._key("started", self.rank), "1")
        t0 = time.monotonic()
        pending = [r for r in range(self.world) if r != self.rank]
        while pending:
            pending = [r for r in pending if self._read("started", r) is None]
            for r in pending:
                reason = self._read("failed", r)
                if reason is not None:
                    raise PeerFailure(r, -1, reason, time.monotonic() - t0)
            if pending and time.monotonic() - t0 > timeout_s:
                raise PeerFailure(pending[0], -1, None, time.monotonic() - t0)
            if pending:
                time.sleep(self.poll_s)

    def finished(self, step: int) -> None:
        """This rank has completed `step` (its O is on the host)."""
        self.store.set(self._key("step", self.rank), str(step))

    def failed(self, reason: str) -> None:
        """This rank is leaving because of an error; peers raise at once."""
        self.store.set(self._key("failed", self.rank), reason or "failed")

    def last_step(self, r: int) -> int:
        v = self._read("step", r)
        return -1 if v is None else int(v)

    def wait_peers(self, step: int) -> None:
        """Return once every peer has finished `step` (no-op for step < 0);
        raise PeerFailure for the first peer that reported a failure, or that
        has not finished `step` when the deadline passes."""
        if step < 0:
            return
        t0 = time.monotonic()
        pending = [r for r in range(self.world) if r != self.rank]
        while True:
            for r in list(pending):
                reason = self._read("failed", r)
                if reason is not None:
                    raise PeerFailure(r, self.last_step(r), reason, time.monotonic() - t0)
                if self.last_step(r) >= step:
                    pending.remove(r)
            if not pending:
                return
            waited = time.monotonic() - t0
            if waited > self.deadline_s:
                r = pending[0]
                raise PeerFailure(r, self.last_step(r), None, waited)
            time.sleep(self.poll_s)
