"""Host-side failure detection for multi-rank runs: heartbeats through the process group's
key-value store.

The reference has no heartbeat (a dead rank surfaces as an NCCL hang until the process-group
timeout). Here every rank runs a `Heartbeat`: a daemon thread that publishes a counter under
`<prefix>/<rank>` every `interval_s` and reads every peer's counter. A peer whose counter
has not advanced for `timeout_s`, or that published the `left` marker (an orderly exit), is
recorded; the training / render loops call `check()` between steps, i.e. before their next
launch or collective, and get a `PeerFailure` naming the ranks instead of entering a
collective that would never complete. Device-side waits have their own bounds (the kernels'
error words); this covers ranks that die or stall on the host.
"""
import threading
import time

import torch.distributed as dist


class PeerFailure(RuntimeError):
    def __init__(self, ranks, reason):
        super().__init__(f"peer rank(s) {sorted(ranks)} {reason}")
        self.ranks = sorted(ranks)
        self.reason = reason


class Heartbeat:
    """Publish this rank's liveness and watch the peers' (see the module docstring)."""

    LEFT = b"left"

    def __init__(self, store=None, rank=None, world=None, interval_s=0.5, timeout_s=5.0,
                 prefix="vdn_hb", clock=time.monotonic):
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store = store
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.interval_s, self.timeout_s = interval_s, timeout_s
        self.prefix = prefix
        self.clock = clock
        self._count = 0
        self._seen = {}            # peer -> (last value, time it changed)
        self._failed = {}          # peer -> reason
        self._stop = threading.Event()
        self._lock = threading.Lock()
        self._thread = None

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def beat(self):
        self._count += 1
        self.store.set(self._key(self.rank), str(self._count))

    def poll(self):
        """Read every peer once; record those that left or went silent for timeout_s."""
        now = self.clock()
        for r in range(self.world):
            if r == self.rank or r in self._failed:
                continue
            try:
                keys = [self._key(r)]
                if not self.store.check(keys):
                    val = None
                else:
                    val = self.store.get(self._key(r))
            except Exception:   # the store itself is gone: the coordinator (rank 0) died
                val = None
            if val == self.LEFT:
                with self._lock:
                    self._failed[r] = "left the run"
                continue
            last = self._seen.get(r)
            if last is None or last[0] != val:
                self._seen[r] = (val, now)
            elif now - last[1] > self.timeout_s:
                with self._lock:
                    self._failed[r] = f"silent for more than {self.timeout_s:.1f} s"

    def _run(self):
        while not self._stop.is_set():
            try:
                self.beat()
            except Exception:
                pass
            self.poll()
            self._stop.wait(self.interval_s)

    def start(self):
        self.beat()
        self._thread = threading.Thread(target=self._run, name="vdn-heartbeat", daemon=True)
        self._thread.start()
        return self

    def failed(self):
        with self._lock:
            return dict(self._failed)

    def check(self):
        """Raise PeerFailure if any peer failed; call between steps."""
        f = self.failed()
        if f:
            reasons = sorted(set(f.values()))
            raise PeerFailure(f.keys(), "; ".join(reasons))

    def leave(self):
        """Orderly exit: stop beating and tell the peers this rank is gone on purpose."""
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval_s + 1)
        try:
            self.store.set(self._key(self.rank), self.LEFT.decode())
        except Exception:
            pass

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval_s + 1)
