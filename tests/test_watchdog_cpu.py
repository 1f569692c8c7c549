"""Host-side failure detection on gloo ranks (no GPU): a rank that goes silent, leaves, or
dies is reported to the others by the heartbeat before their next collective."""
import os
import queue
import socket
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from vdn_minimax_h3_b200.utils.watchdog import Heartbeat, PeerFailure


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    hb = Heartbeat(interval_s=0.1, timeout_s=1.0).start()
    try:
        dist.barrier()
        if mode == "healthy":
            time.sleep(1.5)
            hb.check()
            dist.barrier()
            hb.stop()
            q.put((rank, "ok"))
            return
        victim = world - 1
        if rank == victim:
            if mode == "silent":
                hb.stop()              # alive but no longer beating (a host-side hang)
                time.sleep(3.0)
            elif mode == "leave":
                hb.leave()
            elif mode == "die":
                os._exit(3)            # abrupt exit, nothing cleaned up
            q.put((rank, "victim"))
            return
        t0 = time.monotonic()
        while time.monotonic() - t0 < 10:
            try:
                hb.check()             # between steps: before the next collective
            except PeerFailure as exc:
                q.put((rank, (exc.ranks, exc.reason)))
                hb.stop()
                return
            time.sleep(0.05)
        q.put((rank, "not detected"))
    finally:
        # os._exit skips the queue's feeder thread: flush the result before leaving
        q.close()
        q.join_thread()
        if mode == "healthy":
            dist.destroy_process_group()
        else:
            os._exit(0)                # the group is broken; leave without collectives


@pytest.mark.timeout(120)
@pytest.mark.parametrize("mode", ["healthy", "silent", "leave", "die"])
def test_heartbeat(mode):
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    expected = world - 1 if mode == "die" else world
    deadline = time.monotonic() + 60
    while len(res) < expected and time.monotonic() < deadline:
        try:
            r, v = q.get(timeout=1.0)
        except queue.Empty:
            continue
        res[r] = v
    for p in procs:
        p.join(timeout=30)
    if mode == "healthy":
        assert res == {0: "ok", 1: "ok", 2: "ok"}, res
        return
    for r in (0, 1):
        ranks, reason = res[r]
        assert ranks == [2], res
        assert ("left" in reason) if mode == "leave" else ("silent" in reason), res


def test_poll_logic_with_fake_store():
    """Deterministic clock: silence is reported only after timeout_s without a change."""
    class Store:
        def __init__(self):
            self.kv = {}

        def set(self, k, v):
            self.kv[k] = v.encode() if isinstance(v, str) else v

        def get(self, k):
            return self.kv[k]

        def check(self, keys):
            return all(k in self.kv for k in keys)

    now = [0.0]
    st = Store()
    hb = Heartbeat(store=st, rank=0, world=2, timeout_s=2.0, clock=lambda: now[0])
    st.set("vdn_hb/1", "1")
    hb.poll()
    now[0] = 1.5
    hb.poll()
    hb.check()
    st.set("vdn_hb/1", "2")
    now[0] = 3.0
    hb.poll()
    hb.check()                         # changed: fresh again
    now[0] = 5.5
    hb.poll()
    with pytest.raises(PeerFailure):
        hb.check()
