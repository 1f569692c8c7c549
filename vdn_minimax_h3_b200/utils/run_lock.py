"""A RUNNING lock per output directory so two jobs never train into the same place
(reference src/utils/run_lock.py:29-155). The lock records a job id (SLURM_JOB_ID, else
host:pid); a lock whose job has finished (slurm says a terminal state, or the pid is gone
on this host) is stale and may be taken over."""
import json
import os
import socket
import subprocess
import time

LOCK = "RUNNING"
RELEASED_STATES = ("COMPLETED", "FAILED", "CANCELLED", "TIMEOUT", "PREEMPTED", "NODE_FAIL",
                   "OUT_OF_MEMORY", "BOOT_FAIL", "DEADLINE")


def my_job_id():
    return os.environ.get("SLURM_JOB_ID") or f"{socket.gethostname()}:{os.getpid()}"


def _job_alive(job_id, attempts=3):
    if ":" in job_id:
        host, pid = job_id.rsplit(":", 1)
        if host != socket.gethostname():
            return True            # cannot tell from here: treat as alive
        try:
            os.kill(int(pid), 0)
            return True
        except (OSError, ValueError):
            return False
    for _ in range(attempts):
        try:
            out = subprocess.run(["sacct", "-j", job_id, "-n", "-X", "-o", "State"],
                                 capture_output=True, text=True, timeout=20).stdout.split()
            if out:
                return out[0].rstrip("+") not in RELEASED_STATES
        except (OSError, subprocess.SubprocessError):
            time.sleep(1)
    return True


def read_lock(output_dir):
    path = os.path.join(output_dir, LOCK)
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f)


def check(output_dir, job_id=None):
    """None when the directory is free (or locked by us / a dead job); else the holder."""
    job_id = job_id or my_job_id()
    lock = read_lock(output_dir)
    if lock is None or lock.get("job_id") == job_id or not _job_alive(lock.get("job_id", "")):
        return None
    return lock


def acquire(output_dir, job_id=None):
    job_id = job_id or my_job_id()
    holder = check(output_dir, job_id)
    if holder is not None:
        raise RuntimeError(f"{output_dir} is being trained by job {holder['job_id']}")
    os.makedirs(output_dir, exist_ok=True)
    tmp = os.path.join(output_dir, LOCK + ".tmp")
    with open(tmp, "w") as f:
        json.dump({"job_id": job_id, "since": time.time()}, f)
    os.replace(tmp, os.path.join(output_dir, LOCK))
    return job_id


def release(output_dir, job_id=None):
    job_id = job_id or my_job_id()
    lock = read_lock(output_dir)
    if lock is not None and lock.get("job_id") == job_id:
        os.remove(os.path.join(output_dir, LOCK))
