"""The lr schedule as a pure function of the step (linear warm-up, cosine to min_lr), the
schedule stamp stored in a train state, and the loud-but-non-fatal check on resume.
Reference parity: src/utils/lr_schedule.py:13-64."""
import math
from types import SimpleNamespace

SCHEDULE_ARGS = ("lr", "min_lr", "warmup_steps", "max_steps")


def lr_at(step, args):
    if step < args.warmup_steps:
        return args.lr * (step + 1) / args.warmup_steps
    progress = (step - args.warmup_steps) / max(args.max_steps - args.warmup_steps, 1)
    return args.min_lr + 0.5 * (args.lr - args.min_lr) * (1 + math.cos(math.pi * progress))


def schedule_sum(ran_steps, lr, min_lr, warmup_steps, max_steps):
    a = SimpleNamespace(lr=lr, min_lr=min_lr, warmup_steps=warmup_steps, max_steps=max_steps)
    return sum(lr_at(s, a) for s in range(ran_steps))


def schedule_stamp(args):
    return {k: getattr(args, k) for k in SCHEDULE_ARGS if hasattr(args, k)}


def check_schedule_stamp(saved, args, rank=0, step=0):
    """Returns the changed keys (and prints a banner on rank 0); never raises."""
    if not saved:
        return {}
    now = schedule_stamp(args)
    diff = {k: (saved.get(k), now.get(k)) for k in now if saved.get(k) != now.get(k)}
    if diff and rank == 0:
        print("=" * 78 + "\nWARNING: lr schedule args CHANGED across this resume:", flush=True)
        for k, (a, b) in diff.items():
            print(f"    {k}: {a} -> {b}", flush=True)
        old = SimpleNamespace(**{**now, **saved})
        print(f"    lr at the resume step ({step}): {lr_at(step, old):.3e} -> {lr_at(step, args):.3e}\n"
              + "=" * 78, flush=True)
    return diff
