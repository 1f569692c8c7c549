"""Resumable sampler: re-enters an epoch at a data cursor without loading the samples
before it, so a resumed run sees exactly the order an uninterrupted run would have.

Behaviour parity: src/utils/samplers.py (the reference's `SkipFirst`): the wrapped sampler
is still iterated from its start (its permutation is a function of seed and epoch), only the
first `skip` indices are dropped.
"""
import itertools

import torch


class SkipFirst(torch.utils.data.Sampler):
    """Wraps `sampler`; the next pass drops its first `skip` indices. `skip` stays set
    until the caller clears it (the trainer clears it when the resumed epoch ends), and
    `set_epoch` is forwarded so a DistributedSampler keeps reshuffling per epoch."""

    def __init__(self, sampler, skip: int = 0):
        self.sampler = sampler
        self.skip = int(skip)

    def set_epoch(self, epoch: int) -> None:
        if hasattr(self.sampler, "set_epoch"):
            self.sampler.set_epoch(epoch)

    def __iter__(self):
        return itertools.islice(iter(self.sampler), max(self.skip, 0), None)

    def __len__(self):
        return max(len(self.sampler) - max(self.skip, 0), 0)
