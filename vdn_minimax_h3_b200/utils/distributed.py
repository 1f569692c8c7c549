"""Rank-0 init semantics and a bitwise cross-rank proof, before sharding (reference
src/utils/distributed.py:6-33): broadcast the freshly initialised trainables from rank 0,
then compare an fp64 fingerprint of EVERY parameter and raise on any mismatch."""
import torch
import torch.distributed as dist


def fingerprint(model, device):
    return torch.tensor([p.detach().double().sum().item() for _, p in model.named_parameters()],
                        dtype=torch.float64, device=device)


def broadcast_and_verify_init(model, params_to_broadcast, device):
    for p in params_to_broadcast:
        t = p.data.to(device)
        dist.broadcast(t, src=0)
        p.data.copy_(t.to(p.data.device))
    names = [n for n, _ in model.named_parameters()]
    sums = fingerprint(model, device)
    ref = sums.clone()
    dist.broadcast(ref, src=0)
    bad = (sums != ref).nonzero().flatten().tolist()
    if bad:
        raise RuntimeError(f"rank {dist.get_rank()}: {len(bad)} parameters differ from rank 0 "
                           f"before sharding, e.g. {[names[i] for i in bad[:5]]}")
