"""The output head under sequence parallelism: each rank runs norm_out + proj_out (and the
audio projection) on the video / audio rows it already owns, and only those outputs are
gathered -- never the residual stream.

The reference all-gathers the whole [T, 5376] residual and every rank then runs the head on
all T rows, text rows included (src/inference/utils/ulysses_runtime.py:478-495, then the
model's norm_out / proj_out). The head is row-wise, so the same result comes from each rank
projecting its own rows: the gathered bytes drop from T x 5376 bf16 (1.1 GB at H3 scale) to
the video and audio output channels (~20 MB), and no rank projects text rows.
"""
import weakref
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist


class ShardedHead:
    """bounds[p] = (first, end) packed rows owned by rank p (contiguous, ascending)."""

    def __init__(self, group=None):
        self.group = group
        self._plans = {}

    def _plan(self, indices: torch.Tensor, bounds: Sequence[Tuple[int, int]]):
        """Per-rank (first, end) positions in `indices` of the rows each rank owns. Cached
        per index TENSOR (held weakly, checked against its in-place version counter), so a
        later request whose indices reuse the same memory is never served stale cuts."""
        bounds = tuple(tuple(b) for b in bounds)
        entry = self._plans.get(id(indices))
        if (entry is not None and entry[0]() is indices and entry[1] == indices._version
                and entry[2] == bounds):
            return entry[3]
        if indices.numel() > 1 and not bool((indices[1:] > indices[:-1]).all()):
            raise ValueError("sharded head needs ascending output row indices")
        edges = torch.tensor([b[0] for b in bounds] + [bounds[-1][1]], device=indices.device,
                             dtype=indices.dtype)
        cuts = torch.searchsorted(indices, edges).tolist()        # one small D2H per new tensor
        plan = [(cuts[p], cuts[p + 1]) for p in range(len(bounds))]
        self._plans = {k: v for k, v in self._plans.items() if v[0]() is not None}
        self._plans[id(indices)] = (weakref.ref(indices), indices._version, bounds, plan)
        return plan

    def _gather(self, local: torch.Tensor, spans: List[Tuple[int, int]]) -> torch.Tensor:
        counts = [b - a for a, b in spans]
        width = max(counts) if counts else 0
        P = len(spans)
        pad = local.new_zeros(width, local.shape[-1])
        pad[:local.shape[0]].copy_(local)
        full = local.new_empty(P * width, local.shape[-1])
        dist.all_gather_into_tensor(full, pad, group=self.group)
        parts = [full[p * width:p * width + counts[p]] for p in range(P)]
        return torch.cat(parts) if parts else full[:0]

    def __call__(self, model, x_local, bounds, rank, temb, timestep_indices, video_indices,
                 audio_indices):
        """x_local: this rank's residual rows bounds[rank]; returns (video [1, Nv, Cv],
        audio [1, Na, Ca]) identical on every rank, ordered like the index tensors."""
        row0 = bounds[rank][0]
        tidx = timestep_indices
        outs = []
        for indices, proj, channels in ((video_indices, model.proj_out, None),
                                        (audio_indices, getattr(model, "audio_proj_out", None),
                                         model.config.audio_in_channels)):
            if indices.numel() == 0 or proj is None:
                outs.append(x_local.new_zeros(1, 0, channels or model.proj_out.out_features))
                continue
            spans = self._plan(indices, bounds)
            a, b = spans[rank]
            rows = indices[a:b]
            h = model.norm_out(x_local.index_select(0, rows - row0).unsqueeze(0), temb,
                               tidx.index_select(0, rows)).to(proj.weight.dtype)
            local = proj(h)[0]
            outs.append(self._gather(local.contiguous(), spans).unsqueeze(0))
        return outs[0], outs[1]
