"""Block-streamed inference (inference/offload.py) on CPU: the engine with its blocks kept on
the host and brought in per block gives the same output as the resident engine, two model
evaluations in a row, and the packed weights keep aliasing the module weights on each trip."""
import copy

import torch

from tests.test_model_cpu import _forward_inputs, tiny_model
from vdn_minimax_h3_b200.inference.engine import InferenceEngine
from vdn_minimax_h3_b200.inference.offload import enable_block_offload
from vdn_minimax_h3_b200.inference.render import render_geometry
from vdn_minimax_h3_b200.models.h3 import h3_tiny_config
from vdn_minimax_h3_b200.models.hybrid_transform import set_layout


@torch.no_grad()
def test_block_offload_matches_resident_engine():
    cfg = h3_tiny_config()
    model = tiny_model()
    geo = render_geometry(cfg, 5, latent_h=16, latent_w=16, audio=False, num_latent_frames=4)
    kw, layout = _forward_inputs(cfg, geo, 32)
    set_layout(model, layout)
    ref_v, _ = InferenceEngine(copy.deepcopy(model))(**kw, layout=layout)

    eng = InferenceEngine(copy.deepcopy(model))
    streamer = enable_block_offload(eng, "cpu")
    assert enable_block_offload(eng) is streamer
    assert streamer.host_bytes() > 0 and not any(b.resident for b in streamer.blocks)
    seen = []
    acquire = streamer.acquire

    def spy(i):
        acquire(i)
        pb, blk = eng.blocks[i], eng.model.transformer_blocks[i]
        q = blk.attn.orig.to_q.weight
        # the module's to_q weight is still a view of the packed QKV weight
        seen.append(q.untyped_storage().data_ptr() == pb.w_qkvg.untyped_storage().data_ptr())
        assert streamer.blocks[i].resident

    streamer.acquire = spy
    for _ in range(2):
        out_v, _ = eng(**kw, layout=layout)
        torch.testing.assert_close(out_v, ref_v, rtol=0, atol=0)
    assert seen and all(seen)
    # only block 0 stays resident: prefetched for the next model evaluation
    assert [b.resident for b in streamer.blocks] == [True] + [False] * (len(streamer.blocks) - 1)


def test_module_offload_keeps_tied_tensors_and_outputs():
    """Eager block streaming (forward hooks): a parameter tied between two blocks stays
    resident (never re-pointed), every other block tensor lives on its host copy between
    forwards, and the outputs equal the resident model's."""
    import torch
    import torch.nn as nn
    from vdn_minimax_h3_b200.inference.offload import enable_module_offload

    class Blocks(nn.Module):
        def __init__(self):
            super().__init__()
            self.transformer_blocks = nn.ModuleList(nn.Linear(8, 8) for _ in range(3))
            self.transformer_blocks[2].weight = self.transformer_blocks[0].weight   # tied

        def forward(self, x):
            for b in self.transformer_blocks:
                x = torch.tanh(b(x))
            return x

    torch.manual_seed(0)
    m = Blocks()
    x = torch.randn(4, 8)
    want = m(x)
    tied = m.transformer_blocks[0].weight
    streamer = enable_module_offload(m, torch.device("cpu"))
    assert enable_module_offload(m, torch.device("cpu")) is streamer           # idempotent
    for _ in range(2):
        torch.testing.assert_close(m(x), want, rtol=0, atol=0)
    assert m.transformer_blocks[0].weight is tied
    assert streamer.host_bytes() == sum(b.nbytes() for b in streamer.blocks) > 0
    # the tied weight is in no block's streamed groups
    key = tied.untyped_storage().data_ptr()
    for b in streamer.blocks:
        assert all(k[2] != key for k in b.groups)
