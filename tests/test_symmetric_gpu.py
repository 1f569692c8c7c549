"""The device flag barrier gives up after its time limit and reports it (one GPU, no peers:
the flag of the missing rank is one that nothing sets)."""
import pytest
import torch

from vdn_minimax_h3_b200.ops._ext import KernelError, check_device_error, error_word, ext

pytestmark = pytest.mark.gpu


def test_barrier_single_rank_passes():
    flags = torch.zeros(32, dtype=torch.int64, device="cuda")
    peers = torch.tensor([flags.data_ptr()], dtype=torch.int64, device="cuda")
    for _ in range(3):
        ext().symm_barrier(flags.data_ptr() + 8, flags.data_ptr(), peers, 0, int(1e9),
                           error_word("cuda"))
    torch.cuda.synchronize()
    check_device_error()
    assert flags[0].item() == 3 and flags[1].item() == 3   # my slot, my epoch counter


def test_barrier_times_out_and_context_survives():
    flags = torch.zeros(32, dtype=torch.int64, device="cuda")
    absent = torch.zeros(32, dtype=torch.int64, device="cuda")   # the missing peer's slots
    peers = torch.tensor([flags.data_ptr(), absent.data_ptr()], dtype=torch.int64, device="cuda")
    ext().symm_barrier(flags.data_ptr() + 16, flags.data_ptr(), peers, 0, int(50e6),
                       error_word("cuda"))
    torch.cuda.synchronize()
    with pytest.raises(KernelError, match="peer flag wait timed out"):
        check_device_error()
    assert absent[0].item() == 1          # the flag was published to the peer's slot
    x = torch.arange(10, device="cuda").sum().item()   # the context is still usable
    assert x == 45
    check_device_error()
