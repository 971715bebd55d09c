"""imi_peer_allgather on one GPU: a one-rank exchange copies its block and
advances its epoch on every call; in a two-rank exchange whose second rank
never arrives (its flag word is never written), the wait for it runs out
after its bound, bit 0 of status is set, the present rank's block is still
copied and the kernel returns (nothing hangs)."""
import ctypes

import pytest
import torch

from adaptiveimi_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _gather(world, rank, nbytes, src_ptrs, flag_ptrs, counters, dst, status):
    dev = dst.device
    src = torch.tensor(src_ptrs, dtype=torch.int64, device=dev)
    flg = torch.tensor(flag_ptrs, dtype=torch.int64, device=dev)
    d = _lib.PeerGatherDesc()
    d.world, d.rank, d.bytes = world, rank, nbytes
    d.src_peers, d.flag_peers = src.data_ptr(), flg.data_ptr()
    d.epoch, d.ticket = counters.data_ptr(), counters.data_ptr() + 4
    d.dst, d.status = dst.data_ptr(), status.data_ptr()
    _lib.check(_lib.load().imi_peer_allgather(ctypes.byref(d), ops._stream(dev)), "imi_peer_allgather")
    torch.cuda.synchronize(dev)


def test_one_rank_exchange_copies_and_advances_the_epoch():
    dev = torch.device("cuda")
    block = torch.arange(40000, dtype=torch.int32, device=dev)  # 160 000 bytes: five 32 KB chunks
    flags = torch.zeros((1,), dtype=torch.int32, device=dev)
    counters = torch.zeros((2,), dtype=torch.int32, device=dev)
    status = torch.zeros((1,), dtype=torch.int32, device=dev)
    for call in (1, 2):
        dst = torch.full((40000,), -1, dtype=torch.int32, device=dev)
        _gather(1, 0, block.numel() * 4, [block.data_ptr()], [flags.data_ptr()], counters, dst, status)
        assert torch.equal(dst, block)
        assert int(counters[0]) == call and int(counters[1]) == 0 and int(status[0]) == 0
        assert int(flags[0]) == call


def test_missing_peer_times_out_with_status():
    dev = torch.device("cuda")
    n = 8192
    mine = torch.arange(n, dtype=torch.int32, device=dev)
    absent = torch.zeros(n, dtype=torch.int32, device=dev)
    my_flags = torch.zeros((2,), dtype=torch.int32, device=dev)     # word 1 is never written
    peer_flags = torch.zeros((2,), dtype=torch.int32, device=dev)   # stands in for the absent rank's words
    counters = torch.zeros((2,), dtype=torch.int32, device=dev)
    status = torch.zeros((1,), dtype=torch.int32, device=dev)
    dst = torch.full((2 * n,), -1, dtype=torch.int32, device=dev)
    _gather(2, 0, n * 4, [mine.data_ptr(), absent.data_ptr()], [my_flags.data_ptr(), peer_flags.data_ptr()],
            counters, dst, status)
    assert int(status[0]) & 1
    assert torch.equal(dst[:n], mine)                    # rank 0 (present) was copied
    assert bool((dst[n:] == -1).all())                   # rank 1 (absent) was not
    assert int(peer_flags[0]) == 1 and int(my_flags[0]) == 1  # rank 0 announced itself to both
