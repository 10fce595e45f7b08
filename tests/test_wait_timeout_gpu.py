"""Bounded waits: a peer all-gather whose other rank never writes its rows.

b200q_allgather_peer waits on the device for every other rank's flag. Here
one GPU runs rank 0 of a world of 2 whose "peer" buffer is a second local
buffer: nothing ever writes rank 1's flag into rank 0's buffer, so the wait
runs out. With the limit set to 1 ms (b200q_set_peer_wait_ns) the kernel
records the timeout in the device status word and returns; the host sees it
as B200Q_ETIMEOUT through _native.check_device. Nothing faults or hangs, and
the same context then runs a gather whose flag is already set, which
completes without a timeout. The rank's own rows land in both buffers in
either case.
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ETIMEOUT = -7


def _gather(L, local, rows, n_local, bases, flags_off, counters, st):
    arr = (ctypes.c_void_p * 2)(*bases)
    return L.b200q_allgather_peer(local.data_ptr(), rows, n_local, arr, 0, flags_off, 0, 2, counters.data_ptr(), 0,
                                  None, 0, st)


def test_peer_wait_runs_out_and_is_reported():
    import torch

    from cybel_b200 import _native

    L = _native.lib()
    dev = torch.cuda.current_device()
    torch.cuda.synchronize()
    _native.check_device(dev)  # nothing pending from earlier tests
    rows, n_local, world = 2, 256, 2
    data_bytes = rows * world * n_local * 4
    flags_off = data_bytes
    own = torch.zeros(data_bytes + 256, dtype=torch.uint8, device="cuda")
    fake_peer = torch.zeros_like(own)
    counters = torch.zeros(16, dtype=torch.int32, device="cuda")
    local = torch.arange(rows * n_local, dtype=torch.float32, device="cuda") + 1.0
    st = torch.cuda.current_stream().cuda_stream
    prev = L.b200q_set_peer_wait_ns(1_000_000)  # 1 ms
    try:
        assert L.b200q_set_peer_wait_ns(0) == 1_000_000  # query only
        t0 = time.perf_counter()
        assert _gather(L, local, rows, n_local, [own.data_ptr(), fake_peer.data_ptr()], flags_off, counters, st) == 0
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        with pytest.raises(_native.NativeError) as ei:
            _native.check_device(dev)
        assert ei.value.status == ETIMEOUT
        assert elapsed < 1.0  # the 1 ms limit, not the 2 s default, ended the wait
        _native.check_device(dev)  # cleared by the read
        # this rank's rows reached both receive areas (columns [0, n_local))
        want = local.view(rows, n_local).cpu().numpy()
        for buf in (own, fake_peer):
            got = buf[:data_bytes].view(torch.float32).view(rows, world * n_local)[:, :n_local].cpu().numpy()
            assert np.array_equal(got, want)
        # The context is still usable: with rank 1's flag for the next
        # sequence number already in place, the second gather's wait ends at once.
        own[flags_off + 4:flags_off + 8].view(torch.int32).fill_(2)
        assert _gather(L, local, rows, n_local, [own.data_ptr(), fake_peer.data_ptr()], flags_off, counters, st) == 0
        torch.cuda.synchronize()
        _native.check_device(dev)
        assert counters[:2].cpu().tolist() == [2, 2]
    finally:
        L.b200q_set_peer_wait_ns(prev)
