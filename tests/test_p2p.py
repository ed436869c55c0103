"""Peer-memory exchange of the expert-parallel layer (lmoe_p2p_*).

CPU: the buffer geometry the library reports (size and region offsets) against a plain
restatement of its layout, and argument checks that reject a step before any launch.
GPU (one device, this rank's buffer as its only peer): a wait on a flag that no kernel
raises gives up after its time budget and leaves a timeout code in the state's error word,
with the context still usable; and the counts exchange of a single rank yields its own
segment offsets."""
import ctypes

import pytest
import torch

from light_moe_b200 import capi


def _layout(ep, E, Tc, k, S, d):
    a = lambda x: (x + 255) // 256 * 256
    p = 0
    flags = p; p = a(p + 4 * 3 * ep)
    cnt = p; p = a(p + 4 * ep * E)
    routed = ep * Tc * k
    rows = p; p = a(p + 2 * (routed + S * Tc) * d)
    meta = p; p = a(p + 4 * (routed + S * Tc))
    ret = p; p = a(p + 2 * Tc * k * d)
    return p, rows, ret


@pytest.mark.parametrize("geom", [(1, 8, 64, 2, 0, 4096), (8, 8, 8192, 2, 0, 4096), (4, 64, 40, 6, 2, 2048),
                                  (2, 16, 1, 4, 1, 256)])
def test_buffer_geometry(geom):
    total, rows, ret = _layout(*geom)
    lib = capi.lib()
    assert lib.lmoe_p2p_buffer_bytes(*geom) == total
    r, t = ctypes.c_size_t(), ctypes.c_size_t()
    capi.call("lmoe_p2p_buffer_offsets", *geom, ctypes.byref(r), ctypes.byref(t))
    assert (r.value, t.value) == (rows, ret)
    assert rows % 256 == 0 and ret % 256 == 0


def test_step_arguments_rejected_on_host():
    lib = capi.lib()
    fake = ctypes.c_void_p(16)   # never dereferenced: every call below fails its checks first
    base = (fake, 0, 2, 8, 64, 2, 0, 4096)
    # more tokens than the capacity, experts not divisible by ranks, a rank outside the group,
    # slots that do not fit the 24-bit slot field
    assert lib.lmoe_p2p_wait(*base, 65, fake, 1, None) == -1
    assert lib.lmoe_p2p_wait(fake, 0, 3, 8, 64, 2, 0, 4096, 8, fake, 1, None) == -1
    assert lib.lmoe_p2p_wait(fake, 2, 2, 8, 64, 2, 0, 4096, 8, fake, 1, None) == -1
    assert lib.lmoe_p2p_wait(fake, 0, 2, 8, 1 << 23, 2, 0, 4096, 8, fake, 1, None) == -1
    assert lib.lmoe_p2p_wait(*base, 8, fake, 0, None) == -1   # only rows (1) or returns (2)
    assert lib.lmoe_p2p_buffer_bytes(0, 8, 64, 2, 0, 4096) == 0


def _own_buffer(geom):
    nbytes = capi.lib().lmoe_p2p_buffer_bytes(*geom)
    ptr, handle = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
    capi.call("lmoe_p2p_alloc", nbytes, ctypes.byref(ptr), handle)
    return ptr.value


@pytest.mark.gpu
def test_wait_for_a_flag_nobody_raises_times_out():
    geom = (1, 8, 16, 2, 0, 256)
    own = _own_buffer(geom)
    try:
        dev = torch.device("cuda", 0)
        peers = torch.tensor([own], dtype=torch.int64, device=dev)
        state = torch.zeros(4, dtype=torch.int32, device=dev)
        counts = torch.tensor([4, 0, 4, 0, 8, 0, 0, 0], dtype=torch.int32, device=dev)
        seg = torch.zeros(8 + 2, dtype=torch.int32, device=dev)
        dst = torch.zeros(8, dtype=torch.int32, device=dev)
        args = (peers.data_ptr(), 0, 1, 8, 16, 2, 0, 256, 8, state.data_ptr())
        s = capi.stream_handle()
        capi.call("lmoe_p2p_exchange_counts", *args, counts.data_ptr(), seg.data_ptr(), dst.data_ptr(), s)
        torch.cuda.synchronize()
        # one rank: its own counts come back, its segments are its experts, then the hole
        assert state[0].item() == 1 and state[1].item() == 0
        assert seg.tolist() == [0, 4, 4, 8, 8, 16, 16, 16, 16, 32]
        assert dst.tolist() == [0, 4, 4, 8, 8, 16, 16, 16]
        # no dispatch ran, so the row flag never reaches this step's epoch: the wait gives up
        capi.call("lmoe_p2p_wait", *args, 1, s)
        torch.cuda.synchronize()
        err = state[1].item() & 0xffffffff
        assert err >> 24 == 1, hex(err)   # timeout code
        # the context is still usable
        assert (torch.ones(4, device=dev) * 2).sum().item() == 8
    finally:
        torch.cuda.synchronize()
        capi.call("lmoe_p2p_free", own)
