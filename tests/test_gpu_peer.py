"""The head split's peer-memory all-reduce (orch_peer_allreduce) on one GPU.

Its job is to sum a buffer over the GPUs of a box, but its arithmetic and its waits can be
checked with one process: two regions on this GPU stand for rank 0's and rank 1's, rank 1's
slot is written from the host (as rank 1's kernel would write it over NVLink: each 64-bit
word the call number over the fp32 bits), and one launch as rank 0 must return x0 + x1 bit
for bit, on both banks of slots, and write its own words into both regions. A third call
whose rank-1 words nobody writes must give up after its bounded wait and report device
check bit 512, with the context still usable. The two-shot form is checked the same way.
The layout follows
orchard_b200/csrc/peer_allreduce.cu (header 4096 bytes, then [bank][rank][cap] 64-bit
words). The two-GPU form runs in tests/test_gpu_split.py.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

SLOTS = 4096


@pytest.fixture(scope="module")
def lib():
    from orchard_b200 import _lib
    _lib.call("orch_init", 0, None)
    torch.cuda.set_device(0)
    return _lib


def _region(lib, world, cap):
    n = lib.lib().orch_peer_region_bytes(world, cap)
    assert n == SLOTS + 2 * world * cap * 8
    t = torch.zeros(n // 8, dtype=torch.int64, device="cuda")  # 256-byte aligned by torch
    assert t.data_ptr() % 256 == 0
    return t


def _words(x, call_no):
    return (x.reshape(-1).view(torch.int32).to(torch.int64) & 0xFFFFFFFF) | (call_no << 32)


def _slot(region, bank, q, world, cap, n):
    off = (SLOTS + (bank * world + q) * cap * 8) // 8
    return region[off:off + n]


def test_peer_allreduce_sums_seeded_peer_bit_exact(lib):
    world, H, rows_max = 2, 4096, 8
    cap = rows_max * H
    A, B = _region(lib, world, cap), _region(lib, world, cap)
    bases = (C.c_void_p * 2)(A.data_ptr(), B.data_ptr())
    s = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(7)
    for call_no, rows in ((1, 3), (2, 8), (3, 1)):  # banks 1, 0, 1; 1..64 blocks
        n = rows * H
        x0 = torch.randn((rows_max, H), generator=g, device="cuda")
        x1 = torch.randn((rows, H), generator=g, device="cuda")
        tail = x0[rows:].clone()
        _slot(A, call_no & 1, 1, world, cap, n).copy_(_words(x1, call_no))
        want = x0[:rows] + x1
        sent = x0[:rows].clone()
        lib.call("orch_peer_allreduce", C.addressof(bases), 0, world, cap, x0, n, 1, s)
        torch.cuda.synchronize()
        assert torch.equal(x0[:rows], want)
        assert torch.equal(x0[rows:], tail)  # values past n untouched
        assert int(A[0].item()) & 0xFFFFFFFF == call_no  # rank 0's call counter advanced once
        # rank 0's words landed in "rank 1's" region as well as in its own
        assert torch.equal(_slot(B, call_no & 1, 0, world, cap, n), _words(sent, call_no))
        assert torch.equal(_slot(A, call_no & 1, 0, world, cap, n), _words(sent, call_no))
    flags = C.c_uint32(0)
    lib.call("orch_device_check", C.byref(flags), s)
    assert flags.value == 0


def _pairs(region, pair_off, n):
    off = SLOTS // 8 + 2 * pair_off
    return region[off:off + n]


def test_peer_allreduce_two_shots_seeded_peer_bit_exact(lib):
    """The two-shot form as rank 0 of two: chunk 1 of x0 goes to "rank 1", chunk 0 is summed
    here with rank 1's seeded part and sent to both regions, chunk 1's sum is rank 1's
    (seeded) -- x0 + x1 bit for bit, on both banks."""
    world, H, rows_max = 2, 4096, 8
    cap = rows_max * H
    cap2 = cap // 2
    cs = (cap2 + world - 1) // world
    A, B = _region(lib, world, cap), _region(lib, world, cap)
    bases = (C.c_void_p * 2)(A.data_ptr(), B.data_ptr())
    s = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(11)
    for call_no, rows in ((1, 3), (2, 8), (3, 1)):
        n = rows * H
        cp = (n // 2 + world - 1) // world
        bank0 = (call_no & 1) * world * cap2
        x0 = torch.randn(cap, generator=g, device="cuda")
        x1 = torch.randn(n, generator=g, device="cuda")
        want = x0[:n] + x1
        sent = x0[:n].clone()
        c0, c1 = slice(0, 2 * cp), slice(2 * cp, n)
        _pairs(A, bank0 + 1 * cs, 2 * cp).copy_(_words(x1[c0], call_no))  # rank 1's part of chunk 0
        _pairs(A, bank0 + (world + 1) * cs, n - 2 * cp).copy_(_words(want[c1], call_no))  # chunk 1's sum
        lib.call("orch_peer_allreduce", C.addressof(bases), 0, world, cap, x0, n, 2, s)
        torch.cuda.synchronize()
        assert torch.equal(x0[:n], want)
        assert int(A[0].item()) & 0xFFFFFFFF == call_no
        assert torch.equal(_pairs(B, bank0, n - 2 * cp), _words(sent[c1], call_no))  # chunk 1 to rank 1
        assert torch.equal(_pairs(B, bank0 + world * cs, 2 * cp), _words(want[c0], call_no))  # chunk 0's sum
    flags = C.c_uint32(0)
    lib.call("orch_device_check", C.byref(flags), s)
    assert flags.value == 0


def test_peer_allreduce_bounded_wait_reports_bit_512(lib):
    """Rank 1's words never arrive: the call gives up after its bounded wait (~5 s), flags bit
    512 and returns; the GPU keeps working."""
    world, cap = 2, 4096
    A, B = _region(lib, world, cap), _region(lib, world, cap)
    bases = (C.c_void_p * 2)(A.data_ptr(), B.data_ptr())
    s = torch.cuda.current_stream().cuda_stream
    x = torch.ones(cap, device="cuda")
    lib.call("orch_peer_allreduce", C.addressof(bases), 0, world, cap, x, cap, 0, s)
    torch.cuda.synchronize()
    flags = C.c_uint32(0)
    lib.call("orch_device_check", C.byref(flags), s)
    assert flags.value & 512
    y = torch.arange(16, device="cuda", dtype=torch.float32) * 2
    assert float(y.sum().item()) == 240.0  # the context is still usable


def test_peer_allreduce_rejects_bad_arguments(lib):
    from orchard_b200._lib import OrchardError
    world, cap = 2, 4096
    A = _region(lib, world, cap)
    bases = (C.c_void_p * 2)(A.data_ptr(), None)
    x = torch.zeros(cap, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    with pytest.raises(OrchardError):  # a missing peer region
        lib.call("orch_peer_allreduce", C.addressof(bases), 0, world, cap, x, cap, 0, s)
    ok = (C.c_void_p * 2)(A.data_ptr(), A.data_ptr())
    with pytest.raises(OrchardError):  # n beyond the slots
        lib.call("orch_peer_allreduce", C.addressof(ok), 0, world, cap, x, cap + 4, 0, s)
    with pytest.raises(OrchardError):  # n not a multiple of 4
        lib.call("orch_peer_allreduce", C.addressof(ok), 0, world, cap, x, 6, 0, s)
    with pytest.raises(OrchardError):  # rank outside the world
        lib.call("orch_peer_allreduce", C.addressof(ok), 2, world, cap, x, cap, 0, s)
    with pytest.raises(OrchardError):  # no such algorithm
        lib.call("orch_peer_allreduce", C.addressof(ok), 0, world, cap, x, cap, 3, s)
    assert lib.lib().orch_peer_region_bytes(9, 4096) == 0
