"""Allocation-free decode attention (GPU), collected last on purpose.

Some callers cannot allocate device memory: a host that is capturing its own CUDA graph,
a real-time host whose memory is fixed at start-up, or a plugin host that hands the
library only the tensors of a call. ``orch_attention_decode_noalloc`` serves them with
scratch that lives inside the library. This test calls it through the C ABI and checks
it against ``orch_attention_decode`` (caller workspace) on two calls in a row, with the
attention tests' tolerance: max|a - b| / max|b| <= 1e-2.
"""

import numpy as np
import pytest
import torch

from conftest import rel_err
from orchard_b200 import _lib
from orchard_b200._lib import call

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available()
    call("orch_init", 0, None)


def _inputs(seed, M, nh, hd, max_seq, L):
    g = np.random.default_rng([20261201, 91, seed])
    kc = torch.from_numpy(g.standard_normal((M, nh, max_seq, hd), dtype=np.float32).astype(np.float16)).cuda()
    vc = torch.from_numpy(g.standard_normal((M, nh, max_seq, hd), dtype=np.float32).astype(np.float16)).cuda()
    q = torch.from_numpy(g.standard_normal((M, nh * hd), dtype=np.float32).astype(np.float16)).cuda()
    pos = torch.tensor([L - 1 - (i % 5) for i in range(M)], dtype=torch.int32, device="cuda")
    return q, kc, vc, pos


@pytest.mark.parametrize("M,L", [(1, 577), (4, 640), (16, 200)])
def test_noalloc_matches_workspace_path_twice(M, L):
    nh, hd, max_seq = 32, 128, 640
    st = torch.cuda.current_stream().cuda_stream
    ws_bytes = _lib.lib().orch_attention_workspace_bytes(M, nh, hd, max_seq)
    ws = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device="cuda")
    for rep in range(2):  # two calls in a row: the shared scratch keeps the last call's contents
        q, kc, vc, pos = _inputs(rep * 10 + M, M, nh, hd, max_seq, L)
        ref = torch.empty((M, nh * hd), dtype=torch.float16, device="cuda")
        out = torch.full_like(ref, 7.0)
        call("orch_attention_decode", q, kc, vc, pos, None, ref, M, nh, hd, max_seq, M, ws, ws_bytes, st)
        call("orch_attention_decode_noalloc", q, kc, vc, pos, None, out, M, nh, hd, max_seq, M, st)
        torch.cuda.synchronize()
        assert rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy()) <= 1e-2


def _device_flags():
    torch.cuda.synchronize()
    flags = _lib.C.c_uint32(0)
    call("orch_device_check", _lib.C.byref(flags), None)
    return int(flags.value)


def test_noalloc_reports_rows_outside_the_cache():
    """The allocation-free path checks each row's position and cache slot on the device
    before using them, like the workspace path: a rejected row is skipped (its output row is
    left as it was) and its flag bit (position 2, slot 8) is reported by orch_device_check,
    the library's one place to read device-side input checks. Four rows over 32 heads take
    the split-position kernels, so the shared scratch and the combine pass are exercised."""
    M, nh, hd, max_seq, nslots = 4, 32, 128, 640, 4
    q, kc, vc, _ = _inputs(77, nslots, nh, hd, max_seq, 600)
    q = q[:M].contiguous()
    st = torch.cuda.current_stream().cuda_stream
    pos = torch.tensor([577, max_seq + 3, 500, 12], dtype=torch.int32, device="cuda")
    slots = torch.tensor([2, 0, nslots, 3], dtype=torch.int32, device="cuda")
    ws_bytes = _lib.lib().orch_attention_workspace_bytes(M, nh, hd, max_seq)
    assert ws_bytes > 0  # the split path
    ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device="cuda")
    _device_flags()
    for rep in range(2):
        ref = torch.full((M, nh * hd), 7.0, dtype=torch.float16, device="cuda")
        out = torch.full_like(ref, 7.0)
        call("orch_attention_decode", q, kc, vc, pos, slots, ref, M, nh, hd, max_seq, nslots, ws, ws_bytes, st)
        assert _device_flags() == 2 | 8
        call("orch_attention_decode_noalloc", q, kc, vc, pos, slots, out, M, nh, hd, max_seq, nslots, st)
        assert _device_flags() == 2 | 8
        o, r = out.float().cpu().numpy(), ref.float().cpu().numpy()
        assert np.all(o[1] == 7.0) and np.all(o[2] == 7.0)
        assert rel_err(o[[0, 3]], r[[0, 3]]) <= 1e-2
    assert _device_flags() == 0  # reading clears both words


def test_noalloc_rejects_shapes_beyond_its_scratch():
    assert _lib.lib().orch_attention_noalloc_max_bytes() == 1 << 20
    t = torch.zeros(16, dtype=torch.float16, device="cuda")
    p = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().orch_attention_decode_noalloc(t.data_ptr(), t.data_ptr(), t.data_ptr(), p.data_ptr(), None,
                                                  t.data_ptr(), 1, 64, 128, 65536, 1, None)
    assert rc == 3 and b"scratch" in _lib.lib().orch_last_error()
