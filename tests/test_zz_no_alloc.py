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
        call("orch_attention_decode", q, kc, vc, pos, None, ref, M, nh, hd, max_seq, ws, ws_bytes, st)
        call("orch_attention_decode_noalloc", q, kc, vc, pos, None, out, M, nh, hd, max_seq, st)
        torch.cuda.synchronize()
        assert rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy()) <= 1e-2


def test_noalloc_rejects_shapes_beyond_its_scratch():
    assert _lib.lib().orch_attention_noalloc_max_bytes() == 1 << 20
    t = torch.zeros(16, dtype=torch.float16, device="cuda")
    p = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().orch_attention_decode_noalloc(t.data_ptr(), t.data_ptr(), t.data_ptr(), p.data_ptr(), None,
                                                  t.data_ptr(), 1, 64, 128, 65536, None)
    assert rc == 3 and b"scratch" in _lib.lib().orch_last_error()
