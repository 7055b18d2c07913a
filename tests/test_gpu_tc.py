"""The tcgen05 (TMEM) INT4 GEMM against the oracle and the mma.sync kernel (GPU).

Tolerance: max|gpu - ref| / max|ref| <= 1e-2 against the oracle (fp32); the two GPU
kernels agree to 2e-3 of max|ref| (both round (q-8)*scale to fp16, accumulate in fp32).
"""

import functools

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import ops
from orchard_b200 import _lib, quantizer
from orchard_b200._lib import F16, F32, call

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available()
    call("orch_init", 0, None)
    yield
    call("orch_set_tc_min_m", 17)


def S():
    return torch.cuda.current_stream().cuda_stream


@functools.lru_cache(maxsize=None)
def weights(n, k):
    g = np.random.default_rng([20261201, 55, n, k])
    w = (g.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
    p, s = quantizer.quantize_q4_0(w)
    return p, s, ops.dequantize_q4_0(p, s)


def run_gemm(p, s, x, tc_min):
    M, K = x.shape
    N = p.shape[0]
    call("orch_set_tc_min_m", tc_min)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    call("orch_gemm_q4_0_ex", torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda(),
         F16, y, F32, K, N, M, S())
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("K,N", [(4096, 4096), (11008, 4096), (4096, 12288), (4096, 1000), (96, 200)])
@pytest.mark.parametrize("M", [1, 2, 8, 16, 17, 32, 64, 100, 256, 600])
def test_tc_gemm_matches_oracle(K, N, M):
    if M > 64 and K * N > 4096 * 4096:
        pytest.skip("prefill-sized M covered on the smaller shapes")
    p, s, wd = weights(N, K)
    x = np.random.default_rng([7, M, K]).standard_normal((M, K), dtype=np.float32).astype(np.float16)
    ref = x.astype(np.float32) @ wd.T
    y_tc = run_gemm(p, s, x, 1)
    assert rel_err(y_tc, ref) <= 1e-2
    if M <= 64:
        y_mma = run_gemm(p, s, x, 0)
        assert rel_err(y_tc, y_mma) <= 2e-3


def test_tc_flag_clear_after_runs():
    flags = _lib.C.c_uint32(0)
    call("orch_device_check", _lib.C.byref(flags), None)
    assert flags.value & 256 == 0


@pytest.mark.parametrize("M", [32, 64])
def test_tc_fused_epilogues_match_mma_path(M):
    """QKV+RoPE+KV append, gate/up+SwiGLU and down+residual on both kernels."""
    H, F, nh, hd, max_seq = 4096, 11008, 32, 128, 64
    g = np.random.default_rng([9, M])
    pq, sq, _ = weights(3 * H, H)
    p13, s13, _ = weights(2 * F, H)
    p2, s2, _ = weights(H, F)
    x = g.standard_normal((M, H), dtype=np.float32).astype(np.float16)
    h_in = g.standard_normal((M, F), dtype=np.float32).astype(np.float16)
    pos = torch.tensor(g.integers(0, max_seq, M), dtype=torch.int32, device="cuda")
    c, sn = ops.precompute_freqs_cis(hd, 2048)
    cd, sd = torch.from_numpy(c).cuda(), torch.from_numpy(sn).cuda()
    outs = []
    for tc in (1, 0):
        call("orch_set_tc_min_m", tc)
        q = torch.zeros((M, H), dtype=torch.float16, device="cuda")
        kc = torch.zeros((M, nh, max_seq, hd), dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        call("orch_q4_qkv_rope", torch.from_numpy(pq).cuda(), torch.from_numpy(sq).cuda(), torch.from_numpy(x).cuda(),
             M, H, H, nh, pos, None, cd, sd, 2048, q, kc, vc, max_seq, M, None, None, 0, S())
        h = torch.zeros((M, F), dtype=torch.float16, device="cuda")
        call("orch_q4_linear_swiglu", torch.from_numpy(p13).cuda(), torch.from_numpy(s13).cuda(),
             torch.from_numpy(x).cuda(), h, M, H, F, None, None, 0, S())
        r = torch.ones((M, H), dtype=torch.float32, device="cuda")
        call("orch_q4_linear_resid", torch.from_numpy(p2).cuda(), torch.from_numpy(s2).cuda(),
             torch.from_numpy(h_in).cuda(), r, M, F, H, None, None, 0, S())
        torch.cuda.synchronize()
        outs.append([t.float().cpu().numpy() for t in (q, kc, vc, h, r)])
    for a, b in zip(*outs):
        assert rel_err(a, b) <= 5e-3


@pytest.mark.parametrize("r", [16, 6])
def test_tc_fused_epilogues_with_lora_prefill_rows(r):
    """Prefill-sized batch (a full 256-row tile and a partial one) with rank-r LoRA terms on
    the three fused entry points: the tensor-core kernel (LoRA operands staged in shared
    memory after the K loop; RoPE pairs read t once, as float4 when r % 4 == 0) against the
    mma.sync kernel (LoRA operands read from global memory); same kernel-to-kernel tolerance
    as above."""
    M, H, F, nh, hd, max_seq = 300, 4096, 11008, 32, 128, 512
    g = np.random.default_rng([10, M, r])
    pq, sq, _ = weights(3 * H, H)
    p13, s13, _ = weights(2 * F, H)
    p2, s2, _ = weights(H, F)
    x = g.standard_normal((M, H), dtype=np.float32).astype(np.float16)
    h_in = g.standard_normal((M, F), dtype=np.float32).astype(np.float16)
    pos = torch.tensor(np.arange(M) % max_seq, dtype=torch.int32, device="cuda")
    c, sn = ops.precompute_freqs_cis(hd, 2048)
    cd, sd = torch.from_numpy(c).cuda(), torch.from_numpy(sn).cuda()

    def lora(regions, width):
        t = torch.from_numpy(g.standard_normal((M, regions, r), dtype=np.float32) * 0.1).cuda()
        b = torch.from_numpy(g.standard_normal((regions, r, width), dtype=np.float32) * 0.1).cuda()
        return t, b

    lt3, lb3 = lora(3, H)
    lt2, lb2 = lora(2, F)
    lt1, lb1 = lora(1, H)
    outs = []
    for tc in (1, 0):
        call("orch_set_tc_min_m", tc)
        q = torch.zeros((M, H), dtype=torch.float16, device="cuda")
        kc = torch.zeros((M, nh, max_seq, hd), dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        call("orch_q4_qkv_rope", torch.from_numpy(pq).cuda(), torch.from_numpy(sq).cuda(), torch.from_numpy(x).cuda(),
             M, H, H, nh, pos, None, cd, sd, 2048, q, kc, vc, max_seq, M, lt3, lb3, r, S())
        h = torch.zeros((M, F), dtype=torch.float16, device="cuda")
        call("orch_q4_linear_swiglu", torch.from_numpy(p13).cuda(), torch.from_numpy(s13).cuda(),
             torch.from_numpy(x).cuda(), h, M, H, F, lt2, lb2, r, S())
        res = torch.ones((M, H), dtype=torch.float32, device="cuda")
        call("orch_q4_linear_resid", torch.from_numpy(p2).cuda(), torch.from_numpy(s2).cuda(),
             torch.from_numpy(h_in).cuda(), res, M, F, H, lt1, lb1, r, S())
        torch.cuda.synchronize()
        outs.append([t.float().cpu().numpy() for t in (q, kc, vc, h, res)])
    call("orch_set_tc_min_m", 17)
    for a, b in zip(*outs):
        assert rel_err(a, b) <= 5e-3
