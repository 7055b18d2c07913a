"""Tiled INT4 weights: the device re-layout and the GEMMs that read it (GPU).

* ``orch_q4t_pack`` is checked byte for byte against a NumPy statement of the layout
  (rows in tiles of 128, k in blocks of 256, per block four 64-k stages of
  [2 halves][128 rows][16 B] then the block's scales [8][128] fp16, nibbles of each word
  stored k0 k2 k4 k6 k1 k3 k5 k7, padding = nibble 8 / scale 0).
* ``orch_q4t_gemm`` against the oracle (max|gpu - ref| / max|ref| <= 1e-2) and against the
  reference-layout tensor-core GEMM: the same arithmetic and order for M > 64 (<= 1e-6 of
  max|ref|); for 8 < M <= 64 the tiled path may be the persistent stream-K kernel (each case
  runs with it chosen automatically, forced and off), whose K split points differ, so its
  fp32 partial sums are added in another order (<= 1e-5: sqrt(K) x 2^-24 ~ 6e-6 at K =
  11008); for M <= 8 it is the mma.sync GEMV (<= 2e-3, the kernel-to-kernel tolerance of the
  other GEMM tests).
* The fused tiled entry points against the reference-layout ones (same tolerances; fp16
  outputs of the stream-K range may also differ by one fp16 rounding step).
"""


def kernel_tol(M):
    return 1e-6 if M > 64 else (1e-5 if M > 8 else 2e-3)

import functools

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import ops
from orchard_b200 import _lib, quantizer
from orchard_b200._lib import F16, F32, call

pytestmark = pytest.mark.gpu

PERM = [0, 2, 4, 6, 1, 3, 5, 7]  # nibble p of a tiled word holds k = PERM[p]


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available()
    call("orch_init", 0, None)
    yield
    call("orch_set_tc_min_m", 17)


def S():
    return torch.cuda.current_stream().cuda_stream


def tile_np(p: np.ndarray, s: np.ndarray) -> np.ndarray:
    """NumPy statement of the tiled layout for packed [N, K/2] uint8 + scales [N, K/32] fp16."""
    N, K = p.shape[0], p.shape[1] * 2
    nt, nb = -(-N // 128), -(-K // 256)
    pp = np.full((nt * 128, nb * 128), 0x88, np.uint8)
    pp[:N, : K // 2] = p
    ss = np.zeros((nt * 128, nb * 8), np.float16)
    ss[:N, : K // 32] = s
    words = pp.view("<u4")  # [rows, nb*32] words of 8 nibbles (k in natural order)
    nib = [(words >> (4 * q)) & 0xF for q in range(8)]
    tw = np.zeros_like(words)
    for pos, q in enumerate(PERM):
        tw |= nib[q] << (4 * pos)
    out = np.zeros((nt, nb, 18432), np.uint8)
    tw = tw.reshape(nt, 128, nb, 4, 2, 4)  # tile, row, block, stage, half, word
    out[:, :, :16384] = tw.transpose(0, 2, 3, 4, 1, 5).reshape(nt, nb, 16384 // 4).view(np.uint8).reshape(nt, nb, 16384)
    sc = ss.reshape(nt, 128, nb, 8).transpose(0, 2, 3, 1)  # tile, block, group, row
    out[:, :, 16384:] = np.ascontiguousarray(sc).view(np.uint8).reshape(nt, nb, 2048)
    return out.reshape(-1)


@functools.lru_cache(maxsize=None)
def weights(n, k):
    g = np.random.default_rng([20261201, 77, n, k])
    w = (g.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
    p, s = quantizer.quantize_q4_0(w)
    return p, s, ops.dequantize_q4_0(p, s)


def pack_dev(p, s):
    N, K = p.shape[0], p.shape[1] * 2
    nbytes = _lib.lib().orch_q4t_bytes(N, K)
    t = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    call("orch_q4t_pack", torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda(), N, K, t, S())
    return t


@pytest.mark.parametrize("K,N", [(4096, 256), (11008, 128), (96, 300), (4096, 1000)])
def test_pack_matches_layout_statement(K, N):
    p, s, _ = weights(N, K)
    t = pack_dev(p, s)
    torch.cuda.synchronize()
    assert t.numel() == -(-N // 128) * -(-K // 256) * 18432
    assert np.array_equal(t.cpu().numpy(), tile_np(p, s))


def gemm_ref_layout(p, s, x):
    M, K = x.shape
    N = p.shape[0]
    call("orch_set_tc_min_m", 1)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    call("orch_gemm_q4_0_ex", torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda(),
         F16, y, F32, K, N, M, S())
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.fixture(params=[0, 1, 2], ids=["sk-never", "sk-always", "sk-auto"])
def stream_k(request):
    """Batched-decode GEMM selection (orch_set_stream_k): never (the per-tile kernel, the
    default), always the persistent stream-K kernel, automatic."""
    call("orch_set_stream_k", request.param)
    yield request.param
    call("orch_set_stream_k", 0)


@pytest.mark.parametrize("K,N", [(4096, 4096), (11008, 4096), (4096, 22016), (4096, 1000), (96, 200)])
@pytest.mark.parametrize("M", [1, 2, 8, 16, 17, 32, 64, 100, 256, 600])
def test_tiled_gemm_matches_oracle(K, N, M, stream_k):
    if M > 64 and K * N > 4096 * 4096:
        pytest.skip("prefill-sized M covered on the smaller shapes")
    if stream_k != 0 and not 8 < M <= 64:
        pytest.skip("the stream-K switch only concerns 9..64 rows")
    p, s, wd = weights(N, K)
    x = np.random.default_rng([8, M, K]).standard_normal((M, K), dtype=np.float32).astype(np.float16)
    t = pack_dev(p, s)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    call("orch_q4t_gemm", t, torch.from_numpy(x).cuda(), y, F32, K, N, M, S())
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    ref = x.astype(np.float32) @ wd.T
    assert rel_err(y, ref) <= 1e-2
    if K % 256 == 0:
        assert rel_err(y, gemm_ref_layout(p, s, x)) <= kernel_tol(M)


def test_tiled_gemm_fp16_output():
    p, s, wd = weights(4096, 4096)
    x = np.random.default_rng(3).standard_normal((5, 4096), dtype=np.float32).astype(np.float16)
    t = pack_dev(p, s)
    y = torch.empty((5, 4096), dtype=torch.float16, device="cuda")
    call("orch_q4t_gemm", t, torch.from_numpy(x).cuda(), y, F16, 4096, 4096, 5, S())
    torch.cuda.synchronize()
    assert rel_err(y.float().cpu().numpy(), x.astype(np.float32) @ wd.T) <= 1e-2


def test_stream_k_mode_rejects_bad_values():
    with pytest.raises(_lib.OrchardError):
        call("orch_set_stream_k", 3)


def test_tiled_rejects_bad_arguments():
    p, s, _ = weights(256, 4096)
    t = pack_dev(p, s)
    x = torch.zeros((2, 4096), dtype=torch.float16, device="cuda")
    y = torch.empty((2, 256), dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.OrchardError):
        call("orch_q4t_gemm", t[8:], x, y, F32, 4096, 256, 2, S())
    with pytest.raises(_lib.OrchardError):
        call("orch_q4t_pack", torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda(), 256, 100, t, S())
    # H = 512 heads x 128 = 65536: beyond the epilogue's head-index arithmetic (H < 65536);
    # rejected on the host before any launch, so the small buffers are never touched
    small = torch.zeros(16, dtype=torch.float32, device="cuda")
    pos = torch.zeros(2, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.OrchardError):
        call("orch_q4t_qkv_rope", t, x, 2, 4096, 65536, 512, pos, None, small, small, 16, small, small, small, 4,
             2, None, None, 0, S())


@pytest.mark.parametrize("M", [1, 5, 16, 64, 200])
def test_tiled_fused_match_reference_layout(M, stream_k):
    if stream_k != 0 and not 8 < M <= 64:
        pytest.skip("the stream-K switch only concerns 9..64 rows")
    """QKV+RoPE+KV append, gate/up+SwiGLU, down+residual (with LoRA) on both layouts."""
    H, F, nh, hd, max_seq, r = 4096, 11008, 32, 128, 64, 8
    g = np.random.default_rng([19, M])
    pq, sq, _ = weights(3 * H, H)
    p13, s13, _ = weights(2 * F, H)
    p2, s2, _ = weights(H, F)
    tq, t13, t2 = pack_dev(pq, sq), pack_dev(p13, s13), pack_dev(p2, s2)
    x = torch.from_numpy(g.standard_normal((M, H), dtype=np.float32).astype(np.float16)).cuda()
    h_in = torch.from_numpy(g.standard_normal((M, F), dtype=np.float32).astype(np.float16)).cuda()
    pos = torch.tensor(g.integers(0, max_seq, M), dtype=torch.int32, device="cuda")
    c, sn = ops.precompute_freqs_cis(hd, 2048)
    cd, sd = torch.from_numpy(c).cuda(), torch.from_numpy(sn).cuda()
    lt3 = torch.from_numpy(g.standard_normal((M, 3, r), dtype=np.float32) * 0.1).cuda()
    lb3 = torch.from_numpy(g.standard_normal((3, r, H), dtype=np.float32) * 0.1).cuda()
    lt1 = torch.from_numpy(g.standard_normal((M, 1, r), dtype=np.float32) * 0.1).cuda()
    lb1 = torch.from_numpy(g.standard_normal((1, r, H), dtype=np.float32) * 0.1).cuda()
    call("orch_set_tc_min_m", 1)
    outs = []
    for tiled in (True, False):
        q = torch.zeros((M, H), dtype=torch.float16, device="cuda")
        kc = torch.zeros((M, nh, max_seq, hd), dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        h = torch.zeros((M, F), dtype=torch.float16, device="cuda")
        res = torch.ones((M, H), dtype=torch.float32, device="cuda")
        if tiled:
            call("orch_q4t_qkv_rope", tq, x, M, H, H, nh, pos, None, cd, sd, 2048, q, kc, vc, max_seq, M, lt3, lb3, r, S())
            call("orch_q4t_linear_swiglu", t13, x, h, M, H, F, None, None, 0, S())
            call("orch_q4t_linear_resid", t2, h_in, res, M, F, H, lt1, lb1, r, S())
        else:
            call("orch_q4_qkv_rope", torch.from_numpy(pq).cuda(), torch.from_numpy(sq).cuda(), x, M, H, H, nh, pos,
                 None, cd, sd, 2048, q, kc, vc, max_seq, M, lt3, lb3, r, S())
            call("orch_q4_linear_swiglu", torch.from_numpy(p13).cuda(), torch.from_numpy(s13).cuda(), x, h, M, H, F,
                 None, None, 0, S())
            call("orch_q4_linear_resid", torch.from_numpy(p2).cuda(), torch.from_numpy(s2).cuda(), h_in, res, M, F,
                 H, lt1, lb1, r, S())
        torch.cuda.synchronize()
        outs.append([t.float().cpu().numpy() for t in (q, kc, vc, h, res)])
    for i, (a, b) in enumerate(zip(*outs)):
        if i < 4 and 8 < M <= 64:
            # fp16 outputs of fp32 sums taken in another order: at most one fp16 rounding step
            # apart (plus the fp32 tolerance)
            ulp = np.spacing(np.abs(b).astype(np.float16)).astype(np.float32)
            assert np.all(np.abs(a - b) <= ulp + kernel_tol(M) * np.abs(b).max())
        else:
            assert rel_err(a, b) <= kernel_tol(M)


@pytest.mark.parametrize("M", [4, 64, 300])
def test_qkv_append_rejects_slots_outside_the_cache(M):
    """A row whose cache slot is outside [0, num_slots) still gets its q but appends no K/V
    and sets device check bit 8; every other row's K/V land exactly where valid slots put
    them. M = 4 runs the mma.sync GEMV epilogue, 64 the tensor-core register epilogue, 300
    the receive-buffer epilogue of the prefill tiles."""
    H, nh, hd, max_seq = 4096, 32, 128, 8
    g = np.random.default_rng([23, M])
    pq, sq, _ = weights(3 * H, H)
    tq = pack_dev(pq, sq)
    x = torch.from_numpy(g.standard_normal((M, H), dtype=np.float32).astype(np.float16)).cuda()
    pos = torch.tensor(g.integers(0, max_seq, M), dtype=torch.int32, device="cuda")
    c, sn = ops.precompute_freqs_cis(hd, 64)
    cd, sd = torch.from_numpy(c).cuda(), torch.from_numpy(sn).cuda()
    good = torch.arange(M, dtype=torch.int32, device="cuda")
    bad = good.clone()
    bad[1] = M + 5
    bad[M - 1] = -1
    res = []
    for slots in (good, bad):
        q = torch.zeros((M, H), dtype=torch.float16, device="cuda")
        kc = torch.zeros((M, nh, max_seq, hd), dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        call("orch_q4t_qkv_rope", tq, x, M, H, H, nh, pos, slots, cd, sd, 64, q, kc, vc, max_seq, M, None, None, 0,
             S())
        torch.cuda.synchronize()
        flags = _lib.C.c_uint32(0)
        call("orch_device_check", _lib.C.byref(flags), None)
        res.append((flags.value, q.cpu(), kc.cpu(), vc.cpu()))
    (f0, q0, k0, v0), (f1, q1, k1, v1) = res
    assert f0 == 0 and f1 == 8
    assert torch.equal(q0, q1)
    keep = [m for m in range(M) if m not in (1, M - 1)]
    assert torch.equal(k1[keep], k0[keep]) and torch.equal(v1[keep], v0[keep])
    assert not k1[[1, M - 1]].any() and not v1[[1, M - 1]].any()


@pytest.mark.parametrize("M", [1, 3, 8, 16])
def test_rmsnorm_fused_projections_match_unfused(M):
    """orch_q4t_rms_qkv_rope / orch_q4t_rms_linear_swiglu (RMSNorm computed inside the GEMV for
    up to 8 rows) against orch_rmsnorm_ex followed by the unfused entry points. The fused norm
    sums x^2 in another order, so an element of the normalised row may round to the other
    neighbouring fp16: outputs within 2e-3 of max|ref|; the q / K / V rows and h otherwise
    identical in layout and position. M = 16 takes the two-launch path (bit-identical)."""
    H, F, nh, hd, max_seq = 4096, 11008, 32, 128, 16
    g = np.random.default_rng([29, M])
    pq, sq, _ = weights(3 * H, H)
    p13, s13, _ = weights(2 * F, H)
    tq, t13 = pack_dev(pq, sq), pack_dev(p13, s13)
    x = torch.from_numpy(g.standard_normal((M, H), dtype=np.float32) * 2.0).cuda()
    gam = torch.from_numpy((1 + 0.1 * g.standard_normal(H)).astype(np.float32)).cuda()
    pos = torch.tensor(g.integers(0, max_seq, M), dtype=torch.int32, device="cuda")
    c, sn = ops.precompute_freqs_cis(hd, 64)
    cd, sd = torch.from_numpy(c).cuda(), torch.from_numpy(sn).cuda()
    outs = []
    for fused in (True, False):
        xn = torch.zeros((M, H), dtype=torch.float16, device="cuda")
        q = torch.zeros((M, H), dtype=torch.float16, device="cuda")
        kc = torch.zeros((M, nh, max_seq, hd), dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        h = torch.zeros((M, F), dtype=torch.float16, device="cuda")
        if fused:
            call("orch_q4t_rms_qkv_rope", tq, x, gam, 1e-5, xn, M, H, H, nh, pos, None, cd, sd, 64, q, kc, vc,
                 max_seq, M, S())
            call("orch_q4t_rms_linear_swiglu", t13, x, gam, 1e-5, xn, h, M, H, F, S())
        else:
            call("orch_rmsnorm_ex", x, F32, gam, F32, xn, F16, 1e-5, H, M, S())
            call("orch_q4t_qkv_rope", tq, xn, M, H, H, nh, pos, None, cd, sd, 64, q, kc, vc, max_seq, M, None, None,
                 0, S())
            call("orch_q4t_linear_swiglu", t13, xn, h, M, H, F, None, None, 0, S())
        torch.cuda.synchronize()
        outs.append([t.float().cpu().numpy() for t in (q, kc, vc, h)])
    for a, b in zip(*outs):
        if M > 8:
            np.testing.assert_array_equal(a, b)
        else:
            assert rel_err(a, b) <= 2e-3
    # the oracle: RMSNorm (orchard/kernels/rmsnorm.metal:23-35), the gate/up projection (rows
    # interleaved in blocks of 16: 32b + i gate, 32b + 16 + i up) and SwiGLU, within 1e-2
    xn_ref = ops.rmsnorm(x.cpu().numpy(), gam.cpu().numpy(), 1e-5).astype(np.float16).astype(np.float32)
    y = ops.gemm_q4_0(p13, s13, xn_ref)
    j = np.arange(F)
    gate, up = y[:, 32 * (j // 16) + j % 16], y[:, 32 * (j // 16) + 16 + j % 16]
    assert rel_err(outs[0][3], ops.mul(ops.silu(gate), up)) <= 1e-2


def test_tiled_flag_clear_after_runs():
    flags = _lib.C.c_uint32(0)
    call("orch_device_check", _lib.C.byref(flags), None)
    assert flags.value & 256 == 0
