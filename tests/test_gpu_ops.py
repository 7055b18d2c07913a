"""CUDA kernels through the C ABI against the oracle (GPU).

Tolerances (stated per op): INT4/INT8 packing bit-exact; GEMV/GEMM
max|gpu - ref| / max|ref| <= 1e-2 (fp16 weights*scale rounding, fp16 activations);
RMSNorm / RoPE 1e-3 of max|ref|; softmax atol 1e-3 (examples/full_test.py:113).
"""

import functools

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import ops
from orchard_b200 import _lib, quantizer
from orchard_b200._lib import F16, F32, call, ptr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    call("orch_init", 0, None)
    yield torch.device("cuda", 0)
    torch.cuda.synchronize()
    flags = _lib.C.c_uint32(0)
    call("orch_device_check", _lib.C.byref(flags), None)


def D(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def S():
    return torch.cuda.current_stream().cuda_stream


def rng(*key):
    return np.random.default_rng([20261201, 77, *key])


@functools.lru_cache(maxsize=None)
def q4_weights(n, k, key=0):
    w = (rng(1, n, k, key).standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
    return quantizer.quantize_q4_0(w)


@functools.lru_cache(maxsize=None)
def q4_dense(n, k, key=0):
    p, s = q4_weights(n, k, key)
    return ops.dequantize_q4_0(p, s)


# ---------------------------------------------------------------- INT4 GEMV / GEMM
SHAPES = [(32, 1), (4096, 4096), (4096, 11008), (11008, 4096), (4096, 32000), (256, 100), (96, 37)]


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 4, 8, 16, 64])
def test_q4_gemm_matches_oracle(K, N, M):
    if M > 8 and K * N > 4096 * 11008:
        pytest.skip("large-M sweep covered on the 4096x4096/4096x11008 shapes")
    p, s = q4_weights(N, K)
    x = rng(2, M, K).standard_normal((M, K), dtype=np.float32).astype(np.float16)
    ref = x.astype(np.float32) @ q4_dense(N, K).T
    y = torch.empty((M, N), dtype=torch.float16, device="cuda")
    call("orch_gemm_q4_0", D(p), D(s), D(x), ptr(y), K, N, M, S())
    assert rel_err(y.float().cpu().numpy(), ref) <= 1e-2
    yf = torch.empty((M, N), dtype=torch.float32, device="cuda")
    call("orch_gemm_q4_0_ex", D(p), D(s), D(x.astype(np.float32)), F32, ptr(yf), F32, K, N, M, S())
    assert rel_err(yf.cpu().numpy(), ref) <= 1e-2


def test_gemv_kat_0x99():
    """examples/simple_test.py:83-103: 0x99 bytes, scale 1, ones -> 32.0."""
    p = np.full((1, 16), 0x99, np.uint8)
    s = np.ones((1, 1), np.float16)
    x = np.ones(32, np.float16)
    y = torch.zeros(1, dtype=torch.float16, device="cuda")
    call("orch_gemv_q4_0", D(p), D(s), D(x), ptr(y), 32, 1, S())
    assert float(y.item()) == 32.0


def test_q4_gemm_repeatable_and_m_independent():
    """A row's result does not depend on which other rows share the launch config."""
    K, N = 4096, 4096
    p, s = q4_weights(N, K, 3)
    x = rng(4).standard_normal((8, K), dtype=np.float32).astype(np.float16)
    y1 = torch.empty((8, N), dtype=torch.float32, device="cuda")
    y2 = torch.empty_like(y1)
    call("orch_gemm_q4_0_ex", D(p), D(s), D(x), F16, ptr(y1), F32, K, N, 8, S())
    call("orch_gemm_q4_0_ex", D(p), D(s), D(x), F16, ptr(y2), F32, K, N, 8, S())
    assert torch.equal(y1, y2)


# ---------------------------------------------------------------- INT8
@pytest.mark.parametrize("K,N", [(4096, 4096), (11008, 4096), (64, 33)])
@pytest.mark.parametrize("M", [1, 4, 8])
def test_q8_group_and_per_channel(K, N, M):
    w = (rng(5, K, N).standard_normal((N, K), dtype=np.float32) * 0.02)
    x = rng(6, M, K).standard_normal((M, K), dtype=np.float32).astype(np.float16)
    q, s = quantizer.quantize_q8_0(w)
    ref = ops.gemv_q8_0(q, s, x.astype(np.float32))
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    call("orch_gemm_q8_0_ex", D(q), D(s), D(x), F16, ptr(y), F32, K, N, M, S())
    assert rel_err(y.cpu().numpy(), ref) <= 1e-2
    qp, sp = quantizer.quantize_q8_pc(w)
    ref = ops.gemm_q8_pc(qp, sp, x.astype(np.float32))
    call("orch_gemm_q8_pc", D(qp), D(sp), D(x), F16, ptr(y), F32, K, N, M, S())
    assert rel_err(y.cpu().numpy(), ref) <= 1e-2


# ---------------------------------------------------------------- on-device packers
@pytest.mark.parametrize("shape", [(64, 256), (4096, 4096), (3, 96)])
@pytest.mark.parametrize("src", ["f32", "f16"])
def test_device_quantizer_bit_exact(shape, src):
    w = (rng(7, *shape).standard_normal(shape, dtype=np.float32) * 0.02)
    w[0, :32] = 0.0                                   # zero block
    if shape[1] >= 64:
        w[0, 32:48] = [7.0, 0.5, 1.5, -0.5, 2.5, -1.5, 3.5, -2.5, 4.5, -3.5, 5.5, -4.5, 6.5, -5.5, -6.5, 0]
    if src == "f16":
        w16 = w.astype(np.float16)
        hp, hs = quantizer.quantize_q4_0(w16.astype(np.float32))
        wd, dt = D(w16), F16
    else:
        hp, hs = quantizer.quantize_q4_0(w)
        wd, dt = D(w), F32
    n, k = shape
    p = torch.empty((n, k // 2), dtype=torch.uint8, device="cuda")
    s = torch.empty((n, k // 32), dtype=torch.float16, device="cuda")
    call("orch_quantize_q4_0", ptr(wd), dt, ptr(p), ptr(s), n, k, S())
    np.testing.assert_array_equal(p.cpu().numpy(), hp)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), hs.view(np.uint16))


def test_device_quantizer_matches_reference_fixture(golden_q4):
    for case in ("normal", "edges", "k32"):
        w = golden_q4[f"{case}_w"]
        n, k = w.shape
        p = torch.empty((n, k // 2), dtype=torch.uint8, device="cuda")
        s = torch.empty((n, k // 32), dtype=torch.float16, device="cuda")
        call("orch_quantize_q4_0", D(w), F32, ptr(p), ptr(s), n, k, S())
        np.testing.assert_array_equal(p.cpu().numpy(), golden_q4[f"{case}_packed"])
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), golden_q4[f"{case}_scales"].view(np.uint16))


def test_device_q8_packers_bit_exact():
    w = rng(8).standard_normal((33, 128), dtype=np.float32)
    w[1] = 0
    q = torch.empty((33, 128), dtype=torch.int8, device="cuda")
    s = torch.empty((33, 4), dtype=torch.float16, device="cuda")
    call("orch_quantize_q8_0", D(w), F32, ptr(q), ptr(s), 33, 128, S())
    hq, hs = quantizer.quantize_q8_0(w)
    np.testing.assert_array_equal(q.cpu().numpy(), hq)
    np.testing.assert_array_equal(s.cpu().numpy(), hs)
    sp = torch.empty(33, dtype=torch.float16, device="cuda")
    call("orch_quantize_q8_pc", D(w), F32, ptr(q), ptr(sp), 33, 128, S())
    hq, hs = quantizer.quantize_q8_pc(w)
    np.testing.assert_array_equal(q.cpu().numpy(), hq)
    np.testing.assert_array_equal(sp.cpu().numpy(), hs)


# ---------------------------------------------------------------- elementwise family
@pytest.mark.parametrize("B", [1, 8, 64])
def test_rmsnorm(B):
    x = rng(9, B).standard_normal((B, 4096), dtype=np.float32)
    g = (1 + 0.1 * rng(10).standard_normal(4096, dtype=np.float32))
    ref = ops.rmsnorm(x, g, 1e-5)
    y = torch.empty((B, 4096), dtype=torch.float32, device="cuda")
    call("orch_rmsnorm_ex", D(x), F32, D(g), F32, ptr(y), F32, 1e-5, 4096, B, S())
    assert rel_err(y.cpu().numpy(), ref) <= 1e-5
    yh = torch.empty((B, 4096), dtype=torch.float16, device="cuda")
    call("orch_rmsnorm", D(x.astype(np.float16)), D(g.astype(np.float16)), ptr(yh), 1e-5, 4096, B, S())
    ref16 = ops.rmsnorm(x.astype(np.float16), g.astype(np.float16), 1e-5)
    assert rel_err(yh.float().cpu().numpy(), ref16) <= 1e-3


@pytest.mark.parametrize("B", [1, 8, 64])
def test_rope_per_row(B):
    x = rng(11, B).standard_normal((B, 32, 128), dtype=np.float32)
    pos = rng(12, B).integers(0, 4096, B)
    c, s = ops.precompute_freqs_cis(128, 4096)
    ref = ops.rope(x, c[pos], s[pos])
    y = torch.empty_like(D(x))
    call("orch_rope_ex", D(x), F32, D(c[pos]), D(s[pos]), F32, ptr(y), F32, 128, 32, B, S())
    assert rel_err(y.cpu().numpy(), ref) <= 1e-5
    yh = torch.empty((B, 32, 128), dtype=torch.float16, device="cuda")
    call("orch_rope", D(x.astype(np.float16)), D(c[pos].astype(np.float16)),
         D(s[pos].astype(np.float16)), ptr(yh), 128, 32, B, S())
    ref16 = ops.rope(x.astype(np.float16), c[pos].astype(np.float16), s[pos].astype(np.float16))
    assert rel_err(yh.float().cpu().numpy(), ref16) <= 1e-3


@pytest.mark.parametrize("B,L", [(1, 128), (8, 1024), (64, 4096), (10, 128), (3, 1)])
def test_softmax(B, L):
    rows = max(1, B * (32 if L > 1 else 1))
    x = rng(13, B, L).standard_normal((rows, L), dtype=np.float32) * 3
    ref = ops.softmax_rows(x)
    y = torch.empty((rows, L), dtype=torch.float16, device="cuda")
    call("orch_softmax", D(x.astype(np.float16)), ptr(y), rows, L, S())
    np.testing.assert_allclose(y.float().cpu().numpy(), ops.softmax_rows(x.astype(np.float16)), atol=1e-3)
    yf = torch.empty((rows, L), dtype=torch.float32, device="cuda")
    call("orch_softmax_ex", D(x), F32, ptr(yf), F32, rows, L, S())
    np.testing.assert_allclose(yf.cpu().numpy(), ref, atol=1e-6, rtol=1e-4)


@pytest.mark.parametrize("B", [1, 8, 64])
def test_swiglu_elementwise(B):
    g = rng(14, B).standard_normal((B, 11008), dtype=np.float32)
    u = rng(15, B).standard_normal((B, 11008), dtype=np.float32)
    n = B * 11008
    for dt, npdt, tol in ((F32, np.float32, 1e-6), (F16, np.float16, 1e-3)):
        gd, ud = D(g.astype(npdt)), D(u.astype(npdt))
        t = torch.empty_like(gd)
        call("orch_silu_ex", ptr(gd), ptr(t), dt, n, S())
        call("orch_binary_ex", 1, ptr(t), ptr(ud), ptr(t), dt, n, S())
        ref = ops.mul(ops.silu(g.astype(npdt)), u.astype(npdt))
        np.testing.assert_allclose(t.float().cpu().numpy(), ref, atol=tol * 4, rtol=tol * 4)
        call("orch_binary_ex", 0, ptr(gd), ptr(ud), ptr(t), dt, n, S())
        np.testing.assert_allclose(t.float().cpu().numpy(), ops.add(g.astype(npdt), u.astype(npdt)), atol=tol * 8, rtol=tol)
        # the one-pass form: fp32 silu(g) * u, rounded once
        f = torch.empty_like(gd)
        call("orch_swiglu_ex", ptr(gd), ptr(ud), ptr(f), dt, n, S())
        ref1 = ops.mul(ops.silu(g.astype(npdt).astype(np.float32)), u.astype(npdt).astype(np.float32))
        np.testing.assert_allclose(f.float().cpu().numpy(), ref1, atol=tol * 4, rtol=tol * 4)
        if dt == F16:  # odd length and offset views take the scalar kernel
            call("orch_swiglu_ex", ptr(gd) + 2, ptr(ud) + 2, ptr(f), dt, n - 3, S())
            np.testing.assert_allclose(f.float().cpu().numpy().reshape(-1)[: n - 3], ref1.reshape(-1)[1:n - 2],
                                       atol=tol * 4, rtol=tol * 4)


def test_full_test_kats():
    """examples/full_test.py: add/mul/silu on 1024 fp16, softmax [10,128], embedding ids [1,50,99,0]."""
    a = rng(16).random(1024).astype(np.float16)
    b = rng(17).random(1024).astype(np.float16)
    c = torch.empty(1024, dtype=torch.float16, device="cuda")
    call("orch_add", D(a), D(b), ptr(c), 1024, S())
    np.testing.assert_allclose(c.cpu().numpy(), a + b, atol=1e-3)
    call("orch_mul", D(a), D(b), ptr(c), 1024, S())
    np.testing.assert_allclose(c.cpu().numpy(), a * b, atol=1e-3)
    call("orch_silu", D(a), ptr(c), 1024, S())
    af = a.astype(np.float32)
    np.testing.assert_allclose(c.cpu().numpy(), (af / (1 + np.exp(-af))).astype(np.float16), atol=1e-3)
    ids = np.array([1, 50, 99, 0], np.int32)
    table = rng(18).random((100, 64)).astype(np.float16)
    out = torch.empty((4, 64), dtype=torch.float16, device="cuda")
    call("orch_embedding", D(ids), D(table), ptr(out), 4, 64, 100, S())
    np.testing.assert_array_equal(out.cpu().numpy(), table[ids])


def test_embedding_rejects_out_of_range_ids():
    ids = np.array([3, 100, -1], np.int32)
    table = rng(19).random((100, 8)).astype(np.float16)
    out = torch.full((3, 8), 7.0, dtype=torch.float16, device="cuda")
    flags = _lib.C.c_uint32(0)
    call("orch_device_check", _lib.C.byref(flags), None)
    call("orch_embedding", D(ids), D(table), ptr(out), 3, 8, 100, S())
    call("orch_device_check", _lib.C.byref(flags), None)
    assert flags.value & 4
    o = out.cpu().numpy()
    np.testing.assert_array_equal(o[0], table[3])
    assert np.all(o[1:] == 0)


@pytest.mark.parametrize("M,N,K", [(16, 16, 16), (128, 128, 128), (100, 37, 4096), (1, 16, 4096)])
def test_dense_matmuls(M, N, K):
    a = rng(20, M, K).random((M, K), dtype=np.float32)
    b = rng(21, K, N).random((K, N), dtype=np.float32)
    c = torch.empty((M, N), dtype=torch.float32, device="cuda")
    call("orch_matmul", D(a), D(b), ptr(c), M, N, K, S())
    np.testing.assert_allclose(c.cpu().numpy(), ops.matmul(a, b), rtol=1e-5, atol=1e-4 * K / 16)
    ch = torch.empty((M, N), dtype=torch.float16, device="cuda")
    call("orch_matmul_simd", D(a.astype(np.float16)), D(b.astype(np.float16)), ptr(ch), M, N, K, S())
    ref = ops.matmul(a.astype(np.float16), b.astype(np.float16))
    assert rel_err(ch.float().cpu().numpy(), ref) <= 2e-3


def test_argmax_first_max():
    lg = rng(22).standard_normal((5, 32000), dtype=np.float32)
    lg[2, 7] = lg[2, 9] = 100.0
    lg[4, :] = 1.0
    out = torch.empty(5, dtype=torch.int32, device="cuda")
    call("orch_argmax_rows", D(lg), 5, 32000, ptr(out), S())
    np.testing.assert_array_equal(out.cpu().numpy(), np.argmax(lg, axis=1))


def test_argmax_nan_in_any_lane():
    """np.argmax returns the first NaN of a row. NaNs placed where different threads, warps
    and lanes of the block reduction hold them (not only thread 0) must still win, the lowest
    index among several, in both the plain argmax and the (max, id) pairs of the vocabulary
    split."""
    V = 32000
    lg = rng(24).standard_normal((6, V), dtype=np.float32)
    lg[0, 5] = np.nan                      # thread 5, warp 0
    lg[1, 1000 + 37] = np.nan              # thread 13 of warp 1, second sweep
    lg[2, [31999, 4500, 20001]] = np.nan   # three NaNs in different warps: the first wins
    lg[3, 64] = np.inf                     # an infinity is a number: it wins only without NaN
    lg[3, 700] = np.nan
    lg[4, 3] = 50.0                        # no NaN: the plain maximum
    lg[5, :] = -np.inf
    lg[5, 31000] = np.nan
    out = torch.empty(6, dtype=torch.int32, device="cuda")
    call("orch_argmax_rows", D(lg), 6, V, ptr(out), S())
    np.testing.assert_array_equal(out.cpu().numpy(), np.argmax(lg, axis=1))
    pairs = torch.empty((6, 2), dtype=torch.float32, device="cuda")
    call("orch_argmax_pairs", D(lg), 6, V, 0, ptr(pairs), S())
    np.testing.assert_array_equal(pairs.cpu().numpy()[:, 1].astype(np.int64), np.argmax(lg, axis=1))


def _device_flags():
    torch.cuda.synchronize()
    flags = _lib.C.c_uint32(0)
    call("orch_device_check", _lib.C.byref(flags), None)
    return int(flags.value)


def test_attention_rejects_rows_outside_the_cache():
    """A row whose slot is outside [0, num_slots) or whose position is outside the cache is
    skipped (no cache read, output row left as it was) and reported by orch_device_check
    (slot: bit 8, position: bit 2); the other rows match the oracle. Every index is checked
    on the device before it is used, so the bad rows touch no memory."""
    M, nh, hd, max_seq, nslots = 4, 32, 128, 96, 4
    g = rng(25)
    kc = g.standard_normal((nslots, nh, max_seq, hd), dtype=np.float32).astype(np.float16)
    vc = g.standard_normal((nslots, nh, max_seq, hd), dtype=np.float32).astype(np.float16)
    q = g.standard_normal((M, nh * hd), dtype=np.float32).astype(np.float16)
    pos = np.array([50, max_seq, 60, 20], np.int32)      # row 1: position past the cache
    slots = np.array([3, 0, nslots + 2, 1], np.int32)    # row 2: slot past the cache
    ws_bytes = _lib.lib().orch_attention_workspace_bytes(M, nh, hd, max_seq)
    ws = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device="cuda")
    _device_flags()
    out = torch.full((M, nh * hd), 7.0, dtype=torch.float16, device="cuda")
    call("orch_attention_decode", D(q), D(kc), D(vc), D(pos), D(slots), ptr(out),
         M, nh, hd, max_seq, nslots, ptr(ws), ws_bytes, S())
    assert _device_flags() == 2 | 8
    o = out.float().cpu().numpy()
    assert np.all(o[1] == 7.0) and np.all(o[2] == 7.0)
    for m in (0, 3):
        ref = ops.attention_one(q[m].reshape(nh, hd).astype(np.float32),
                                kc[slots[m], :, :pos[m] + 1].astype(np.float32),
                                vc[slots[m], :, :pos[m] + 1].astype(np.float32))
        assert rel_err(o[m].reshape(nh, hd), ref) <= 1e-2
    # prefill attention: a unit whose slot is outside the cache is skipped the same way
    units = np.array([[0, 2, 0, 0], [2, 2, nslots, 0]], np.int32)
    out2 = torch.full((M, nh * hd), 7.0, dtype=torch.float16, device="cuda")
    call("orch_attention_prefill", D(q), D(kc), D(vc), D(units), 2, ptr(out2), M, nh, hd, max_seq, nslots, S())
    assert _device_flags() == 8
    assert np.all(out2.float().cpu().numpy()[2:] == 7.0)


# ---------------------------------------------------------------- attention over the KV cache
@pytest.mark.parametrize("M,L,hd", [(1, 1, 128), (1, 128, 128), (1, 576, 128), (16, 640, 128),
                                    (64, 513, 128), (3, 1500, 64), (2, 40, 32)])
def test_attention_decode(M, L, hd):
    nh, max_seq = 4 if hd != 128 else 32, max(L, 1) + 7
    g = rng(23, M, L, hd)
    kc = g.standard_normal((M, nh, max_seq, hd), dtype=np.float32).astype(np.float16)
    vc = g.standard_normal((M, nh, max_seq, hd), dtype=np.float32).astype(np.float16)
    q = g.standard_normal((M, nh * hd), dtype=np.float32).astype(np.float16)
    pos = np.array([max(0, L - 1 - (i % 3)) for i in range(M)], np.int32)
    slots = np.arange(M, dtype=np.int32)[::-1].copy()
    ws_bytes = _lib.lib().orch_attention_workspace_bytes(M, nh, hd, max_seq)
    ws = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device="cuda")
    out = torch.empty((M, nh * hd), dtype=torch.float16, device="cuda")
    call("orch_attention_decode", D(q), D(kc), D(vc), D(pos), D(slots), ptr(out),
         M, nh, hd, max_seq, M, ptr(ws), ws_bytes, S())
    o = out.float().cpu().numpy()
    for m in range(M):
        sl, L_m = slots[m], pos[m] + 1
        ref = ops.attention_one(q[m].reshape(nh, hd).astype(np.float32), kc[sl, :, :L_m].astype(np.float32),
                                vc[sl, :, :L_m].astype(np.float32))
        assert rel_err(o[m].reshape(nh, hd), ref) <= 1e-2


@pytest.mark.parametrize("M,K,R", [(5, 4096, 48), (300, 4096, 48), (4096, 4096, 48), (1000, 96, 16), (4096, 512, 80),
                                   (4096, 4096, 32), (257, 11008, 32), (512, 4096, 30)])
def test_lora_xa(M, K, R):
    """t = x.A (the first LoRA factor, orchard/model.py:60-76): fp16 x, fp32 A, fp32 t. Small M,
    R > 64 or R % 4 != 0 take the one-row-per-CTA fp32 kernel; M >= 256 otherwise the tiled
    tensor-core one (TF32 with A split in two terms, each 8-k step added in fp32, 32 or 64
    columns). Both are fp32-accurate: max|gpu - ref| / max|ref| <= 1e-5 against fp32 NumPy."""
    g = np.random.default_rng([31, M, K, R])
    x = g.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    a = (g.standard_normal((K, R), dtype=np.float32) * 0.01).astype(np.float32)
    t = torch.empty((M, R), dtype=torch.float32, device="cuda")
    call("orch_lora_xa", D(x), D(a), t, M, K, R, S())
    torch.cuda.synchronize()
    ref = x.astype(np.float32) @ a
    assert rel_err(t.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("lens,starts", [([1, 13, 64, 65, 200], [0, 0, 0, 3, 100]), ([512, 512], [0, 0]),
                                         ([70, 1, 129], [500, 7, 0])])
def test_attention_prefill(lens, starts):
    """Prefill attention (tensor cores, 64 rows per CTA) against the decode kernel run per row
    and the oracle. Cache positions after each sequence's last row hold NaN: the kernel must
    never read them. Same 1e-2 bound against the oracle as decode attention; against the
    decode kernel (both fp32-accurate, fp16 outputs) <= 2e-3 of max|out|."""
    from orchard_b200.model import prefill_units

    nh, hd = 32, 128
    nseq = len(lens)
    max_seq = max(s + n for s, n in zip(starts, lens)) + 5
    g = rng(41, nseq, sum(lens))
    kc = g.standard_normal((nseq, nh, max_seq, hd), dtype=np.float32).astype(np.float16)
    vc = g.standard_normal((nseq, nh, max_seq, hd), dtype=np.float32).astype(np.float16)
    for i in range(nseq):
        kc[i, :, starts[i] + lens[i]:] = np.nan
        vc[i, :, starts[i] + lens[i]:] = np.nan
    pos = np.concatenate([np.arange(s, s + n) for s, n in zip(starts, lens)]).astype(np.int32)
    slots = np.concatenate([np.full(n, i) for i, n in enumerate(lens)]).astype(np.int32)
    M = len(pos)
    q = g.standard_normal((M, nh * hd), dtype=np.float32).astype(np.float16)
    units = prefill_units(pos, slots)
    out = torch.empty((M, nh * hd), dtype=torch.float16, device="cuda")
    call("orch_attention_prefill", D(q), D(kc), D(vc), D(units), len(units), ptr(out), M, nh, hd, max_seq, kc.shape[0], S())
    ws_bytes = _lib.lib().orch_attention_workspace_bytes(M, nh, hd, max_seq)
    ws = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device="cuda")
    out_d = torch.empty((M, nh * hd), dtype=torch.float16, device="cuda")
    call("orch_attention_decode", D(q), D(kc), D(vc), D(pos), D(slots), ptr(out_d), M, nh, hd, max_seq, kc.shape[0], ptr(ws),
         ws_bytes, S())
    o, od = out.float().cpu().numpy(), out_d.float().cpu().numpy()
    assert np.all(np.isfinite(o))
    assert np.abs(o - od).max() <= 2e-3 * np.abs(od).max()
    for m in range(0, M, 7):
        sl, L_m = slots[m], pos[m] + 1
        ref = ops.attention_one(q[m].reshape(nh, hd).astype(np.float32), kc[sl, :, :L_m].astype(np.float32),
                                vc[sl, :, :L_m].astype(np.float32))
        assert rel_err(o[m].reshape(nh, hd), ref) <= 1e-2
