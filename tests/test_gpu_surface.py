"""The reference's operator surface on the GPU: ``orchard_core`` (pybind11) and the C ABI's
buffer calls.

``LlamaLayer.forward`` (orchard/model.py:78-195) is the reference's own client of the surface.
The reference package itself is not importable where these tests run, so the test below
drives ``orchard_core`` (registered by ``install_as_orchard_core()``) through the same calls
in the same order -- Float32 activation tensors, Int8 packed weights with Float16 scales,
``run_gemv_q4_0`` for one row and ``run_gemm_q4_0`` for a batch, RoPE in place, attention on
the host over per-sequence caches laid out as the reference keeps them (K [heads, hd, L],
V [heads, L, hd]), ``run_add`` residuals, ``run_silu`` then ``run_mul`` -- and compares with
``tests/golden/layer_trace.npz``, which ``make_golden.py`` recorded by running the
reference's ``LlamaLayer.forward`` itself: ten single-token steps of one sequence, then a
batch of two rows at positions 10 and 0. Tolerance: max|gpu - ref| / max|ref| <= 1e-2 on
each layer output (the layer-output bound), 1e-3 on the caches.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err
from orchard_b200 import _lib, install_as_orchard_core, quantizer

pytestmark = pytest.mark.gpu

PROJ = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj", "wo": "self_attn.o_proj",
        "w1": "mlp.gate_proj", "w3": "mlp.up_proj", "w2": "mlp.down_proj"}


@pytest.fixture(scope="module")
def core():
    assert torch.cuda.is_available()
    return install_as_orchard_core()


def upload(core, be, arr, dtype):
    t = core.Tensor(be, list(arr.shape), dtype)
    t.copy_from_host(np.ascontiguousarray(arr))
    return t


class SurfaceLayer:
    """Layer 0 of the tiny checkpoint on the surface, called as orchard/model.py:78-195 calls it."""

    def __init__(self, core, be, cfg, ckpt):
        self.core, self.be = core, be
        self.H = cfg["hidden_size"]
        self.F = cfg["intermediate_size"]
        self.nh = cfg["num_attention_heads"]
        self.hd = self.H // self.nh
        self.eps = cfg["rms_norm_eps"]
        self.w = {}
        for name, hf in PROJ.items():  # the loader's cast and packer (orchard/loader.py:106-138)
            p, s = quantizer.quantize_q4_0(np.asarray(ckpt[f"model.layers.0.{hf}.weight"], np.float32))
            self.w[name] = (upload(core, be, p.view(np.int8), core.DType.Int8),
                            upload(core, be, s, core.DType.Float16))
        self.attn_norm = upload(core, be, np.asarray(ckpt["model.layers.0.input_layernorm.weight"], np.float32),
                                core.DType.Float32)
        self.ffn_norm = upload(core, be, np.asarray(ckpt["model.layers.0.post_attention_layernorm.weight"],
                                                    np.float32), core.DType.Float32)
        self.k_cache, self.v_cache = {}, {}

    def f32(self, n):
        return self.core.Tensor(self.be, [n], self.core.DType.Float32)

    def proj(self, name, x, out, K, N, B):
        w, s = self.w[name]
        if B == 1:
            self.be.run_gemv_q4_0(w, s, x, out, K, N)
        else:
            self.be.run_gemm_q4_0(w, s, x, out, K, N, B)

    def forward(self, x, cos, sin, slots):
        be, H, F, nh, hd = self.be, self.H, self.F, self.nh, self.hd
        B = len(slots)
        xn = self.f32(B * H)
        be.run_rmsnorm(x, self.attn_norm, xn, self.eps, H, B)
        q, k, v = self.f32(B * H), self.f32(B * H), self.f32(B * H)
        for name, t in (("wq", q), ("wk", k), ("wv", v)):
            self.proj(name, xn, t, H, H, B)
        be.run_rope(q, cos, sin, q, hd, nh, B)
        be.run_rope(k, cos, sin, k, hd, nh, B)
        qh = q.copy_to_host().reshape(B, nh, hd)
        kh = k.copy_to_host().reshape(B, nh, hd)
        vh = v.copy_to_host().reshape(B, nh, hd)
        att = np.zeros((B, nh, hd), np.float32)
        for i, sl in enumerate(slots):  # host attention over per-sequence caches
            kc = self.k_cache.get(sl, np.zeros((nh, hd, 0), np.float32))
            vc = self.v_cache.get(sl, np.zeros((nh, 0, hd), np.float32))
            self.k_cache[sl] = kc = np.concatenate([kc, kh[i][:, :, None]], axis=2)
            self.v_cache[sl] = vc = np.concatenate([vc, vh[i][:, None, :]], axis=1)
            for h in range(nh):
                sc = (qh[i, h] @ kc[h]) / np.sqrt(hd)
                e = np.exp(sc - sc.max())
                att[i, h] = (e / e.sum()) @ vc[h]
        attn = self.f32(B * H)
        attn.copy_from_host(att.reshape(-1))
        o = self.f32(B * H)
        self.proj("wo", attn, o, H, H, B)
        be.run_add(x, o, x, B * H)
        xf = self.f32(B * H)
        be.run_rmsnorm(x, self.ffn_norm, xf, self.eps, H, B)
        gate, up = self.f32(B * F), self.f32(B * F)
        self.proj("w1", xf, gate, H, F, B)
        self.proj("w3", xf, up, H, F, B)
        be.run_silu(gate, gate, B * F)
        be.run_mul(gate, up, gate, B * F)
        d = self.f32(B * H)
        self.proj("w2", gate, d, F, H, B)
        be.run_add(x, d, x, B * H)
        return x


def test_reference_layer_flow_through_orchard_core(core, golden_model, golden_trace):
    cfg, tr = golden_model["config"], golden_trace
    be = core.MetalBackend()
    be.initialize("")
    assert be.is_available() and "B200" in be.get_device_name()
    layer = SurfaceLayer(core, be, cfg, golden_model["ckpt"])
    hd = layer.hd
    inv = 1.0 / (10000.0 ** (np.arange(0, hd, 2)[: hd // 2].astype(np.float32) / hd))  # orchard/model.py:7-13
    ang = np.outer(np.arange(cfg["max_position_embeddings"]).astype(np.float32), inv)
    cos_t, sin_t = np.cos(ang), np.sin(ang)

    def call(xrows, positions, slots):
        B = len(slots)
        x = layer.f32(B * layer.H)
        x.copy_from_host(np.ascontiguousarray(xrows, np.float32).reshape(-1))
        fc, fs = layer.f32(B * hd // 2), layer.f32(B * hd // 2)
        fc.copy_from_host(np.ascontiguousarray(cos_t[positions]).reshape(-1))
        fs.copy_from_host(np.ascontiguousarray(sin_t[positions]).reshape(-1))
        layer.forward(x, fc, fs, slots)
        return x.copy_to_host().reshape(B, layer.H)

    for p in range(tr["seq_x_in"].shape[0]):
        out = call(tr["seq_x_in"][p:p + 1], [p], [20])
        assert rel_err(out, tr["seq_x_out"][p:p + 1]) <= 1e-2, p
    out = call(tr["batch_x_in"], [int(v) for v in tr["batch_pos"]], [20, 21])
    assert rel_err(out, tr["batch_x_out"]) <= 1e-2
    assert rel_err(layer.k_cache[20], tr["k_cache_a"]) <= 1e-3
    assert rel_err(layer.v_cache[20], tr["v_cache_a"]) <= 1e-3


def test_tensor_buffer_semantics(core):
    """src/runtime/tensor.cpp:60-72, src/bindings.cpp:67-79: exact byte count in, a large
    enough destination out, shape / numel / size_bytes per dtype (4 / 2 / 1 bytes)."""
    be = core.MetalBackend()
    be.initialize("")
    for dt, npdt in ((core.DType.Float32, np.float32), (core.DType.Float16, np.float16), (core.DType.Int8, np.int8)):
        t = core.Tensor(be, [3, 5], dt)
        assert t.shape() == [3, 5] and t.numel() == 15 and t.size_bytes() == 15 * np.dtype(npdt).itemsize
        src = (np.arange(15) - 7).astype(npdt)
        t.copy_from_host(src)
        dst = np.zeros(15, npdt)
        t.copy_to_host(dst)
        np.testing.assert_array_equal(dst, src)
        np.testing.assert_array_equal(t.copy_to_host().reshape(-1), src)
        with pytest.raises(RuntimeError):
            t.copy_from_host(np.zeros(14, npdt))
        with pytest.raises(RuntimeError):
            t.copy_to_host(np.zeros(14, npdt))
    empty = core.Tensor(be, [0], core.DType.Float32)  # the reference allocates a tiny buffer
    assert empty.numel() == 0 and empty.size_bytes() == 0


def test_c_abi_buffers():
    """orch_alloc / orch_h2d / orch_d2h / orch_memset / orch_free (metal_backend.h:19-22):
    a round trip of a host buffer, an offset copy, a memset, and the null-pointer errors."""
    lib = _lib.lib()
    _lib.call("orch_init", 0, None)
    ptr = ctypes.c_void_p()
    _lib.call("orch_alloc", 4096, ctypes.byref(ptr))
    assert ptr.value
    src = np.arange(1024, dtype=np.float32)
    _lib.call("orch_h2d", ptr.value, src.ctypes.data, src.nbytes, None)
    back = np.zeros_like(src)
    _lib.call("orch_d2h", back.ctypes.data, ptr.value, back.nbytes, None)
    np.testing.assert_array_equal(back, src)
    part = np.zeros(16, np.float32)
    _lib.call("orch_d2h", part.ctypes.data, ptr.value + 64 * 4, part.nbytes, None)
    np.testing.assert_array_equal(part, src[64:80])
    _lib.call("orch_memset", ptr.value, 0, 4096, None)
    _lib.call("orch_sync", None)
    _lib.call("orch_d2h", back.ctypes.data, ptr.value, back.nbytes, None)
    assert not back.any()
    assert lib.orch_h2d(None, src.ctypes.data, 16, None) == 1
    assert lib.orch_d2h(back.ctypes.data, None, 16, None) == 1
    _lib.call("orch_free", ptr.value)
    zero = ctypes.c_void_p()
    _lib.call("orch_alloc", 0, ctypes.byref(zero))  # an empty tensor still gets a buffer
    assert zero.value
    _lib.call("orch_free", zero.value)
