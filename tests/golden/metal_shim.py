"""A NumPy stand-in for the reference's ``orchard_core`` module, used ONLY by
``make_golden.py`` to run the reference's own Python (orchard/model.py,
orchard/loader.py, orchard/quantizer.py) on the CPU of this container.

Each ``run_*`` is a literal transcription of the Metal kernel it replaces, in the
kernel's float32 arithmetic and accumulation order (vectorised over output rows
only), so the fixtures it produces are an independent check on the vectorised
oracle in ``oracle/ops.py``.

Decisions where the reference disagrees with itself:
* F4 (dtype blindness): a tensor's values are read and written in the dtype the
  host declared for it (the reference host declares Float32 activations).
* F3 (``gemm_q4_0`` nibble order): the batched op uses the quantizer/GEMV order.
* F6 (RoPE row): each row uses its own row of angles.
* F5 (``copy_to_host()`` without a destination): returns a fresh array.
"""

from __future__ import annotations

import enum

import numpy as np

F32 = np.float32


class DType(enum.Enum):
    Float32 = 0
    Float16 = 1
    Int8 = 2


Float32, Float16, Int8 = DType.Float32, DType.Float16, DType.Int8
_NP = {DType.Float32: np.float32, DType.Float16: np.float16, DType.Int8: np.int8}


class Tensor:
    """src/runtime/tensor.cpp:17-72 semantics on a NumPy buffer."""

    def __init__(self, backend, shape, dtype):
        self.backend = backend
        self._shape = [int(s) for s in shape]
        self.dtype = dtype
        n = int(np.prod(self._shape)) if self._shape else 0
        self.buf = np.zeros(n, dtype=_NP[dtype])

    def copy_from_host(self, data):
        a = np.ascontiguousarray(data)
        if a.nbytes != self.buf.nbytes:  # tensor.cpp:60-65
            raise RuntimeError("Size mismatch in copy_from_host")
        self.buf[:] = np.frombuffer(a.tobytes(), dtype=self.buf.dtype)

    def copy_to_host(self, out=None):
        if out is None:
            return self.buf.copy()
        o = np.asarray(out)
        if o.nbytes < self.buf.nbytes:  # bindings.cpp:71-79
            raise RuntimeError("Buffer too small")
        o.reshape(-1).view(np.uint8)[: self.buf.nbytes] = self.buf.view(np.uint8)
        return o

    def shape(self):
        return list(self._shape)

    def numel(self):
        return self.buf.size

    def size_bytes(self):
        return self.buf.nbytes

    # values as float32 (activations) / raw views (weights)
    def f(self):
        return self.buf.astype(F32)

    def put(self, v):
        v = np.asarray(v, dtype=F32).reshape(-1)
        self.buf[: v.size] = v.astype(self.buf.dtype)


def _dot4(a, b):
    """Sequential fp32 4-term dot product."""
    s = (a[..., 0] * b[0]).astype(F32)
    s = (s + a[..., 1] * b[1]).astype(F32)
    s = (s + a[..., 2] * b[2]).astype(F32)
    return (s + a[..., 3] * b[3]).astype(F32)


class MetalBackend:
    def __init__(self):
        self.ready = False

    def initialize(self, resource_path=None):
        self.ready = True

    def is_available(self):
        return True

    def get_device_name(self):
        return "metal-shim (numpy)"

    # gemv_int4.metal:10-74, literal order
    def _q4_row_dot(self, w, s, x, K, N):
        w = w.buf.view(np.uint8).reshape(N, K // 2)
        s = s.buf.view(np.float16).reshape(N, K // 32)
        acc = np.zeros(N, dtype=F32)
        for k in range(0, K, 32):
            scale = s[:, k // 32].astype(F32)
            for j in range(4):
                p = w[:, k // 2 + 4 * j: k // 2 + 4 * j + 4]
                lo = (p & 0x0F).astype(F32) - F32(8.0)
                hi = (p >> 4).astype(F32) - F32(8.0)
                x03 = x[k + 8 * j: k + 8 * j + 4]
                x47 = x[k + 8 * j + 4: k + 8 * j + 8]
                ev = np.array([x03[0], x03[2], x47[0], x47[2]], dtype=F32)
                od = np.array([x03[1], x03[3], x47[1], x47[3]], dtype=F32)
                acc = (acc + _dot4(lo, ev) * scale).astype(F32)
                acc = (acc + _dot4(hi, od) * scale).astype(F32)
        return acc

    def run_gemv_q4_0(self, w, s, inp, out, K, N):
        out.put(self._q4_row_dot(w, s, inp.f()[:K], K, N))

    def run_gemm_q4_0(self, w, s, inp, out, K, N, B):
        x = inp.f()
        res = np.zeros((B, N), dtype=F32)
        for b in range(B):
            res[b] = self._q4_row_dot(w, s, x[b * K:(b + 1) * K], K, N)
        out.put(res)

    # gemv_int8.metal:13-55
    def run_gemv_q8_0(self, w, s, inp, out, K, N):
        w8 = w.buf.view(np.int8).reshape(N, K).astype(F32)
        sc = s.buf.view(np.float16).reshape(N, K // 32).astype(F32)
        x = inp.f()
        acc = np.zeros(N, dtype=F32)
        for k in range(0, K, 32):
            for i in range(0, 32, 4):
                acc = (acc + _dot4(w8[:, k + i: k + i + 4], x[k + i: k + i + 4]) * sc[:, k // 32]).astype(F32)
        out.put(acc)

    # rmsnorm.metal:4-36
    def run_rmsnorm(self, inp, weight, out, eps, N, count):
        x = inp.f().reshape(-1)[: N * count].reshape(count, N)
        w = weight.f()
        ss = np.zeros(count, dtype=F32)
        for i in range(N):
            ss = (ss + x[:, i] * x[:, i]).astype(F32)
        r = (F32(1.0) / np.sqrt((ss / F32(N) + F32(eps)).astype(F32))).astype(F32)
        out.put((x * r[:, None]).astype(F32) * w[None, :N])

    # rope.metal:4-50 with per-row angles
    def run_rope(self, inp, fcos, fsin, out, head_dim, num_heads, seq_len):
        x = inp.f()[: seq_len * num_heads * head_dim].reshape(seq_len, num_heads, head_dim)
        c = fcos.f().reshape(-1, head_dim // 2)
        s = fsin.f().reshape(-1, head_dim // 2)
        c = np.broadcast_to(c[:seq_len] if c.shape[0] >= seq_len else c[:1], (seq_len, head_dim // 2))
        s = np.broadcast_to(s[:seq_len] if s.shape[0] >= seq_len else s[:1], (seq_len, head_dim // 2))
        x0, x1 = x[..., 0::2], x[..., 1::2]
        o = np.empty_like(x)
        o[..., 0::2] = (x0 * c[:, None, :] - x1 * s[:, None, :]).astype(F32)
        o[..., 1::2] = (x0 * s[:, None, :] + x1 * c[:, None, :]).astype(F32)
        out.put(o)

    # elementwise.metal:4-30
    def run_add(self, a, b, c, size):
        c.put(a.f()[:size] + b.f()[:size])

    def run_mul(self, a, b, c, size):
        c.put(a.f()[:size] * b.f()[:size])

    def run_silu(self, inp, out, size):
        x = inp.f()[:size]
        out.put(x * (F32(1.0) / (F32(1.0) + np.exp(-x))))

    # softmax.metal:4-56
    def run_softmax(self, inp, out, rows, cols):
        x = inp.f()[: rows * cols].reshape(rows, cols)
        m = x.max(axis=1, keepdims=True)
        e = np.exp(x - m)
        out.put(e / e.sum(axis=1, keepdims=True))

    # matmul.metal:4-23 (sequential K)
    def run_matmul(self, a, b, c, M, N, K):
        A = a.f()[: M * K].reshape(M, K)
        Bm = b.f()[: K * N].reshape(K, N)
        acc = np.zeros((M, N), dtype=F32)
        for k in range(K):
            acc = (acc + A[:, k:k + 1] * Bm[k:k + 1, :]).astype(F32)
        c.put(acc)

    def run_matmul_simd(self, a, b, c, M, N, K):
        A = a.buf.view(np.float16)[: M * K].reshape(M, K).astype(F32)
        Bm = b.buf.view(np.float16)[: K * N].reshape(K, N).astype(F32)
        c.put(A @ Bm)

    # embedding.metal:4-17
    def run_embedding(self, ids, weights, out, num_tokens, hidden_dim):
        i = ids.buf.view(np.int32)[:num_tokens].astype(np.int64)
        w = weights.buf.view(np.float16).reshape(-1, hidden_dim)
        out.put(w[i].astype(F32))
