"""Vectorised NumPy restatement of the reference's hot-path arithmetic.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Every function cites the
reference file:line it restates (paths relative to the Orchard project root).

Conventions
-----------
* Weights are ``[N, K]`` (out, in) row-major, as the reference quantizer and the
  Metal kernels assume (``orchard/quantizer.py:12-16``).
* Activations are computed in float32, the arithmetic type of every Metal kernel
  (``orchard/kernels/*.metal`` accumulate in ``float``). Returned arrays are
  float32; callers that emulate a ``half`` store cast with ``.astype(np.float16)``.
"""

from __future__ import annotations

import numpy as np

GROUP = 32
FP16_ZERO_SCALE = np.float16(1e-5)  # orchard/quantizer.py:33 (stored as fp16 subnormal)


# --------------------------------------------------------------------------------------
# INT4 "Q4_0-like" packing
# --------------------------------------------------------------------------------------

def quantize_q4_0(weight: np.ndarray, group_size: int = GROUP):
    """Restates ``quantize_q4_0`` (orchard/quantizer.py:3-78).

    scale = fp16(max|w_g| / 7) per group of ``group_size`` (quantizer.py:25-30),
    zero scales -> fp16(1e-5) (quantizer.py:33), q = clip(round_half_even(w/scale + 8),
    0, 15) (quantizer.py:49-53), low nibble = even index (quantizer.py:67-73).
    The arithmetic is done in the dtype NumPy's promotion gives for ``weight``
    (float32 for the loader's fp32 cast, orchard/loader.py:121-124).
    """
    w = np.asarray(weight)
    n, k = w.shape
    assert k % group_size == 0, f"K={k} not divisible by group size {group_size}"
    g = w.reshape(n, k // group_size, group_size)
    scales = (np.abs(g).max(axis=2) / 7.0).astype(np.float16)
    scales[scales == 0] = FP16_ZERO_SCALE
    q = np.rint(g / scales[:, :, None] + 8.0).astype(np.int8)
    q = np.clip(q, 0, 15).astype(np.uint8).reshape(n, k // 2, 2)
    packed = (q[:, :, 1] << 4) | q[:, :, 0]
    return packed.astype(np.uint8), scales


def unpack_q4_0(packed: np.ndarray) -> np.ndarray:
    """Nibbles -> uint8 codes ``[N, K]``: low nibble even k, high nibble odd k
    (orchard/kernels/gemv_int4.metal:45-49, 65-69)."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty((p.shape[0], p.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = p & 0x0F
    out[:, 1::2] = p >> 4
    return out


def dequantize_q4_0(packed, scales, group_size: int = GROUP) -> np.ndarray:
    """``(q - 8) * scale`` in float32 (gemv_int4.metal:48-49, 69). Exact in fp32."""
    q = unpack_q4_0(packed).astype(np.float32) - 8.0
    n, k = q.shape
    s = np.asarray(scales, dtype=np.float16).astype(np.float32)
    return (q.reshape(n, k // group_size, group_size) * s[:, :, None]).reshape(n, k)


# --------------------------------------------------------------------------------------
# INT8 group-32 (reference) and per-channel (new) formats
# --------------------------------------------------------------------------------------

def _round_half_away(v: np.ndarray) -> np.ndarray:
    """C ``std::round`` (src/main.cpp:58): halves away from zero, exact in fp32."""
    t = np.trunc(v)
    return t + np.sign(v) * (np.abs(v - t) >= 0.5)


def quantize_q8_0(weight: np.ndarray, group_size: int = GROUP):
    """Restates the only INT8 quantizer, ``quantize_q8_0`` (src/main.cpp:35-64):
    scale = fp16(max|w_g|/127), zero -> 1.0, q = (int8) std::round(w / scale)."""
    w = np.asarray(weight, dtype=np.float32)
    n, k = w.shape
    assert k % group_size == 0
    g = w.reshape(n, k // group_size, group_size)
    scales = (np.abs(g).max(axis=2) / np.float32(127.0)).astype(np.float16)
    scales[scales == 0] = np.float16(1.0)
    q = _round_half_away(g / scales.astype(np.float32)[:, :, None])
    q = np.clip(q, -127, 127).astype(np.int8)
    return q.reshape(n, k), scales


def quantize_q8_pc(weight: np.ndarray):
    """Per-output-channel INT8 (the BASELINE sweep's INT8 variant, no reference
    counterpart): same rule as ``quantize_q8_0`` with one group spanning the row."""
    w = np.asarray(weight, dtype=np.float32)
    scales = (np.abs(w).max(axis=1) / np.float32(127.0)).astype(np.float16)
    scales[scales == 0] = np.float16(1.0)
    q = np.clip(_round_half_away(w / scales.astype(np.float32)[:, None]), -127, 127)
    return q.astype(np.int8), scales


def dequantize_q8_0(w8, scales, group_size: int = GROUP) -> np.ndarray:
    q = np.asarray(w8, dtype=np.int8).astype(np.float32)
    n, k = q.shape
    s = np.asarray(scales, dtype=np.float16).astype(np.float32)
    return (q.reshape(n, k // group_size, group_size) * s[:, :, None]).reshape(n, k)


def dequantize_q8_pc(w8, scales) -> np.ndarray:
    q = np.asarray(w8, dtype=np.int8).astype(np.float32)
    return q * np.asarray(scales, dtype=np.float16).astype(np.float32)[:, None]


# --------------------------------------------------------------------------------------
# GEMV / skinny GEMM
# --------------------------------------------------------------------------------------

def _as_rows(x) -> np.ndarray:
    x = np.asarray(x).astype(np.float32)
    return x.reshape(1, -1) if x.ndim == 1 else x


def gemm_q4_0(packed, scales, x) -> np.ndarray:
    """``y[b, n] = sum_g s[n,g] * sum_{i in g} (q[n,i]-8) * x[b,i]`` in fp32.

    B = 1 restates ``gemv_q4_0`` (orchard/kernels/gemv_int4.metal:10-74). For B > 1 the
    reference ``gemm_q4_0`` (orchard/kernels/gemm_int4.metal:47-62) pairs nibbles with
    the wrong inputs; the oracle follows the quantizer + GEMV nibble order instead
    (reference defect, documented)."""
    w = dequantize_q4_0(packed, scales)
    return _as_rows(x) @ w.T


def gemv_q8_0(w8, scales, x) -> np.ndarray:
    """orchard/kernels/gemv_int8.metal:13-55 (group-32 scales)."""
    return _as_rows(x) @ dequantize_q8_0(w8, scales).T


def gemm_q8_pc(w8, scales, x) -> np.ndarray:
    """Per-channel INT8: ``y = s[n] * sum_i q[n,i] x[b,i]``."""
    return _as_rows(x) @ dequantize_q8_pc(w8, scales).T


# --------------------------------------------------------------------------------------
# Normalisation, RoPE, softmax, elementwise
# --------------------------------------------------------------------------------------

def rmsnorm(x, weight, eps: float) -> np.ndarray:
    """orchard/kernels/rmsnorm.metal:23-35: ``x * rsqrt(sum(x^2)/N + eps) * w``."""
    x = _as_rows(x)
    n = x.shape[1]
    ss = (x.astype(np.float64) ** 2).sum(axis=1) / n
    r = (1.0 / np.sqrt(ss + eps)).astype(np.float32)
    return x * r[:, None] * np.asarray(weight, dtype=np.float32)[None, :]


def precompute_freqs_cis(dim: int, end: int, theta: float = 10000.0):
    """orchard/model.py:7-13 (float32 tables ``[end, dim/2]``)."""
    freqs = 1.0 / (theta ** (np.arange(0, dim, 2)[: dim // 2].astype(np.float32) / dim))
    t = np.arange(end).astype(np.float32)
    f = np.outer(t, freqs)
    return np.cos(f), np.sin(f)


def rope(x, cos, sin) -> np.ndarray:
    """Interleaved-pair rotation (orchard/kernels/rope.metal:26-49) with per-row
    angles: ``x`` is ``[rows, heads, hd]``, ``cos``/``sin`` are ``[rows, hd/2]``.

    The Metal kernel indexes ``freqs[i]`` for every row (rope.metal:39-40) although the
    host passes one row of angles per sequence (orchard/model.py:322-341); the oracle
    uses the row's own angles (reference defect, documented)."""
    x = np.asarray(x, dtype=np.float32)
    c = np.asarray(cos, dtype=np.float32)[:, None, :]
    s = np.asarray(sin, dtype=np.float32)[:, None, :]
    x0 = x[..., 0::2]
    x1 = x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def softmax_rows(x) -> np.ndarray:
    """orchard/kernels/softmax.metal:18-55: max, sum of exp, normalise (fp32)."""
    x = np.asarray(x, dtype=np.float32)
    m = x.max(axis=1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=1, keepdims=True)


def add(a, b):
    """orchard/kernels/elementwise.metal:4-11."""
    return np.asarray(a, np.float32) + np.asarray(b, np.float32)


def mul(a, b):
    """orchard/kernels/elementwise.metal:13-20."""
    return np.asarray(a, np.float32) * np.asarray(b, np.float32)


def silu(x):
    """orchard/kernels/elementwise.metal:22-30: ``x / (1 + exp(-x))`` in fp32."""
    x = np.asarray(x, np.float32)
    return x * (np.float32(1.0) / (np.float32(1.0) + np.exp(-x)))


def matmul(a, b):
    """orchard/kernels/matmul.metal:4-23: fp32 ``C[M,N] = A[M,K] @ B[K,N]``."""
    return np.asarray(a, np.float32) @ np.asarray(b, np.float32)


def embedding(ids, table):
    """orchard/kernels/embedding.metal:4-17: ``out[t] = W[ids[t]]``."""
    return np.asarray(table)[np.asarray(ids, dtype=np.int64)]


def attention_one(q, k_cache, v_cache) -> np.ndarray:
    """Per-sequence attention of one new token over its cache, as the reference's
    host loop does it (orchard/model.py:117-137): per head
    ``softmax(q.K / sqrt(hd)) . V`` over positions 0..pos inclusive.

    ``q``: ``[H, hd]``; ``k_cache``/``v_cache``: ``[H, L, hd]`` (fp32)."""
    hd = q.shape[-1]
    scale = np.float32(1.0 / np.sqrt(hd))
    s = np.einsum("hd,hld->hl", q.astype(np.float32), k_cache.astype(np.float32)) * scale
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=1, keepdims=True)
    return np.einsum("hl,hld->hd", p, v_cache.astype(np.float32))
