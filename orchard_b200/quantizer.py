"""Host-side packers for the quantised weight formats.

``quantize_q4_0`` produces exactly the bytes of the reference packer
(orchard/quantizer.py:3-78): ``packed uint8 [N, K/2]`` (low nibble = even k) and
``scales fp16 [N, K/group]`` with ``scale = fp16(max|w|/7)``, zero scales replaced by
fp16(1e-5), ``q = clip(round_half_even(w/scale + 8), 0, 15)``. The same rule runs on
the GPU in ``orch_quantize_q4_0`` (bit-identical, much faster for 7B-sized models).

INT8: ``quantize_q8_0`` follows the reference's C++ packer (src/main.cpp:35-64: group 32,
``scale = fp16(max|w|/127)``, zero -> 1.0, round half away from zero);
``quantize_q8_pc`` is the per-output-channel variant (one scale per row).
"""

from __future__ import annotations

import numpy as np

__all__ = ["quantize_q4_0", "quantize_q8_0", "quantize_q8_pc", "Q4_ZERO_SCALE"]

Q4_ZERO_SCALE = np.float16(1e-5)


def quantize_q4_0(weight_fp32, group_size: int = 32):
    """Pack ``weight_fp32 [N, K]`` (out, in) into the Q4_0-like format.

    Arithmetic happens in the dtype of the input, as in the reference (its loader and
    optimizer pass float32, orchard/loader.py:121-124, orchard/optimizer.py:50-53)."""
    w = np.asarray(weight_fp32)
    if w.ndim != 2:
        raise ValueError(f"expected a 2-D [N, K] weight, got shape {w.shape}")
    n, k = w.shape
    if group_size <= 0 or k % group_size != 0:
        raise ValueError(f"K = {k} is not a whole number of {group_size}-wide scale groups")
    blocks = w.reshape(n, k // group_size, group_size)
    scale = (np.max(np.abs(blocks), axis=2) / 7.0).astype(np.float16)
    scale[scale == 0] = Q4_ZERO_SCALE
    codes = np.clip(np.round(blocks / scale[:, :, None] + 8.0).astype(np.int8), 0, 15)
    codes = codes.astype(np.uint8).reshape(n, k // 2, 2)
    packed = codes[..., 0] | (codes[..., 1] << 4)
    return packed.astype(np.uint8), scale


def _round_away(v):
    """C ``std::round``: nearest integer, halves away from zero (exact in fp32)."""
    t = np.trunc(v)
    return t + np.sign(v) * (np.abs(v - t) >= 0.5)


def quantize_q8_0(weight_fp32, group_size: int = 32):
    """INT8 group-32: ``int8 [N, K]`` + ``fp16 [N, K/32]``."""
    w = np.asarray(weight_fp32, dtype=np.float32)
    n, k = w.shape
    if k % group_size:
        raise ValueError(f"K={k} must be divisible by {group_size}")
    blocks = w.reshape(n, k // group_size, group_size)
    scale = (np.max(np.abs(blocks), axis=2) / np.float32(127.0)).astype(np.float16)
    scale[scale == 0] = np.float16(1.0)
    q = np.clip(_round_away(blocks / scale.astype(np.float32)[:, :, None]), -127, 127)
    return q.astype(np.int8).reshape(n, k), scale


def quantize_q8_pc(weight_fp32):
    """INT8 per output channel: ``int8 [N, K]`` + ``fp16 [N]``."""
    w = np.asarray(weight_fp32, dtype=np.float32)
    scale = (np.max(np.abs(w), axis=1) / np.float32(127.0)).astype(np.float16)
    scale[scale == 0] = np.float16(1.0)
    q = np.clip(_round_away(w / scale.astype(np.float32)[:, None]), -127, 127)
    return q.astype(np.int8), scale
