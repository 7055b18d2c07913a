"""orchard_b200: Orchard's quantised Llama-layer path on NVIDIA B200 (sm_100a).

* ``orchard_b200.Llama`` -- ``orchard.Llama`` (orchard/model.py:197-381) on fused CUDA kernels.
* ``orchard_b200.quantize_q4_0`` -- the reference packer (orchard/quantizer.py:3-78).
* ``orchard_b200.orchard_core`` -- the reference's pybind11 operator surface
  (src/bindings.cpp) over the same kernels; ``install_as_orchard_core()`` registers it
  under the top-level name ``orchard_core`` so code written against the reference's
  module imports it unchanged.
* ``include/orchard_b200.h`` -- the C ABI of ``lib/liborchard_b200.so``.
"""

from __future__ import annotations

import importlib
import sys

from .quantizer import quantize_q4_0, quantize_q8_0, quantize_q8_pc  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    if name in ("Llama", "LlamaConfig", "DecodeEngine", "precompute_freqs_cis"):
        from . import model
        return getattr(model, name)
    if name == "orchard_core":
        return importlib.import_module(".orchard_core", __name__)
    raise AttributeError(name)


def install_as_orchard_core():
    """Makes ``import orchard_core`` resolve to this package's operator surface."""
    mod = importlib.import_module(".orchard_core", __name__)
    sys.modules["orchard_core"] = mod
    return mod
