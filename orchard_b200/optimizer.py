"""``orchard optimize`` on the GPU: write a pre-quantised checkpoint.

Same output as the reference's ``optimize_model`` (orchard/optimizer.py:8-64): every file of
the input directory that is not ``*.safetensors`` is copied; in each ``*.safetensors`` the
transformer-block weights (``model.layers.*`` keys containing ``weight`` but not ``norm``)
and ``lm_head.weight`` are replaced by ``<name>.weight_packed`` (uint8 ``[N, K/2]``, low
nibble = even k) and ``<name>.weight_scales`` (fp16 ``[N, K/32]``), everything else is kept
as is. The quantisation runs on the device packer, bit-identical to the reference's
``quantize_q4_0`` for fp32 input (the reference casts every weight to fp32 first).
"""

from __future__ import annotations

import glob
import os
import shutil

import numpy as np
import torch

from .model import quantize_on_device


def _should_quantize(key: str) -> bool:
    return ("model.layers" in key and "weight" in key and "norm" not in key) or "lm_head.weight" in key


def optimize_model(input_path: str, output_path: str, device=0, verbose: bool = False) -> None:
    from safetensors.numpy import load_file, save_file

    if not torch.cuda.is_available():
        raise RuntimeError("orchard_b200.optimizer needs a CUDA device (there is no CPU fallback)")
    os.makedirs(output_path, exist_ok=True)
    for name in os.listdir(input_path):
        src = os.path.join(input_path, name)
        if not name.endswith(".safetensors") and not os.path.isdir(src):
            shutil.copyfile(src, os.path.join(output_path, name))
    dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    for path in sorted(glob.glob(os.path.join(input_path, "*.safetensors"))):
        tensors = load_file(path)
        out = {}
        for key, t in tensors.items():
            if _should_quantize(key):
                w = np.ascontiguousarray(t, dtype=np.float32)  # the reference's fp32 cast
                packed, scales = quantize_on_device(w, dev)
                out[key.replace(".weight", ".weight_packed")] = packed.cpu().numpy()
                out[key.replace(".weight", ".weight_scales")] = scales.cpu().numpy()
                if verbose:
                    print(f"  quantised {key} {tuple(w.shape)}")
            else:
                out[key] = t
        save_file(out, os.path.join(output_path, os.path.basename(path)))
