"""Checkpoint ingest with the reference's naming and packed format.

Reads ``config.json`` and every ``*.safetensors`` under a model directory, as
``load_weights`` does (orchard/loader.py:9-104):

* ``model.layers.{i}.self_attn.{q,k,v,o}_proj.weight`` -> wq, wk, wv, wo;
  ``model.layers.{i}.mlp.{gate,up,down}_proj.weight`` -> w1, w3, w2
  (orchard/loader.py:53-62). A key ending ``.weight_packed`` with its
  ``.weight_scales`` partner is the pre-quantised format written by
  ``orchard optimize`` (orchard/optimizer.py:40-56) and is used as is; a plain
  ``.weight`` is quantised with the reference rule (on the GPU, bit-identically).
* ``input_layernorm`` / ``post_attention_layernorm`` / ``model.norm`` -> fp32 norms.
* ``model.embed_tokens.weight`` -> embeddings; ``lm_head.weight[_packed]`` -> output head.

LoRA adapters follow ``load_lora_adapter`` (orchard/loader.py:150-254): ``r`` and
``lora_alpha`` from ``adapter_config.json`` (defaults 8 and 16), A stored as
``[in, r]``, B as ``[r, out]`` pre-multiplied by ``alpha / r``.
"""

from __future__ import annotations

import glob
import json
import os
from typing import Dict, Optional, Tuple

import numpy as np

PROJ = {
    ("self_attn", "q_proj"): "wq",
    ("self_attn", "k_proj"): "wk",
    ("self_attn", "v_proj"): "wv",
    ("self_attn", "o_proj"): "wo",
    ("mlp", "gate_proj"): "w1",
    ("mlp", "up_proj"): "w3",
    ("mlp", "down_proj"): "w2",
}


class Checkpoint:
    """Host-side view of a checkpoint: per-layer entries hold either a float array
    (``("dense", w)``) or the packed pair (``("packed", packed, scales)``)."""

    def __init__(self, config: dict):
        self.config = config
        n = config["num_hidden_layers"]
        self.layers = [dict() for _ in range(n)]
        self.embed: Optional[np.ndarray] = None
        self.norm: Optional[np.ndarray] = None
        self.lm_head: Optional[tuple] = None

    def complete(self) -> bool:
        need = set(PROJ.values()) | {"attn_norm", "ffn_norm"}
        return (self.embed is not None and self.norm is not None and self.lm_head is not None
                and all(need <= set(l) for l in self.layers))


def _route(ck: Checkpoint, key: str, get) -> None:
    if key.endswith("_scales"):
        return
    parts = key.split(".")
    packed = key.endswith("_packed")
    if parts[0] == "model" and len(parts) > 2 and parts[1] == "layers":
        li = int(parts[2])
        if li >= len(ck.layers):
            return
        mod = parts[3]
        if mod in ("self_attn", "mlp"):
            name = PROJ.get((mod, parts[4]))
            if name is None:
                return
            if packed:
                ck.layers[li][name] = ("packed", get(key), get(key.replace("_packed", "_scales")))
            else:
                ck.layers[li][name] = ("dense", get(key))
        elif mod == "input_layernorm":
            ck.layers[li]["attn_norm"] = np.asarray(get(key), dtype=np.float32)
        elif mod == "post_attention_layernorm":
            ck.layers[li]["ffn_norm"] = np.asarray(get(key), dtype=np.float32)
    elif parts[0] == "model" and len(parts) > 1 and parts[1] == "norm":
        ck.norm = np.asarray(get(key), dtype=np.float32)
    elif parts[0] == "model" and len(parts) > 1 and parts[1] == "embed_tokens":
        ck.embed = np.asarray(get(key))
    elif parts[0] == "lm_head":
        if packed:
            ck.lm_head = ("packed", get(key), get(key.replace("_packed", "_scales")))
        else:
            ck.lm_head = ("dense", get(key))


def from_tensors(config: dict, tensors: Dict[str, np.ndarray]) -> Checkpoint:
    ck = Checkpoint(config)
    for k in tensors:
        _route(ck, k, lambda name: tensors[name])
    return ck


def load_checkpoint(model_path: str) -> Checkpoint:
    """config.json + *.safetensors (orchard/loader.py:13-40)."""
    from safetensors import safe_open

    with open(os.path.join(model_path, "config.json")) as f:
        config = json.load(f)
    files = sorted(glob.glob(os.path.join(model_path, "*.safetensors")))
    if not files:
        raise FileNotFoundError("No .safetensors files found")
    ck = Checkpoint(config)
    for fn in files:
        with safe_open(fn, framework="numpy", device="cpu") as f:
            keys = list(f.keys())
            for k in keys:
                _route(ck, k, f.get_tensor)
    return ck


def load_lora(adapter_path: str, n_layers: int) -> Tuple[Dict[int, Dict[str, tuple]], int, float]:
    """Returns ``{layer: {module: (A [in, r] fp32, B [r, out] fp32 scaled)}}``, r, alpha."""
    from safetensors import safe_open

    with open(os.path.join(adapter_path, "adapter_config.json")) as f:
        cfg = json.load(f)
    r = cfg.get("r", 8)
    alpha = cfg.get("lora_alpha", 16)
    scaling = alpha / r
    files = sorted(glob.glob(os.path.join(adapter_path, "*.safetensors")))
    if not files:
        raise FileNotFoundError("No adapter weights found")
    out: Dict[int, Dict[str, list]] = {}
    for fn in files:
        with safe_open(fn, framework="numpy", device="cpu") as f:
            for key in f.keys():
                parts = key.split(".")
                if "layers" not in parts:
                    continue
                try:
                    li = int(parts[parts.index("layers") + 1])
                    mod, proj = parts[parts.index("layers") + 2], parts[parts.index("layers") + 3]
                except (ValueError, IndexError):
                    continue
                if li >= n_layers:
                    continue
                name = PROJ.get((mod, proj))
                if name is None:
                    continue
                is_a, is_b = "lora_A" in parts, "lora_B" in parts
                if not (is_a or is_b):
                    continue
                t = f.get_tensor(key)
                slot = out.setdefault(li, {}).setdefault(name, [None, None])
                if is_a:
                    slot[0] = np.ascontiguousarray(t.T.astype(np.float32))
                else:
                    slot[1] = np.ascontiguousarray(t.T.astype(np.float32) * np.float32(scaling))
    return {li: {k: tuple(v) for k, v in d.items()} for li, d in out.items()}, r, alpha
