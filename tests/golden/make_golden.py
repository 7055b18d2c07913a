"""Generate the golden fixtures in this directory from the reference itself.

Runs where a checkout of the reference exists; its path comes from the
``ORCHARD_REFERENCE`` environment variable (or the first argument). The fixtures it
writes are committed so the tests never need the reference at run time.

* ``q4_quantizer.npz``   -- the reference ``quantize_q4_0`` (orchard/quantizer.py:3-78)
  on seeded N(0, 0.02) weights and on hand-made edge blocks (all-zero block, exact
  .5 ties, one-sided blocks, K = 32).
* ``tiny_model.npz``     -- a 2-layer Llama-shaped checkpoint written as HF
  safetensors, loaded by the reference loader (orchard/loader.py:9-104, which
  quantises with the reference quantizer) and run through the reference
  ``Llama.generate_batch`` (orchard/model.py:254-381) at temperature 0, with and
  without a rank-4 LoRA adapter (orchard/loader.py:150-254). Logits of every
  decode step are captured from ``Llama._sample``. A third run samples at temperature
  0.7 from ``np.random.seed(20261201)`` (``Llama._sample``'s ``np.random.choice``).
* ``layer_trace.npz``    -- ``LlamaLayer.forward`` (orchard/model.py:78-195) called
  token by token on one sequence, then on a batch of two sequences at different
  positions.

The reference's compute backend is Metal; here ``metal_shim.py`` (a literal
float32 transcription of the Metal kernels) stands in for ``orchard_core``.

Usage:  ORCHARD_REFERENCE=<reference checkout> python tests/golden/make_golden.py
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ORCHARD_REFERENCE", "")

CONFIG = {
    "hidden_size": 64,
    "num_attention_heads": 2,
    "intermediate_size": 160,
    "num_hidden_layers": 2,
    "vocab_size": 64,
    "rms_norm_eps": 1e-5,
    "max_position_embeddings": 64,
}
PROMPTS = [[5, 17, 33, 8, 61], [12, 40, 3, 29, 50, 7, 44]]
MAX_TOKENS = 6
SAMPLE_T, SAMPLE_SEED, SAMPLE_TOKENS = 0.7, 20261201, 16  # sampled run (np.random.choice)
LORA_R, LORA_ALPHA = 4, 8


def load_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "orchard")):
        raise SystemExit("make_golden.py: set ORCHARD_REFERENCE (or pass the path) to a reference checkout")
    sys.path.insert(0, HERE)
    import metal_shim
    sys.modules["orchard_core"] = metal_shim
    spec = importlib.util.spec_from_file_location(
        "orchard", os.path.join(REF, "orchard", "__init__.py"),
        submodule_search_locations=[os.path.join(REF, "orchard")])
    pkg = importlib.util.module_from_spec(spec)
    sys.modules["orchard"] = pkg
    spec.loader.exec_module(pkg)
    import orchard.quantizer  # noqa: F401
    import orchard.model  # noqa: F401
    import orchard.loader  # noqa: F401
    return sys.modules["orchard"]


def quantizer_cases(qz):
    cases = {}
    rng = np.random.default_rng([20261201, 0, 0, 0])
    w = (rng.standard_normal((64, 256), dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
    cases["normal"] = w
    e = np.zeros((4, 128), dtype=np.float32)
    # row 0: block 0 all zero (scale -> fp16(1e-5)), block 1 exact .5 ties at scale 1.0
    ties = [7.0, 0.5, 1.5, -0.5, 2.5, -1.5, 3.5, -2.5, 4.5, -3.5, 5.5, -4.5, 6.5, -5.5, -6.5, 0.0]
    e[0, 32:48] = ties
    e[0, 48:64] = -np.array(ties, dtype=np.float32)
    e[0, 64:96] = rng.uniform(-1e-3, 1e-3, 32).astype(np.float32)
    e[0, 96:128] = 1e-9
    # row 1: large values; row 2: one-sided negative; row 3: max at negative end
    e[1] = rng.uniform(-300.0, 300.0, 128).astype(np.float32)
    e[2] = -np.abs(rng.standard_normal(128).astype(np.float32))
    e[3] = rng.standard_normal(128).astype(np.float32)
    e[3, ::32] = -9.0
    cases["edges"] = e
    cases["k32"] = rng.standard_normal((1, 32)).astype(np.float32)
    out = {}
    for name, w in cases.items():
        p, s = qz(w)
        out[f"{name}_w"] = w
        out[f"{name}_packed"] = p
        out[f"{name}_scales"] = s
    return out


def make_checkpoint(path):
    from safetensors.numpy import save_file
    H, F, V = CONFIG["hidden_size"], CONFIG["intermediate_size"], CONFIG["vocab_size"]
    t = {}
    g = np.random.default_rng([20261201, 1, 0, 0])

    def w(shape, std=0.02):
        return (g.standard_normal(shape, dtype=np.float32) * std).astype(np.float16)

    t["model.embed_tokens.weight"] = w((V, H), 1.0)
    for i in range(CONFIG["num_hidden_layers"]):
        p = f"model.layers.{i}."
        for nm in ("q_proj", "k_proj", "v_proj", "o_proj"):
            t[p + f"self_attn.{nm}.weight"] = w((H, H))
        t[p + "mlp.gate_proj.weight"] = w((F, H))
        t[p + "mlp.up_proj.weight"] = w((F, H))
        t[p + "mlp.down_proj.weight"] = w((H, F))
        t[p + "input_layernorm.weight"] = (1.0 + w((H,), 0.1).astype(np.float32)).astype(np.float16)
        t[p + "post_attention_layernorm.weight"] = (1.0 + w((H,), 0.1).astype(np.float32)).astype(np.float16)
    t["model.norm.weight"] = (1.0 + w((H,), 0.1).astype(np.float32)).astype(np.float16)
    t["lm_head.weight"] = w((V, H))
    os.makedirs(path, exist_ok=True)
    save_file(t, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(CONFIG, f)
    return t


def make_adapter(path):
    from safetensors.numpy import save_file
    H = CONFIG["hidden_size"]
    g = np.random.default_rng([20261201, 2, 0, 0])
    t = {}
    for i in range(CONFIG["num_hidden_layers"]):
        for nm in ("q_proj", "v_proj"):
            base = f"base_model.model.model.layers.{i}.self_attn.{nm}."
            t[base + "lora_A.weight"] = (g.standard_normal((LORA_R, H), dtype=np.float32) * 0.6).astype(np.float16)
            t[base + "lora_B.weight"] = (g.standard_normal((H, LORA_R), dtype=np.float32) * 0.6).astype(np.float16)
    os.makedirs(path, exist_ok=True)
    save_file(t, os.path.join(path, "adapter_model.safetensors"))
    with open(os.path.join(path, "adapter_config.json"), "w") as f:
        json.dump({"r": LORA_R, "lora_alpha": LORA_ALPHA}, f)
    return t


class IdTokenizer:
    """Prompts are space-separated token ids; decode joins ids back."""

    class _Enc:
        def __init__(self, ids):
            self.ids = ids

    def encode(self, text):
        return self._Enc([int(v) for v in text.split()])

    def decode(self, ids):
        return " ".join(str(int(v)) for v in ids)


def run_generate(orchard, model_dir, adapter_dir=None, temperature=0.0, max_tokens=MAX_TOKENS, seed=None):
    llama = orchard.model.Llama(model_dir)
    if adapter_dir:
        llama.load_lora(adapter_dir)
    llama.tokenizer = IdTokenizer()
    logits = []
    orig = llama._sample

    def rec(lg, temperature=0.7):
        logits.append(np.array(lg, dtype=np.float32).copy())
        return orig(lg, temperature)

    llama._sample = rec
    if seed is not None:
        np.random.seed(seed)
    texts = llama.generate_batch([" ".join(map(str, p)) for p in PROMPTS],
                                 max_tokens=max_tokens, temperature=temperature)
    toks = [[int(v) for v in s.split()] for s in texts]
    return llama, toks, logits


def layer_trace(orchard, llama):
    core = sys.modules["orchard_core"]
    layer = llama.layers[0]
    H = CONFIG["hidden_size"]
    hd = H // CONFIG["num_attention_heads"]
    cos_t, sin_t = orchard.model.precompute_freqs_cis(hd, CONFIG["max_position_embeddings"])
    g = np.random.default_rng([20261201, 3, 0, 0])
    slot_a, slot_b = 20, 21
    for s in (slot_a, slot_b):
        layer.k_cache_np[s] = np.zeros((layer.heads, hd, 0), np.float32)
        layer.v_cache_np[s] = np.zeros((layer.heads, 0, hd), np.float32)
    xs_in, xs_out, pos_a = [], [], []

    def call(xrows, positions, slots):
        B = len(slots)
        x = core.Tensor(llama.backend, [B * H], core.DType.Float32)
        x.copy_from_host(xrows.reshape(-1).astype(np.float32))
        fc = core.Tensor(llama.backend, [B * (hd // 2)], core.DType.Float32)
        fs = core.Tensor(llama.backend, [B * (hd // 2)], core.DType.Float32)
        fc.copy_from_host(cos_t[positions].reshape(-1).astype(np.float32))
        fs.copy_from_host(sin_t[positions].reshape(-1).astype(np.float32))
        layer.forward(x, fc, fs, slots)
        return x.copy_to_host().reshape(B, H)

    T = 10
    for p in range(T):
        xi = g.standard_normal((1, H), dtype=np.float32)
        xs_in.append(xi)
        xs_out.append(call(xi, [p], [slot_a]))
        pos_a.append(p)
    xb = g.standard_normal((2, H), dtype=np.float32)
    yb = call(xb, [T, 0], [slot_a, slot_b])
    return {"seq_x_in": np.concatenate(xs_in), "seq_x_out": np.concatenate(xs_out),
            "batch_x_in": xb, "batch_x_out": yb, "batch_pos": np.array([T, 0]),
            "k_cache_a": layer.k_cache_np[slot_a], "v_cache_a": layer.v_cache_np[slot_a]}


def main():
    orchard = load_reference()
    qz = orchard.quantizer.quantize_q4_0
    np.savez_compressed(os.path.join(HERE, "q4_quantizer.npz"), **quantizer_cases(qz))

    with tempfile.TemporaryDirectory() as td:
        mdir = os.path.join(td, "model")
        adir = os.path.join(td, "adapter")
        ckpt = make_checkpoint(mdir)
        adapter = make_adapter(adir)
        llama, toks, logits = run_generate(orchard, mdir)
        trace = layer_trace(orchard, llama)
        _, toks_l, logits_l = run_generate(orchard, mdir, adir)
        _, toks_s, _ = run_generate(orchard, mdir, temperature=SAMPLE_T, max_tokens=SAMPLE_TOKENS, seed=SAMPLE_SEED)

    pad = max(len(t) for t in toks + toks_l)
    out = {f"ckpt/{k}": v for k, v in ckpt.items()}
    out.update({f"adapter/{k}": v for k, v in adapter.items()})
    out["config_json"] = np.array(json.dumps(CONFIG))
    out["prompts"] = np.array([p + [-1] * (8 - len(p)) for p in PROMPTS])
    out["max_tokens"] = np.array(MAX_TOKENS)
    out["lora_r_alpha"] = np.array([LORA_R, LORA_ALPHA])
    out["tokens"] = np.array([t + [-1] * (pad - len(t)) for t in toks])
    out["tokens_lora"] = np.array([t + [-1] * (pad - len(t)) for t in toks_l])
    out["logits"] = np.stack(logits)
    out["logits_lora"] = np.stack(logits_l)
    pad_s = max(len(t) for t in toks_s)
    out["tokens_sampled"] = np.array([t + [-1] * (pad_s - len(t)) for t in toks_s])
    out["sample_t_seed_tokens"] = np.array([SAMPLE_T, SAMPLE_SEED, SAMPLE_TOKENS])
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), **out)
    np.savez_compressed(os.path.join(HERE, "layer_trace.npz"), **trace)
    print("tokens", toks, "tokens_lora", toks_l)


if __name__ == "__main__":
    main()
