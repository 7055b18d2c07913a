"""NumPy restatement of the reference's Llama layer, decode step and greedy
``generate_batch`` (orchard/model.py).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Activation tensors are float32, as the reference's host allocates them
(orchard/model.py:86,90-92,143,160,164-165,183); attention and the KV cache are the
reference's float32 NumPy host code (orchard/model.py:112-144). Quantised weights are
``(packed uint8 [N,K/2], scales fp16 [N,K/32])`` pairs.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import ops

EOS_ID = 2  # orchard/model.py:370-371


@dataclass
class OracleLayer:
    wq: Tuple[np.ndarray, np.ndarray]
    wk: Tuple[np.ndarray, np.ndarray]
    wv: Tuple[np.ndarray, np.ndarray]
    wo: Tuple[np.ndarray, np.ndarray]
    w1: Tuple[np.ndarray, np.ndarray]  # gate
    w2: Tuple[np.ndarray, np.ndarray]  # down
    w3: Tuple[np.ndarray, np.ndarray]  # up
    attn_norm: np.ndarray
    ffn_norm: np.ndarray
    # module name -> (A [in, r], B [r, out] already scaled by alpha/r), orchard/loader.py:240-254
    lora: Dict[str, Tuple[np.ndarray, np.ndarray]] = field(default_factory=dict)


class OracleModel:
    """The reference model's arithmetic with a per-sequence host KV cache."""

    def __init__(self, config: dict, layers: List[OracleLayer], embed: np.ndarray,
                 norm: np.ndarray, lm_head: Tuple[np.ndarray, np.ndarray],
                 cache_dequant: bool = False):
        self.config = config
        self.layers = layers
        self.embed = np.asarray(embed, dtype=np.float32)
        self.norm = np.asarray(norm, dtype=np.float32)
        self.lm_head = lm_head
        self.hidden = config["hidden_size"]
        self.heads = config["num_attention_heads"]
        self.head_dim = self.hidden // self.heads
        self.eps = config["rms_norm_eps"]
        self.freqs_cos, self.freqs_sin = ops.precompute_freqs_cis(
            self.head_dim, config.get("max_position_embeddings", 2048))
        self._dq: Dict[int, np.ndarray] = {}
        self.cache_dequant = cache_dequant
        self.reset()

    # -- KV cache -------------------------------------------------------------------
    def reset(self):
        """Empty per-layer, per-sequence caches (orchard/model.py:277-284)."""
        self.k_cache: List[Dict[int, np.ndarray]] = [dict() for _ in self.layers]
        self.v_cache: List[Dict[int, np.ndarray]] = [dict() for _ in self.layers]

    def _lin(self, w, x):
        if not self.cache_dequant:
            return ops.gemm_q4_0(w[0], w[1], x)
        key = id(w[0])
        if key not in self._dq:
            self._dq[key] = ops.dequantize_q4_0(w[0], w[1])
        return np.asarray(x, np.float32) @ self._dq[key].T

    @staticmethod
    def _lora(layer: OracleLayer, name: str, x, out):
        """orchard/model.py:60-76: ``out += (x @ A) @ B``."""
        if name in layer.lora:
            a, b = layer.lora[name]
            out = out + (np.asarray(x, np.float32) @ a.astype(np.float32)) @ b.astype(np.float32)
        return out

    # -- layer -----------------------------------------------------------------------
    def layer_forward(self, li: int, x: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                      seq_ids: List[int]) -> np.ndarray:
        """orchard/model.py:78-195 for ``len(seq_ids)`` rows; returns the new residual."""
        L = self.layers[li]
        B = len(seq_ids)
        H, hd = self.heads, self.head_dim
        x = np.asarray(x, np.float32).reshape(B, self.hidden)
        xn = ops.rmsnorm(x, L.attn_norm, self.eps)                          # :86-87
        q = self._lora(L, "wq", xn, self._lin(L.wq, xn))                     # :94-106
        k = self._lora(L, "wk", xn, self._lin(L.wk, xn))
        v = self._lora(L, "wv", xn, self._lin(L.wv, xn))
        q = ops.rope(q.reshape(B, H, hd), cos, sin)                          # :109-110
        k = ops.rope(k.reshape(B, H, hd), cos, sin)
        v = v.reshape(B, H, hd)
        attn = np.zeros((B, H, hd), np.float32)
        for i, b in enumerate(seq_ids):                                      # :120-137
            kc = self.k_cache[li].get(b, np.zeros((H, 0, hd), np.float32))
            vc = self.v_cache[li].get(b, np.zeros((H, 0, hd), np.float32))
            kc = np.concatenate([kc, k[i][:, None, :]], axis=1)
            vc = np.concatenate([vc, v[i][:, None, :]], axis=1)
            self.k_cache[li][b] = kc
            self.v_cache[li][b] = vc
            attn[i] = ops.attention_one(q[i], kc, vc)
        attn = attn.reshape(B, self.hidden)
        o = self._lora(L, "wo", attn, self._lin(L.wo, attn))                 # :147-154
        x = x + o                                                            # :157
        xf = ops.rmsnorm(x, L.ffn_norm, self.eps)                            # :160-161
        g = self._lora(L, "w1", xf, self._lin(L.w1, xf))                     # :167-176
        u = self._lora(L, "w3", xf, self._lin(L.w3, xf))
        h = ops.mul(ops.silu(g), u)                                          # :179-180
        d = self._lora(L, "w2", h, self._lin(L.w2, h))                       # :184-190
        return x + d                                                         # :193

    # -- decode step -----------------------------------------------------------------
    def forward_tokens(self, tokens: List[int], positions: List[int],
                       seq_ids: List[int], logits: bool = True) -> Optional[np.ndarray]:
        """One token per listed sequence through every layer (orchard/model.py:318-356)."""
        x = self.embed[np.asarray(tokens, dtype=np.int64)].astype(np.float32)
        cos = self.freqs_cos[np.asarray(positions)]
        sin = self.freqs_sin[np.asarray(positions)]
        for li in range(len(self.layers)):
            x = self.layer_forward(li, x, cos, sin, seq_ids)
        if not logits:
            return None
        xn = ops.rmsnorm(x, self.norm, self.eps)                             # :348
        return self._lin(self.lm_head, xn)                                   # :353-356

    def generate_greedy(self, prompts: List[List[int]], max_tokens: int,
                        ignore_eos: bool = False) -> List[List[int]]:
        """``generate_batch(..., temperature=0)`` token flow (orchard/model.py:254-381):
        token-by-token prefill per sequence, the last prompt token fed again as the first
        decode input at position ``len(prompt)``, greedy argmax, EOS id 2 retires a row."""
        return self.generate(prompts, max_tokens, 0.0, ignore_eos)

    def generate(self, prompts: List[List[int]], max_tokens: int, temperature: float,
                 ignore_eos: bool = False) -> List[List[int]]:
        """``generate_batch`` token flow (orchard/model.py:254-381) with its sampler
        (orchard/model.py:244-252): argmax at temperature 0, otherwise
        ``np.random.choice`` over ``softmax((logits - max) / T)`` in float32, one call per
        active row in row order (so the draws follow the global NumPy RNG stream)."""
        self.reset()
        cur = []
        for b, ids in enumerate(prompts):
            for i, t in enumerate(ids):
                self.forward_tokens([t], [i], [b], logits=False)
            cur.append(ids[-1])
        gen: List[List[int]] = [[] for _ in prompts]
        active = list(range(len(prompts)))
        for _ in range(max_tokens):
            if not active:
                break
            toks = [cur[b] for b in active]
            pos = [len(prompts[b]) + len(gen[b]) for b in active]
            lg = self.forward_tokens(toks, pos, active)
            nxt = []
            for i, b in enumerate(active):
                t = int(np.argmax(lg[i])) if temperature == 0 else sample(lg[i], temperature)
                gen[b].append(t)
                cur[b] = t
                if ignore_eos or t != EOS_ID:
                    nxt.append(b)
            active = nxt
        return gen


def sample(logits: np.ndarray, temperature: float) -> int:
    """orchard/model.py:247-252: shift by the max, float32 softmax of logits / T, then
    ``np.random.choice`` (one uniform from the global RNG; the first index whose normalised
    running sum exceeds it)."""
    lg = np.asarray(logits, np.float32)
    lg = lg - np.max(lg)
    probs = np.exp(lg / temperature) / np.sum(np.exp(lg / temperature))
    return int(np.random.choice(len(probs), p=probs))


def random_model(config: dict, seed: int = 0, lora_rank: int = 0,
                 lora_modules=("wq", "wv")) -> Tuple[OracleModel, dict]:
    """Seeded random-init model in the reference's packed format.

    Weights N(0, 0.02) drawn as float32, cast to fp16 and back (the loader's fp32 cast
    of fp16 checkpoints, orchard/loader.py:121-122), then quantised. Norm weights
    N(1, 0.1); embeddings N(0, 1) fp16. Returns the oracle model and the raw arrays."""
    H = config["hidden_size"]
    F = config["intermediate_size"]
    V = config["vocab_size"]
    nl = config["num_hidden_layers"]
    layers = []
    raw: dict = {"layers": []}
    for li in range(nl):
        def rng(tid):
            return np.random.default_rng([20261201, seed, li, tid])
        shapes = {"wq": (H, H), "wk": (H, H), "wv": (H, H), "wo": (H, H),
                  "w1": (F, H), "w3": (F, H), "w2": (H, F)}
        q = {}
        rl = {}
        for tid, (name, shp) in enumerate(shapes.items()):
            w = (rng(tid).standard_normal(shp, dtype=np.float32) * 0.02).astype(np.float16)
            rl[name] = w
            q[name] = ops.quantize_q4_0(w.astype(np.float32))
        an = (1.0 + 0.1 * rng(10).standard_normal(H, dtype=np.float32)).astype(np.float16)
        fn = (1.0 + 0.1 * rng(11).standard_normal(H, dtype=np.float32)).astype(np.float16)
        lora = {}
        if lora_rank:
            for j, m in enumerate(lora_modules):
                a = (rng(20 + j).standard_normal((H, lora_rank), dtype=np.float32) * 0.01)
                bb = (rng(30 + j).standard_normal((lora_rank, H), dtype=np.float32) * 0.01)
                lora[m] = (a.astype(np.float16).astype(np.float32),
                           bb.astype(np.float16).astype(np.float32))
        layers.append(OracleLayer(wq=q["wq"], wk=q["wk"], wv=q["wv"], wo=q["wo"],
                                  w1=q["w1"], w2=q["w2"], w3=q["w3"],
                                  attn_norm=an.astype(np.float32),
                                  ffn_norm=fn.astype(np.float32), lora=lora))
        raw["layers"].append({"fp16": rl, "attn_norm": an, "ffn_norm": fn})
    g = np.random.default_rng([20261201, seed, 1000, 0])
    embed = g.standard_normal((V, H), dtype=np.float32).astype(np.float16)
    norm = (1.0 + 0.1 * np.random.default_rng([20261201, seed, 1000, 1])
            .standard_normal(H, dtype=np.float32)).astype(np.float16)
    lm = (np.random.default_rng([20261201, seed, 1000, 2])
          .standard_normal((V, H), dtype=np.float32) * 0.02).astype(np.float16)
    lm_q = ops.quantize_q4_0(lm.astype(np.float32))
    raw.update(embed=embed, norm=norm, lm_head=lm)
    model = OracleModel(config, layers, embed.astype(np.float32), norm.astype(np.float32), lm_q)
    return model, raw


def from_hf_tensors(config: dict, tensors: dict, adapter: Optional[dict] = None,
                    lora_r: int = 8, lora_alpha: float = 16) -> OracleModel:
    """Build the oracle from HF-named fp16/fp32 tensors the way the reference loader
    does (orchard/loader.py:9-104): linear weights cast to fp32 and quantised, norms
    and embeddings kept fp32; LoRA A transposed to ``[In, r]`` and B transposed and
    scaled by ``alpha / r`` to ``[r, Out]`` (orchard/loader.py:156-160, 236-254)."""
    nl = config["num_hidden_layers"]
    proj = {"self_attn.q_proj": "wq", "self_attn.k_proj": "wk", "self_attn.v_proj": "wv",
            "self_attn.o_proj": "wo", "mlp.gate_proj": "w1", "mlp.up_proj": "w3",
            "mlp.down_proj": "w2"}
    layers = []
    for i in range(nl):
        p = f"model.layers.{i}."
        q = {v: ops.quantize_q4_0(np.asarray(tensors[p + k + ".weight"], np.float32))
             for k, v in proj.items()}
        lora = {}
        if adapter:
            scaling = lora_alpha / lora_r
            for k, v in proj.items():
                base = f"base_model.model.model.layers.{i}.{k}."
                if base + "lora_A.weight" in adapter:
                    a = np.asarray(adapter[base + "lora_A.weight"]).T.astype(np.float32)
                    b = np.asarray(adapter[base + "lora_B.weight"]).T.astype(np.float32) * scaling
                    lora[v] = (a, b.astype(np.float32))
        layers.append(OracleLayer(
            attn_norm=np.asarray(tensors[p + "input_layernorm.weight"], np.float32),
            ffn_norm=np.asarray(tensors[p + "post_attention_layernorm.weight"], np.float32),
            lora=lora, **q))
    lm = ops.quantize_q4_0(np.asarray(tensors["lm_head.weight"], np.float32))
    return OracleModel(config, layers, np.asarray(tensors["model.embed_tokens.weight"], np.float32),
                       np.asarray(tensors["model.norm.weight"], np.float32), lm,
                       cache_dequant=True)
