"""Shared fixtures. GPU tests are marked ``gpu``; the rest run on a CPU-only host."""

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device and the built library")


@pytest.fixture(scope="session")
def golden_model():
    d = np.load(os.path.join(GOLDEN, "tiny_model.npz"))
    cfg = json.loads(str(d["config_json"]))
    ckpt = {k[5:]: d[k] for k in d.files if k.startswith("ckpt/")}
    adapter = {k[8:]: d[k] for k in d.files if k.startswith("adapter/")}
    prompts = [[int(v) for v in row if v >= 0] for row in d["prompts"]]
    return {
        "config": cfg, "ckpt": ckpt, "adapter": adapter, "prompts": prompts,
        "max_tokens": int(d["max_tokens"]), "lora_r_alpha": tuple(int(v) for v in d["lora_r_alpha"]),
        "tokens": [[int(v) for v in r if v >= 0] for r in d["tokens"]],
        "tokens_lora": [[int(v) for v in r if v >= 0] for r in d["tokens_lora"]],
        "logits": d["logits"], "logits_lora": d["logits_lora"],
        "tokens_sampled": [[int(v) for v in r if v >= 0] for r in d["tokens_sampled"]],
        "sample_t": float(d["sample_t_seed_tokens"][0]), "sample_seed": int(d["sample_t_seed_tokens"][1]),
        "sample_tokens": int(d["sample_t_seed_tokens"][2]),
    }


@pytest.fixture(scope="session")
def golden_q4():
    return np.load(os.path.join(GOLDEN, "q4_quantizer.npz"))


@pytest.fixture(scope="session")
def golden_trace():
    return np.load(os.path.join(GOLDEN, "layer_trace.npz"))


def rel_err(got, ref):
    """max |got - ref| / max |ref| (the tolerance metric used for GEMV/GEMM/layer outputs)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / den)
