"""Host-side logic of the model driver that needs no GPU."""

import numpy as np
import torch

import oracle
from orchard_b200 import loader, model


def test_freqs_match_oracle():
    c, s = model.precompute_freqs_cis(128, 4096)
    oc, os_ = oracle.ops.precompute_freqs_cis(128, 4096)
    np.testing.assert_array_equal(c, oc)
    np.testing.assert_array_equal(s, os_)
    assert c.dtype == np.float32 and c.shape == (4096, 64)


def test_interleave_gate_up_layout():
    F, KB = 48, 8
    p1 = torch.arange(F * KB, dtype=torch.int32).view(F, KB)
    p3 = -torch.arange(F * KB, dtype=torch.int32).view(F, KB) - 1
    s1 = torch.arange(F * 2, dtype=torch.int32).view(F, 2)
    s3 = -s1 - 1
    w, s = model.interleave_gate_up(p1, s1, p3, s3)
    assert w.shape == (2 * F, KB)
    for b in range(F // 16):
        assert torch.equal(w[32 * b:32 * b + 16], p1[16 * b:16 * b + 16])
        assert torch.equal(w[32 * b + 16:32 * b + 32], p3[16 * b:16 * b + 16])
        assert torch.equal(s[32 * b + 16:32 * b + 32], s3[16 * b:16 * b + 16])


def test_loader_routes_reference_keys(golden_model):
    g = golden_model
    ck = loader.from_tensors(g["config"], g["ckpt"])
    assert ck.complete()
    assert set(ck.layers[0]) == {"wq", "wk", "wv", "wo", "w1", "w2", "w3", "attn_norm", "ffn_norm"}
    assert ck.layers[1]["w1"][0] == "dense"
    assert ck.layers[0]["attn_norm"].dtype == np.float32
    # pre-packed keys (orchard/optimizer.py:55-56) are taken as they are
    t = dict(g["ckpt"])
    w = t.pop("model.layers.0.self_attn.q_proj.weight")
    p, s = oracle.ops.quantize_q4_0(w.astype(np.float32))
    t["model.layers.0.self_attn.q_proj.weight_packed"] = p
    t["model.layers.0.self_attn.q_proj.weight_scales"] = s
    ck2 = loader.from_tensors(g["config"], t)
    assert ck2.layers[0]["wq"][0] == "packed"
    assert ck2.layers[0]["wq"][1] is p


def test_lora_loader_matches_reference_layout(tmp_path, golden_model):
    from safetensors.numpy import save_file
    import json
    g = golden_model
    r, alpha = g["lora_r_alpha"]
    save_file(g["adapter"], str(tmp_path / "adapter_model.safetensors"))
    (tmp_path / "adapter_config.json").write_text(json.dumps({"r": r, "lora_alpha": alpha}))
    per_layer, rr, aa = loader.load_lora(str(tmp_path), g["config"]["num_hidden_layers"])
    assert rr == r and aa == alpha
    m = oracle.model.from_hf_tensors(g["config"], g["ckpt"], g["adapter"], r, alpha)
    for li in range(g["config"]["num_hidden_layers"]):
        assert set(per_layer[li]) == {"wq", "wv"}
        for name in ("wq", "wv"):
            np.testing.assert_array_equal(per_layer[li][name][0], m.layers[li].lora[name][0])
            np.testing.assert_array_equal(per_layer[li][name][1], m.layers[li].lora[name][1])
