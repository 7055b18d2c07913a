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


def test_prefill_units_cover_rows_in_runs():
    """Work units of the prefill attention kernel: every row exactly once and in order; a
    unit never spans a change of cache slot or a gap in positions, and holds at most
    max_rows rows (the kernel's 64-row tile)."""
    pos, slots = [], []
    for slot, (start, n) in enumerate([(0, 130), (5, 1), (0, 64), (300, 65), (7, 3)]):
        pos += list(range(start, start + n))
        slots += [slot] * n
    pos[200] += 3  # a gap in positions inside slot 3's run
    u = model.prefill_units(pos, slots)
    assert u.dtype == np.int32 and u.shape[1] == 4
    rows = np.concatenate([np.arange(r0, r0 + n) for r0, n, _, _ in u])
    np.testing.assert_array_equal(rows, np.arange(len(pos)))
    for r0, n, slot, p0 in u:
        assert 1 <= n <= 64
        assert all(slots[r0 + i] == slot and pos[r0 + i] == p0 + i for i in range(n))
    # unit starts are exactly the run starts plus every 64th row of a run
    brk = [0] + [i for i in range(1, len(pos)) if slots[i] != slots[i - 1] or pos[i] != pos[i - 1] + 1]
    ends = brk[1:] + [len(pos)]
    expect = [r for a, e in zip(brk, ends) for r in range(a, e, 64)]
    assert u[:, 0].tolist() == expect
    assert model.prefill_units([], []).shape == (0, 4)
    assert model.prefill_units(list(range(10)), [0] * 10, max_rows=4)[:, 1].tolist() == [4, 4, 2]
