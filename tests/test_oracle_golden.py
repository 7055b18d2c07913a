"""The oracle and the host packers against fixtures produced by the reference itself."""

import numpy as np
import pytest

import oracle
from oracle import ops
from orchard_b200 import quantizer

CASES = ("normal", "edges", "k32")


@pytest.mark.parametrize("case", CASES)
def test_oracle_quantizer_bit_exact(golden_q4, case):
    p, s = ops.quantize_q4_0(golden_q4[f"{case}_w"])
    np.testing.assert_array_equal(p, golden_q4[f"{case}_packed"])
    np.testing.assert_array_equal(s.view(np.uint16), golden_q4[f"{case}_scales"].view(np.uint16))


@pytest.mark.parametrize("case", CASES)
def test_product_quantizer_bit_exact(golden_q4, case):
    p, s = quantizer.quantize_q4_0(golden_q4[f"{case}_w"])
    assert p.dtype == np.uint8 and s.dtype == np.float16
    np.testing.assert_array_equal(p, golden_q4[f"{case}_packed"])
    np.testing.assert_array_equal(s.view(np.uint16), golden_q4[f"{case}_scales"].view(np.uint16))


def test_edge_block_semantics(golden_q4):
    s = golden_q4["edges_scales"]
    p = golden_q4["edges_packed"]
    assert s[0, 0].view(np.uint16) == 0x00A8          # all-zero block -> fp16(1e-5)
    assert np.all(p[0, :16] == 0x88)                  # zero weights -> code 8
    codes = ops.unpack_q4_0(p)
    # ties at scale 1.0: w + 8 = x.5 rounds half to even
    assert s[0, 1] == np.float16(1.0)
    ties = golden_q4["edges_w"][0, 32:48]
    expect = np.rint(ties + 8).astype(np.int64)
    np.testing.assert_array_equal(codes[0, 32:48], np.clip(expect, 0, 15))


def test_dequant_roundtrip_error_bound(golden_q4):
    w = golden_q4["normal_w"]
    p, s = ops.quantize_q4_0(w)
    d = ops.dequantize_q4_0(p, s)
    step = np.repeat(s.astype(np.float32), 32, axis=1)
    assert np.all(np.abs(d - w) <= 0.5 * step * (1 + 1e-3) + 1e-12)


def test_gemv_kat_0x99():
    """examples/simple_test.py:53-105: bytes 0x99, scale 1, ones -> 32.0."""
    p = np.full((1, 16), 0x99, np.uint8)
    s = np.ones((1, 1), np.float16)
    y = ops.gemm_q4_0(p, s, np.ones(32, np.float32))
    assert y.shape == (1, 1) and y[0, 0] == 32.0


def test_q8_round_half_away():
    w = np.array([[127.0, 2.5, -2.5, 0.5, -0.5, 1.49999, 0.0] + [0.0] * 25], np.float32)
    q, s = quantizer.quantize_q8_0(w)
    assert s[0, 0] == np.float16(1.0)
    np.testing.assert_array_equal(q[0, :7], [127, 3, -3, 1, -1, 1, 0])
    q2, s2 = ops.quantize_q8_0(w)
    np.testing.assert_array_equal(q, q2)
    qp, sp = quantizer.quantize_q8_pc(w)
    qp2, sp2 = ops.quantize_q8_pc(w)
    np.testing.assert_array_equal(qp, qp2)
    np.testing.assert_array_equal(sp, sp2)


@pytest.mark.parametrize("with_lora", [False, True])
def test_oracle_generate_matches_reference(golden_model, with_lora):
    g = golden_model
    m = oracle.model.from_hf_tensors(g["config"], g["ckpt"], g["adapter"] if with_lora else None,
                                     *g["lora_r_alpha"])
    seen = []
    orig = m.forward_tokens

    def rec(*a, **k):
        r = orig(*a, **k)
        if r is not None:
            seen.extend(list(r))
        return r

    m.forward_tokens = rec
    toks = m.generate_greedy(g["prompts"], g["max_tokens"])
    assert toks == (g["tokens_lora"] if with_lora else g["tokens"])
    ref = g["logits_lora"] if with_lora else g["logits"]
    np.testing.assert_allclose(np.array(seen), ref, atol=1e-5, rtol=1e-5)


def test_oracle_sampled_generate_matches_reference(golden_model):
    """temperature 0.7 from a seeded global NumPy RNG: the reference's tokens, including a
    row that samples EOS and retires (so later draws skip it)."""
    g = golden_model
    m = oracle.model.from_hf_tensors(g["config"], g["ckpt"])
    np.random.seed(g["sample_seed"])
    toks = m.generate(g["prompts"], g["sample_tokens"], g["sample_t"])
    assert toks == g["tokens_sampled"]
    assert any(t[-1] == 2 for t in toks)


def test_oracle_layer_trace(golden_model, golden_trace):
    g = golden_model
    m = oracle.model.from_hf_tensors(g["config"], g["ckpt"])
    H = g["config"]["hidden_size"]
    for p in range(golden_trace["seq_x_in"].shape[0]):
        cos, sin = m.freqs_cos[[p]], m.freqs_sin[[p]]
        y = m.layer_forward(0, golden_trace["seq_x_in"][p:p + 1], cos, sin, [0])
        np.testing.assert_allclose(y, golden_trace["seq_x_out"][p:p + 1], atol=2e-5, rtol=1e-5)
    pos = golden_trace["batch_pos"]
    y = m.layer_forward(0, golden_trace["batch_x_in"], m.freqs_cos[pos], m.freqs_sin[pos], [0, 1])
    np.testing.assert_allclose(y, golden_trace["batch_x_out"], atol=2e-5, rtol=1e-5)
    # the reference stores K as [H, hd, S]; the oracle as [H, S, hd]
    np.testing.assert_allclose(m.k_cache[0][0].transpose(0, 2, 1), golden_trace["k_cache_a"], atol=1e-5)
    np.testing.assert_allclose(m.v_cache[0][0], golden_trace["v_cache_a"], atol=1e-5)
    assert H == golden_trace["seq_x_in"].shape[1]
