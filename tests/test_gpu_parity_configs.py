"""The benchmarked configurations against the oracle (GPU), with the kernels the bench runs.

* Config 1 exactly: one 7B-shaped layer, batch 1, 127 cached N(0,1) fp16 positions, the
  current position 127, input hidden state N(0,1) fp16. Layer output and its update
  (output - input) within 1e-2 of max|ref| (max|gpu - ref| / max|ref|); RMSNorm and RoPE
  within 1e-3 (orchard/model.py:78-195, orchard/kernels/rmsnorm.metal:23-35,
  orchard/kernels/rope.metal:26-49).
* Batched decode at the bench's batch sizes (64 and 16 sequences) on a 2-layer 7B-shaped
  slice, 515 cached positions, three steps through the captured decode graph with the
  default kernel selection (tiled weights, the tcgen05 GEMMs with their split-K and
  register epilogues): every row's logits within 1e-2 of that row's max|ref|
  (orchard/model.py:318-356).
* Config-5 prefill: two 300-token prompts with a rank-16 LoRA on Q and V (A, B ~ N(0, 0.01))
  through ``Llama.prefill`` (256-row tensor-core tiles, the TF32 LoRA term in the QKV
  tile, the tensor-core prefill attention) against the reference's token-by-token prefill
  (orchard/model.py:285-305): the K and V caches of both layers, then the next decode
  step's logits, within 1e-2.

Weights are seeded N(0, 0.02) fp16 packed by the reference rule on the device (bit-exact
with the host packer, tests/test_gpu_ops.py); the oracle runs the same packed weights.
"""

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import ops
from orchard_b200 import loader
from orchard_b200._lib import F16, F32, call, ptr
from orchard_b200.model import Llama
from test_gpu_model import seven_b_slice

pytestmark = pytest.mark.gpu


def S():
    return torch.cuda.current_stream().cuda_stream


def row_rel_err(got, ref):
    """max over rows of max|got - ref| / max|ref| of that row."""
    return max(rel_err(g, r) for g, r in zip(np.asarray(got), np.asarray(ref)))


# ------------------------------------------------------------------------------ config 1
def test_config1_single_layer_decode_batch1():
    cfg, t, om = seven_b_slice(n_layers=1, seed=31)
    om.cache_dequant = True
    llm = Llama(checkpoint=loader.from_tensors(cfg, t), max_batch=1, max_seq=256)
    eng = llm.engine
    g = np.random.default_rng([20261201, 1, 0, 0])
    x = g.standard_normal((1, 4096), dtype=np.float32).astype(np.float16)
    kc = g.standard_normal((32, 127, 128), dtype=np.float32).astype(np.float16)
    vc = g.standard_normal((32, 127, 128), dtype=np.float32).astype(np.float16)
    eng.k_cache[0, 0, :, :127].copy_(torch.from_numpy(kc))
    eng.v_cache[0, 0, :, :127].copy_(torch.from_numpy(vc))
    eng.x[:1].copy_(torch.from_numpy(x.astype(np.float32)))
    eng.pos[:1].fill_(127)
    eng.run_layer(0, 1)
    torch.cuda.synchronize()
    out = eng.x[:1].cpu().numpy()
    k_new = eng.k_cache[0, 0, :, 127].float().cpu().numpy()
    v_new = eng.v_cache[0, 0, :, 127].float().cpu().numpy()

    om.k_cache[0][0] = kc.astype(np.float32)
    om.v_cache[0][0] = vc.astype(np.float32)
    cos, sin = om.freqs_cos[[127]], om.freqs_sin[[127]]
    x32 = x.astype(np.float32)
    ref = om.layer_forward(0, x32, cos, sin, [0])
    assert rel_err(out, ref) <= 1e-2
    assert rel_err(out - x32, ref - x32) <= 1e-2          # the layer's own contribution
    assert rel_err(k_new, om.k_cache[0][0][:, 127]) <= 1e-2  # RoPE'd key appended at 127
    assert rel_err(v_new, om.v_cache[0][0][:, 127]) <= 1e-2

    # RMSNorm alone (fp32 in, fp32 out) and RoPE alone at position 127, 1e-3
    L = om.layers[0]
    xn = torch.empty((1, 4096), dtype=torch.float32, device="cuda")
    call("orch_rmsnorm_ex", torch.from_numpy(x32).cuda(), F32, torch.from_numpy(L.attn_norm).cuda(), F32, ptr(xn),
         F32, 1e-5, 4096, 1, S())
    xn_ref = ops.rmsnorm(x32, L.attn_norm, 1e-5)
    assert rel_err(xn.cpu().numpy(), xn_ref) <= 1e-3
    q = ops.gemm_q4_0(L.wq[0], L.wq[1], xn_ref).astype(np.float16)  # the projection RoPE rotates
    qr = torch.empty((1, 32, 128), dtype=torch.float32, device="cuda")
    call("orch_rope_ex", torch.from_numpy(q).cuda(), F16, torch.from_numpy(np.ascontiguousarray(cos)).cuda(),
         torch.from_numpy(np.ascontiguousarray(sin)).cuda(), F32, ptr(qr), F32, 128, 32, 1, S())
    q_ref = ops.rope(q.astype(np.float32).reshape(1, 32, 128), cos, sin)
    assert rel_err(qr.cpu().numpy(), q_ref) <= 1e-3


# ------------------------------------------------------------------ batched decode (config 4)
@pytest.mark.parametrize("B", [64, 16])
def test_batched_decode_7b_slice_matches_oracle(B):
    """B sequences with 515 cached positions each (seeded N(0,1) fp16 K/V, identical in the
    device cache and the oracle's), three greedy steps at positions 515..517 through the
    decode graph. The oracle follows the GPU's tokens so both see the same inputs."""
    cfg, t, om = seven_b_slice(n_layers=2, seed=7)
    om.cache_dequant = True
    P, steps = 515, 3
    llm = Llama(checkpoint=loader.from_tensors(cfg, t), max_batch=B, max_seq=640)
    eng = llm.engine
    gen = torch.Generator(device="cuda").manual_seed(1000 + B)
    for li in range(2):
        k = torch.randn((B, 32, P, 128), generator=gen, device="cuda").half()
        v = torch.randn((B, 32, P, 128), generator=gen, device="cuda").half()
        eng.k_cache[li, :B, :, :P].copy_(k)
        eng.v_cache[li, :B, :, :P].copy_(v)
        kh, vh = k.float().cpu().numpy(), v.float().cpu().numpy()
        for b in range(B):
            om.k_cache[li][b] = kh[b]
            om.v_cache[li][b] = vh[b]
        del k, v, kh, vh
    cur = np.random.default_rng([20261201, 4, B]).integers(0, 32000, B).astype(np.int32)
    for s in range(steps):
        eng.tok_in[:B].copy_(torch.from_numpy(cur))
        eng.pos[:B].fill_(P + s)
        eng.step(B, logits=True)  # the captured graph, default kernel selection
        lg = eng.logits[:B].cpu().numpy()
        ref = om.forward_tokens(cur.tolist(), [P + s] * B, list(range(B)))
        assert row_rel_err(lg, ref) <= 1e-2, s
        tok = eng.tok_out[:B].cpu().numpy()
        top2 = np.sort(ref, axis=1)[:, -2:]
        clear = top2[:, 1] - top2[:, 0] > 1e-2 * np.abs(ref).max(axis=1)
        assert np.array_equal(tok[clear], np.argmax(ref, axis=1)[clear])
        cur = tok.astype(np.int32)


# ------------------------------------------------------------------------- prefill (config 5)
def test_prefill_with_lora_matches_token_by_token_oracle():
    """The oracle runs each prompt's rows in position order through its layer, appending
    each row's K/V before that row attends: the reference's token-by-token prefill, row for
    row (its projections are row-independent)."""
    cfg, t, om = seven_b_slice(n_layers=2, seed=9)
    om.cache_dequant = True
    r, n = 16, 300
    g = np.random.default_rng([20261201, 5, 1])
    per_layer = {}
    for li in range(2):
        mods = {m: ((g.standard_normal((4096, r)) * 0.01).astype(np.float32),
                    (g.standard_normal((r, 4096)) * 0.01).astype(np.float32) * 2.0) for m in ("wq", "wv")}
        per_layer[li] = mods
        om.layers[li].lora = dict(mods)
    prompts = g.integers(0, 32000, (2, n)).tolist()
    llm = Llama(checkpoint=loader.from_tensors(cfg, t), max_batch=2, max_seq=320)
    eng = llm.engine
    eng.set_lora(per_layer, r)
    llm.prefill(prompts)
    om.reset()
    for b, p in enumerate(prompts):
        om.forward_tokens(p, list(range(n)), [b] * n, logits=False)
    torch.cuda.synchronize()
    for li in range(2):
        for b in range(2):
            kd = eng.k_cache[li, b, :, :n].float().cpu().numpy()
            vd = eng.v_cache[li, b, :, :n].float().cpu().numpy()
            assert rel_err(kd, om.k_cache[li][b]) <= 1e-2, (li, b)
            assert rel_err(vd, om.v_cache[li][b]) <= 1e-2, (li, b)
    # the first decode step: the last prompt token again at position n (orchard/model.py:305)
    last = [p[-1] for p in prompts]
    eng.tok_in[:2].copy_(torch.tensor(last, dtype=torch.int32))
    eng.pos[:2].fill_(n)
    eng.step(2, logits=True)
    ref = om.forward_tokens(last, [n, n], [0, 1])
    assert row_rel_err(eng.logits[:2].cpu().numpy(), ref) <= 1e-2
