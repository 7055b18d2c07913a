"""Host logic of the multi-GPU column split (CPU; two gloo ranks for the collectives).

The split plan (which FFN / vocabulary columns a rank holds), the merge of per-rank
(max, id) pairs, and the order of operations in ``parallel.ffn_column_split`` /
``head_column_split`` are checked here with NumPy kernels built on the oracle: two ranks
each hold half of the FFN columns and half of the vocabulary, and their result must equal
the unsplit computation (fp32 sums split in K: max-rel <= 1e-5; tokens exact).

The head split (``attention_head_split`` / ``ffn_head_split`` / ``vocab_head_split``) is
checked the same way against the oracle's own layer (``OracleModel.layer_forward``, which
restates orchard/model.py:78-195): two ranks with half of the attention heads (their Q/K/V
rows, O columns and KV cache) each, all rows on both ranks, bit-identical residuals after
the all-reduces. The set-up of its peer-memory all-reduce is checked against a fake
library: a rank that cannot map a region, or gets a wrong known sum, makes every rank keep
NCCL.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ops
from orchard_b200.parallel import ColumnSplit, ffn_column_split, head_column_split, local_rows, merge_argmax, shard_range


@pytest.mark.parametrize("n,world,align", [(11008, 2, 32), (11008, 4, 32), (11008, 8, 32), (32000, 8, 16),
                                           (4096, 8, 32), (100, 3, 16), (64, 2, 16)])
def test_shard_range_covers_and_aligns(n, world, align):
    spans = [shard_range(n, world, r, align) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    for lo, hi in spans:
        assert lo % align == 0 and (hi % align == 0 or hi == n)
        assert hi > lo
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= align


def test_plan_7b_shapes():
    for world in (2, 4, 8):
        parts = [ColumnSplit.plan(11008, 32000, world, r) for r in range(world)]
        assert sum(p.f_local for p in parts) == 11008 and sum(p.v_local for p in parts) == 32000
        assert all(p.f_local % 32 == 0 for p in parts)  # down-projection K slices start on a group
        assert all(p.f_local % 16 == 0 for p in parts)  # gate/up interleave blocks
    assert ColumnSplit.plan(11008, 32000, 8, 0).f_local == 1376


def test_local_rows():
    assert local_rows(64, 8, 3) == (24, 32)
    with pytest.raises(ValueError):
        local_rows(10, 4, 0)


def test_merge_argmax_matches_np_argmax():
    g = np.random.default_rng(3)
    world, B, per = 4, 50, 7
    logits = g.integers(-3, 3, (B, world * per)).astype(np.float32)  # many ties
    logits[5, 9] = np.nan
    logits[6, 20] = np.nan
    logits[6, 3] = np.nan
    vals = np.empty((world, B), np.float32)
    idx = np.empty((world, B), np.int64)
    for r in range(world):
        sl = logits[:, r * per:(r + 1) * per]
        i = np.argmax(sl, axis=1)
        vals[r] = sl[np.arange(B), i]
        idx[r] = r * per + i
    assert np.array_equal(merge_argmax(vals, idx), np.argmax(logits, axis=1))


# ------------------------------------------------------------------------------------------
# two gloo ranks running the split orchestration with oracle kernels
# ------------------------------------------------------------------------------------------

H, F, V, B, EPS = 64, 192, 64, 4, 1e-5


def model(seed=11):
    g = np.random.default_rng(seed)

    def q(n, k):
        return ops.quantize_q4_0((g.standard_normal((n, k)) * 0.05).astype(np.float32))

    return {"w1": q(F, H), "w3": q(F, H), "w2": q(H, F), "lm": q(V, H),
            "ffn_norm": (1 + 0.1 * g.standard_normal(H)).astype(np.float32),
            "norm": (1 + 0.1 * g.standard_normal(H)).astype(np.float32),
            "x": g.standard_normal((B, H)).astype(np.float32)}


class NpOps:
    """The ops interface of parallel.py with oracle arithmetic on CPU tensors."""

    def __init__(self, m, plan):
        self.m, self.p = m, plan
        w1, s1, w3, s3, w2, s2 = plan.ffn_shard(*m["w1"], *m["w3"], *m["w2"])
        self.w1 = ops.dequantize_q4_0(w1, s1)
        self.w3 = ops.dequantize_q4_0(w3, s3)
        self.w2 = ops.dequantize_q4_0(np.ascontiguousarray(w2), np.ascontiguousarray(s2))
        self.lm = ops.dequantize_q4_0(*plan.lm_shard(*m["lm"]))

    def rmsnorm(self, x, w, xn, rows):
        w = self.m["norm"] if w is None else w
        xn[:rows] = torch.from_numpy(ops.rmsnorm(x[:rows].numpy(), w, EPS).astype(np.float16))

    def gate_up_swiglu(self, layer, xn_all, h, rows):
        a = xn_all[:rows].float().numpy()
        h[:rows] = torch.from_numpy((ops.silu(a @ self.w1.T) * (a @ self.w3.T)).astype(np.float16))

    def down_partial(self, layer, h, part, rows):
        part[:rows] = torch.from_numpy(h[:rows].float().numpy() @ self.w2.T)

    def add(self, x, red, rows):
        x[:rows] += red[:rows]

    def lm_partial(self, xn_all, logits, rows):
        logits[:rows] = torch.from_numpy(xn_all[:rows].float().numpy() @ self.lm.T)

    def argmax_pairs(self, logits, pairs, rows):
        lg = logits[:rows].numpy()
        i = np.argmax(lg, axis=1)
        pairs[:rows, 0] = torch.from_numpy(lg[np.arange(rows), i])
        pairs[:rows, 1] = torch.from_numpy((self.p.v0 + i).astype(np.float32))

    def merge_pairs(self, pairs_all, tok, rows):
        pa = pairs_all[:self.p.world * self.p.world * rows].numpy().reshape(self.p.world, self.p.world * rows, 2)
        t = merge_argmax(pa[..., 0], pa[..., 1].astype(np.int64))
        tok[:rows] = torch.from_numpy(t[self.p.rank * rows:(self.p.rank + 1) * rows].astype(np.int32))


class GlooComm:
    """all_gather / reduce_scatter on CPU tensors (the reduce-scatter as an all-reduce of
    the whole buffer and a slice: same result)."""

    def __init__(self, world, rank):
        self.world, self.rank = world, rank

    def all_gather(self, out, inp, rows):
        parts = [torch.empty_like(inp[:rows]) for _ in range(self.world)]
        dist.all_gather(parts, inp[:rows].contiguous())
        out[:self.world * rows] = torch.cat(parts)

    def reduce_scatter(self, out, inp, rows):
        full = inp[:self.world * rows].clone()
        dist.all_reduce(full)
        out[:rows] = full[self.rank * rows:(self.rank + 1) * rows]


class Bufs:
    def __init__(self, plan, x_local):
        W, R = plan.world, x_local.shape[0]
        self.x = x_local.clone()
        self.xn = torch.zeros((R, H), dtype=torch.float16)
        self.xn_all = torch.zeros((W * R, H), dtype=torch.float16)
        self.h = torch.zeros((W * R, plan.f_local), dtype=torch.float16)
        self.part = torch.zeros((W * R, H), dtype=torch.float32)
        self.red = torch.zeros((R, H), dtype=torch.float32)
        self.logits = torch.zeros((W * R, plan.v_local), dtype=torch.float32)
        self.pairs = torch.zeros((W * R, 2), dtype=torch.float32)
        self.pairs_all = torch.zeros((W * W * R, 2), dtype=torch.float32)
        self.tok = torch.zeros(R, dtype=torch.int32)


class Layer:
    def __init__(self, m):
        self.ffn_norm = m["ffn_norm"]


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = model()
        plan = ColumnSplit.plan(F, V, world, rank)
        r0, r1 = local_rows(B, world, rank)
        bufs = Bufs(plan, torch.from_numpy(m["x"][r0:r1]))
        o, c = NpOps(m, plan), GlooComm(world, rank)
        ffn_column_split(o, c, Layer(m), bufs, r1 - r0)
        x_after = bufs.x.numpy().copy()
        head_column_split(o, c, bufs, r1 - r0)
        q.put((rank, x_after, bufs.tok.numpy().copy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_column_split_two_gloo_ranks_match_unsplit():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, x, t = q.get(timeout=120)
        res[r] = (x, t)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # unsplit reference
    m = model()
    d = {k: ops.dequantize_q4_0(*m[k]) for k in ("w1", "w3", "w2", "lm")}
    xn = ops.rmsnorm(m["x"], m["ffn_norm"], EPS).astype(np.float16).astype(np.float32)
    h = (ops.silu(xn @ d["w1"].T) * (xn @ d["w3"].T)).astype(np.float16).astype(np.float32)
    x_ref = m["x"] + h @ d["w2"].T
    xn2 = ops.rmsnorm(x_ref, m["norm"], EPS).astype(np.float16).astype(np.float32)
    tok_ref = np.argmax(xn2 @ d["lm"].T, axis=1)
    x_split = np.concatenate([res[r][0] for r in range(world)])
    tok_split = np.concatenate([res[r][1] for r in range(world)])
    assert np.abs(x_split - x_ref).max() / np.abs(x_ref).max() <= 1e-5
    assert np.array_equal(tok_split, tok_ref)


# ------------------------------------------------------------------------------------------
# the head split: two gloo ranks, each with half the attention heads, FFN and vocabulary,
# run one decode step of every row; the result must equal the oracle's unsplit layer
# ------------------------------------------------------------------------------------------

HCFG = {"hidden_size": 128, "num_attention_heads": 4, "intermediate_size": 192, "num_hidden_layers": 1,
        "vocab_size": 64, "rms_norm_eps": 1e-5, "max_position_embeddings": 64}
HPOS = [5, 3, 7]  # each row's position; its cache holds positions 0 .. pos-1


def head_split_case():
    """The oracle model, the rows' input residual and their caches (N(0,1), all heads)."""
    from oracle.model import random_model
    m, _ = random_model(HCFG, seed=5)
    H, nh = HCFG["hidden_size"], HCFG["num_attention_heads"]
    hd = H // nh
    g = np.random.default_rng(17)
    x = g.standard_normal((len(HPOS), H)).astype(np.float32)
    kc = [g.standard_normal((nh, p, hd)).astype(np.float32) for p in HPOS]
    vc = [g.standard_normal((nh, p, hd)).astype(np.float32) for p in HPOS]
    return m, x, kc, vc


class NpHeadOps:
    """The head split's ops interface (parallel.py) with oracle arithmetic on this rank's
    slices; bufs hold CPU torch tensors, the cache is a list of per-row arrays."""

    def __init__(self, m, plan, kc, vc):
        L = m.layers[0]
        self.m, self.p, self.hd = m, plan, HCFG["hidden_size"] // HCFG["num_attention_heads"]
        wq, sq, wk, sk, wv, sv, wo, so = plan.attn_shard(*L.wq, *L.wk, *L.wv, *L.wo, self.hd)
        w1, s1, w3, s3, w2, s2 = plan.ffn_shard(*L.w1, *L.w3, *L.w2)
        c = np.ascontiguousarray
        self.wq, self.wk, self.wv = (wq, sq), (wk, sk), (wv, sv)
        self.wo, self.w1, self.w3, self.w2 = (c(wo), c(so)), (w1, s1), (w3, s3), (c(w2), c(s2))
        self.lm = plan.lm_shard(*m.lm_head)
        self.kc = [k[plan.h0:plan.h1] for k in kc]
        self.vc = [v[plan.h0:plan.h1] for v in vc]
        self.L = L

    def qkv_local(self, ctx, b, rows):
        x = b.x[:rows].numpy()
        xn = ops.rmsnorm(x, self.L.attn_norm, EPS)
        hl = self.p.h_local
        cos, sin = self.m.freqs_cos[HPOS], self.m.freqs_sin[HPOS]
        q = ops.rope(ops.gemm_q4_0(*self.wq, xn).reshape(rows, hl, self.hd), cos, sin)
        k = ops.rope(ops.gemm_q4_0(*self.wk, xn).reshape(rows, hl, self.hd), cos, sin)
        v = ops.gemm_q4_0(*self.wv, xn).reshape(rows, hl, self.hd)
        for i in range(rows):
            self.kc[i] = np.concatenate([self.kc[i], k[i][:, None, :]], axis=1)
            self.vc[i] = np.concatenate([self.vc[i], v[i][:, None, :]], axis=1)
        b.q = q

    def attention_local(self, ctx, b, rows):
        b.attn = np.stack([ops.attention_one(b.q[i], self.kc[i], self.vc[i]).reshape(-1) for i in range(rows)])

    def o_partial(self, ctx, b, rows, resid):
        p = torch.from_numpy(ops.gemm_q4_0(*self.wo, b.attn).astype(np.float32))
        b.x[:rows] = b.x[:rows] + p if resid else p

    def gate_up_local(self, ctx, b, rows):
        xf = ops.rmsnorm(b.x[:rows].numpy(), self.L.ffn_norm, EPS)
        b.h = ops.mul(ops.silu(ops.gemm_q4_0(*self.w1, xf)), ops.gemm_q4_0(*self.w3, xf))

    def down_partial_resid(self, ctx, b, rows, resid):
        p = torch.from_numpy(ops.gemm_q4_0(*self.w2, b.h).astype(np.float32))
        b.x[:rows] = b.x[:rows] + p if resid else p

    def rmsnorm(self, x, w, xn, rows):
        xn[:rows] = torch.from_numpy(ops.rmsnorm(x[:rows].numpy(), self.m.norm, EPS))

    def lm_partial(self, xn, logits, rows):
        logits[:rows] = torch.from_numpy(ops.gemm_q4_0(*self.lm, xn[:rows].numpy()).astype(np.float32))

    def argmax_pairs(self, logits, pairs, rows):
        lg = logits[:rows].numpy()
        i = np.argmax(lg, axis=1)
        pairs[:rows, 0] = torch.from_numpy(lg[np.arange(rows), i])
        pairs[:rows, 1] = torch.from_numpy((self.p.v0 + i).astype(np.float32))

    def merge_all_pairs(self, pairs_all, tok, rows):
        pa = pairs_all[:self.p.world * rows].numpy().reshape(self.p.world, rows, 2)
        tok[:rows] = torch.from_numpy(merge_argmax(pa[..., 0], pa[..., 1].astype(np.int64)).astype(np.int32))


class HeadComm(GlooComm):
    def all_reduce(self, x, rows):
        dist.all_reduce(x[:rows])


class HeadBufs:
    def __init__(self, plan, x):
        R, H = x.shape
        self.x = torch.from_numpy(x.copy())
        self.xn = torch.zeros((R, H), dtype=torch.float32)
        self.logits = torch.zeros((R, plan.v_local), dtype=torch.float32)
        self.pairs = torch.zeros((R, 2), dtype=torch.float32)
        self.pairs_all = torch.zeros((plan.world * R, 2), dtype=torch.float32)
        self.tok = torch.zeros(R, dtype=torch.int32)


def _head_rank(rank, world, port, q):
    from orchard_b200.parallel import attention_head_split, ffn_head_split, vocab_head_split
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, x, kc, vc = head_split_case()
        hd = HCFG["hidden_size"] // HCFG["num_attention_heads"]
        plan = ColumnSplit.plan(HCFG["intermediate_size"], HCFG["vocab_size"], world, rank,
                                HCFG["num_attention_heads"], hd)
        o, c, b = NpHeadOps(m, plan, kc, vc), HeadComm(world, rank), HeadBufs(plan, x)
        attention_head_split(o, c, None, b, len(HPOS))
        ffn_head_split(o, c, None, b, len(HPOS))
        x_after = b.x.numpy().copy()
        vocab_head_split(o, c, b, len(HPOS))
        q.put((rank, x_after, b.tok.numpy().copy(), plan.h0, plan.h1))
    finally:
        dist.destroy_process_group()


def test_head_split_plan():
    parts = [ColumnSplit.plan(11008, 32000, 8, r, 32, 128) for r in range(8)]
    assert [(p.h0, p.h1) for p in parts] == [(4 * r, 4 * r + 4) for r in range(8)]
    assert all(p.heads for p in parts) and not ColumnSplit.plan(11008, 32000, 8, 0).heads
    with pytest.raises(ValueError):
        ColumnSplit.plan(11008, 32000, 8, 0, 4, 128)  # fewer heads than ranks
    with pytest.raises(ValueError):
        ColumnSplit.plan(11008, 32000, 2, 0, 32, 48)  # O columns would split a scale group
    with pytest.raises(ValueError):
        ColumnSplit.plan(11008, 32000, 2, 0).attn_shard(*([None] * 8), 128)


def test_head_split_two_gloo_ranks_match_oracle_layer():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_head_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, x, t, h0, h1 = q.get(timeout=120)
        res[r] = (x, t, h0, h1)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [(res[r][2], res[r][3]) for r in range(world)] == [(0, 2), (2, 4)]
    # unsplit: the oracle's own layer (orchard/model.py:78-195) over the same caches
    m, x, kc, vc = head_split_case()
    for i, (k, v) in enumerate(zip(kc, vc)):
        m.k_cache[0][i], m.v_cache[0][i] = k, v
    x_ref = m.layer_forward(0, x, m.freqs_cos[HPOS], m.freqs_sin[HPOS], list(range(len(HPOS))))
    tok_ref = np.argmax(m._lin(m.lm_head, ops.rmsnorm(x_ref, m.norm, EPS)), axis=1)
    for r in range(world):  # every rank holds every row, bit-identical after the all-reduces
        assert np.array_equal(res[r][0], res[0][0])
        assert np.array_equal(res[r][1], tok_ref)
    assert np.abs(res[0][0] - x_ref).max() / np.abs(x_ref).max() <= 1e-5


# ------------------------------------------------------------------------------------------
# the head split's peer all-reduce set-up: every rank keeps NCCL when any rank fails
# ------------------------------------------------------------------------------------------

def _peer_setup_rank(rank, world, port, fail_rank, fail_test_rank, q):
    """One gloo rank building _PeerAllReduce against a fake library: region size, IPC calls
    and the self-test are stubbed; `fail_rank` fails to map a peer's region and
    `fail_test_rank` gets a wrong known sum."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import orchard_b200.model as M
        from orchard_b200 import _lib

        class FakeLib:
            def orch_peer_region_bytes(self, w, n):
                return 4096 + 16 * w * n

        def fake_call(name, *args):
            if name == "orch_ipc_open" and rank == fail_rank:
                raise _lib.OrchardError(name, 2, "mapping refused")
            return 0

        M._lib.lib = lambda: FakeLib()
        M.call = fake_call
        torch.cuda.synchronize = lambda *a, **k: None
        M._PeerAllReduce._self_test = lambda self, dev: rank != fail_test_rank
        p = M._PeerAllReduce(dist.group.WORLD, world, rank, 4096, "cpu")
        q.put((rank, p.ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank,fail_test_rank,want", [(-1, -1, True), (1, -1, False), (-1, 0, False)])
def test_peer_allreduce_setup_is_collective(fail_rank, fail_test_rank, want):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_setup_rank, args=(r, world, port, fail_rank, fail_test_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == {0: want, 1: want}
