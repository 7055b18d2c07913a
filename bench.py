"""Benchmark: 7B-shape INT4 batched decode tokens/s on B200.

Workload (the reference's headline decode configuration): a 32-layer Llama-2-7B-shaped
random-init INT4 model (hidden 4096, 32 heads x 128, FFN 11008, vocab 32000, group-32
scales); B independent sequences with a 512-token random prompt prefilled into the fp16
KV cache, then greedy decode. One step = one token for each of the B sequences through
all 32 layers, the final norm, the lm_head and the argmax. Timed steps run at positions
515..639 (average ~577, the middle of the 513..640 decode window). Every step streams
3.7 GB of weights plus the KV cache, so inputs are far larger than L2 (126 MB).

Our arm:   python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B]
Reference: python bench.py --impl reference ...  (the reference's CPU path, restated in
           oracle/, timed on the host cores; the Metal backend cannot run here)

Under torchrun each rank runs its own B sequences (sequence data parallelism, no
collective on the data path): scaling "weak"; the reported value is the sum over ranks
of tokens / (max over ranks of the timed region).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG7B = {"hidden_size": 4096, "num_attention_heads": 32, "intermediate_size": 11008, "num_hidden_layers": 32,
         "vocab_size": 32000, "rms_norm_eps": 1e-5, "max_position_embeddings": 2048}
PROMPT = 512
MAX_SEQ = 640
METRIC = "7B-shape INT4 decode tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=125)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--extra-batches", default="1,16", help="also time these batch sizes (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-column-split", action="store_true", help="at N > 1 skip the column-split measurement")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--only-decode", action="store_true",
                    help="time the decode step alone (no per-batch, split, e2e, prefill, sweep or CPU sections): "
                         "for launch-list captures")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ------------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                for line in out.stdout.strip().splitlines():
                    self.rows.append([c.strip() for c in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------------------------------------
# model construction (random init on the device, packed with the reference rule)
# ------------------------------------------------------------------------------------------------
def build_model(cfg, device, max_batch, seed=1234, group=None, split_heads=False):
    import torch

    from orchard_b200 import loader
    from orchard_b200.model import Llama, quantize_on_device

    H, F, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    gen = torch.Generator(device=device).manual_seed(seed)

    def packed(n, k):
        w = (torch.randn((n, k), generator=gen, device=device, dtype=torch.float32) * 0.02).half()
        p, s = quantize_on_device(w, device)
        del w
        return ("packed", p, s)

    ck = loader.Checkpoint(cfg)
    for li in range(cfg["num_hidden_layers"]):
        e = ck.layers[li]
        for nm, shp in (("wq", (H, H)), ("wk", (H, H)), ("wv", (H, H)), ("wo", (H, H)),
                        ("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F))):
            e[nm] = packed(*shp)
        e["attn_norm"] = (1 + 0.1 * torch.randn(H, generator=gen, device=device)).half().float().cpu().numpy()
        e["ffn_norm"] = (1 + 0.1 * torch.randn(H, generator=gen, device=device)).half().float().cpu().numpy()
    ck.embed = torch.randn((V, H), generator=gen, device=device).half()
    ck.norm = (1 + 0.1 * torch.randn(H, generator=gen, device=device)).half().float().cpu().numpy()
    ck.lm_head = packed(V, H)
    return Llama(checkpoint=ck, device=device, max_batch=max_batch, max_seq=MAX_SEQ, group=group,
                 split_heads=split_heads)


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
def time_decode(llm, B, steps, warmup, start_pos):
    """Device-timed decode steps (graph replays) for rows [0, B) starting at start_pos."""
    import torch

    eng = llm.engine
    dev = eng.device
    eng.pos[:B].fill_(start_pos)
    for _ in range(warmup):
        eng.step(B, logits=True)
        eng.tok_in[:B].copy_(eng.tok_out[:B])
        eng.pos[:B].add_(1)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push(f"timed_decode_b{B}")  # ncu --nvtx-include selects these launches
    s.record()
    for _ in range(steps):
        eng.step(B, logits=True)
        eng.tok_in[:B].copy_(eng.tok_out[:B])
        eng.pos[:B].add_(1)
    e.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    return s.elapsed_time(e) / 1000.0


# INT4 GEMM entry points: argument index of M, K and N, N multiplier, output bytes per element
QGEMM_ARGS = {"orch_q4t_rms_qkv_rope": (5, 6, 7, 3, 2), "orch_q4t_rms_linear_swiglu": (6, 7, 8, 2, 1),
              "orch_q4_qkv_rope": (3, 4, 5, 3, 2), "orch_q4_linear_swiglu": (4, 5, 6, 2, 1),
              "orch_q4_linear_resid": (4, 5, 6, 1, 8), "orch_gemm_q4_0_ex": (8, 6, 7, 1, 4),
              "orch_q4t_qkv_rope": (2, 3, 4, 3, 2), "orch_q4t_linear_swiglu": (3, 4, 5, 2, 1),
              "orch_q4t_linear_resid": (3, 4, 5, 1, 8), "orch_q4t_gemm": (6, 4, 5, 1, 4)}


SPLIT_FAMILIES = {"orch_q4t_qkv_rope": "attn_proj_gemm (replicated weights)",
                  "orch_q4t_linear_resid": "attn_proj_gemm (replicated weights)",
                  "orch_q4t_linear_swiglu": "ffn_vocab_slice_gemm", "orch_q4t_gemm": "ffn_vocab_slice_gemm",
                  "nccl": "nccl", "orch_attention_decode": "attention"}
# the head split: every projection is a slice; the all-reduces are timed around the
# collective (peer-memory kernel or NCCL), so the peer kernel's own launch is not counted twice
HEAD_FAMILIES = {"orch_q4t_rms_qkv_rope": "slice_gemm", "orch_q4t_qkv_rope": "slice_gemm",
                 "orch_q4t_linear_resid": "slice_gemm", "orch_q4t_rms_linear_swiglu": "slice_gemm",
                 "orch_q4t_linear_swiglu": "slice_gemm", "orch_q4t_gemm": "slice_gemm",
                 "nccl": "allreduce / all-gather", "orch_peer_allreduce": None,
                 "orch_attention_decode": "attention"}


def kernel_profile(llm, B, pos, reps=3, split=False):
    """Per-kernel-family device time of one eager decode step (CUDA events around each
    launch on the launching stream), with each family's algorithmic bytes. With `split`
    (the column split) the families are the replicated attention projections, the FFN /
    vocabulary slice GEMMs, attention, the NCCL collectives and the rest; for the head split,
    the slice GEMMs, attention, the all-reduces / all-gather and the rest."""
    import torch

    from orchard_b200 import _lib
    eng = llm.engine
    cfg = eng.cfg
    H, F, V, nh, hd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.num_attention_heads, cfg.head_dim
    fam = {}
    orig = _lib.call

    def timed(name, *args):
        st = torch.cuda.current_stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        rc = orig(name, *args)
        b.record(st)
        fam.setdefault(name, []).append((a, b, args))
        return rc

    import orchard_b200.model as M
    M.call = timed
    comm = getattr(eng, "_comm", None)
    saved = {}

    def timed_collective(fn, *args):
        st = torch.cuda.current_stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        rc = fn(*args)
        b.record(st)
        fam.setdefault("nccl", []).append((a, b, args))
        return rc

    if split and comm is not None:
        for nm in ("all_gather", "reduce_scatter", "all_reduce"):
            saved[nm] = getattr(comm, nm)
            setattr(comm, nm, lambda *args, _fn=saved[nm]: timed_collective(_fn, *args))

    try:
        for _ in range(reps):
            eng.pos[:B].fill_(pos)
            eng.step(B, logits=True, graph=False)
        torch.cuda.synchronize()
    finally:
        M.call = orig
        for nm, fn in saved.items():
            setattr(comm, nm, fn)
    L = pos + 1
    out = {}
    if split:
        table = HEAD_FAMILIES if getattr(eng, "heads_split", False) else SPLIT_FAMILIES
        for name, ev in fam.items():
            key = table.get(name, "other")
            if key is None:
                continue
            d = out.setdefault(key, {"ms": 0.0, "launches": 0})
            d["ms"] += sum(a.elapsed_time(b) for a, b, _ in ev) / reps
            d["launches"] += len(ev) // reps
        return out
    for name, ev in fam.items():
        ms = sum(a.elapsed_time(b) for a, b, _ in ev) / reps
        n = len(ev) // reps
        if name in QGEMM_ARGS:
            # weights + scales once, activations in, outputs out (fp16 in, fp16/fp32 out);
            # padding of the tiled layout is not counted
            byts = 0
            im, ik, inn, nmul, out_b = QGEMM_ARGS[name]
            for _, _, args in ev[:n]:
                Mr, K, N = args[im], args[ik], nmul * args[inn]
                byts += N * K // 2 + N * K // 16 + 2 * Mr * K + out_b * Mr * N
            out["qgemm"] = out.get("qgemm", {"ms": 0.0, "bytes": 0, "launches": 0})
            out["qgemm"]["ms"] += ms
            out["qgemm"]["bytes"] += byts
            out["qgemm"]["launches"] += n
        elif name == "orch_attention_decode":
            byts = n * (2 * B * nh * L * hd * 2 + 2 * 2 * B * nh * hd)
            out["attention"] = {"ms": ms, "bytes": byts, "launches": n}
        else:
            out.setdefault("other", {"ms": 0.0, "bytes": 0, "launches": 0})
            out["other"]["ms"] += ms
            out["other"]["launches"] += n
    return out


def time_prefill_lora(llm, reps=3, seqs=8, length=512, rank=16, seed=11):
    """Config 5: batched prefill of seqs x length random tokens with a rank-16 LoRA on Q and V
    (A, B ~ N(0, 0.01)); device-timed, tensor-core INT4 GEMMs with M = seqs * length."""
    import torch

    eng = llm.engine
    H = eng.cfg.hidden_size
    g = np.random.default_rng([20261201, 5, seed, seqs])
    per_layer = {li: {m: ((g.standard_normal((H, rank)) * 0.01).astype(np.float32),
                          (g.standard_normal((rank, H)) * 0.01).astype(np.float32) * 2.0)
                      for m in ("wq", "wv")} for li in range(eng.cfg.num_hidden_layers)}
    eng.set_lora(per_layer, rank)
    prompts = g.integers(0, eng.cfg.vocab_size, (seqs, length)).tolist()
    llm.prefill(prompts)
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        llm.prefill(prompts)
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) / 1000.0)
    eng.set_lora({}, rank)
    t = float(np.median(ts))
    tokens = seqs * length
    lin = 2.0 * 6_476_005_376 * tokens            # dense-equivalent projection flops (32 layers + lm_head)
    lin -= 2.0 * 4096 * 32000 * tokens            # prefill computes no logits
    attn = 4.0 * 32 * 32 * 128 * seqs * length * (length + 1) / 2   # QK^T and PV, causal
    lora = 2.0 * 32 * 2 * tokens * (H * rank + rank * H)
    flops = lin + attn + lora
    return {"workload": f"batched prefill {seqs}x{length} tokens, LoRA r={rank} on Q and V", "ms": round(t * 1e3, 3),
            "tok_s": round(tokens / t, 1), "tflops": round(flops / t / 1e12, 2), "flops": flops, "s": t}


def time_column_split(cfg, dev, global_batch, steps, warmup, rank, world, check_steps=0):
    """The column split (sequences sharded, FFN and vocabulary projections split by columns,
    two NCCL collectives per layer): global_batch sequences, global_batch / world per rank,
    512-token prompts, greedy decode steps timed on the device (max over ranks). With fewer
    sequences than ranks every rank runs the same sequence (attention replicated), counted
    once. `check_steps` > 0: before timing, that many eager steps of the split engine are
    compared with the unsplit engine on the same weights and prompts (same input tokens each
    step): the tokens of this rank's rows (argmax over the whole vocabulary, merged across
    ranks) and the logits of its vocabulary slice."""
    import torch
    import torch.distributed as dist

    replicated = global_batch < world
    B = 1 if replicated else global_batch // world
    llm = build_model(cfg, dev, B, seed=4321, group=dist.group.WORLD)  # same weights on every rank
    eng = llm.engine
    g = np.random.default_rng([20261201, 6, 0 if replicated else rank])
    prompts = g.integers(0, cfg["vocab_size"], (B, PROMPT)).tolist()
    llm.prefill(prompts)
    out = {"global_batch": global_batch, "per_rank_batch": B, "steps": steps,
           "rows": "the same sequence on every rank" if replicated else "sequences sharded over the ranks"}
    check = None
    if check_steps:
        sp = eng.split
        last = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=dev)
        eng.tok_in[:B].copy_(last)
        tin, tout, lgs = [], [], []
        for s in range(check_steps):
            eng.pos[:B].fill_(PROMPT + s)
            tin.append(eng.tok_in[:B].clone())
            eng.step(B, logits=True, graph=False)
            tout.append(eng.tok_out[:B].clone())
            lgs.append(eng.sdec.logits[rank * B:(rank + 1) * B].clone())
            eng.tok_in[:B].copy_(eng.tok_out[:B])
        check = (sp.v0, sp.v1, tin, tout, lgs)
    start = PROMPT + 3 - warmup if warmup <= 3 else PROMPT
    eng.pos[:B].fill_(PROMPT)
    eng.step(B, logits=True)  # capture the graph (with its NCCL calls) before timing
    torch.cuda.synchronize(dev)
    dist.barrier()
    secs = time_decode(llm, B, steps, warmup, start)
    t = torch.tensor([secs], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    secs = float(t.item())
    out.update(tok_s=round(global_batch * steps / secs, 2), ms_per_step=round(secs / steps * 1000, 4))
    if check_steps:
        fam = kernel_profile(llm, B, start + warmup + steps // 2, split=True)
        out["families_ms"] = {k: round(v["ms"], 4) for k, v in fam.items()}
    eng.release_graphs()
    del llm, eng
    torch.cuda.empty_cache()
    if check is not None:
        v0, v1, tin, tout, lgs = check
        ref = build_model(cfg, dev, B, seed=4321)  # unsplit, same weights
        ref.prefill(prompts)
        out["check"] = split_check(ref.engine, prompts, tin, tout, lgs, v0, v1, B, dev)
        del ref
        torch.cuda.empty_cache()
    return out


def split_check(eng_ref, prompts, tin, tout, lgs, v0, v1, rows, dev):
    """Decode steps of an unsplit engine on the inputs a split engine saw (`tin`, one tensor of
    input tokens per step) against the split's tokens `tout` and its vocabulary slice of the
    logits `lgs` (rows [0, rows) of both); summed over the ranks."""
    import torch
    import torch.distributed as dist

    match, total, err, clear, clear_match, tie_ok = 0, 0, 0.0, 0, 0, 0
    for s in range(len(tin)):
        eng_ref.pos[:rows].fill_(PROMPT + s)
        eng_ref.tok_in[:rows].copy_(tin[s])
        eng_ref.step(rows, logits=True, graph=False)
        same = eng_ref.tok_out[:rows] == tout[s]
        match += int(same.sum().item())
        total += rows
        full = eng_ref.logits[:rows, v0:v1]
        err = max(err, float((lgs[s] - full).abs().max().item() / max(full.abs().max().item(), 1e-30)))
        # a row whose two best logits are more than 1e-2 of max |logit| apart must pick the
        # same token; closer rows may differ by summation order, but the split's pick must
        # then be within that margin of the best logit
        lg = eng_ref.logits[:rows]
        tol = 1e-2 * lg.abs().amax(dim=1)
        top2 = torch.topk(lg, 2, dim=1).values
        is_clear = (top2[:, 0] - top2[:, 1]) > tol
        clear += int(is_clear.sum().item())
        clear_match += int((same & is_clear).sum().item())
        picked = lg.gather(1, tout[s].long().view(-1, 1)).view(-1)
        tie_ok += int(((~same) & ~is_clear & (top2[:, 0] - picked <= tol)).sum().item())
    st = torch.tensor([match, total, clear, clear_match, tie_ok], dtype=torch.float64, device=dev)
    dist.all_reduce(st)
    e = torch.tensor([err], device=dev)
    dist.all_reduce(e, op=dist.ReduceOp.MAX)
    m, n, c, cm, ok = (int(v) for v in st.tolist())
    return {"steps": len(tin),
            "tokens_match": bool(cm == c and m + ok == n and e.item() <= 1e-2),
            "tokens_matched": f"{m}/{n}", "clear_rows_matched": f"{cm}/{c}",
            "other_rows_within_tie_margin": f"{ok}/{n - c}",
            "logits_max_rel": float(e.item()),
            "rule": "rows with a top-2 gap > 1e-2 of max|logit| pick the same token; the rest pick a "
                    "token within that margin of the best; logits of each rank's vocabulary slice "
                    "within 1e-2 (max|split - unsplit| / max|unsplit|)",
            "against": "unsplit engine, same weights, prompts and input tokens"}


def time_head_split(cfg, dev, batches, steps, warmup, world, check_steps=8):
    """The head split (every rank runs all sequences; attention heads, FFN and vocabulary
    divided over the ranks; two all-reduces of the residual per layer): for each global
    batch in `batches` (one engine sized for the largest), greedy decode steps timed on the
    device (max over ranks). Before timing the largest batch, `check_steps` eager steps are
    compared with the unsplit engine on the same weights, prompts and input tokens."""
    import torch
    import torch.distributed as dist

    Bmax = max(batches)
    llm = build_model(cfg, dev, Bmax, seed=4321, group=dist.group.WORLD, split_heads=True)
    eng = llm.engine
    g = np.random.default_rng([20261201, 7, 0])  # the same prompts on every rank
    prompts = g.integers(0, cfg["vocab_size"], (Bmax, PROMPT)).tolist()
    llm.prefill(prompts)
    sp = eng.split
    out = {"heads_per_rank": sp.h_local, "by_global_batch": {},
           "allreduce": (f"peer-memory kernel (orch_peer_allreduce) up to {eng._comm.peer.max_floats // cfg['hidden_size']}"
                         " rows, NCCL above" if eng.peer_allreduce else "NCCL")}
    check = None
    if check_steps:
        last = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=dev)
        eng.tok_in[:Bmax].copy_(last)
        tin, tout, lgs = [], [], []
        for s in range(check_steps):
            eng.pos[:Bmax].fill_(PROMPT + s)
            tin.append(eng.tok_in[:Bmax].clone())
            eng.step(Bmax, logits=True, graph=False)
            tout.append(eng.tok_out[:Bmax].clone())
            lgs.append(eng.sdec.logits[:Bmax].clone())
            eng.tok_in[:Bmax].copy_(eng.tok_out[:Bmax])
        check = (tin, tout, lgs)
    start = PROMPT + 3 - warmup if warmup <= 3 else PROMPT
    for B in sorted(batches, reverse=True):
        eng.pos[:B].fill_(PROMPT)
        eng.step(B, logits=True)  # capture the graph (with its NCCL calls) before timing
        torch.cuda.synchronize(dev)
        dist.barrier()
        secs = time_decode(llm, B, steps, warmup, start)
        t = torch.tensor([secs], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
        out["by_global_batch"][str(B)] = {"tok_s": round(B * steps / secs, 2),
                                          "ms_per_step": round(secs / steps * 1000, 4), "steps": steps}
        fam = kernel_profile(llm, B, start + warmup + steps // 2, split=True)
        out["by_global_batch"][str(B)]["families_ms"] = {k: round(v["ms"], 4) for k, v in fam.items()}
    v0, v1 = sp.v0, sp.v1
    eng.release_graphs()
    del llm, eng
    torch.cuda.empty_cache()
    if check is not None:
        ref = build_model(cfg, dev, Bmax, seed=4321)  # unsplit, same weights
        ref.prefill(prompts)
        out["check"] = split_check(ref.engine, prompts, *check, v0, v1, Bmax, dev)
        del ref
        torch.cuda.empty_cache()
    return out


def time_allreduce(dev, world, rows_list=(1, 8, 64), calls=32):
    """The head split's all-reduce of fp32 residual rows [rows, 4096] alone: NCCL against the
    peer-memory kernel (orch_peer_allreduce; its automatic choice, and its two-shot form
    forced), `calls` dependent calls captured in one CUDA graph, us per call (max over
    ranks), and the bytes each rank sends over NVLink per call (NCCL ring: 2 (world - 1) /
    world of the buffer; the peer kernel a 64-bit word per value: one shot to each other
    rank, two shots 2 (world - 1) / world of the buffer)."""
    import torch
    import torch.distributed as dist

    from orchard_b200.model import _PeerAllReduce
    H = CFG7B["hidden_size"]
    peer = _PeerAllReduce(dist.group.WORLD, world, dist.get_rank(), max(rows_list) * H, dev)
    out = {"calls_per_graph": calls, "peer_self_test": peer.ok}
    x = torch.randn((max(rows_list), H), device=dev) * 1e-3
    for rows in rows_list:
        n = rows * H
        res = {}
        for kind in ("nccl", "peer", "peer_two_shot"):
            if kind != "nccl" and not peer.ok:
                continue

            def one():
                if kind == "nccl":
                    dist.all_reduce(x[:rows], op=dist.ReduceOp.SUM)
                else:
                    peer(x, n, algo=2 if kind == "peer_two_shot" else 0)
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(3):
                    one()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(calls):
                    one()
            g.replay()
            torch.cuda.synchronize(dev)
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize(dev)
            t = torch.tensor([a.elapsed_time(b) / calls * 1000.0], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            one_shot = kind == "peer" and (world <= 2 or 8 * n * (world - 1) <= (1 << 20))
            sent = 8 * n * (world - 1) if one_shot else (16 if kind != "nccl" else 8) * n * (world - 1) / world
            res[kind] = {"us": round(float(t.item()), 2), "sent_bytes": int(sent),
                         "GBps_out": round(sent / (float(t.item()) * 1e-6) / 1e9, 1)}
            del g
        out[str(rows)] = res
    torch.cuda.synchronize(dev)
    return out


class OracleStepSample:
    """The oracle's decode step (the reference's arithmetic restated in NumPy) on the host
    cores, measured in bounded samples: one sample is one of the 32 layers of a batch-B step
    at `L0` cached positions (the GPU arm's mean timed position); the final norm + lm_head
    is timed once. step time = 32 x (mean layer sample) + head. Weights are random codes with
    unit-ish scales (timing does not depend on values), dequantised once and kept (the
    fastest host form of the oracle's GEMMs)."""

    def __init__(self, B: int, L0: int, seed: int = 7):
        import oracle

        self.oracle = oracle
        H, F, V = 4096, 11008, 32000
        g = np.random.default_rng(seed)

        def q(n, k):
            return (g.integers(0, 256, (n, k // 2), dtype=np.uint8), np.full((n, k // 32), 0.01, np.float16))

        layer = oracle.model.OracleLayer(wq=q(H, H), wk=q(H, H), wv=q(H, H), wo=q(H, H), w1=q(F, H), w3=q(F, H),
                                         w2=q(H, F), attn_norm=np.ones(H, np.float32),
                                         ffn_norm=np.ones(H, np.float32))
        cfg = dict(CFG7B, num_hidden_layers=1)
        self.om = oracle.model.OracleModel(cfg, [layer], g.standard_normal((V, H), dtype=np.float32),
                                           np.ones(H, np.float32), q(V, H), cache_dequant=True)
        self.B, self.L0 = B, L0
        for b in range(B):
            self.om.k_cache[0][b] = g.standard_normal((32, L0, 128), dtype=np.float32)
            self.om.v_cache[0][b] = g.standard_normal((32, L0, 128), dtype=np.float32)
        self.x = self.om.embed[np.arange(B) % V]
        self.cos, self.sin = self.om.freqs_cos[[L0] * B], self.om.freqs_sin[[L0] * B]

    def layer(self) -> float:
        t0 = time.perf_counter()
        self.om.layer_forward(0, self.x, self.cos, self.sin, list(range(self.B)))
        t = time.perf_counter() - t0
        for b in range(self.B):  # keep the cache at L0 positions
            self.om.k_cache[0][b] = self.om.k_cache[0][b][:, :self.L0]
            self.om.v_cache[0][b] = self.om.v_cache[0][b][:, :self.L0]
        return t

    def head(self) -> float:
        t0 = time.perf_counter()
        self.om._lin(self.om.lm_head, self.oracle.ops.rmsnorm(self.x, self.om.norm, 1e-5))
        return time.perf_counter() - t0

    @staticmethod
    def cores() -> dict:
        try:
            import threadpoolctl
            blas = max((i.get("num_threads", 1) for i in threadpoolctl.threadpool_info()), default=1)
        except Exception:
            blas = None
        return {"blas_threads": blas, "os_cpu_count": os.cpu_count()}


def timed_positions(steps: int, warmup: int):
    """First warm-up position, first and last timed positions of the GPU arm."""
    start = PROMPT + 3 - warmup if warmup <= 3 else PROMPT
    return start, start + warmup, start + warmup + steps - 1


def cpu_baseline_sample(B, L0, target_s=12.0):
    """cpu_baseline of our arm's line: layer samples for about `target_s` seconds."""
    smp = OracleStepSample(B, L0)
    smp.layer()  # warm (dequantises the weights once)
    head = min(smp.head(), smp.head())
    ts = []
    t_start = time.perf_counter()
    while not ts or time.perf_counter() - t_start < target_s:
        ts.append(smp.layer())
    step_s = 32 * float(np.mean(ts)) + head
    cores = OracleStepSample.cores()
    return {"value": B / step_s, "unit": "tok/s", "cores": int(cores["blas_threads"] or cores["os_cpu_count"] or 1),
            "kind": "port", **cores,
            "sample": f"oracle decode step, batch {B}, {L0} cached positions: {len(ts)} samples of one of the 32 "
                      f"layers ({np.mean(ts) * 1e3:.0f} ms each) x 32 + final norm and lm_head ({head * 1e3:.0f} ms)",
            "step_s": step_s}


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    cfg = dict(CFG7B, num_hidden_layers=args.layers)
    B = args.batch
    extra = [int(b) for b in args.extra_batches.split(",") if b] if (world == 1) else []
    max_b = max([B] + extra)
    llm = build_model(cfg, dev, max_b, seed=1234 + rank)
    eng = llm.engine
    g = np.random.default_rng([20261201, 4, rank])
    prompts = g.integers(0, cfg["vocab_size"], (max_b, PROMPT)).tolist()
    t0 = time.perf_counter()
    llm.prefill(prompts)
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0
    start, first, last = timed_positions(args.steps, args.warmup)
    assert last < MAX_SEQ, "steps + warmup exceed the 640-position decode window"
    # capture the graph before timing
    eng.pos[:B].fill_(PROMPT)
    eng.step(B, logits=True)
    torch.cuda.synchronize(dev)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        secs = time_decode(llm, B, args.steps, args.warmup, start)
    t = torch.tensor([secs], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    secs_max = float(t.item())
    tokens = B * args.steps * world
    value = tokens / secs_max

    # kernel families of one step at the mean timed position; roofline of the dominant one
    mid = first + args.steps // 2
    prof = kernel_profile(llm, B, mid)
    dom = max(("qgemm", "attention"), key=lambda k: prof.get(k, {"ms": 0})["ms"])
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    d = prof[dom]
    achieved = d["bytes"] / (d["ms"] / 1000.0) / 1e9
    step_ms = secs_max / args.steps * 1000.0
    prof_ms = sum(v["ms"] for v in prof.values())
    fam = {k: {"ms": round(v["ms"], 4), "GBps": round(v["bytes"] / (v["ms"] / 1000.0) / 1e9, 1) if v["bytes"] else None,
               "launches": v["launches"]} for k, v in prof.items()}
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": "measured" if peaks else "fallback",
                "traffic": None, "traffic_note": "DRAM bytes of the same kernels from ncu are summarised in profiles/",
                "launches_per_step": d["launches"], "bytes_per_step": d["bytes"],
                "share_of_eager_step": round(d["ms"] / prof_ms, 3), "families": fam}
    step_bytes = sum(v["bytes"] for v in prof.values())
    line = {"metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights x fp16 activations, fp32 accumulate",
            "data": "synthetic (seeded random-init weights N(0,0.02) packed by the reference rule; random prompts)",
            "config": {"workload": f"llama-2-7b-shape INT4 batched decode, batch {B}/GPU, prompt {PROMPT}, "
                                   f"positions {first}..{last}",
                       "model": "llama-2-7b-shape (32 layers, hidden 4096, 32x128 heads, FFN 11008, vocab 32000)",
                       "global_batch": B * world, "seq_len": MAX_SEQ, "parallelism": f"dp{world} (sequence replicas)",
                       "l2": "no flush needed: each step streams 3.7 GB of weights + KV (> 126 MB L2)"},
            "step_hbm_bytes": step_bytes, "step_hbm_frac": round(step_bytes / (step_ms / 1000) / 1e9 / peak, 4),
            "prefill_s": round(prefill_s, 2), "roofline": roofline,
            "gpu_launches": eng.kernel_launches_per_step(B) * args.steps}
    if rank == 0:
        line["clocks"] = clk.summary()
    if args.only_decode:
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    # per-batch lines (N = 1 only)
    if world == 1:
        per = {}
        for b in extra:
            if b == B:
                continue
            eng.pos[:b].fill_(PROMPT)
            eng.step(b, logits=True)
            sb = time_decode(llm, b, args.steps, args.warmup, start)
            per[str(b)] = {"tok_s": round(b * args.steps / sb, 2), "ms_per_step": round(sb / args.steps * 1000, 4)}
        line["per_batch"] = per
    # the column split, measured beside the replicas (N > 1): global batch 64 (with the token
    # check against the unsplit engine and the per-family breakdown), 16 and 1
    if world > 1 and not args.no_column_split:
        del llm, eng
        torch.cuda.empty_cache()
        splits = {}
        for gb in (B, 16, 1):
            if gb != B and (gb in splits or (gb >= world and gb % world)):
                continue
            splits[str(gb)] = time_column_split(cfg, dev, gb, min(args.steps, 32), args.warmup, rank, world,
                                                check_steps=8 if gb == B else 0)
        line["column_split"] = {"note": "FFN and lm_head column-split over NCCL; attention data-parallel "
                                        "(replicated attention weights); two collectives per layer",
                                "by_global_batch": splits}
        try:  # a failure here (the same on every rank) must not cost the line
            hs = time_head_split(cfg, dev, sorted({B, 1}), min(args.steps, 32), args.warmup, world)
            hs["note"] = ("attention heads (Q/K/V rows, O columns, KV cache), FFN and lm_head split over NCCL; "
                          "every rank runs all sequences; two all-reduces of the fp32 residual per layer")
        except Exception as e:
            hs = {"error": repr(e)[:300]}
            torch.cuda.empty_cache()
        line["head_split"] = hs
        try:
            line["allreduce_fp32_rows"] = time_allreduce(dev, world)
        except Exception as e:
            line["allreduce_fp32_rows"] = {"error": repr(e)[:300]}
        llm = build_model(cfg, dev, max_b, seed=1234 + rank)
        eng = llm.engine
        llm.prefill(prompts)
    # end to end through the public API: generate_batch_ids with per-step H2D/D2H; the
    # batch's decode graph is captured before (as at N = 1, where the timing above did it)
    eng.pos[:B].fill_(PROMPT)
    eng.step(B, logits=True)
    torch.cuda.synchronize(dev)
    stats = {}
    e2e_prompts = g.integers(0, cfg["vocab_size"], (B, PROMPT)).tolist()
    llm.generate_batch_ids(e2e_prompts, max_tokens=args.steps, temperature=0, ignore_eos=True, stats=stats)
    tt = torch.tensor([stats["decode_s"]], device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    line["e2e"] = {"value": round(B * stats["steps"] * world / float(tt.item()), 2), "unit": "tok/s",
                   "h2d_bytes_per_step": stats["h2d_bytes_per_step"], "d2h_bytes_per_step": stats["d2h_bytes_per_step"],
                   "api": "Llama.generate_batch_ids (greedy), decode phase; graph captured before timing",
                   "prefill_s": round(stats["prefill_s"], 2)}
    # config 5: 8 sequences x 512 tokens with Q/V LoRA, sequences sharded over the ranks
    seqs = max(1, 8 // world)
    pf = time_prefill_lora(llm, seqs=seqs)
    pt = torch.tensor([pf["s"]], device=dev)
    if world > 1:
        dist.all_reduce(pt, op=dist.ReduceOp.MAX)
    t_pf = float(pt.item())
    peaks_bf16 = float(peaks.get("bf16_tflops", 1590.0))
    flops = pf["flops"] * world
    line["prefill_config5"] = {"workload": f"batched prefill {seqs * world}x512 tokens, LoRA r=16 on Q and V, "
                                           f"{seqs} sequence(s) per GPU",
                               "ms": round(t_pf * 1e3, 3), "tok_s": round(seqs * world * 512 / t_pf, 1),
                               "tflops": round(flops / t_pf / 1e12, 2), "flops": flops,
                               "frac_of_bf16_peak": round(flops / t_pf / 1e12 / (peaks_bf16 * world), 4),
                               "time": "max over ranks, median of 3"}
    if rank == 0 and world == 1:
        from orchard_b200 import kbench
        line["gemv_sweep"] = {"peak_GBps": peak, "cases": kbench.gemv_sweep(reps=30, peak_gbs=peak),
                              "what": "orch_q4t_gemm (INT4 g32, tiled) and orch_gemm_q8_pc (INT8 per channel), "
                                      "fp16 out, graph-timed over weight copies > 4 x L2"}
        line["elementwise_config2"] = kbench.elementwise_config(reps=50)
        if not args.no_cpu_baseline:
            cb = cpu_baseline_sample(B, (first + last) // 2)
            cb.pop("step_s", None)
            line["cpu_baseline"] = cb
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    """The reference arm: the oracle's decode step on the host cores (the reference's compute
    backend is Apple Metal; its CPU path is the NumPy arithmetic restated in oracle/), same
    workload, metric and positions as our arm. Each step is a bounded sample: one of the 32
    layers of the batch's decode step; the value extrapolates 32 layers + the lm_head."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    start, first, last = timed_positions(args.steps, args.warmup)
    L0 = (first + last) // 2
    smp = OracleStepSample(args.batch, L0)
    head = min(smp.head(), smp.head())
    for _ in range(max(1, args.warmup)):
        smp.layer()
    ts = [smp.layer() for _ in range(args.steps)]
    layer_s = float(np.mean(ts))
    step_s = 32 * layer_s + head
    value = args.batch / step_s
    cores = OracleStepSample.cores()
    sample = (f"oracle decode step, batch {args.batch}, {L0} cached positions: {args.steps} timed samples of one of "
              f"the 32 layers ({layer_s * 1e3:.0f} ms each) x 32 + final norm and lm_head ({head * 1e3:.0f} ms)")
    line = {"metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(layer_s * 1000, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, fp32 NumPy arithmetic",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": f"llama-2-7b-shape INT4 batched decode, batch {args.batch}, prompt {PROMPT}, "
                                   f"positions {first}..{last} (sampled at {L0})",
                       "model": "llama-2-7b-shape", "global_batch": args.batch, "seq_len": MAX_SEQ,
                       "parallelism": "host cores"},
            "step_unit": "one of the 32 layers of a decode step (bounded sample); value = batch / (32 x layer + head)",
            "extrapolated_ms_per_step": round(step_s * 1000, 1),
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "kind": "port",
                             "cores": int(cores["blas_threads"] or cores["os_cpu_count"] or 1), **cores,
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's compute backend is Apple Metal (unavailable on this box); its CPU path "
                    "(orchard/model.py with the kernel arithmetic in NumPy) is the oracle port"}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)
