"""Kernel-level timing of the decode path's kernels at the 7B shapes.

    python -m orchard_b200.kbench [--kernel q4|q4t|q8pc|attn|attn_prefill|sweep|elementwise|all]
                                  [--M 1,16,64] [--reps 50]

q4: reference-layout INT4 weights (orch_gemm_q4_0_ex); q4t: tiled INT4 weights (orch_q4t_gemm).

Each INT4/INT8 GEMM shape is timed over enough distinct weight copies that the set
exceeds the 126 MB L2 (so every launch streams its weights from HBM), with CUDA events on
the launching stream after warm-up. Reported GB/s use the algorithmic bytes: packed
weights + scales + activations in + outputs out. One JSON line per case.
"""

from __future__ import annotations

import argparse
import json

import numpy as np

import torch

from . import _lib
from ._lib import F16, F32, call

DECODE_SHAPES = [("qkv", 4096, 12288), ("o", 4096, 4096), ("gate_up", 4096, 22016), ("down", 11008, 4096),
                 ("lm_head", 4096, 32000)]
L2_BYTES = 126 * 1024 * 1024


_SIDE = {}


def _capture_stream() -> torch.cuda.Stream:
    """One capture stream per device for every timed graph (the library keeps per-stream
    workspaces, so a fresh stream per case would allocate a new one each time)."""
    d = torch.cuda.current_device()
    if d not in _SIDE:
        _SIDE[d] = torch.cuda.Stream()
    return _SIDE[d]


def _graph_time(run, n: int, reps: int) -> float:
    """Microseconds per launch: `reps` launches (rotating over `n` inputs) captured in one
    CUDA graph and replayed, so host launch overhead is not measured."""
    for i in range(2 * n):
        run(i)
    torch.cuda.synchronize()
    side = _capture_stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for i in range(reps):
            run(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000 / reps


def _copies(nbytes: int) -> int:
    return max(2, -(-4 * L2_BYTES // nbytes))


def time_q4(M: int, K: int, N: int, reps: int, fmt: str = "q4", out_f16: bool = False):
    dev = "cuda"
    wbytes = N * K // 2 if fmt in ("q4", "q4t") else N * K
    sbytes = N * K // 16 if fmt in ("q4", "q4t") else 2 * N
    n = min(_copies(wbytes + sbytes), 64)
    ws = []
    for i in range(n):
        if fmt in ("q4", "q4t"):
            w = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev)
            s = (torch.rand((N, K // 32), device=dev) * 0.01).half()
            if fmt == "q4t":
                t = torch.empty(_lib.lib().orch_q4t_bytes(N, K), dtype=torch.uint8, device=dev)
                call("orch_q4t_pack", w, s, N, K, t, torch.cuda.current_stream().cuda_stream)
                w, s = t, None
        else:
            w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
            s = (torch.rand(N, device=dev) * 0.01).half()
        ws.append((w, s))
    x = torch.randn((M, K), device=dev).half()
    odt = F16 if out_f16 else F32
    y = torch.empty((M, N), device=dev, dtype=torch.float16 if out_f16 else torch.float32)
    fn = "orch_gemm_q4_0_ex" if fmt == "q4" else "orch_gemm_q8_pc"

    def run(i):
        w, s = ws[i % n]
        if fmt == "q4t":
            call("orch_q4t_gemm", w, x, y, odt, K, N, M, torch.cuda.current_stream().cuda_stream)
        else:
            call(fn, w, s, x, F16, y, odt, K, N, M, torch.cuda.current_stream().cuda_stream)

    us = _graph_time(run, n, reps)
    byts = wbytes + sbytes + 2 * M * K + (2 if out_f16 else 4) * M * N
    return {"kernel": f"qgemm_{fmt}", "M": M, "K": K, "N": N, "us": round(us, 3),
            "GBps": round(byts / us / 1e3, 1), "bytes": byts, "weight_copies": n}


# the INT4 / INT8 GEMV sweep: activation rows x (K, N)
SWEEP_M = (1, 2, 4, 8)
SWEEP_KN = ((4096, 4096), (4096, 11008), (11008, 4096), (4096, 32000))


def gemv_sweep(reps: int = 30, peak_gbs: float = 0.0):
    """INT4 group-32 (tiled device layout, the engine's path) and INT8 per-channel weights,
    fp16 activations N(0,1) scale, fp16 outputs, fp32 accumulation; each case over weight
    copies totalling > 4 x L2. Bytes: N K / 2 + N K / 16 + 2 M K + 2 M N (INT4),
    N K + 2 N + 2 M K + 2 M N (INT8)."""
    out = []
    for fmt in ("q4t", "q8pc"):
        for K, N in SWEEP_KN:
            for M in SWEEP_M:
                r = time_q4(M, K, N, reps, fmt, out_f16=True)
                r["format"] = "int4 g32" if fmt == "q4t" else "int8 per-channel"
                if peak_gbs:
                    r["frac"] = round(r["GBps"] / peak_gbs, 4)
                out.append(r)
                torch.cuda.empty_cache()
    return out


def _rotating(make, nbytes: int, cap: int = 64):
    """Enough independent input copies that one pass over them exceeds L2 (at most `cap`)."""
    n = max(1, min(cap, -(-2 * L2_BYTES // max(nbytes, 1))))
    return [make() for _ in range(n)], n


def elementwise_config(reps: int = 50):
    """Config 2: RMSNorm [B,4096] (gamma N(1,0.1)), RoPE of Q and K [B,32,128] at positions
    U[0,4095], row softmax [B*32, L] (logits N(0,3)), SwiGLU [B,11008] x 2, fp16 in and out,
    B in {1, 8, 64}, L in {128, 1024, 4096}. Launches rotate over input copies (up to 64;
    the small cases stay L2-resident: they measure launch and latency cost)."""
    dev = "cuda"
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    rows = []
    for B in (1, 8, 64):
        gam = (1 + 0.1 * torch.randn(4096, device=dev)).half()
        xs, n = _rotating(lambda: torch.randn((B, 4096), device=dev).half(), 4 * B * 4096)
        y = torch.empty((B, 4096), device=dev, dtype=torch.float16)
        us = _graph_time(lambda i: call("orch_rmsnorm", xs[i % n], gam, y, 1e-5, 4096, B, st()), n, reps)
        byts = 4 * B * 4096 + 8192
        rows.append({"op": "rmsnorm", "B": B, "us": round(us, 3), "GBps": round(byts / us / 1e3, 1), "bytes": byts})

        pos = torch.randint(0, 4096, (B,), device=dev)
        inv = 1.0 / (10000.0 ** (torch.arange(0, 128, 2, device=dev).float() / 128))
        ang = pos.float()[:, None] * inv[None, :]
        cs, sn = torch.cos(ang).half(), torch.sin(ang).half()
        qk, n = _rotating(lambda: (torch.randn((B, 32, 128), device=dev).half(),
                                   torch.randn((B, 32, 128), device=dev).half()), 8 * B * 32 * 128)
        qo, ko = torch.empty_like(qk[0][0]), torch.empty_like(qk[0][1])

        def rope(i):
            q, k = qk[i % n]
            call("orch_rope", q, cs, sn, qo, 128, 32, B, st())
            call("orch_rope", k, cs, sn, ko, 128, 32, B, st())
        us = _graph_time(rope, n, reps)
        byts = 2 * (2 * B * 32 * 128 * 2) + 2 * B * 64 * 2
        rows.append({"op": "rope_q_and_k", "B": B, "us": round(us, 3), "GBps": round(byts / us / 1e3, 1),
                     "bytes": byts, "launches": 2})

        for L in (128, 1024, 4096):
            ls, n = _rotating(lambda: (torch.randn((B * 32, L), device=dev) * 3).half(), 4 * B * 32 * L)
            so = torch.empty((B * 32, L), device=dev, dtype=torch.float16)
            us = _graph_time(lambda i: call("orch_softmax", ls[i % n], so, B * 32, L, st()), n, reps)
            byts = 4 * B * 32 * L
            rows.append({"op": "softmax", "B": B, "L": L, "us": round(us, 3), "GBps": round(byts / us / 1e3, 1),
                         "bytes": byts})

        gu, n = _rotating(lambda: (torch.randn((B, 11008), device=dev).half(),
                                   torch.randn((B, 11008), device=dev).half()), 6 * B * 11008)
        h = torch.empty((B, 11008), device=dev, dtype=torch.float16)
        us = _graph_time(lambda i: call("orch_swiglu_ex", gu[i % n][0], gu[i % n][1], h, F16, B * 11008, st()),
                         n, reps)
        byts = 6 * B * 11008
        rows.append({"op": "swiglu", "B": B, "us": round(us, 3), "GBps": round(byts / us / 1e3, 1), "bytes": byts})
    return rows


def time_attn(M: int, L: int, reps: int, nh: int = 32, hd: int = 128, max_seq: int = 640):
    dev = "cuda"
    n = max(1, min(16, -(-4 * L2_BYTES // (2 * M * nh * max_seq * hd * 2))))
    caches = [(torch.randn((M, nh, max_seq, hd), device=dev).half(), torch.randn((M, nh, max_seq, hd), device=dev).half())
              for _ in range(n)]
    q = torch.randn((M, nh * hd), device=dev).half()
    out = torch.empty_like(q)
    pos = torch.full((M,), L - 1, dtype=torch.int32, device=dev)
    wsb = _lib.lib().orch_attention_workspace_bytes(M, nh, hd, max_seq)
    ws = torch.empty(max(wsb // 4, 1), dtype=torch.float32, device=dev)
    def run(i):
        kc, vc = caches[i % n]
        call("orch_attention_decode", q, kc, vc, pos, None, out, M, nh, hd, max_seq, M, ws, wsb,
             torch.cuda.current_stream().cuda_stream)

    us = _graph_time(run, n, reps)
    byts = 2 * M * nh * L * hd * 2 + 2 * 2 * M * nh * hd
    return {"kernel": "attention_decode", "M": M, "L": L, "us": round(us, 3), "GBps": round(byts / us / 1e3, 1),
            "bytes": byts, "cache_copies": n}


def time_attn_prefill(seqs: int, L: int, reps: int, nh: int = 32, hd: int = 128, max_seq: int = 640):
    """Causal prefill attention (orch_attention_prefill) for `seqs` sequences of L tokens at
    positions 0..L-1: q [seqs*L, nh*hd], K / V caches of `seqs` slots. One copy of the inputs
    (the kernel is tensor-bound; with 8 x 512 tokens q + K + V = 100 MB)."""
    from .model import prefill_units

    dev = "cuda"
    M = seqs * L
    q = torch.randn((M, nh * hd), device=dev).half()
    kc = torch.randn((seqs, nh, max_seq, hd), device=dev).half()
    vc = torch.randn_like(kc)
    units = torch.from_numpy(prefill_units(np.tile(np.arange(L), seqs), np.repeat(np.arange(seqs), L))).to(dev)
    out = torch.empty_like(q)

    def run(i):
        call("orch_attention_prefill", q, kc, vc, units, units.shape[0], out, M, nh, hd, max_seq, kc.shape[0],
             torch.cuda.current_stream().cuda_stream)

    us = _graph_time(run, 1, reps)
    flops = 2 * 2 * seqs * nh * (L * (L + 1) // 2) * hd  # QK^T and PV over the causal pairs
    return {"kernel": "attention_prefill", "seqs": seqs, "L": L, "us": round(us, 3),
            "TFLOPs": round(flops / us / 1e6, 1), "flops": flops}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default="all",
                    choices=["q4", "q4t", "q8pc", "attn", "attn_prefill", "sweep", "elementwise", "all"])
    ap.add_argument("--M", default="1,16,64", help="activation rows (attn_prefill: sequences)")
    ap.add_argument("--L", type=int, default=512, help="attn_prefill: tokens per sequence")
    ap.add_argument("--shape", default="", help="only this decode shape name (qkv, o, gate_up, down, lm_head)")
    ap.add_argument("--shapes", default="", help="extra GEMM shapes K:N,K:N,... (timed instead of the decode shapes)")
    ap.add_argument("--reps", type=int, default=50)
    a = ap.parse_args()
    call("orch_init", 0, None)
    if a.kernel == "sweep":
        for r in gemv_sweep(a.reps):
            print(json.dumps(r), flush=True)
        return
    if a.kernel == "elementwise":
        for r in elementwise_config(a.reps):
            print(json.dumps(r), flush=True)
        return
    Ms = [int(v) for v in a.M.split(",")]
    for M in Ms:
        if a.kernel in ("q4", "q4t", "q8pc", "all"):
            shapes = DECODE_SHAPES
            if a.shapes:
                shapes = [(f"{k}x{n}", int(k), int(n)) for k, n in (v.split(":") for v in a.shapes.split(","))]
            for name, K, N in shapes:
                if a.shape and name != a.shape:
                    continue
                for fmt in (("q4t", "q4", "q8pc") if a.kernel == "all" else (a.kernel,)):
                    r = time_q4(M, K, N, a.reps, fmt)
                    r["shape"] = name
                    print(json.dumps(r), flush=True)
        if a.kernel in ("attn", "all"):
            print(json.dumps(time_attn(M, 577, a.reps)), flush=True)
        if a.kernel == "attn_prefill":
            print(json.dumps(time_attn_prefill(M, a.L, a.reps)), flush=True)


if __name__ == "__main__":
    main()
