"""Llama decode on B200: the reference's Python API over the fused sm_100a kernels.

Reference API: ``orchard.Llama(model_path)``, ``load_lora``, ``generate_batch(prompts,
max_tokens=50, temperature=0.7)`` (orchard/model.py:197-381). Arithmetic follows
``LlamaLayer.forward`` (orchard/model.py:78-195); the per-layer sequence of the
reference's ~14 synchronous ops plus host attention becomes seven launches:

  1. RMSNorm (fp32 residual -> fp16)                          rmsnorm.metal
  2. Q/K/V INT4 projection + LoRA + RoPE + KV-cache append     model.py:94-124
  3. attention over the device KV cache (+ a combine launch when positions are split)
                                                               model.py:117-137
  4. O INT4 projection + LoRA + residual add                   model.py:147-157
  5. RMSNorm, gate/up INT4 projection + LoRA + SwiGLU, down projection + residual
     (three launches)                                          model.py:160-193

At 1-8 rows, on projections without a LoRA term, each RMSNorm is folded into the GEMV that
follows it (the GEMV normalises the fp32 residual itself), leaving five. Then come the final
RMSNorm, the INT4 lm_head and a row argmax. A whole decode step for a batch size is
captured once in a CUDA graph and replayed.

Token flow of ``generate_batch`` is the reference's: prompts are prefilled one position
at a time (all sequences of the batch together), the last prompt token is fed again as
the first decode input at position ``len(prompt)`` (orchard/model.py:305,325-329), the
next token is the argmax for temperature 0 and ``np.random.choice`` over
``softmax(logits / T)`` otherwise (orchard/model.py:244-252), and id 2 ends a row.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import F16, F32, call, ptr
from .loader import Checkpoint, from_tensors, load_checkpoint, load_lora
from .parallel import (ColumnSplit, attention_head_split, ffn_column_split, ffn_head_split, head_column_split,
                       vocab_head_split)

EOS_ID = 2


@dataclass
class LlamaConfig:
    hidden_size: int
    num_attention_heads: int
    intermediate_size: int
    num_hidden_layers: int
    vocab_size: int
    rms_norm_eps: float = 1e-5
    max_position_embeddings: int = 2048
    rope_theta: float = 10000.0

    @classmethod
    def from_dict(cls, d: dict) -> "LlamaConfig":
        return cls(hidden_size=d["hidden_size"], num_attention_heads=d["num_attention_heads"],
                   intermediate_size=d["intermediate_size"],
                   num_hidden_layers=d["num_hidden_layers"], vocab_size=d["vocab_size"],
                   rms_norm_eps=d.get("rms_norm_eps", 1e-5),
                   max_position_embeddings=d.get("max_position_embeddings", 2048),
                   rope_theta=d.get("rope_theta", 10000.0))

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


def precompute_freqs_cis(dim: int, end: int, theta: float = 10000.0):
    """float32 cos/sin tables ``[end, dim/2]`` computed exactly as orchard/model.py:7-13."""
    inv = 1.0 / (theta ** (np.arange(0, dim, 2)[: dim // 2].astype(np.float32) / dim))
    ang = np.outer(np.arange(end).astype(np.float32), inv)
    return np.cos(ang), np.sin(ang)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


# --------------------------------------------------------------------------------------
# device weights
# --------------------------------------------------------------------------------------

def quantize_on_device(w, device) -> tuple:
    """Reference INT4 packing (orchard/quantizer.py:3-78) on the GPU: returns
    ``(packed uint8 [N, K/2], scales fp16 [N, K/32])`` device tensors, bit-identical to
    the host packer for fp32 input or fp16 input cast to fp32 (the loader's cast)."""
    t = torch.as_tensor(w).to(device)
    if t.dtype not in (torch.float16, torch.float32):
        t = t.float()
    t = t.contiguous()
    n, k = t.shape
    packed = torch.empty((n, k // 2), dtype=torch.uint8, device=device)
    scales = torch.empty((n, k // 32), dtype=torch.float16, device=device)
    call("orch_quantize_q4_0", ptr(t), F16 if t.dtype == torch.float16 else F32, ptr(packed),
         ptr(scales), n, k, _stream())
    return packed, scales


def _as_device(a, device, np_dtype=None) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device).contiguous()
    a = np.ascontiguousarray(a)
    if np_dtype is not None:
        a = a.view(np_dtype) if a.dtype.itemsize == np.dtype(np_dtype).itemsize else a.astype(np_dtype)
    return torch.as_tensor(a).to(device)


def _packed_on_device(entry, device) -> tuple:
    """A checkpoint entry -> (packed, scales) device tensors. Entries are
    ("packed", packed, scales) -- host arrays or device tensors -- or ("dense", weight)."""
    if entry[0] == "packed":
        p = _as_device(entry[1], device, np.uint8)
        s = _as_device(entry[2], device, np.float16)
        if p.dtype != torch.uint8:
            p = p.view(torch.uint8)
        return p, s.to(torch.float16)
    return quantize_on_device(entry[1], device)


def interleave_gate_up(p1, s1, p3, s3):
    """Rows of gate (w1) and up (w3) interleaved in blocks of 16: rows 32b..32b+15 = gate
    16b..16b+15, rows 32b+16..32b+31 = up 16b..16b+15 (the SwiGLU epilogue's layout)."""
    F = p1.shape[0]
    assert F % 16 == 0 and p3.shape[0] == F

    def il(a, b):
        return torch.stack([a.view(F // 16, 16, -1), b.view(F // 16, 16, -1)], dim=1).reshape(2 * F, -1)

    return il(p1, p3).contiguous(), il(s1, s3).contiguous()


def prefill_units(positions, slots, max_rows: int = 64) -> np.ndarray:
    """Work units of orch_attention_prefill for the rows of a prefill chunk: runs of
    consecutive rows in one cache slot at consecutive positions, cut into pieces of at most
    `max_rows`; one int32 record (row0, rows, slot, pos0) each."""
    pos = np.asarray(positions, np.int64)
    sl = np.asarray(slots, np.int64)
    n = len(pos)
    if n == 0:
        return np.zeros((0, 4), np.int32)
    brk = np.ones(n, bool)
    brk[1:] = (sl[1:] != sl[:-1]) | (pos[1:] != pos[:-1] + 1)
    starts = np.flatnonzero(brk)
    ends = np.append(starts[1:], n)
    out = []
    for a, e in zip(starts.tolist(), ends.tolist()):
        for r in range(a, e, max_rows):
            out.append((r, min(max_rows, e - r), sl[r], pos[r]))
    return np.asarray(out, np.int32).reshape(-1, 4)


def tile_q4(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """Re-lays a packed INT4 weight (reference layout, on the device) into the tiled layout
    the tensor-core GEMM streams (rows in tiles of 128, k in blocks of 256, each block one
    contiguous run of nibbles and scales; see include/orchard_b200.h)."""
    N, K = w.shape[0], w.shape[1] * 2
    t = torch.empty(_lib.lib().orch_q4t_bytes(N, K), dtype=torch.uint8, device=w.device)
    call("orch_q4t_pack", ptr(w), ptr(s), N, K, ptr(t), _stream())
    return t


class DeviceLayer:
    """One layer's device weights: fused [Wq;Wk;Wv], Wo, gate/up interleaved, Wdown, either in
    the tiled layout (`tiled`, the default: tcgen05 GEMM for every row count) or in the
    reference layout (mma.sync GEMV below the tensor-core threshold)."""

    def __init__(self, entries: dict, cfg: LlamaConfig, device, tiled: bool = True,
                 split: Optional[ColumnSplit] = None):
        H, F = cfg.hidden_size, cfg.intermediate_size
        q = {n: _packed_on_device(entries[n], device) for n in ("wq", "wk", "wv", "wo", "w1", "w3", "w2")}
        if split is not None:  # this rank's FFN columns: gate/up rows f0:f1, down columns f0:f1
            w1, s1, w3, s3, w2, s2 = split.ffn_shard(*q["w1"], *q["w3"], *q["w2"])
            q["w1"], q["w3"], q["w2"] = (w1, s1), (w3, s3), (w2.contiguous(), s2.contiguous())
            F = split.f_local
        Ha = H  # width of this rank's Q (= K = V) rows and of the O projection's K
        if split is not None and split.heads:  # this rank's heads: Q/K/V rows, O columns
            wq, sq, wk, sk, wv, sv, wo, so = split.attn_shard(*q["wq"], *q["wk"], *q["wv"], *q["wo"], cfg.head_dim)
            q["wq"], q["wk"], q["wv"] = (wq, sq), (wk, sk), (wv, sv)
            q["wo"] = (wo.contiguous(), so.contiguous())
            Ha = split.h_local * cfg.head_dim
        self.wqkv = torch.cat([q["wq"][0], q["wk"][0], q["wv"][0]]).contiguous()
        self.sqkv = torch.cat([q["wq"][1], q["wk"][1], q["wv"][1]]).contiguous()
        self.wo, self.so = q["wo"]
        self.w13, self.s13 = interleave_gate_up(q["w1"][0], q["w1"][1], q["w3"][0], q["w3"][1])
        self.w2, self.s2 = q["w2"]
        del q
        self.attn_norm = torch.as_tensor(np.asarray(entries["attn_norm"], np.float32)).to(device)
        self.ffn_norm = torch.as_tensor(np.asarray(entries["ffn_norm"], np.float32)).to(device)
        assert self.wqkv.shape == (3 * Ha, H // 2) and self.w13.shape == (2 * F, H // 2)
        assert self.w2.shape == (H, F // 2) and self.wo.shape == (H, Ha // 2)
        self.f_local = F
        self.h_attn = Ha
        self.tiled = tiled
        if tiled:
            self.tqkv = tile_q4(self.wqkv, self.sqkv)
            self.to = tile_q4(self.wo, self.so)
            self.t13 = tile_q4(self.w13, self.s13)
            self.t2 = tile_q4(self.w2, self.s2)
            torch.cuda.current_stream().synchronize()
            self.wqkv = self.sqkv = self.wo = self.so = self.w13 = self.s13 = self.w2 = self.s2 = None
        self.lora: Dict[str, tuple] = {}

    def weight_bytes(self) -> int:
        ts = (self.tqkv, self.to, self.t13, self.t2) if self.tiled else \
            (self.wqkv, self.sqkv, self.wo, self.so, self.w13, self.s13, self.w2, self.s2)
        return sum(t.numel() * t.element_size() for t in ts)

    def set_lora(self, mods: Dict[str, tuple], cfg: LlamaConfig, r: int, device):
        """Packs adapters per fused projection: A_cat [K, R*r] and B_cat [R, r, width]."""
        H, F = cfg.hidden_size, cfg.intermediate_size
        groups = {"qkv": (("wq", "wk", "wv"), H, H), "o": (("wo",), H, H),
                  "gu": (("w1", "w3"), H, F), "down": (("w2",), F, H)}
        self.lora = {}
        for g, (names, k_in, width) in groups.items():
            if not any(n in mods for n in names):
                continue
            R = len(names)
            a = np.zeros((k_in, R * r), np.float32)
            b = np.zeros((R, r, width), np.float32)
            for i, n in enumerate(names):
                if n in mods:
                    A, Bm = mods[n]
                    a[:, i * r:(i + 1) * r] = A
                    b[i] = Bm
            self.lora[g] = (torch.as_tensor(a).to(device), torch.as_tensor(b).to(device), R)


# --------------------------------------------------------------------------------------
# engine
# --------------------------------------------------------------------------------------

class RowBuffers:
    """Activation buffers for up to `rows` token rows: fp32 residual, fp16 GEMM inputs and
    outputs, per-row token / position / cache slot, LoRA x.A rows and the attention
    workspace."""

    def __init__(self, rows: int, cfg: "LlamaConfig", max_seq: int, device, logits: bool, heads: int = 0):
        H, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
        nh, hd = cfg.num_attention_heads, cfg.head_dim
        self.rows = rows
        self.x = torch.zeros((rows, H), dtype=torch.float32, device=device)
        self.xn = torch.zeros((rows, H), dtype=torch.float16, device=device)
        self.q = torch.zeros((rows, H), dtype=torch.float16, device=device)
        self.attn = torch.zeros((rows, H), dtype=torch.float16, device=device)
        self.h = torch.zeros((rows, F), dtype=torch.float16, device=device)
        self.logits = torch.zeros((rows, V), dtype=torch.float32, device=device) if logits else None
        self.tok_in = torch.zeros(rows, dtype=torch.int32, device=device)
        self.tok_out = torch.zeros(rows, dtype=torch.int32, device=device)
        self.pos = torch.zeros(rows, dtype=torch.int32, device=device)
        self.slots = torch.arange(rows, dtype=torch.int32, device=device)
        self.uniforms = torch.full((rows,), 0.5, dtype=torch.float32, device=device)  # sampler draws
        self.lora_t = torch.zeros((rows, 3 * 64), dtype=torch.float32, device=device)
        lib = _lib.lib()
        ms = list(range(1, min(rows, 256) + 1)) + [rows]  # splits only happen for few rows
        # a rank of the head split runs fewer heads per row (its split count may differ)
        ws = max(lib.orch_attention_workspace_bytes(m, h, hd, max_seq) for m in ms for h in {nh, heads or nh})
        self.attn_ws = torch.zeros(max(ws, 16) // 4 + 1, dtype=torch.float32, device=device)
        self.attn_ws_bytes = ws


class _SplitBuffers:
    """Buffers of the column-split FFN and head for up to ``rb.rows`` local rows: the
    gathered rows of every rank (rank-major), this rank's FFN slice of them, the fp32
    partial down projection and its reduced local rows, the vocabulary slice's logits and
    the (max, id) pairs."""

    def __init__(self, rb: RowBuffers, split: ColumnSplit, cfg: "LlamaConfig", device):
        H = cfg.hidden_size
        W, R = split.world, rb.rows
        self.x, self.xn, self.tok = rb.x, rb.xn, rb.tok_out
        self.xn_all = torch.zeros((W * R, H), dtype=torch.float16, device=device)
        self.h = torch.zeros((W * R, split.f_local), dtype=torch.float16, device=device)
        self.part = torch.zeros((W * R, H), dtype=torch.float32, device=device)
        self.red = torch.zeros((R, H), dtype=torch.float32, device=device)
        self.logits = torch.zeros((W * R, split.v_local), dtype=torch.float32, device=device)
        self.pairs = torch.zeros((W * R, 2), dtype=torch.float32, device=device)
        self.pairs_all = torch.zeros((W * W * R, 2), dtype=torch.float32, device=device)


class _HeadSplitBuffers:
    """Buffers of the head split's lm_head for up to ``rb.rows`` rows (every rank holds all
    rows): the vocabulary slice's logits, this rank's (max, id) pairs and every rank's."""

    def __init__(self, rb: RowBuffers, split: ColumnSplit, device):
        R = rb.rows
        self.x, self.xn, self.tok = rb.x, rb.xn, rb.tok_out
        self.logits = torch.zeros((R, split.v_local), dtype=torch.float32, device=device)
        self.pairs = torch.zeros((R, 2), dtype=torch.float32, device=device)
        self.pairs_all = torch.zeros((split.world * R, 2), dtype=torch.float32, device=device)


class _LayerCtx:
    """What the head split's ops need of one layer: its weights, its slice of the KV cache
    and, for a prefill chunk, the attention work units."""

    def __init__(self, layer: "DeviceLayer", kc: torch.Tensor, vc: torch.Tensor, units: Optional[torch.Tensor]):
        self.L, self.kc, self.vc, self.units = layer, kc, vc, units


class _CudaSplitOps:
    """The column split's and the head split's kernels on this rank (parallel.py names the
    order)."""

    def __init__(self, eng: "DecodeEngine"):
        self.e = eng

    # -- head split (all rows on every rank, RowBuffers b) --------------------------------
    def qkv_local(self, ctx, b, rows):
        e, L, c = self.e, ctx.L, self.e.cfg
        call("orch_q4t_rms_qkv_rope", ptr(L.tqkv), ptr(b.x), ptr(L.attn_norm), c.rms_norm_eps, ptr(b.xn), rows,
             c.hidden_size, L.h_attn, e.nh_local, ptr(b.pos), ptr(b.slots), ptr(e.cos), ptr(e.sin), e.max_pos,
             ptr(b.q), ptr(ctx.kc), ptr(ctx.vc), e.max_seq, e.num_slots, _stream())

    def attention_local(self, ctx, b, rows):
        e, hd = self.e, self.e.cfg.head_dim
        if ctx.units is not None:
            call("orch_attention_prefill", ptr(b.q), ptr(ctx.kc), ptr(ctx.vc), ptr(ctx.units), ctx.units.shape[0],
                 ptr(b.attn), rows, e.nh_local, hd, e.max_seq, e.num_slots, _stream())
        else:
            call("orch_attention_decode", ptr(b.q), ptr(ctx.kc), ptr(ctx.vc), ptr(b.pos), ptr(b.slots),
                 ptr(b.attn), rows, e.nh_local, hd, e.max_seq, e.num_slots, ptr(b.attn_ws), b.attn_ws_bytes,
                 _stream())

    def o_partial(self, ctx, b, rows, resid):
        L, H = ctx.L, self.e.cfg.hidden_size
        if resid:
            call("orch_q4t_linear_resid", ptr(L.to), ptr(b.attn), ptr(b.x), rows, L.h_attn, H, None, None, 0,
                 _stream())
        else:
            call("orch_q4t_gemm", ptr(L.to), ptr(b.attn), ptr(b.x), F32, L.h_attn, H, rows, _stream())

    def gate_up_local(self, ctx, b, rows):
        L, c = ctx.L, self.e.cfg
        call("orch_q4t_rms_linear_swiglu", ptr(L.t13), ptr(b.x), ptr(L.ffn_norm), c.rms_norm_eps, ptr(b.xn),
             ptr(b.h), rows, c.hidden_size, L.f_local, _stream())

    def down_partial_resid(self, ctx, b, rows, resid):
        L, H = ctx.L, self.e.cfg.hidden_size
        if resid:
            call("orch_q4t_linear_resid", ptr(L.t2), ptr(b.h), ptr(b.x), rows, L.f_local, H, None, None, 0,
                 _stream())
        else:
            call("orch_q4t_gemm", ptr(L.t2), ptr(b.h), ptr(b.x), F32, L.f_local, H, rows, _stream())

    def merge_all_pairs(self, pairs_all, tok, rows):
        call("orch_argmax_merge", ptr(pairs_all), self.e.split.world, rows, 0, rows, ptr(tok), _stream())

    # -- column split and shared -----------------------------------------------------------

    def rmsnorm(self, x, w, xn, rows):
        c = self.e.cfg
        call("orch_rmsnorm_ex", ptr(x), F32, ptr(self.e.norm if w is None else w), F32, ptr(xn), F16,
             c.rms_norm_eps, c.hidden_size, rows, _stream())

    def gate_up_swiglu(self, layer, xn_all, h, rows):
        call("orch_q4t_linear_swiglu", ptr(layer.t13), ptr(xn_all), ptr(h), rows, self.e.cfg.hidden_size,
             layer.f_local, None, None, 0, _stream())

    def down_partial(self, layer, h, part, rows):
        call("orch_q4t_gemm", ptr(layer.t2), ptr(h), ptr(part), F32, layer.f_local, self.e.cfg.hidden_size, rows,
             _stream())

    def add(self, x, red, rows):
        call("orch_binary_ex", 0, ptr(x), ptr(red), ptr(x), F32, rows * self.e.cfg.hidden_size, _stream())

    def lm_partial(self, xn_all, logits, rows):
        sp = self.e.split
        call("orch_q4t_gemm", ptr(self.e.lm_t), ptr(xn_all), ptr(logits), F32, self.e.cfg.hidden_size, sp.v_local,
             rows, _stream())

    def argmax_pairs(self, logits, pairs, rows):
        sp = self.e.split
        call("orch_argmax_pairs", ptr(logits), rows, sp.v_local, sp.v0, ptr(pairs), _stream())

    def merge_pairs(self, pairs_all, tok, rows):
        sp = self.e.split
        call("orch_argmax_merge", ptr(pairs_all), sp.world, sp.world * rows, sp.rank * rows, rows, ptr(tok),
             _stream())


class _PeerAllReduce:
    """The head split's all-reduce of fp32 rows through peer memory (orch_peer_allreduce):
    this rank's region (up to ``max_floats`` floats per rank and bank) allocated and zeroed
    here, exported by CUDA IPC, every other rank's region opened; a collective makes sure no
    rank writes into a region before it is zeroed. ``ok`` is False on every rank when any
    rank could not map a region or got a wrong known sum. The regions stay mapped for the
    life of the process."""

    def __init__(self, group, world: int, rank: int, max_floats: int, device):
        import ctypes as C

        import torch.distributed as dist
        lib = _lib.lib()
        self.world, self.rank, self.max_floats = world, rank, max_floats
        nbytes = lib.orch_peer_region_bytes(world, max_floats)
        if nbytes == 0:
            raise ValueError(f"no peer all-reduce for {world} ranks")
        base = C.c_void_p()
        call("orch_alloc", nbytes, C.byref(base))
        call("orch_memset", base.value, 0, nbytes, None)
        handle = (C.c_uint8 * 64)()
        call("orch_ipc_handle", base.value, C.addressof(handle))
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        every = torch.empty(world * 64, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().numpy()
        bases = []
        opened = True
        try:
            for q in range(world):
                if q == rank:
                    bases.append(base.value)
                    continue
                h = (C.c_uint8 * 64)(*every[q * 64:(q + 1) * 64].tolist())
                peer = C.c_void_p()
                call("orch_ipc_open", C.addressof(h), C.byref(peer))
                bases.append(peer.value)
        except _lib.OrchardError:
            opened = False
        self._bases = (C.c_void_p * world)(*(bases if opened else [None] * world))
        self.bases_addr = C.addressof(self._bases)
        torch.cuda.synchronize(device)
        # every rank mapped every region (or all of them give up), and none writes into a
        # region before it is zeroed
        ok = torch.tensor([1 if opened else 0], dtype=torch.int32, device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        self.ok = bool(ok.item())
        if not self.ok:
            return
        # known sums over every rank; the ranks agree on the outcome, and on a failure they
        # all keep the library collective
        ok.fill_(1 if self._self_test(device) else 0)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        self.ok = bool(ok.item())

    def _self_test(self, device) -> bool:
        """Known sums at the largest size and at one row, twice each (both banks of slots):
        the algorithms the automatic choice takes at this world size."""
        import ctypes as C
        good = True
        for n in (self.max_floats - self.max_floats % 4, min(4096, self.max_floats) // 4 * 4):
            pattern = (1 + torch.arange(n, device=device) % 7).float()
            want = pattern * (self.world * (self.world + 1) // 2)
            for _ in range(2):
                x = pattern * (self.rank + 1)
                self(x, n)
                torch.cuda.synchronize(device)
                good = good and bool(torch.equal(x, want))
        flags = C.c_uint32(0)
        call("orch_device_check", C.byref(flags), _stream())
        return good and (flags.value & 512) == 0

    def __call__(self, x, n: int, algo: int = 0):
        call("orch_peer_allreduce", self.bases_addr, self.rank, self.world, self.max_floats, ptr(x), n, algo,
             _stream())


class _NcclComm:
    """Collectives of the column split over a torch.distributed (NCCL) group; buffers are
    row-major, the first ``rows`` rows of the input and ``world * rows`` of the output. The
    head split's all-reduce of the residual goes through peer memory (``peer``) when its
    rows fit the regions, through NCCL otherwise (prefill chunks)."""

    def __init__(self, group, world: int, rank: int, peer: Optional[_PeerAllReduce] = None):
        self.group, self.world, self.rank = group, world, rank
        self.peer = peer

    def all_reduce(self, x, rows):
        n = rows * x.shape[1]
        if self.peer is not None and n <= self.peer.max_floats:
            self.peer(x, n)
            return
        import torch.distributed as dist
        dist.all_reduce(x[:rows], op=dist.ReduceOp.SUM, group=self.group)

    def all_gather(self, out, inp, rows):
        import torch.distributed as dist
        dist.all_gather_into_tensor(out[:self.world * rows], inp[:rows], group=self.group)

    def reduce_scatter(self, out, inp, rows):
        import torch.distributed as dist
        dist.reduce_scatter_tensor(out[:rows], inp[:self.world * rows], op=dist.ReduceOp.SUM, group=self.group)


class DecodeEngine:
    """Device state for up to ``max_batch`` sequences of up to ``max_seq`` positions.
    With ``group`` (a torch.distributed NCCL group of several ranks, one GPU each) the
    sequences are sharded over the ranks and the FFN and vocabulary projections are split
    by columns (parallel.py); ``M`` then counts this rank's rows, equal on every rank.
    With ``group`` and ``split_heads`` every rank runs the same rows (the same prompts and
    tokens on every rank) and holds a slice of the attention heads (their Q/K/V/O weights
    and KV cache) beside its FFN and vocabulary columns; ``M`` counts all rows."""

    def __init__(self, ck: Checkpoint, device=0, max_batch: int = 32, max_seq: Optional[int] = None,
                 tiled: bool = True, group=None, split_heads: bool = False):
        if not torch.cuda.is_available():
            raise RuntimeError("orchard_b200 needs a CUDA device (there is no CPU fallback)")
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        torch.cuda.set_device(self.device)
        call("orch_init", self.device.index or 0, None)
        self.cfg = cfg = LlamaConfig.from_dict(ck.config)
        if not ck.complete():
            raise ValueError("checkpoint is missing tensors")
        H, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
        self.max_batch = max_batch
        self.max_seq = max_seq or cfg.max_position_embeddings
        self.max_pos = max(self.max_seq, cfg.max_position_embeddings)
        dev = self.device
        self.tiled = tiled
        # column split over the ranks of `group` (torch.distributed, NCCL): sequences sharded,
        # FFN and vocabulary projections split by columns (parallel.py)
        self.group = group
        self.split: Optional[ColumnSplit] = None
        if group is not None:
            import torch.distributed as dist
            world, rank = dist.get_world_size(group), dist.get_rank(group)
            if world > 1:
                if not tiled:
                    raise ValueError("the column split runs on tiled weights")
                if split_heads:
                    self.split = ColumnSplit.plan(F, V, world, rank, cfg.num_attention_heads, cfg.head_dim)
                else:
                    self.split = ColumnSplit.plan(F, V, world, rank)
        self.layers = [DeviceLayer(e, cfg, dev, tiled, self.split) for e in ck.layers]
        emb = ck.embed if isinstance(ck.embed, torch.Tensor) else torch.as_tensor(np.asarray(ck.embed))
        if emb.dtype not in (torch.float16, torch.float32):
            emb = emb.float()
        self.embed = emb.to(dev).contiguous()
        self.norm = torch.as_tensor(np.asarray(ck.norm, np.float32)).to(dev)
        self.lm_w, self.lm_s = _packed_on_device(ck.lm_head, dev)
        if self.split is not None:
            w, sc = self.split.lm_shard(self.lm_w, self.lm_s)
            self.lm_w, self.lm_s = w.contiguous(), sc.contiguous()
        if tiled:
            self.lm_t = tile_q4(self.lm_w, self.lm_s)
            torch.cuda.current_stream().synchronize()
            self.lm_w = self.lm_s = None
        cos, sin = precompute_freqs_cis(cfg.head_dim, self.max_pos, cfg.rope_theta)
        self.cos = torch.as_tensor(cos).to(dev)
        self.sin = torch.as_tensor(sin).to(dev)
        nl, nh, hd = cfg.num_hidden_layers, cfg.num_attention_heads, cfg.head_dim
        self.heads_split = self.split is not None and self.split.heads
        self.peer_allreduce = False  # the head split's all-reduces through peer memory
        self.nh_local = self.split.h_local if self.heads_split else nh  # heads in this rank's cache
        # with the column split one extra slot takes the padding rows of a prefill whose
        # token count is below another rank's (their K/V land there and are never read)
        self.columns_split = self.split is not None and not self.heads_split
        self.scratch_slot = max_batch if self.columns_split else -1
        # prefill attention on the tensor-core kernel (head_dim 128); False: the decode kernel
        # per row (ORCHARD_PREFILL_ATTN=decode)
        self.prefill_attention = os.environ.get("ORCHARD_PREFILL_ATTN", "tc") != "decode"
        nslots = max_batch + (1 if self.columns_split else 0)
        self.num_slots = nslots
        self.k_cache = torch.zeros((nl, nslots, self.nh_local, self.max_seq, hd), dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.lora_r = 0
        self.dec = RowBuffers(max_batch, cfg, self.max_seq, dev, logits=self.split is None, heads=self.nh_local)
        self.pre: Optional[RowBuffers] = None
        self.sdec = None
        if self.heads_split:
            self.sdec = _HeadSplitBuffers(self.dec, self.split, dev)
        elif self.split is not None:
            self.sdec = _SplitBuffers(self.dec, self.split, cfg, dev)
        self.spre: Optional[_SplitBuffers] = None
        if self.split is not None:
            self._split_ops = _CudaSplitOps(self)
            peer = None
            # the head split's all-reduces of decode rows through peer memory (on two GPUs
            # 4.8 / 5.2 / 9.5 us per call at 1 / 8 / 64 rows against NCCL's 15.2 / 16.8 / 19.9;
            # on more GPUs the larger rows take the kernel's two-shot form); prefill chunks take
            # NCCL. ORCHARD_PEER_ALLREDUCE=0: NCCL for every size
            if self.heads_split and os.environ.get("ORCHARD_PEER_ALLREDUCE", "1") != "0":
                peer = _PeerAllReduce(group, self.split.world, self.split.rank, max_batch * H, dev)
                if not peer.ok:
                    import warnings
                    warnings.warn("peer-memory all-reduce failed its self-test; the head split uses NCCL")
                    peer = None
            self.peer_allreduce = peer is not None
            self._comm = _NcclComm(group, self.split.world, self.split.rank, peer)
        self.graphs: Dict[tuple, torch.cuda.CUDAGraph] = {}
        torch.cuda.synchronize(dev)

    # decode buffers, by name
    x = property(lambda self: self.dec.x)
    xn = property(lambda self: self.dec.xn)
    logits = property(lambda self: self.dec.logits)
    tok_in = property(lambda self: self.dec.tok_in)
    tok_out = property(lambda self: self.dec.tok_out)
    pos = property(lambda self: self.dec.pos)
    slots = property(lambda self: self.dec.slots)

    # -- lora --------------------------------------------------------------------------
    def set_lora(self, per_layer: Dict[int, Dict[str, tuple]], r: int):
        if r > 64:
            raise ValueError("LoRA rank above 64 is not supported by the fused epilogues")
        if self.heads_split and any(per_layer.values()):
            raise ValueError("LoRA adapters are not supported with the head split")
        for li, layer in enumerate(self.layers):
            layer.set_lora(per_layer.get(li, {}), self.cfg, r, self.device)
        self.lora_r = r
        self.graphs.clear()

    def _lora(self, layer, g, x, M, s, bufs):
        if g not in layer.lora:
            return None, None, 0
        a, b, R = layer.lora[g]
        K = a.shape[0]
        call("orch_lora_xa", ptr(x), ptr(a), ptr(bufs.lora_t), M, K, R * self.lora_r, s)
        return ptr(bufs.lora_t), ptr(b), self.lora_r

    # -- one step ----------------------------------------------------------------------
    def run_layers(self, M: int, bufs: Optional[RowBuffers] = None, units: Optional[torch.Tensor] = None):
        """All layers for rows [0, M) of `bufs` (default: the decode buffers): token ids in
        tok_in, positions in pos, cache slots in slots. `units` (prefill: a device copy of
        prefill_units for these rows) routes attention to the tensor-core prefill kernel,
        which reads each sequence's keys once per 64 rows instead of once per row."""
        b = bufs if bufs is not None else self.dec
        cfg = self.cfg
        call("orch_embed_rows", ptr(b.tok_in), ptr(self.embed), F16 if self.embed.dtype == torch.float16 else F32,
             ptr(b.x), M, cfg.hidden_size, cfg.vocab_size, _stream())
        for li in range(len(self.layers)):
            self.run_layer(li, M, b, units)

    def run_layer(self, li: int, M: int, bufs: Optional[RowBuffers] = None, units: Optional[torch.Tensor] = None):
        """Layer `li` (LlamaLayer.forward, orchard/model.py:78-195) on the fp32 residual rows
        [0, M) of `bufs`.x in place, at the rows' positions and cache slots."""
        b = bufs if bufs is not None else self.dec
        cfg, s = self.cfg, _stream()
        H, F = cfg.hidden_size, cfg.intermediate_size
        nh, hd, eps = cfg.num_attention_heads, cfg.head_dim, cfg.rms_norm_eps
        L = self.layers[li]
        kc, vc = self.k_cache[li], self.v_cache[li]
        if self.heads_split:  # all rows here, this rank's heads and FFN columns (parallel.py)
            ctx = _LayerCtx(L, kc, vc, units)
            attention_head_split(self._split_ops, self._comm, ctx, b, M)
            ffn_head_split(self._split_ops, self._comm, ctx, b, M)
            return
        if L.tiled and "qkv" not in L.lora:
            # RMSNorm fused in front of the projection (one launch for up to 8 rows)
            call("orch_q4t_rms_qkv_rope", ptr(L.tqkv), ptr(b.x), ptr(L.attn_norm), eps, ptr(b.xn), M, H, H, nh,
                 ptr(b.pos), ptr(b.slots), ptr(self.cos), ptr(self.sin), self.max_pos, ptr(b.q), ptr(kc), ptr(vc),
                 self.max_seq, self.num_slots, s)
        else:
            call("orch_rmsnorm_ex", ptr(b.x), F32, ptr(L.attn_norm), F32, ptr(b.xn), F16, eps, H, M, s)
            lt, lb, lr = self._lora(L, "qkv", b.xn, M, s, b)
            if L.tiled:
                call("orch_q4t_qkv_rope", ptr(L.tqkv), ptr(b.xn), M, H, H, nh, ptr(b.pos), ptr(b.slots),
                     ptr(self.cos), ptr(self.sin), self.max_pos, ptr(b.q), ptr(kc), ptr(vc), self.max_seq,
                     self.num_slots, lt, lb, lr, s)
            else:
                call("orch_q4_qkv_rope", ptr(L.wqkv), ptr(L.sqkv), ptr(b.xn), M, H, H, nh, ptr(b.pos),
                     ptr(b.slots), ptr(self.cos), ptr(self.sin), self.max_pos, ptr(b.q), ptr(kc), ptr(vc),
                     self.max_seq, self.num_slots, lt, lb, lr, s)
        if units is not None:
            call("orch_attention_prefill", ptr(b.q), ptr(kc), ptr(vc), ptr(units), units.shape[0],
                 ptr(b.attn), M, nh, hd, self.max_seq, self.num_slots, s)
        else:
            call("orch_attention_decode", ptr(b.q), ptr(kc), ptr(vc), ptr(b.pos), ptr(b.slots),
                 ptr(b.attn), M, nh, hd, self.max_seq, self.num_slots, ptr(b.attn_ws), b.attn_ws_bytes, s)
        lt, lb, lr = self._lora(L, "o", b.attn, M, s, b)
        if L.tiled:
            call("orch_q4t_linear_resid", ptr(L.to), ptr(b.attn), ptr(b.x), M, H, H, lt, lb, lr, s)
        else:
            call("orch_q4_linear_resid", ptr(L.wo), ptr(L.so), ptr(b.attn), ptr(b.x), M, H, H, lt, lb, lr, s)
        if L.tiled and self.split is None and "gu" not in L.lora:
            call("orch_q4t_rms_linear_swiglu", ptr(L.t13), ptr(b.x), ptr(L.ffn_norm), eps, ptr(b.xn), ptr(b.h), M,
                 H, F, s)
            lt, lb, lr = self._lora(L, "down", b.h, M, s, b)
            call("orch_q4t_linear_resid", ptr(L.t2), ptr(b.h), ptr(b.x), M, F, H, lt, lb, lr, s)
            return
        call("orch_rmsnorm_ex", ptr(b.x), F32, ptr(L.ffn_norm), F32, ptr(b.xn), F16, eps, H, M, s)
        if self.split is not None:
            if "gu" in L.lora or "down" in L.lora:
                raise ValueError("LoRA on the FFN projections is not supported with the column split")
            sb = self.sdec if b is self.dec else self._split_bufs(b)
            ffn_column_split(self._split_ops, self._comm, L, sb, M)
            return
        lt, lb, lr = self._lora(L, "gu", b.xn, M, s, b)
        if L.tiled:
            call("orch_q4t_linear_swiglu", ptr(L.t13), ptr(b.xn), ptr(b.h), M, H, F, lt, lb, lr, s)
        else:
            call("orch_q4_linear_swiglu", ptr(L.w13), ptr(L.s13), ptr(b.xn), ptr(b.h), M, H, F, lt, lb, lr, s)
        lt, lb, lr = self._lora(L, "down", b.h, M, s, b)
        if L.tiled:
            call("orch_q4t_linear_resid", ptr(L.t2), ptr(b.h), ptr(b.x), M, F, H, lt, lb, lr, s)
        else:
            call("orch_q4_linear_resid", ptr(L.w2), ptr(L.s2), ptr(b.h), ptr(b.x), M, F, H, lt, lb, lr, s)

    def run_head(self, M: int, temperature: float = 0.0):
        """Final RMSNorm, INT4 lm_head (fp32 logits) and the next token into tok_out: the
        argmax, or for temperature > 0 a draw from softmax(logits / T) with the row's
        uniform in ``uniforms`` (orchard/model.py:244-252)."""
        b = self.dec
        cfg, s = self.cfg, _stream()
        H, V = cfg.hidden_size, cfg.vocab_size
        if self.heads_split:
            vocab_head_split(self._split_ops, self._comm, self.sdec, M)
            return
        if self.split is not None:
            head_column_split(self._split_ops, self._comm, self.sdec, M)
            return
        call("orch_rmsnorm_ex", ptr(b.x), F32, ptr(self.norm), F32, ptr(b.xn), F16, cfg.rms_norm_eps, H, M, s)
        if self.tiled:
            call("orch_q4t_gemm", ptr(self.lm_t), ptr(b.xn), ptr(b.logits), F32, H, V, M, s)
        else:
            call("orch_gemm_q4_0_ex", ptr(self.lm_w), ptr(self.lm_s), ptr(b.xn), F16, ptr(b.logits), F32,
                 H, V, M, s)
        if temperature > 0:
            call("orch_sample_rows", ptr(b.logits), M, V, float(temperature), ptr(b.uniforms), ptr(b.tok_out), s)
        else:
            call("orch_argmax_rows", ptr(b.logits), M, V, ptr(b.tok_out), s)

    def prefill_rows(self, tokens: np.ndarray, positions: np.ndarray, slots: np.ndarray, chunk: int = 4096):
        """Batched prefill: every prompt token is a row with its own position and cache slot,
        all layers run once per chunk of rows (rows of one sequence in position order). The
        projections take the tensor-core GEMM; attention is causal per row (each row attends
        to positions 0..pos of its slot, written by this or an earlier chunk)."""
        n = len(tokens)
        if self.split is not None:
            # every rank runs the same chunks (the FFN collectives): pad to the largest count
            import torch.distributed as dist
            cnt = torch.tensor([n, -n], dtype=torch.int64, device=self.device)
            dist.all_reduce(cnt, op=dist.ReduceOp.MAX, group=self.group)
            pad = int(cnt[0].item()) - n
            if self.heads_split and (pad or int(cnt[1].item()) != -n):
                raise ValueError("the head split runs the same rows on every rank: token counts differ")
            if pad:
                tokens = np.concatenate([np.asarray(tokens, np.int32), np.zeros(pad, np.int32)])
                positions = np.concatenate([np.asarray(positions, np.int32), np.zeros(pad, np.int32)])
                slots = np.concatenate([np.asarray(slots, np.int32), np.full(pad, self.scratch_slot, np.int32)])
                n += pad
        if n == 0:
            return
        rows = min(chunk, n)
        if self.pre is None or self.pre.rows < rows:
            self.pre = RowBuffers(rows, self.cfg, self.max_seq, self.device, logits=False, heads=self.nh_local)
        b = self.pre
        t_d = torch.as_tensor(np.asarray(tokens, np.int32)).to(self.device)
        p_d = torch.as_tensor(np.asarray(positions, np.int32)).to(self.device)
        s_d = torch.as_tensor(np.asarray(slots, np.int32)).to(self.device)
        pos_h, slots_h = np.asarray(positions, np.int32), np.asarray(slots, np.int32)
        for r0 in range(0, n, rows):
            m = min(rows, n - r0)
            b.tok_in[:m].copy_(t_d[r0:r0 + m])
            b.pos[:m].copy_(p_d[r0:r0 + m])
            b.slots[:m].copy_(s_d[r0:r0 + m])
            units = None
            if self.prefill_attention and self.cfg.head_dim == 128:
                units = torch.as_tensor(prefill_units(pos_h[r0:r0 + m], slots_h[r0:r0 + m])).to(self.device)
            self.run_layers(m, b, units)

    def _split_bufs(self, b: RowBuffers) -> _SplitBuffers:
        if self.spre is None or self.spre.x is not b.x:
            self.spre = _SplitBuffers(b, self.split, self.cfg, self.device)
        return self.spre

    def kernel_launches_per_step(self, M: int, logits: bool = True) -> int:
        """Kernels of this library one step launches (for reporting)."""
        L0 = self.layers[0]
        small = M <= _lib.lib().orch_gemv_max_rows()  # the GEMV normalises its own rows
        if self.heads_split:  # norm (above 8 rows) + qkv, attention, o, norm + gate/up, down
            per_layer = 5 + (0 if small else 2)
            if self.peer_allreduce and M * self.cfg.hidden_size <= self._comm.peer.max_floats:
                per_layer += 2  # the two all-reduces are this library's kernel
            if _lib.lib().orch_attention_workspace_bytes(M, self.nh_local, self.cfg.head_dim, self.max_seq) > 0:
                per_layer += 1
            return 1 + per_layer * len(self.layers) + (4 if logits else 0)
        per_layer = 7 + len(L0.lora)
        per_layer -= int(L0.tiled and "qkv" not in L0.lora and small)
        per_layer -= int(L0.tiled and self.split is None and "gu" not in L0.lora and small)
        if self.split is not None:
            per_layer += 1  # the residual add after the reduce-scatter
        n = 1 + per_layer * len(self.layers)
        if _lib.lib().orch_attention_workspace_bytes(M, self.cfg.num_attention_heads, self.cfg.head_dim,
                                                     self.max_seq) > 0:
            n += len(self.layers)
        return n + ((4 if self.split is not None else 3) if logits else 0)

    def step(self, M: int, logits: bool = True, graph: bool = True, temperature: float = 0.0):
        """One decode (or prefill) step for rows [0, M); with `graph` the step is replayed
        from a captured CUDA graph. ``temperature`` > 0 samples with the uniforms in
        ``self.dec.uniforms`` instead of taking the argmax."""
        if temperature > 0 and self.split is not None:
            raise ValueError("the column split samples greedily")
        key = (M, logits, float(temperature))
        if not graph:
            self.run_layers(M)
            if logits:
                self.run_head(M, temperature)
            return
        g = self.graphs.get(key)
        if g is None:
            # warm once outside capture (sets kernel attributes), then capture
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self.run_layers(M)
                if logits:
                    self.run_head(M, temperature)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.run_layers(M)
                if logits:
                    self.run_head(M, temperature)
            self.graphs[key] = g
            # capture only records; the step itself still has to run
        g.replay()

    def release_graphs(self):
        """Drops the captured steps (those of a column split hold NCCL calls and must go
        before the process group is destroyed)."""
        self.graphs.clear()
        torch.cuda.synchronize(self.device)

    def reset_cache(self):
        self.k_cache.zero_()
        self.v_cache.zero_()


# --------------------------------------------------------------------------------------
# public API
# --------------------------------------------------------------------------------------

class Llama:
    """``orchard.Llama`` on B200 (orchard/model.py:197-381).

    ``group`` (a torch.distributed NCCL group, one GPU per rank) splits the model over the
    ranks: by default each rank passes its own sequences and the FFN and vocabulary
    projections are split by columns; with ``split_heads`` every rank passes the same
    sequences and the attention heads are split as well (parallel.py)."""

    def __init__(self, model_path: Optional[str] = None, *, checkpoint: Optional[Checkpoint] = None,
                 device=0, max_batch: int = 32, max_seq: Optional[int] = None, tokenizer=None,
                 use_graphs: bool = True, tiled: bool = True, group=None, split_heads: bool = False):
        ck = checkpoint if checkpoint is not None else load_checkpoint(model_path)
        self.config = dict(ck.config)
        self.engine = DecodeEngine(ck, device=device, max_batch=max_batch, max_seq=max_seq, tiled=tiled,
                                   group=group, split_heads=split_heads)
        self.use_graphs = use_graphs
        self.tokenizer = tokenizer
        if tokenizer is None and model_path is not None:
            tp = os.path.join(model_path, "tokenizer.json")
            if os.path.exists(tp):
                try:
                    from tokenizers import Tokenizer
                    self.tokenizer = Tokenizer.from_file(tp)
                except ImportError:
                    self.tokenizer = None

    @classmethod
    def from_tensors(cls, config: dict, tensors: Dict[str, np.ndarray], **kw) -> "Llama":
        return cls(checkpoint=from_tensors(config, tensors), **kw)

    def load_lora(self, adapter_path: str):
        per_layer, r, _alpha = load_lora(adapter_path, self.engine.cfg.num_hidden_layers)
        self.engine.set_lora(per_layer, r)

    # -- sampling (orchard/model.py:244-252) --------------------------------------------
    @staticmethod
    def _sample(logits: np.ndarray, temperature: float) -> int:
        if temperature == 0:
            return int(np.argmax(logits))
        logits = logits - np.max(logits)
        probs = np.exp(logits / temperature) / np.sum(np.exp(logits / temperature))
        return int(np.random.choice(len(probs), p=probs))

    def generate_batch(self, prompts: List[str], max_tokens: int = 50, temperature: float = 0.7):
        if self.tokenizer is None:
            raise RuntimeError("Tokenizer not available")
        ids = [self.tokenizer.encode(p).ids for p in prompts]
        out = self.generate_batch_ids(ids, max_tokens=max_tokens, temperature=temperature)
        return [self.tokenizer.decode(seq) for seq in out]

    def prefill(self, prompt_ids: Sequence[Sequence[int]], chunk: int = 4096):
        """Fills the KV cache with every prompt in one batched pass per chunk of tokens (the
        reference feeds them one token at a time through the decode path, orchard/model.py:
        285-303; the cache contents are the same)."""
        eng = self.engine
        B = len(prompt_ids)
        if B > eng.max_batch:
            raise ValueError(f"batch {B} exceeds max_batch {eng.max_batch}")
        if any(len(p) == 0 for p in prompt_ids):
            raise ValueError("empty prompt")
        if max(len(p) for p in prompt_ids) + 1 > eng.max_seq:
            raise ValueError("prompt longer than the KV cache")
        toks = np.concatenate([np.asarray(p, np.int32) for p in prompt_ids])
        pos = np.concatenate([np.arange(len(p), dtype=np.int32) for p in prompt_ids])
        slots = np.concatenate([np.full(len(p), b, np.int32) for b, p in enumerate(prompt_ids)])
        eng.prefill_rows(toks, pos, slots, chunk=chunk)

    def generate_batch_ids(self, prompt_ids: Sequence[Sequence[int]], max_tokens: int = 50,
                           temperature: float = 0.7, ignore_eos: bool = False,
                           stats: Optional[dict] = None) -> List[List[int]]:
        """Token ids in, token ids out; the reference's generate_batch token flow.

        Every decode step copies that step's positions host->device (pinned) and the sampled
        tokens device->host. With temperature 0 the host reads a step's tokens two steps
        later, so one step is always queued behind the running one and the GPU never waits on
        the host; a row that produced EOS keeps computing for up to two steps (those tokens
        are dropped), which leaves every row's result unchanged. With temperature > 0 the softmax and the draw run on the
        device too: the host draws one uniform per active row from the global NumPy RNG, in
        row order (the draws np.random.choice makes in the reference), and copies them in
        with the positions. ``stats`` (optional dict) receives the prefill and decode
        wall times, steps run and bytes copied per step."""
        import time

        eng = self.engine
        B = len(prompt_ids)
        if eng.split is not None and temperature != 0:
            raise ValueError("the column split samples greedily on the device (temperature 0)")
        lens = np.array([len(p) for p in prompt_ids], np.int32)
        total = int(lens.max()) + max_tokens
        if total > eng.max_seq:
            raise ValueError(f"prompt + max_tokens ({total}) exceeds max_seq {eng.max_seq}")
        t0 = time.perf_counter()
        self.prefill(prompt_ids)
        torch.cuda.synchronize(eng.device)
        t1 = time.perf_counter()
        last = np.array([p[-1] for p in prompt_ids], np.int32)
        eng.tok_in[:B].copy_(torch.as_tensor(last).to(eng.device))
        pos_host = torch.empty((max_tokens, B), dtype=torch.int32, pin_memory=True)
        pos_host.copy_(torch.as_tensor(lens[None, :] + np.arange(max_tokens, dtype=np.int32)[:, None]))
        tok_host = torch.empty((max_tokens, B), dtype=torch.int32, pin_memory=True)
        u_host = torch.empty((max_tokens, B), dtype=torch.float32, pin_memory=True)
        gen: List[List[int]] = [[] for _ in range(B)]
        active = np.ones(B, dtype=bool)
        greedy = temperature == 0
        stream = torch.cuda.current_stream(eng.device)
        events: List[torch.cuda.Event] = []

        def consume(step):
            events[step].synchronize()
            nxt = tok_host[step].numpy()
            for b in np.nonzero(active)[0]:
                gen[b].append(int(nxt[b]))
                if not ignore_eos and nxt[b] == EOS_ID:
                    active[b] = False

        LAG = 2  # greedy: steps enqueued ahead of the host's reading of their tokens
        steps = 0
        consumed = 0
        for step in range(max_tokens):
            if greedy and step >= LAG:
                consume(step - LAG)
                consumed = step - LAG + 1
            if not active.any() and eng.split is None:  # split ranks stay in step together
                break
            eng.pos[:B].copy_(pos_host[step], non_blocking=True)
            if not greedy:  # one uniform per active row, in row order (the reference's draws)
                u = np.full(B, 0.5, np.float32)
                act = np.nonzero(active)[0]
                u[act] = np.random.random_sample(len(act))
                u_host[step].copy_(torch.as_tensor(u))
                eng.dec.uniforms[:B].copy_(u_host[step], non_blocking=True)
            eng.step(B, logits=True, graph=self.use_graphs, temperature=temperature)
            if greedy:
                eng.tok_in[:B].copy_(eng.tok_out[:B])
                tok_host[step].copy_(eng.tok_out[:B], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(stream)
                events.append(ev)
            else:
                tok_host[step].copy_(eng.tok_out[:B], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(stream)
                ev.synchronize()
                nxt = tok_host[step].numpy()
                for b in np.nonzero(active)[0]:
                    gen[b].append(int(nxt[b]))
                    if not ignore_eos and nxt[b] == EOS_ID:
                        active[b] = False
                eng.tok_in[:B].copy_(eng.tok_out[:B])
            steps += 1
        if greedy:
            for st in range(consumed, steps):
                if not active.any():
                    break
                consume(st)
        torch.cuda.synchronize(eng.device)
        t2 = time.perf_counter()
        if stats is not None:
            stats.update(prefill_s=t1 - t0, decode_s=t2 - t1, steps=steps, batch=B,
                         h2d_bytes_per_step=4 * B if greedy else 8 * B, d2h_bytes_per_step=4 * B)
        return gen
