"""Column split of the large-N projections across the GPUs of one box, and the head split.

Two arrangements. In the column split sequences are sharded data-parallel (each rank owns
``B / world`` rows with their KV cache, attention and Q/K/V/O projections, whose weights
every rank holds), and the two large-N projections are split by columns:

* FFN: rank r holds gate/up rows ``F[f0:f1]`` and the matching down-projection columns
  ``W2[:, f0:f1]`` (a K split). Per layer: all-gather the normed hidden state of every
  rank's rows, gate/up + SwiGLU on the local slice for all rows, the down projection of
  the local slice (a partial sum over K) for all rows, a reduce-scatter that sums the
  partials and hands each rank its own rows, and the residual add: two collectives.
* vocab: rank r holds lm_head rows ``V[v0:v1]``; after the final norm the rows are
  all-gathered, each rank takes the (max, argmax) of its vocabulary slice, the pairs are
  all-gathered and merged (highest logit, lowest id on ties, as ``np.argmax``).

The head split (``ColumnSplit.plan(..., num_heads=nh)``) also divides the attention: every
rank runs all rows (the residual is the same on every rank), rank r holds attention heads
``[h0, h1)``: those heads' rows of Wq / Wk / Wv, their K/V cache, and the O projection's
columns ``Wo[:, h0*hd:h1*hd]`` (a K split), beside the FFN and vocabulary slices above.
Per layer two all-reduces of the fp32 residual: after the O projection and after the down
projection, each rank adding its partial sum over K and rank 0 also the residual itself.
Nothing of the model is replicated, so at batch 1 every weight byte and every KV byte is
read by one rank only.

This module holds the split arithmetic and the order of operations; the device buffers,
kernels and collectives are supplied by the caller (``ops`` / ``comm`` objects), so the
same orchestration runs on the GPUs (NCCL) and, in the tests, on CPU ranks (gloo) with
NumPy kernels.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple

import numpy as np


def shard_range(n: int, world: int, rank: int, align: int = 32) -> Tuple[int, int]:
    """Contiguous slice of ``n`` for ``rank``: every boundary is a multiple of ``align``
    (the last slice ends at ``n``); slices differ by at most one ``align`` unit."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    units = -(-n // align)
    lo = (units * rank // world) * align
    hi = min(n, (units * (rank + 1) // world) * align)
    return lo, hi


def local_rows(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """The rows (sequences) rank ``rank`` owns when ``batch`` rows are sharded."""
    if batch % world:
        raise ValueError(f"batch {batch} is not a multiple of world size {world}")
    per = batch // world
    return rank * per, (rank + 1) * per


@dataclass
class ColumnSplit:
    """Which columns of the large-N projections one rank holds."""

    world: int
    rank: int
    f0: int
    f1: int
    v0: int
    v1: int
    h0: int = 0  # attention heads [h0, h1) of the head split; h1 == 0: heads not split
    h1: int = 0

    @classmethod
    def plan(cls, intermediate_size: int, vocab_size: int, world: int, rank: int,
             num_heads: int = 0, head_dim: int = 0) -> "ColumnSplit":
        """``num_heads`` > 0 plans the head split as well (``head_dim`` a multiple of 32, so
        each rank's slice of the O projection's K starts on a scale group)."""
        # FFN slices: multiples of 32 (one INT4 scale group, so the down projection's K
        # slice starts on a group; also the gate/up interleave's 16-row blocks)
        f0, f1 = shard_range(intermediate_size, world, rank, 32)
        v0, v1 = shard_range(vocab_size, world, rank, 16)
        if f1 <= f0 or v1 <= v0:
            raise ValueError("too many ranks for these projection sizes")
        h0 = h1 = 0
        if num_heads:
            if head_dim <= 0 or head_dim % 32:
                raise ValueError("the head split needs a head_dim that is a multiple of 32")
            if num_heads < world:
                raise ValueError(f"{world} ranks cannot split {num_heads} attention heads")
            h0, h1 = shard_range(num_heads, world, rank, 1)
        return cls(world, rank, f0, f1, v0, v1, h0, h1)

    @property
    def heads(self) -> bool:
        """True for the head split (rows replicated, attention heads divided)."""
        return self.h1 > 0

    @property
    def h_local(self) -> int:
        return self.h1 - self.h0

    @property
    def f_local(self) -> int:
        return self.f1 - self.f0

    @property
    def v_local(self) -> int:
        return self.v1 - self.v0

    def ffn_shard(self, w1, s1, w3, s3, w2, s2):
        """Slices of packed INT4 FFN weights (reference layout: packed ``[N, K/2]``, scales
        ``[N, K/32]``; NumPy arrays or torch tensors): gate/up rows ``f0:f1`` and the down
        projection's columns ``f0:f1`` (bytes ``f0/2:f1/2``, scale groups ``f0/32:f1/32``)."""
        f0, f1 = self.f0, self.f1
        return (w1[f0:f1], s1[f0:f1], w3[f0:f1], s3[f0:f1],
                w2[:, f0 // 2:f1 // 2], s2[:, f0 // 32:f1 // 32])

    def lm_shard(self, w, s):
        """lm_head rows ``v0:v1`` (packed and scales)."""
        return w[self.v0:self.v1], s[self.v0:self.v1]

    def attn_shard(self, wq, sq, wk, sk, wv, sv, wo, so, head_dim: int):
        """Slices of packed INT4 attention weights for heads ``h0:h1``: the rows
        ``h0*hd:h1*hd`` of Wq, Wk and Wv, and the same range of the O projection's columns
        (bytes ``/2``, scale groups ``/32``)."""
        if not self.heads:
            raise ValueError("this plan does not split the heads")
        r0, r1 = self.h0 * head_dim, self.h1 * head_dim
        return (wq[r0:r1], sq[r0:r1], wk[r0:r1], sk[r0:r1], wv[r0:r1], sv[r0:r1],
                wo[:, r0 // 2:r1 // 2], so[:, r0 // 32:r1 // 32])


def merge_argmax(vals: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """Merge per-rank (max logit, global id) pairs ``[world, B]`` into the token of each row:
    the highest value; among equal values the lowest id (ranks hold ascending id ranges, so
    this is ``np.argmax`` over the full row). A NaN wins, as in ``np.argmax``."""
    vals = np.asarray(vals, np.float32)
    idx = np.asarray(idx, np.int64)
    out = np.empty(vals.shape[1], np.int64)
    for b in range(vals.shape[1]):
        best_v, best_i = vals[0, b], idx[0, b]
        for r in range(1, vals.shape[0]):
            v, i = vals[r, b], idx[r, b]
            if np.isnan(best_v):
                break
            if np.isnan(v) or v > best_v or (v == best_v and i < best_i):
                best_v, best_i = v, i
        out[b] = best_i
    return out


# ------------------------------------------------------------------------------------------
# order of operations (shared by the GPU engine and the CPU tests)
# ------------------------------------------------------------------------------------------

def ffn_column_split(ops, comm, layer, bufs, rows: int) -> None:
    """FFN half of one layer for this rank's ``rows`` local rows (residual ``bufs.x``):

        xn      = rmsnorm(x)                    local rows
        xn_all  = all_gather(xn)                every rank's rows, rank-major
        h       = silu(xn_all Wg^T) * (xn_all Wu^T)   local F slice, all rows
        part    = h W2[:, slice]^T              partial over K, all rows, fp32
        red     = reduce_scatter(part)          summed, this rank's rows
        x      += red
    """
    ops.rmsnorm(bufs.x, layer.ffn_norm, bufs.xn, rows)
    comm.all_gather(bufs.xn_all, bufs.xn, rows)
    ops.gate_up_swiglu(layer, bufs.xn_all, bufs.h, rows * comm.world)
    ops.down_partial(layer, bufs.h, bufs.part, rows * comm.world)
    comm.reduce_scatter(bufs.red, bufs.part, rows)
    ops.add(bufs.x, bufs.red, rows)


def head_column_split(ops, comm, bufs, rows: int) -> None:
    """Final norm, vocabulary-split lm_head and the merged argmax: ``bufs.tok`` receives
    the next token of each of this rank's ``rows`` rows."""
    ops.rmsnorm(bufs.x, None, bufs.xn, rows)
    comm.all_gather(bufs.xn_all, bufs.xn, rows)
    ops.lm_partial(bufs.xn_all, bufs.logits, rows * comm.world)
    ops.argmax_pairs(bufs.logits, bufs.pairs, rows * comm.world)
    comm.all_gather(bufs.pairs_all, bufs.pairs, rows * comm.world)
    ops.merge_pairs(bufs.pairs_all, bufs.tok, rows)


# ------------------------------------------------------------------------------------------
# head split: every rank runs all rows; attention heads, FFN and vocabulary divided
# ------------------------------------------------------------------------------------------

def attention_head_split(ops, comm, layer, bufs, rows: int) -> None:
    """Attention half of one layer for all ``rows`` rows (the residual ``bufs.x`` is the same
    on every rank):

        q, k, v = rmsnorm(x) [Wq; Wk; Wv][heads h0:h1]^T, RoPE, k / v into this rank's cache
        a       = attention(q, k, v)                 this rank's heads
        x       = x + a Wo[:, h0:h1]^T  on rank 0,   a Wo[:, h0:h1]^T  on the others (fp32)
        x       = all_reduce_sum(x)
    """
    ops.qkv_local(layer, bufs, rows)
    ops.attention_local(layer, bufs, rows)
    ops.o_partial(layer, bufs, rows, comm.rank == 0)
    comm.all_reduce(bufs.x, rows)


def ffn_head_split(ops, comm, layer, bufs, rows: int) -> None:
    """FFN half of one layer for all ``rows`` rows:

        h = silu(rmsnorm(x) Wg[f0:f1]^T) * (rmsnorm(x) Wu[f0:f1]^T)
        x = x + h W2[:, f0:f1]^T  on rank 0,  h W2[:, f0:f1]^T  on the others (fp32)
        x = all_reduce_sum(x)
    """
    ops.gate_up_local(layer, bufs, rows)
    ops.down_partial_resid(layer, bufs, rows, comm.rank == 0)
    comm.all_reduce(bufs.x, rows)


def vocab_head_split(ops, comm, bufs, rows: int) -> None:
    """Final norm and the vocabulary-split lm_head for all ``rows`` rows: each rank's
    (max, id) pair per row, gathered and merged; ``bufs.tok`` receives every row's token."""
    ops.rmsnorm(bufs.x, None, bufs.xn, rows)
    ops.lm_partial(bufs.xn, bufs.logits, rows)
    ops.argmax_pairs(bufs.logits, bufs.pairs, rows)
    comm.all_gather(bufs.pairs_all, bufs.pairs, rows)
    ops.merge_all_pairs(bufs.pairs_all, bufs.tok, rows)
