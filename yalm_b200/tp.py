"""Tensor-parallel partition of one decoder layer, as the engine holds it.

yb_create with tp_size > 1 gives rank r of P (yalm_b200/csrc/engine.cu, shard_table): Wq rows of a
block of whole query heads and the Wo columns of the same heads (row-parallel: partial sums over
heads); Wk, Wv rows of a block of whole kv heads, so each GQA group stays on one rank; W1, W3 rows of
a block of hidden units and the W2 columns of the same units (partial sums); a block of classifier
rows; the embedding and the norm weights replicated.  The only exchanges per layer are the sums of
the wo and w2 partials (added in rank order 0..P-1 on every rank) plus one gather of the logits per
output step.  shard() reads the engine's own table through the C ABI (yb_tp_shard: host
arithmetic, no GPU needed), so tests check the slices the engine uploads.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _lib


@dataclass(frozen=True)
class Shard:
    q_rows: slice      # rows of Wq (and columns of Wo)
    kv_rows: slice     # rows of Wk and Wv
    hidden: slice      # rows of W1 / W3, columns of W2
    vocab: slice       # rows of the classifier


def shard(config, rank: int, world: int) -> Shard:
    """Rank `rank` of `world`'s slices (yb_tp_shard); raises YalmB200Error for a world size the
    engine refuses (it must divide n_kv_heads, vocab_size and hidden_dim / 8)."""
    cfg = config.to_c()
    out = (ctypes.c_longlong * 8)()
    _lib.call("yb_tp_shard", ctypes.byref(cfg), int(rank), int(world), out)
    v = list(out)
    return Shard(q_rows=slice(v[0], v[1]), kv_rows=slice(v[2], v[3]), hidden=slice(v[4], v[5]),
                 vocab=slice(v[6], v[7]))
