"""Tensor-parallel partition of one decoder layer (host-side description).

The engine (yb_create with tp_size > 1, yalm_b200/csrc/engine.cu upload_weights) gives rank r of P:
  Wq rows of query heads [r*nh/P, (r+1)*nh/P)         Wk, Wv rows of kv heads [r*nkv/P, (r+1)*nkv/P)
  Wo columns of the same query heads                  (row-parallel: partial sums over heads)
  W1, W3 rows of hidden units [r*H/P, (r+1)*H/P)      W2 columns of the same hidden units (partials)
  classifier rows of vocabulary [r*V/P, (r+1)*V/P)    embedding and norm weights replicated
so each GQA group stays on one rank, attention needs no exchange, and the only exchanges per layer
are the sums of the wo and w2 partials (added in rank order 0..P-1 on every rank) plus one gather
of the logits per output step.  This module states the same slices for tests and tools.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    q_rows: slice      # rows of Wq (and columns of Wo)
    kv_rows: slice     # rows of Wk and Wv
    hidden: slice      # rows of W1 / W3, columns of W2
    vocab: slice       # rows of the classifier


def shard(config, rank: int, world: int) -> Shard:
    c = config
    if c.n_kv_heads % world or c.hidden_dim % (8 * world) or c.vocab_size % world:
        raise ValueError("world size must divide n_kv_heads, hidden_dim / 8 and vocab_size")
    nh, nkv = c.n_heads // world, c.n_kv_heads // world
    hd = c.head_dim
    h = c.hidden_dim // world
    v = c.vocab_size // world
    return Shard(q_rows=slice(rank * nh * hd, (rank + 1) * nh * hd),
                 kv_rows=slice(rank * nkv * hd, (rank + 1) * nkv * hd),
                 hidden=slice(rank * h, (rank + 1) * h),
                 vocab=slice(rank * v, (rank + 1) * v))
