"""Multi-GPU partitioning of batched decode attention (one process per GPU).

Attention heads are independent once q/k/v exist; a GQA group lives inside
its kv head; sequences are independent.  So a decode step shards with no
exchange until the per-rank outputs are gathered:

* ``kv_heads`` (world == number of kv heads, e.g. 8 GPUs x 8 kv heads): rank r
  holds kv head r (and its q heads) of every sequence;
* ``sequences`` (world < kv heads): rank r holds a length-balanced subset of
  the sequences with every head.

After each layer the per-rank outputs are all-gathered; ``assemble`` turns
the gathered buffer back into the reference output layout
[sequence][q_head * head_dim] (attention_score_cuda.cu:81, output index
head_idx*head_dim + d).  The reference has no multi-GPU mode; this is new.
"""
from __future__ import annotations

import numpy as np


def balance_sequences(lengths, world: int):
    """Deal sequences, longest first, to `world` groups in snake order
    (0..W-1, W-1..0, ...): group sizes differ by at most one (so an all-gather
    of padded per-rank outputs stays uniform) and total lengths stay close.
    Each group is returned sorted."""
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    groups = [[] for _ in range(world)]
    for k, i in enumerate(order):
        rnd, pos = divmod(k, world)
        groups[pos if rnd % 2 == 0 else world - 1 - pos].append(i)
    return [sorted(g) for g in groups]


def plan(world: int, n_kv_heads: int, lengths):
    """Per-rank (sequence indices, kv-head indices) and the mode name."""
    n = len(lengths)
    if world == 1:
        return "replica", [(list(range(n)), list(range(n_kv_heads)))]
    if world >= n_kv_heads:
        if world % n_kv_heads:
            raise ValueError(f"{world} ranks cannot split {n_kv_heads} kv heads evenly")
        # kv heads first; ranks beyond one per head would split sequences too
        reps = world // n_kv_heads
        out = []
        for r in range(world):
            h = r // reps
            groups = balance_sequences(lengths, reps)
            out.append((groups[r % reps], [h]))
        return "kv_heads", out
    groups = balance_sequences(lengths, world)
    return "sequences", [(g, list(range(n_kv_heads))) for g in groups]


def assemble(mode: str, parts, shards, n_seqs: int, n_q_heads: int, head_dim: int):
    """Reference-layout output [n_seqs][n_q_heads*head_dim] from per-rank
    outputs parts[r] of shape [len(seqs_r)][len(heads_r)*group*head_dim]."""
    out = np.zeros((n_seqs, n_q_heads * head_dim), dtype=np.asarray(parts[0]).dtype)
    n_kv = max(h for _, hs in shards for h in hs) + 1
    group = n_q_heads // n_kv
    for part, (seqs, heads) in zip(parts, shards):
        if not len(seqs):
            continue  # a rank without sequences contributes nothing
        part = np.asarray(part).reshape(len(seqs), len(heads), group * head_dim)
        rows = np.asarray(seqs, dtype=np.int64)
        for j, h in enumerate(heads):
            out[rows, h * group * head_dim:(h + 1) * group * head_dim] = part[:, j]
    return out
