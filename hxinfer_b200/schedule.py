"""Host mirror of the split-K decode schedule computed on the device.

The decode kernel (csrc/decode_attention.cu) flattens every (sequence,
kv head) segment into 64-position tiles, ordered sequence-major then kv head
then tile, and gives CTA c of C = min(grid, ceil(T/2)) the tiles
[c*T/C, (c+1)*T/C).  The part of a
segment inside one CTA is a *piece*.  A piece that starts at its segment's
first tile stores its partial result in slot ``seq*hkv + head``; a CTA's
first piece that starts inside a segment stores it in slot ``n_segments + c``.
The combine step merges, for each segment, slot ``seg`` with the slots of the
CTAs whose non-empty range starts strictly inside the segment.

This module restates that arithmetic in Python so CPU tests can check that
every tile is covered once, that no two pieces share a slot and that the
combine step finds every piece, for any lengths and CTA count.
"""
from __future__ import annotations

BLOCK = 64
MIN_TILES_PER_CTA = 2  # the device gives each working CTA at least this many tiles


def tiles_of(length: int) -> int:
    return (max(length, 0) + BLOCK - 1) // BLOCK


def segment_ranges(lengths, hkv):
    """[(seg, a, b)] global tile range of each segment, seg = s*hkv + h."""
    out, run = [], 0
    for s, L in enumerate(lengths):
        t = tiles_of(L)
        for h in range(hkv):
            out.append((s * hkv + h, run, run + t))
            run += t
    return out, run


def effective_ctas(total: int, grid: int) -> int:
    """CTAs that receive work: min(grid, ceil(T / MIN_TILES_PER_CTA)), at least 1."""
    return max(1, min(grid, -(-total // MIN_TILES_PER_CTA)))


def cta_range(total: int, c: int, n_ctas: int):
    return total * c // n_ctas, total * (c + 1) // n_ctas


def pieces(lengths, hkv, n_ctas):
    """Pieces as written by the decode kernel: (cta, seg, first_tile, last_tile, slot, whole)."""
    segs, total = segment_ranges(lengths, hkv)
    n_seg = len(segs)
    n_ctas = effective_ctas(total, n_ctas)
    out = []
    for c in range(n_ctas):
        g0, g1 = cta_range(total, c, n_ctas)
        first = True
        for seg, a, b in segs:
            lo, hi = max(a, g0), min(b, g1)
            if lo >= hi:
                continue
            from_start = lo == a
            slot = seg if from_start else n_seg + c
            assert first or from_start, "only a CTA's first piece can start inside a segment"
            out.append((c, seg, lo, hi, slot, from_start and hi == b))
            first = False
    return out


def combine_slots(lengths, hkv, n_ctas, seg: int):
    """Slots the combine kernel reads for `seg` ([] when one piece wrote the output)."""
    segs, total = segment_ranges(lengths, hkv)
    n_seg = len(segs)
    n_ctas = effective_ctas(total, n_ctas)
    _, a, b = segs[seg]
    if a == b:
        return []

    def cstart(c):
        return total * c // n_ctas

    extra = [n_seg + c for c in range(a * n_ctas // total, n_ctas)
             if cstart(c) < b and cstart(c) > a and cstart(c + 1) > cstart(c)]
    return [seg] + extra if extra else []


def workspace_slots(n_seqs: int, hkv: int, n_ctas: int) -> int:
    return n_seqs * hkv + n_ctas
