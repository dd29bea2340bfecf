"""Host checks of the split-K decode schedule (hxinfer_b200/schedule.py mirrors
the device arithmetic of csrc/decode_attention.cu)."""
import numpy as np
import pytest

from hxinfer_b200 import schedule as S


CASES = [
    ([1025], 4, 148),                 # Qwen decode, one sequence
    ([32769], 4, 148),                # Qwen decode at 32k
    ([1], 8, 148),                    # a single position
    ([64, 65, 63, 1, 128], 2, 7),     # block boundaries, few CTAs
    ([0, 5, 0, 70], 3, 5),            # empty sequences
    (list(np.random.default_rng(4).integers(512, 32769, 64)), 8, 148),  # batched LLaMA-3 shape
    ([3] * 10, 1, 148),               # more CTAs than tiles
    (list(np.random.default_rng(4).integers(512, 32769, 64)), 8, 296),  # two CTAs per SM
    (list(np.random.default_rng(5).integers(1, 4000, 40)), 2, 296),     # wide grid, short segments
]


def test_pieces_per_segment_fit_the_device_bound():
    """The device keeps at most kMaxPieces (300) pieces per segment, and a
    launch uses at most 298 CTAs (kMaxPieces - 2): every segment's slot list
    fits for any lengths."""
    for lengths, hkv in (([32769], 4), ([200000], 1), ([64] * 3, 8)):
        for ctas in (148, 296, 298):
            segs, _ = S.segment_ranges(lengths, hkv)
            for seg, _, _ in segs:
                assert len(S.combine_slots(lengths, hkv, ctas, seg)) <= 300


@pytest.mark.parametrize("lengths,hkv,ctas", CASES)
def test_every_tile_covered_once(lengths, hkv, ctas):
    segs, total = S.segment_ranges(lengths, hkv)
    cover = np.zeros(total, np.int32)
    for c, seg, lo, hi, slot, whole in S.pieces(lengths, hkv, ctas):
        cover[lo:hi] += 1
    assert np.all(cover == 1)


@pytest.mark.parametrize("lengths,hkv,ctas", CASES)
def test_slots_unique_and_in_range(lengths, hkv, ctas):
    ps = S.pieces(lengths, hkv, ctas)
    slots = [p[4] for p in ps if not p[5]]
    assert len(slots) == len(set(slots))
    assert all(0 <= s < S.workspace_slots(len(lengths), hkv, ctas) for s in slots)


@pytest.mark.parametrize("lengths,hkv,ctas", CASES)
def test_combine_finds_exactly_the_pieces(lengths, hkv, ctas):
    ps = S.pieces(lengths, hkv, ctas)
    segs, _ = S.segment_ranges(lengths, hkv)
    for seg, a, b in segs:
        mine = [p for p in ps if p[1] == seg]
        want = sorted(p[4] for p in mine) if len(mine) > 1 else []
        assert sorted(S.combine_slots(lengths, hkv, ctas, seg)) == want
        if len(mine) == 1:
            assert mine[0][5]  # the single piece is whole and writes the output


def test_schedule_invariants_on_random_batches():
    """Seeded random batches (lengths 0..70,000, 1-16 kv heads, grids up to
    298 CTAs): every tile is covered once, piece slots are unique and inside
    the workspace, and the combine finds exactly the split pieces."""
    rng = np.random.default_rng(2026)
    for _ in range(40):
        n = int(rng.integers(1, 40))
        lengths = [int(x) for x in rng.integers(0, 70000, n)]
        if rng.random() < 0.3:
            lengths[int(rng.integers(0, n))] = 0
        hkv = int(rng.choice([1, 2, 4, 8, 16]))
        ctas = int(rng.integers(1, 299))
        test_every_tile_covered_once(lengths, hkv, ctas)
        test_slots_unique_and_in_range(lengths, hkv, ctas)
        test_combine_finds_exactly_the_pieces(lengths, hkv, ctas)
