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
]


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
