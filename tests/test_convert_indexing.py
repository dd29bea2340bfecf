"""The index arithmetic of hx_convert's kernel (hxinfer_b200/csrc/convert.cu:
launch_convert + convert_kernel), restated and checked on the CPU: for every
size, alignment and grid the kernel can get, each element is converted
exactly once and no access leaves [0, n).  Restates, and must track, the CUDA
code: 8-element groups only when both pointers are 16-byte aligned, the
n % 8 tail (or everything) element by element, a grid-stride loop over
groups + tail units, grid = max(1, min(ceil(units / 256), SMs * 8))."""
import numpy as np
import pytest

THREADS = 256


def covered(n: int, aligned: bool, sms: int) -> np.ndarray:
    groups = n // 8 if aligned else 0
    tail = n - 8 * groups
    units = groups + tail
    blocks = max(1, min((units + THREADS - 1) // THREADS, sms * 8))
    stride = blocks * THREADS
    hits = np.zeros(n, np.int64)
    # the grid-stride loop visits each unit u < units once (thread u % stride)
    assert stride >= 1
    u = np.arange(units, dtype=np.int64)
    g = u[u < groups]
    if g.size:
        idx = (8 * g[:, None] + np.arange(8)[None, :]).ravel()  # get8/put8 of group g
        assert idx.min() >= 0 and idx.max() < n
        np.add.at(hits, idx, 1)
    e = 8 * groups + (u[u >= groups] - groups)  # single elements
    if e.size:
        assert e.min() >= 0 and e.max() < n
        np.add.at(hits, e, 1)
    return hits


@pytest.mark.parametrize("sms", [1, 148])
@pytest.mark.parametrize("aligned", [True, False])
def test_every_element_exactly_once(aligned, sms):
    for n in list(range(1, 70)) + [255, 256, 257, 2047, 2048, 2049, 8 * 256 * 148 * 8 + 13,
                                   65533, 65536, 8388613, 4194307]:
        hits = covered(n, aligned, sms)
        assert hits.min() == 1 and hits.max() == 1, (n, aligned, sms)


def test_vector_accesses_stay_16_byte_aligned():
    # with both base pointers 16-byte aligned, group g starts at byte 16 g (2-byte
    # elements) or 32 g (4-byte elements): every uint4 / float4 access is aligned
    for esize in (2, 4):
        for g in range(0, 1000, 37):
            assert (8 * g * esize) % 16 == 0
