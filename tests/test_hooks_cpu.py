"""Staging-ring bookkeeping of the offload hooks (ztcp_b200.hooks.CompactStagingRing), on unpinned host
memory: contiguous views, wrap-around with the skipped tail counted, out-of-order release reclaiming space
in ring order, and the full-ring error."""
from __future__ import annotations

import pytest


def test_ring_views_wrap_and_release_in_ring_order():
    from ztcp_b200.hooks import CompactStagingRing

    r = CompactStagingRing(10, 8, pin=False)
    a = r.reserve(4)
    b = r.reserve(4)
    assert (a.start, b.start, r.free_slots) == (0, 4, 2)
    assert tuple(a.blobs.shape) == (4, 8)
    with pytest.raises(RuntimeError, match="staging ring full"):
        r.reserve(3)  # needs a wrap, but slots 0..3 still belong to a
    r.release(b)      # not the oldest: its space waits for a
    assert r.free_slots == 2
    r.release(a)
    assert r.free_slots == 10
    c = r.reserve(3)  # head is at 8: the 2-slot tail is skipped
    assert (c.start, c.waste, r.free_slots) == (0, 2, 5)
    r.buffer.zero_()
    c.blobs.fill_(5)
    assert int(r.buffer[:3].sum()) == 3 * 8 * 5 and int(r.buffer[3:].sum()) == 0
    d = r.reserve(5)
    assert d.start == 3 and r.free_slots == 0
    with pytest.raises(RuntimeError):
        r.reserve(1)
    r.release(c)
    assert r.free_slots == 5
    with pytest.raises(ValueError):
        r.release(c)
    with pytest.raises(ValueError):
        r.reserve(11)
