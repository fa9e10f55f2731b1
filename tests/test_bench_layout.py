"""bench.py's strong-scaling split: the ranks' shards of every config are
contiguous, disjoint, cover the whole N = 1 tensor, and start at the offset
of their first element in the seeded global stream, so N shards filled by
the device generator are exactly the N = 1 tensor cut into N pieces."""
import numpy as np
import pytest

import bench
from tests import _oracle as O


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_strong_shards_partition_every_config(world):
    for n_attr, off_attr, total, unit in (("n1", "off1", bench.N1, 1), ("n2", "off2", bench.N2, 1),
                                          ("r4", "off4", bench.R4, bench.C4),
                                          ("n5", "off5", bench.N5, 1)):
        pos = 0
        for r in range(world):
            L = bench.Layout(r, world, "strong")
            assert getattr(L, off_attr) == pos * unit
            pos += getattr(L, n_attr)
        assert pos == total
    byte_total = sum(sum(bench.Layout(r, world, "strong").bytes.values()) for r in range(world))
    assert byte_total == sum(bench.BYTES.values())


def test_weak_shards_are_full_size():
    L = bench.Layout(3, 4, "weak")
    assert (L.n1, L.n2, L.r4, L.n5) == (bench.N1, bench.N2, bench.R4, bench.N5)
    assert L.off2 == 3 * bench.N2
    assert L.bytes == bench.BYTES


def test_generator_offsets_reassemble_the_whole_tensor():
    """The oracle's generator (which the device generator matches bit for
    bit, tests/test_parity_gpu.py) gives the same values for a shard filled
    at its offset as for the same slice of the whole tensor."""
    n, world = 100_003, 4
    whole = O.normal(n, 2)
    parts = [O.normal(*(lambda lo, hi: (hi - lo, 2, 0.0, 1.0, lo))(*bench.shard_of(n, r, world)))
             for r in range(world)]
    assert np.array_equal(np.concatenate(parts).view(np.uint32), whole.view(np.uint32))
