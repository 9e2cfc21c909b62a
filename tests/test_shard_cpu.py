"""Host logic of the output-row band sharding (no GPU)."""

import pytest

from torchcst_b200.shard import band


def test_bands_partition_the_chart():
    for n, world in [(8192, 8), (8192, 2), (1024, 4), (512, 1), (6144, 3)]:
        spans = [band(n, r, world) for r in range(world)]
        assert spans[0][0] == 0
        assert all(s + l == spans[k + 1][0] for k, (s, l) in enumerate(spans[:-1]))
        assert sum(l for _, l in spans) == n
        assert all(s % 32 == 0 and l % 32 == 0 for s, l in spans)


@pytest.mark.parametrize("n,world", [(1000, 4), (1024, 3), (96, 2)])
def test_bands_reject_uneven_or_unaligned(n, world):
    with pytest.raises(ValueError):
        band(n, 0, world)


def test_band_rank_range():
    with pytest.raises(ValueError):
        band(1024, 4, 4)
