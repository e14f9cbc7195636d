"""Host logic of the GEMM / scatter overlap: the token-chunk plan (CPU)."""

import pytest

from sparkdiffusion_b200.ulysses import chunk_plan


@pytest.mark.parametrize("rows", [1, 90, 127, 128, 360, 9450, 18900, 37800, 75600, 16380])
def test_chunks_cover_rows_in_whole_tiles(rows):
    plan = chunk_plan(rows, 60, 148)
    assert sum(plan) == rows
    assert all(n > 0 for n in plan)
    assert all(n % 128 == 0 for n in plan[:-1])  # every chunk but the last is whole 128-row tiles


def test_halving_plan_ends_small():
    plan = chunk_plan(9450, 60, 148)  # 8-GPU shard of the 720P layer
    assert plan[0] >= plan[-1] and plan[-1] <= 8 * 128
    # the first chunk fills the 148 persistent CTAs in whole waves (37 M-tiles x 60 N-tiles)
    assert plan[0] == 37 * 128


def test_forced_equal_chunks():
    assert chunk_plan(360, 6, 148, 4) == [128, 128, 104]
    assert chunk_plan(1000, 60, 148, 1) == [1000]
