"""CPU checks of bench.py's host-side arithmetic: the strong-scaling row split, the GEMM tile-wave counts it reports,
the algorithmic op count and the config block, so that the bench line's derived numbers are right before any GPU
time is spent."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench as B  # noqa: E402
from h3q import parallel as P  # noqa: E402


def test_row_split_matches_the_library():
    for world in (1, 2, 4, 8):
        ranges = [B.row_range(B.M_TOKENS, world, r) for r in range(world)]
        assert ranges == [P.row_range(B.M_TOKENS, world, r) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == B.M_TOKENS
    assert B.row_range(B.M_TOKENS, 8, 3) == (12285, 16380)


def test_ops_per_step_counts_the_four_linears():
    want = 2.0 * 32760 * (5120 * 15360 + 5120 * 13824 + 5120 * 5120 + 13824 * 5120)
    assert B.ops_per_step(32760) == want
    assert abs(want / 1e12 - 16.145) < 1e-3


@pytest.mark.parametrize("m,n,tiles,eff", [(32760, 15360, 7680, 0.998), (4095, 5120, 320, 0.865),
                                           (4095, 15360, 960, 0.998), (16380, 5120, 1280, 0.961)])
def test_tile_waves(m, n, tiles, eff):
    t = B.tile_waves(m, n)
    assert t["tiles"] == tiles and t["wave_efficiency"] == eff


def test_config_block_states_the_split():
    c1 = B.config_block(1)
    c8 = B.config_block(8)
    assert c1["M_total"] == c8["M_total"] == 32760
    assert c1["M_per_gpu"] == 32760 and c8["M_per_gpu"] == 4095
    assert "strong" in c8["parallelism"] and "4095-4095" in c8["parallelism"]
    assert "flush" in c1["l2"]
