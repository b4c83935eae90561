"""bench.py's bookkeeping on CPU: the backward's ncu traffic scaled to a
rank's share of the config-2 batch, and this library's kernel count per
config-4 sequence-parallel step for each exchange (what the JSON line's
``roofline.traffic`` and ``gpu_launches`` report)."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "ema-kernels_b200"))
    import bench as b
    return b


def test_traffic_scales_with_the_rank_share(bench):
    full = bench._profile_traffic()
    assert full is not None and full > 3e8  # the committed capture of one whole config-2 backward
    assert bench._profile_traffic(bench.TOKENS) == pytest.approx(full)
    for world in (2, 4, 8):
        assert bench._profile_traffic(bench.TOKENS / world) == pytest.approx(full / world)


def test_sp_kernel_count_per_step(bench):
    # one GPU, 16 sub-spans: per direction the column sums, the expansion fold, dt transpose, scan
    assert bench._sp_launches_per_step(1) == 8
    # several GPUs: plus the summary fold per direction; with "p2p" one exchange kernel
    # replaces both folds
    assert bench._sp_launches_per_step(2, "chain") == 10
    assert bench._sp_launches_per_step(4, "allgather") == 10
    assert bench._sp_launches_per_step(8, "p2p") == 8
