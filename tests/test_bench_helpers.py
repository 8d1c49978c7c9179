"""CPU checks of bench.py's host-side helpers: the figures its JSON line reads from
committed files, and the chunk GEMM's executed-work count."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_profiled_traffic_reads_the_committed_summaries():
    assert bench._profiled_traffic("k_bwd_chunk_cfg4") == pytest.approx(18900.0)
    assert bench._profiled_traffic("no_such_kernel") is None


def test_peaks_have_the_roofline_denominators():
    peaks, source = bench._peaks()
    assert source in ("measured", "fallback")
    for key in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
        assert peaks[key] > 0


def _walk_chunk_gemm(B, N, T, KP1):
    """Executed flops by walking the kernel's work items: every full column block's tiles,
    then the last block's tiles (in pairs when it is at most 128 columns wide, which does
    not change the MMA work), each MMA 128 rows x its width x 16, six per 32-wide block."""
    ntg = (256 // KP1) & ~3
    ntiles = -(-N // ntg)
    last_src = N - (ntiles - 1) * ntg
    ncl = min(256, -(-(last_src * KP1) // 16) * 16)
    tiles_m = -(-B // 16)
    kb = -(-N // 32)
    items = [(n, m, 256) for n in range(ntiles - 1) for m in range(tiles_m)]
    if ncl <= 128:
        items += [(ntiles - 1, m, ncl) for m0 in range(0, tiles_m, 2) for m in (m0, m0 + 1) if m < tiles_m]
    else:
        items += [(ntiles - 1, m, ncl) for m in range(tiles_m)]
    assert len({(n, m) for n, m, _ in items}) == ntiles * tiles_m
    per_chunk = sum(kb * 2 * 3 * 2.0 * 128 * width * 16 for _, _, width in items)
    return per_chunk * -(-T // 8)


@pytest.mark.parametrize("B,N,T,KP1", [(256, 512, 250, 9), (40, 40, 25, 3), (130, 264, 64, 7),
                                       (256, 256, 250, 5), (64, 128, 128, 1), (33, 1024, 17, 9)])
def test_chunk_gemm_executed_flops_matches_a_walk_over_the_work_items(B, N, T, KP1):
    assert bench.chunk_gemm_executed_flops(B, N, T, KP1) == pytest.approx(_walk_chunk_gemm(B, N, T, KP1))


def test_cfg4_chunk_gemm_work():
    # 16 sample tiles x (18 full column blocks of 256 + the last block's 80 columns), the
    # 512-target reduction, 3 products, 32 chunks
    assert bench.chunk_gemm_executed_flops(256, 512, 250, 9) == pytest.approx(
        16 * (18 * 256 + 80) * 2.0 * 128 * 512 * 3 * 32)
